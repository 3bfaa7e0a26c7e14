// kernels.cu — bandwidth-bound kernels of the compressed path:
//   * block compressor (mean pool)          bna/torch/attention_wayfinder_permute.py:1022-1043
//   * two-pool cache append / block close    bna/mlx/compressed_cache.py:104-149
//   * active / decode attention              attention_wayfinder_permute.py:1125-1197,
//                                            bna/mlx/attention.py:1669-1876
//   * device dump of the prefill selection   attention_wayfinder_permute.py:912-966
// All use coalesced 128-bit loads, shared-memory staging and warp-shuffle reductions.
#include <cuda_runtime.h>

#include "common.cuh"
#include "route.cuh"
#include "sm100.cuh"

namespace bna {
// Device error word: kernels that give up a bounded wait record a code here.
__device__ int g_device_error = 0;

int* device_error_word() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
  return static_cast<int*>(p);
}

struct View4 {  // device-side strided [B, H, T, dh] view (element strides)
  void* data;
  int64_t sb, sh, st;
};

static View4 to_view(const bna_tensor4* t) {
  return View4{t->data, t->stride[0], t->stride[1], t->stride[2]};
}

// Row address of token index `idx` of (b, h).
__device__ __forceinline__ uint8_t* row_ptr(const View4& v, int b, int h, int64_t idx) {
  return reinterpret_cast<uint8_t*>(v.data) + 2 * (b * v.sb + h * v.sh + idx * v.st);
}

// ------------------------------------------------------------------------------ compressor
// One CTA (128 threads) per (block, b*h).  Thread = (16-byte chunk of head_dim, token lane);
// fp32 partial sums reduced through shared memory; mean rounded to the storage dtype.
template <typename T>
__device__ __forceinline__ void block_mean(const View4& src, int b, int h, int64_t first_pos, int count,
                                           int64_t pos_base, int64_t ring, int dh, float* red, uint8_t* dst_row) {
  const int chunks = dh >> 3;            // 16-byte chunks per row
  const int lanes = blockDim.x / chunks;  // token lanes
  const int ch = threadIdx.x % chunks, tl = threadIdx.x / chunks;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  // cache index of first_pos (one modulo); rows step from it with a wrap
  const int64_t idx0 = ring > 0 ? first_pos % ring : first_pos - pos_base;
  if (tl < lanes) {
#pragma unroll 8
    for (int j = tl; j < count; j += lanes) {
      int64_t idx = idx0 + j;
      if (ring > 0 && idx >= ring) idx -= ring;
      const uint4 u = ld_nc_128(row_ptr(src, b, h, idx) + ch * 16);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = ElemTraits<T>::unpack2(w[e]);
        acc[2 * e] += f.x;
        acc[2 * e + 1] += f.y;
      }
    }
  }
  __syncthreads();
  if (tl < lanes) {
#pragma unroll
    for (int e = 0; e < 8; ++e) red[tl * dh + ch * 8 + e] = acc[e];
  }
  __syncthreads();
  const float inv_cnt = 1.f / (float)(count > 0 ? count : 1);
  for (int d = threadIdx.x; d < dh; d += blockDim.x) {
    float s = 0.f;
    for (int r = 0; r < lanes; ++r) s += red[r * dh + d];
    const float mval = s * inv_cnt;
    const uint32_t packed = ElemTraits<T>::pack2(mval, 0.f);
    *reinterpret_cast<uint16_t*>(dst_row + 2 * d) = (uint16_t)(packed & 0xFFFFu);
  }
}

struct CompressArgs {
  View4 src, dst, src2, dst2;  // src2/dst2: second tensor of a K/V pair (blockIdx.z == 1)
  int H, dh, block_size;
  int64_t pos0, valid_len, ring, slot0;
};

// 256 threads: 16 head_dim chunks x 16 token lanes, so a 128-token block is one round of
// eight independent 128-bit loads per thread (all in flight together).
constexpr int kCompressThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kCompressThreads) compress_kernel(const CompressArgs a) {
  __shared__ float red[kCompressThreads * 8];
  // programmatic dependent launch: wait for the previous kernel of the stream, then let
  // the next one start launching
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int j = blockIdx.x;
  const int b = blockIdx.y / a.H, h = blockIdx.y % a.H;
  const int64_t first = a.pos0 + (int64_t)j * a.block_size;
  int64_t cnt = a.valid_len - (int64_t)j * a.block_size;
  if (cnt > a.block_size) cnt = a.block_size;
  if (cnt < 1) cnt = 0;
  const bool second = blockIdx.z == 1;
  block_mean<T>(second ? a.src2 : a.src, b, h, first, (int)cnt, a.pos0, a.ring, a.dh, red,
                row_ptr(second ? a.dst2 : a.dst, b, h, a.slot0 + j));
}

// ------------------------------------------------------------------------------ cache append
struct AppendArgs {
  View4 src_k, src_v, ring_k, ring_v;
  int H, dh;
  int64_t pos0, ring;
};

__global__ void __launch_bounds__(128) append_kernel(const AppendArgs a) {
  const int tok = blockIdx.x;
  const int b = blockIdx.y / a.H, h = blockIdx.y % a.H;
  const int chunks = a.dh >> 3;
  const int64_t slot = (a.pos0 + tok) % a.ring;
  for (int c = threadIdx.x; c < 2 * chunks; c += blockDim.x) {
    const bool isv = c >= chunks;
    const int ch = isv ? c - chunks : c;
    const uint4 u = ld_nc_128(row_ptr(isv ? a.src_v : a.src_k, b, h, tok) + ch * 16);
    st_128(row_ptr(isv ? a.ring_v : a.ring_k, b, h, slot) + ch * 16, u);
  }
}

// ------------------------------------------------------------------------------ active / decode
// One CTA (512 threads) per (query index, b * Hkv) serves the G query heads of a KV head.
// One round trip of cp.async brings the raw window rows, the routed summary rows (when the
// host routed them) and the G query rows into shared memory.  Scores: one thread per
// (key, head) dot product; softmax: one warp per head (exp2 domain); weighted sum: one
// thread per (key range, head, 8 columns), the key ranges' partial sums reduced through
// shared memory.  Optionally the CTA also closes one block into the summary pool and
// appends the new token to the ring (fused decode step).
struct ActiveArgs {
  int B, Hq, Hkv, G, Tq, dh, window;
  float scale_log2;
  View4 q, k, v, ks, vs, out;
  int64_t kv_pos0, ring, kv_len, pos0;
  const int64_t* positions;
  int num_summary_limit;
  float* lse;
  int64_t ls_b, ls_h;
  bna_route route;
  // fused decode step (Tq == 1)
  const void* knew;
  const void* vnew;
  int64_t kn_b, kn_h, vn_b, vn_h;
  int64_t close_block, close_slot;
  // routed summaries precomputed on the host (decode step: one known position); -1: on device
  int host_ns;
  int host_ids[kMaxSummaries];
};

constexpr int kDecodeThreads = 512;
constexpr int kDecodeWarps = kDecodeThreads / 32;
constexpr int kKeyParts = kDecodeThreads / 64;  // P.V key ranges summed through shared memory
// reduction buffer (floats): block-mean partials or the P.V partial sums
__host__ __device__ constexpr int decode_red_floats(int G) {
  return kDecodeThreads * 8 > kKeyParts * 128 * G ? kDecodeThreads * 8 : kKeyParts * 128 * G;
}

__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
               "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <typename T, int G>
__global__ void __launch_bounds__(kDecodeThreads) decode_kernel(const ActiveArgs a) {
  extern __shared__ __align__(16) uint8_t dsm_raw[];
  const int maxk = a.window + kMaxSummaries;
  constexpr int kRow = 256 + 16;                                   // padded staged row (bank spread)
  uint8_t* kv = dsm_raw;                                           // [2][maxk][kRow] K rows, V rows
  uint8_t* qraw = kv + 2 * maxk * kRow;                            // [G][256 B] queries as loaded
  float* sc = reinterpret_cast<float*>(qraw + G * 256);            // [G][maxk] scores -> weights
  constexpr int kQRow = 132;  // scaled query row stride (floats): rows of different heads in different banks
  float* qs = sc + G * maxk;                                       // [G][kQRow] scaled queries
  float* red = qs + G * kQRow;                                     // block-mean / P.V reduction
  constexpr int kRed = decode_red_floats(G);
  float* stat = red + kRed;                                        // [G] row sums
  int* sel = reinterpret_cast<int*>(stat + G);                     // [1 + 16] summary count + ids

  // Launched with programmatic stream serialization: this grid may start while the previous
  // kernel of the stream finishes; wait for it (and its memory) before touching anything,
  // then let the next step's grid start launching.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int t = blockIdx.x;
  const int b = blockIdx.y / a.Hkv, kvh = blockIdx.y % a.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t p = a.positions ? a.positions[t] : a.pos0 + t;

  // raw window [lo, hi]; with a fused append the newest row (p) is read from the input
  int64_t lo = max64(0, p - a.window + 1);
  if (a.ring == 0) lo = max64(lo, a.kv_pos0);
  int64_t hi = p;
  if (hi > a.kv_len - 1) hi = a.kv_len - 1;
  const int nraw = hi >= lo ? (int)(hi - lo + 1) : 0;
  const int ring = (int)a.ring;
  const int idx_lo = ring > 0 ? (int)((uint64_t)lo % (uint64_t)a.ring) : (int)(lo - a.kv_pos0);
#pragma unroll 1
  for (int c = threadIdx.x; c < 2 * nraw * 16; c += kDecodeThreads) {
    const int isv = c >= nraw * 16;
    const int e = isv ? c - nraw * 16 : c;
    const int j = e >> 4, ch = e & 15;
    const uint8_t* src;
    if (a.knew && j == nraw - 1) {
      src = reinterpret_cast<const uint8_t*>(isv ? a.vnew : a.knew) +
            2 * (b * (isv ? a.vn_b : a.kn_b) + kvh * (isv ? a.vn_h : a.kn_h));
    } else {
      int idx = idx_lo + j;
      if (ring > 0 && idx >= ring) idx -= ring;
      src = row_ptr(isv ? a.v : a.k, b, kvh, idx);
    }
    cp_async_16(kv + (isv * maxk + j) * kRow + ch * 16, src + ch * 16);
  }
  // host-routed summaries of a step that closes no block: their rows load together with
  // the window rows, in the same round trip (a block closed in this step is written below
  // and may be routed, so such steps load the summaries after the close)
  const bool early_sum = a.host_ns >= 0 && a.close_block < 0;
  if (early_sum) {
#pragma unroll 1
    for (int c = threadIdx.x; c < 2 * a.host_ns * 16; c += kDecodeThreads) {
      const int isv = c >= a.host_ns * 16;
      const int e = isv ? c - a.host_ns * 16 : c;
      const int j = e >> 4, ch = e & 15;
      cp_async_16(kv + (isv * maxk + nraw + j) * kRow + ch * 16,
                  row_ptr(isv ? a.vs : a.ks, b, kvh, a.host_ids[j]) + ch * 16);
    }
  }
  // queries: raw rows in the same round trip as the keys and values, scaled below
  for (int c = threadIdx.x; c < G * 16; c += kDecodeThreads) {
    const int g = c >> 4, ch = c & 15;
    cp_async_16(qraw + g * 256 + ch * 16, row_ptr(a.q, b, kvh * G + g, t) + ch * 16);
  }
  if (a.close_block >= 0) {  // fused block close: mean of the block's tokens from the ring
    const int BS = a.route.block_size;
    block_mean<T>(a.k, b, kvh, a.close_block * BS, BS, 0, a.ring, 128, red, row_ptr(a.ks, b, kvh, a.close_slot));
    __syncthreads();
    block_mean<T>(a.v, b, kvh, a.close_block * BS, BS, 0, a.ring, 128, red, row_ptr(a.vs, b, kvh, a.close_slot));
    __syncthreads();  // the closed block may be routed to below
  }
  if (a.host_ns >= 0) {
    if (threadIdx.x <= kMaxSummaries) sel[threadIdx.x] = threadIdx.x == 0 ? a.host_ns : a.host_ids[threadIdx.x - 1];
  } else if (threadIdx.x == 0) {
    int ids[kMaxSummaries];
    const int n = active_summaries(a.route, p, a.window, a.num_summary_limit, a.route.neighbors, ids);
    sel[0] = n;
    for (int i = 0; i < n; ++i) sel[1 + i] = ids[i];
  }
  __syncthreads();
  const int ns = sel[0];
  const int nk = nraw + ns;
#pragma unroll 1
  for (int c = early_sum ? 2 * ns * 16 : threadIdx.x; c < 2 * ns * 16; c += kDecodeThreads) {
    const int isv = c >= ns * 16;
    const int e = isv ? c - ns * 16 : c;
    const int j = e >> 4, ch = e & 15;
    cp_async_16(kv + (isv * maxk + nraw + j) * kRow + ch * 16,
                row_ptr(isv ? a.vs : a.ks, b, kvh, sel[1 + j]) + ch * 16);
  }
  cp_async_wait_all();
  __syncthreads();
  if (a.knew && threadIdx.x < 32) {
    // fused append: the new token (staged as the last window row) goes to ring slot
    // p % ring; any block close above has already read the ring
    const int slot = (int)((uint64_t)p % (uint64_t)a.ring);
    const int isv = threadIdx.x >= 16;
    const int ch = threadIdx.x & 15;
    st_128(row_ptr(isv ? a.v : a.k, b, kvh, slot) + ch * 16,
           *reinterpret_cast<const uint4*>(kv + (isv * maxk + nraw - 1) * kRow + ch * 16));
  }
#pragma unroll 1
  for (int c = threadIdx.x; c < G * 64; c += kDecodeThreads) {  // queries, scaled to log2 units
    const int g = c >> 6, d = (c & 63) * 2;
    const float2 f = ElemTraits<T>::unpack2(*reinterpret_cast<const uint32_t*>(qraw + g * 256 + d * 2));
    qs[g * kQRow + d] = f.x * a.scale_log2;
    qs[g * kQRow + d + 1] = f.y * a.scale_log2;
  }
  __syncthreads();

  // scores: one thread per (key, head), full 128-wide dot from shared memory
#pragma unroll 1
  for (int e = threadIdx.x; e < nk * G; e += kDecodeThreads) {
    const int j = e / G, g = e - j * G;
    const uint4* kr = reinterpret_cast<const uint4*>(kv + j * kRow);
    const float4* q4 = reinterpret_cast<const float4*>(qs + g * kQRow);
    float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll 4
    for (int c = 0; c < 16; ++c) {
      const uint4 u = kr[c];
      const float4 qa = q4[2 * c], qb = q4[2 * c + 1];
      const float2 f0 = ElemTraits<T>::unpack2(u.x), f1 = ElemTraits<T>::unpack2(u.y);
      const float2 f2 = ElemTraits<T>::unpack2(u.z), f3 = ElemTraits<T>::unpack2(u.w);
      d0 = fmaf(qa.x, f0.x, fmaf(qa.y, f0.y, d0));
      d1 = fmaf(qa.z, f1.x, fmaf(qa.w, f1.y, d1));
      d2 = fmaf(qb.x, f2.x, fmaf(qb.y, f2.y, d2));
      d3 = fmaf(qb.z, f3.x, fmaf(qb.w, f3.y, d3));
    }
    sc[g * maxk + j] = (d0 + d1) + (d2 + d3);
  }
  __syncthreads();
  // softmax: warp g (looping if G > warps) owns head g; weights overwrite the scores
#pragma unroll 1
  for (int g = warp; g < G; g += kDecodeWarps) {
    float* sg = sc + g * maxk;
    float m = -INFINITY;
    for (int j = lane; j < nk; j += 32) m = fmaxf(m, sg[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int j = lane; j < nk; j += 32) {
      const float e = exp2f(sg[j] - m);
      sg[j] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) {
      stat[g] = l;
      if (a.lse) a.lse[b * a.ls_b + (int64_t)(kvh * G + g) * a.ls_h + t] = (m + log2f(l)) * 0.6931471805599453f;
    }
  }
  __syncthreads();
  // weighted values: thread = (key range, head, 8 columns): one 16-byte V load and eight
  // independent FMAs per key; the key ranges' partial sums meet in shared memory
  // (reusing the block-mean buffer)
  constexpr int kOct = G * 16;
  constexpr int kParts = kDecodeThreads / kOct > 0 ? kDecodeThreads / kOct : 1;
  float* part = red;  // [kParts][G * 128]
  const int npairs = G * 64;
#pragma unroll 1
  for (int e = threadIdx.x; e < kParts * kOct; e += kDecodeThreads) {
    const int pi = e / kOct, r = e - pi * kOct;
    const int g = r >> 4, oc = r & 15;
    const float* w = sc + g * maxk;
    const uint8_t* vb = kv + maxk * kRow + oc * 16;
    const int j0 = nk * pi / kParts, j1 = nk * (pi + 1) / kParts;
    float acc[8];
#pragma unroll
    for (int x = 0; x < 8; ++x) acc[x] = 0.f;
#pragma unroll 4
    for (int j = j0; j < j1; ++j) {
      const uint4 u = *reinterpret_cast<const uint4*>(vb + j * kRow);
      const float wj = w[j];
      const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        const float2 f = ElemTraits<T>::unpack2(uw[x]);
        acc[2 * x] = fmaf(wj, f.x, acc[2 * x]);
        acc[2 * x + 1] = fmaf(wj, f.y, acc[2 * x + 1]);
      }
    }
    float4* dst = reinterpret_cast<float4*>(part + pi * G * 128 + g * 128 + oc * 8);
    dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
  __syncthreads();
#pragma unroll 1
  for (int r = threadIdx.x; r < npairs; r += kDecodeThreads) {
    const int g = r >> 6, c = (r & 63) * 2;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int pi = 0; pi < kParts; ++pi) {
      const float2 f = *reinterpret_cast<const float2*>(part + pi * G * 128 + g * 128 + c);
      s0 += f.x;
      s1 += f.y;
    }
    const float l = stat[g];
    const float inv = l > 0.f ? 1.f / l : 0.f;
    *reinterpret_cast<uint32_t*>(row_ptr(a.out, b, kvh * G + g, t) + c * 2) = ElemTraits<T>::pack2(s0 * inv, s1 * inv);
  }
}

// ------------------------------------------------------------------------------ selection dump
__global__ void prefill_selection_kernel(const bna_route r, int window, int32_t* idx, int32_t* cnt) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= r.num_blocks) return;
  int ids[kMaxSummaries];
  const int n = prefill_summaries(r, b, window, r.neighbors, ids);
  for (int i = 0; i < r.max_degree; ++i) idx[(int64_t)b * r.max_degree + i] = i < n ? ids[i] : -1;
  cnt[b] = n;
}

// ------------------------------------------------------------------------------ launchers
int launch_compress(const bna_tensor4* x, bna_tensor4* out, int dtype, int block_size, int64_t pos0,
                    int n_blocks, int64_t valid_len, int64_t ring, int64_t slot0, cudaStream_t stream,
                    const bna_tensor4* x2, bna_tensor4* out2) {
  CompressArgs a{to_view(x), to_view(out), to_view(x2 ? x2 : x), to_view(out2 ? out2 : out), (int)x->size[1],
                 (int)x->size[3], block_size, pos0, valid_len, ring, slot0};
  dim3 grid(n_blocks, (unsigned)(x->size[0] * x->size[1]), x2 ? 2u : 1u);
  if (n_blocks == 0 || grid.y == 0) return BNA_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kCompressThreads);
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (dtype == BNA_BF16)
    cudaLaunchKernelEx(&cfg, compress_kernel<__nv_bfloat16>, a);
  else
    cudaLaunchKernelEx(&cfg, compress_kernel<__half>, a);
  return check_cuda(cudaGetLastError(), "compress_kernel launch");
}

int launch_append(bna_tensor4* rk, bna_tensor4* rv, const bna_tensor4* sk, const bna_tensor4* sv, int64_t pos0,
                  int64_t ring, cudaStream_t stream) {
  AppendArgs a{to_view(sk), to_view(sv), to_view(rk), to_view(rv), (int)sk->size[1], (int)sk->size[3], pos0, ring};
  dim3 grid((unsigned)sk->size[2], (unsigned)(sk->size[0] * sk->size[1]));
  if (grid.x == 0 || grid.y == 0) return BNA_OK;
  append_kernel<<<grid, 128, 0, stream>>>(a);
  return check_cuda(cudaGetLastError(), "append_kernel launch");
}

int launch_active(const bna_tensor4* q, const bna_tensor4* k, const bna_tensor4* v, const bna_tensor4* ks,
                  const bna_tensor4* vs, bna_tensor4* out, float* lse, int64_t ls_b, int64_t ls_h, int dtype,
                  const bna_route* route, int window, const int64_t* positions, int64_t pos0, int64_t kv_pos0,
                  int64_t ring, int64_t kv_len, int num_summary_limit, float scale, const bna_tensor4* knew,
                  const bna_tensor4* vnew, int64_t close_block, int64_t close_slot, cudaStream_t stream) {
  ActiveArgs a{};
  a.host_ns = -1;
  if (!positions && q->size[2] == 1 && route->neighbors == nullptr) {
    // one query at a known position: route it here (same selection code as the device)
    a.host_ns = active_summaries(*route, pos0, window, num_summary_limit, nullptr, a.host_ids);
  }
  a.B = (int)q->size[0];
  a.Hq = (int)q->size[1];
  a.Tq = (int)q->size[2];
  a.dh = (int)q->size[3];
  a.Hkv = (int)k->size[1];
  a.G = a.Hq / a.Hkv;
  a.window = window;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.q = to_view(q);
  a.k = to_view(k);
  a.v = to_view(v);
  a.ks = to_view(ks);
  a.vs = to_view(vs);
  a.out = to_view(out);
  a.kv_pos0 = kv_pos0;
  a.ring = ring;
  a.kv_len = kv_len;
  a.pos0 = pos0;
  a.positions = positions;
  a.num_summary_limit = num_summary_limit;
  a.lse = lse;
  a.ls_b = ls_b;
  a.ls_h = ls_h;
  a.route = *route;
  a.knew = knew ? knew->data : nullptr;
  a.vnew = vnew ? vnew->data : nullptr;
  if (knew) {
    a.kn_b = knew->stride[0];
    a.kn_h = knew->stride[1];
    a.vn_b = vnew->stride[0];
    a.vn_h = vnew->stride[1];
  }
  a.close_block = close_block;
  a.close_slot = close_slot;
  const int maxk = window + kMaxSummaries;
  const size_t smem = (size_t)2 * maxk * (256 + 16) + (size_t)a.G * 256 +
                      sizeof(float) * ((size_t)a.G * maxk + (size_t)a.G * 132 +
                                       (size_t)decode_red_floats(a.G) +
                                       (size_t)a.G) +
                      sizeof(int) * (1 + kMaxSummaries);
  dim3 grid((unsigned)a.Tq, (unsigned)(a.B * a.Hkv));
  if (grid.x == 0 || grid.y == 0) return BNA_OK;
  auto launch = [&](auto kern) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kDecodeThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, a);
  };
  const bool bf = dtype == BNA_BF16;
  switch (a.G) {
    case 1: bf ? launch(decode_kernel<__nv_bfloat16, 1>) : launch(decode_kernel<__half, 1>); break;
    case 2: bf ? launch(decode_kernel<__nv_bfloat16, 2>) : launch(decode_kernel<__half, 2>); break;
    case 4: bf ? launch(decode_kernel<__nv_bfloat16, 4>) : launch(decode_kernel<__half, 4>); break;
    case 8: bf ? launch(decode_kernel<__nv_bfloat16, 8>) : launch(decode_kernel<__half, 8>); break;
    case 16: bf ? launch(decode_kernel<__nv_bfloat16, 16>) : launch(decode_kernel<__half, 16>); break;
    default: return fail(BNA_UNSUPPORTED, "GQA group size must be 1, 2, 4, 8 or 16");
  }
  return check_cuda(cudaGetLastError(), "decode_kernel launch");
}

int launch_selection_dump(const bna_route* r, int window, int32_t* idx, int32_t* cnt, cudaStream_t stream) {
  const int nb = (r->num_blocks + 127) / 128;
  prefill_selection_kernel<<<nb, 128, 0, stream>>>(*r, window, idx, cnt);
  return check_cuda(cudaGetLastError(), "prefill_selection_kernel launch");
}

int take_device_error(int device, int32_t* code) {
  int prev = 0;
  cudaGetDevice(&prev);
  if (device != prev) cudaSetDevice(device);
  int zero = 0, val = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&val, g_device_error, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
  if (device != prev) cudaSetDevice(prev);
  *code = val;
  return check_cuda(e, "reading the device error word");
}

}  // namespace bna
