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
  if (tl < lanes) {
#pragma unroll 8
    for (int j = tl; j < count; j += lanes) {
      const int64_t pos = first_pos + j;
      const int64_t idx = ring > 0 ? pos % ring : pos - pos_base;
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
  View4 src, dst;
  int H, dh, block_size;
  int64_t pos0, valid_len, ring, slot0;
};

// 256 threads: 16 head_dim chunks x 16 token lanes, so a 128-token block is one round of
// eight independent 128-bit loads per thread (all in flight together).
constexpr int kCompressThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kCompressThreads) compress_kernel(const CompressArgs a) {
  __shared__ float red[kCompressThreads * 8];
  const int j = blockIdx.x;
  const int b = blockIdx.y / a.H, h = blockIdx.y % a.H;
  const int64_t first = a.pos0 + (int64_t)j * a.block_size;
  int64_t cnt = a.valid_len - (int64_t)j * a.block_size;
  if (cnt > a.block_size) cnt = a.block_size;
  if (cnt < 1) cnt = 0;
  block_mean<T>(a.src, b, h, first, (int)cnt, a.pos0, a.ring, a.dh, red, row_ptr(a.dst, b, h, a.slot0 + j));
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
// One CTA (128 threads, 4 warps) per (query index, b * Hkv): stages the query's raw window
// and routed summaries in shared memory, then each warp computes one query head's scores
// (lane per key), a warp-shuffle softmax (exp2 domain) and the weighted sum of values
// (lane per 4 head_dim columns).  Optionally first appends the new token to the ring and
// closes one block into the summary pool (fused decode step).
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
};

constexpr int kRowPad = 16;  // bytes of padding per staged row (bank spread)

template <typename T>
__global__ void __launch_bounds__(128) active_kernel(const ActiveArgs a) {
  extern __shared__ uint8_t smem[];
  const int dh = a.dh;  // 128
  const int rowb = dh * 2 + kRowPad;
  const int maxk = a.window + kMaxSummaries;
  uint8_t* sk = smem;
  uint8_t* sv = sk + maxk * rowb;
  float* sq = reinterpret_cast<float*>(sv + maxk * rowb);  // [G][dh]
  float* sp = sq + a.G * dh;                              // [G][maxk]
  float* red = sp + a.G * maxk;                           // [128 * 8] for block means

  const int t = blockIdx.x;
  const int b = blockIdx.y / a.Hkv, kvh = blockIdx.y % a.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t p = a.positions ? a.positions[t] : a.pos0 + t;
  const int chunks = dh >> 3;

  if (a.knew) {  // fused append of the new token at position p
    const int64_t slot = p % a.ring;
    for (int c = threadIdx.x; c < 2 * chunks; c += blockDim.x) {
      const bool isv = c >= chunks;
      const int ch = isv ? c - chunks : c;
      const uint8_t* src = reinterpret_cast<const uint8_t*>(isv ? a.vnew : a.knew) +
                           2 * (b * (isv ? a.vn_b : a.kn_b) + kvh * (isv ? a.vn_h : a.kn_h));
      st_128(row_ptr(isv ? a.v : a.k, b, kvh, slot) + ch * 16, ld_nc_128(src + ch * 16));
    }
  }
  if (a.close_block >= 0) {  // fused block close: mean of the block's tokens from the ring
    const int BS = a.route.block_size;
    block_mean<T>(a.k, b, kvh, a.close_block * BS, BS, 0, a.ring, dh, red, row_ptr(a.ks, b, kvh, a.close_slot));
    __syncthreads();
    block_mean<T>(a.v, b, kvh, a.close_block * BS, BS, 0, a.ring, dh, red, row_ptr(a.vs, b, kvh, a.close_slot));
  }
  __syncthreads();

  // raw window [lo, hi] and routed summaries
  int64_t lo = max64(0, p - a.window + 1);
  if (a.ring == 0) lo = max64(lo, a.kv_pos0);
  int64_t hi = p;
  if (hi > a.kv_len - 1) hi = a.kv_len - 1;
  const int nraw = hi >= lo ? (int)(hi - lo + 1) : 0;
  int ids[kMaxSummaries];
  const int ns = active_summaries(a.route, p, a.window, a.num_summary_limit, a.route.neighbors, ids);
  const int nk = nraw + ns;
  for (int c = threadIdx.x; c < nk * chunks; c += blockDim.x) {
    const int r = c / chunks, ch = c % chunks;
    uint4 ku, vu;
    if (r < nraw) {
      const int64_t pos = lo + r;
      const int64_t idx = a.ring > 0 ? pos % a.ring : pos - a.kv_pos0;
      ku = ld_128(row_ptr(a.k, b, kvh, idx) + ch * 16);
      vu = ld_128(row_ptr(a.v, b, kvh, idx) + ch * 16);
    } else {
      ku = ld_128(row_ptr(a.ks, b, kvh, ids[r - nraw]) + ch * 16);
      vu = ld_128(row_ptr(a.vs, b, kvh, ids[r - nraw]) + ch * 16);
    }
    *reinterpret_cast<uint4*>(sk + r * rowb + ch * 16) = ku;
    *reinterpret_cast<uint4*>(sv + r * rowb + ch * 16) = vu;
  }
  for (int c = threadIdx.x; c < a.G * chunks; c += blockDim.x) {
    const int g = c / chunks, ch = c % chunks;
    const uint4 u = ld_nc_128(row_ptr(a.q, b, kvh * a.G + g, t) + ch * 16);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = ElemTraits<T>::unpack2(w[e]);
      sq[g * dh + ch * 8 + 2 * e] = f.x * a.scale_log2;
      sq[g * dh + ch * 8 + 2 * e + 1] = f.y * a.scale_log2;
    }
  }
  __syncthreads();

  const int nwarps = blockDim.x >> 5;
  for (int g = warp; g < a.G; g += nwarps) {
    const float* qv = sq + g * dh;
    float* pr = sp + g * maxk;
    float m = -INFINITY;
    for (int j = lane; j < nk; j += 32) {
      const uint8_t* kr = sk + j * rowb;
      float s = 0.f;
      for (int ch = 0; ch < chunks; ++ch) {
        const uint4 u = *reinterpret_cast<const uint4*>(kr + ch * 16);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = ElemTraits<T>::unpack2(w[e]);
          s = fmaf(qv[ch * 8 + 2 * e], f.x, s);
          s = fmaf(qv[ch * 8 + 2 * e + 1], f.y, s);
        }
      }
      pr[j] = s;
      m = fmaxf(m, s);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int j = lane; j < nk; j += 32) {
      const float e = exp2f(pr[j] - m);
      pr[j] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    __syncwarp();
    // lane owns head_dim columns [4*lane, 4*lane + 4)
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < nk; ++j) {
      const float w = pr[j];
      const uint2 u = *reinterpret_cast<const uint2*>(sv + j * rowb + lane * 8);
      const float2 f0 = ElemTraits<T>::unpack2(u.x), f1 = ElemTraits<T>::unpack2(u.y);
      acc[0] = fmaf(w, f0.x, acc[0]);
      acc[1] = fmaf(w, f0.y, acc[1]);
      acc[2] = fmaf(w, f1.x, acc[2]);
      acc[3] = fmaf(w, f1.y, acc[3]);
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
    uint8_t* orow = row_ptr(a.out, b, kvh * a.G + g, t);
    uint2 o;
    o.x = ElemTraits<T>::pack2(acc[0] * inv, acc[1] * inv);
    o.y = ElemTraits<T>::pack2(acc[2] * inv, acc[3] * inv);
    *reinterpret_cast<uint2*>(orow + lane * 8) = o;
    if (a.lse && lane == 0)
      a.lse[b * a.ls_b + (int64_t)(kvh * a.G + g) * a.ls_h + t] = (m + log2f(l)) * 0.6931471805599453f;
    __syncwarp();
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
                    int n_blocks, int64_t valid_len, int64_t ring, int64_t slot0, cudaStream_t stream) {
  CompressArgs a{to_view(x), to_view(out), (int)x->size[1], (int)x->size[3], block_size, pos0, valid_len, ring, slot0};
  dim3 grid(n_blocks, (unsigned)(x->size[0] * x->size[1]));
  if (n_blocks == 0 || grid.y == 0) return BNA_OK;
  if (dtype == BNA_BF16)
    compress_kernel<__nv_bfloat16><<<grid, kCompressThreads, 0, stream>>>(a);
  else
    compress_kernel<__half><<<grid, kCompressThreads, 0, stream>>>(a);
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
  const size_t smem = (size_t)2 * maxk * (a.dh * 2 + kRowPad) + sizeof(float) * ((size_t)a.G * a.dh + (size_t)a.G * maxk + 128 * 8);
  dim3 grid((unsigned)a.Tq, (unsigned)(a.B * a.Hkv));
  if (grid.x == 0 || grid.y == 0) return BNA_OK;
  if (dtype == BNA_BF16) {
    auto kern = active_kernel<__nv_bfloat16>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<grid, 128, smem, stream>>>(a);
  } else {
    auto kern = active_kernel<__half>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<grid, 128, smem, stream>>>(a);
  }
  return check_cuda(cudaGetLastError(), "active_kernel launch");
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
