// kernels.cu — bandwidth-bound kernels of the compressed path:
//   * block compressor (mean pool)          bna/torch/attention_wayfinder_permute.py:1022-1043
//   * two-pool cache append / block close    bna/mlx/compressed_cache.py:104-149
//   * active / decode attention              attention_wayfinder_permute.py:1125-1197,
//                                            bna/mlx/attention.py:1669-1876
//   * device dump of the prefill selection   attention_wayfinder_permute.py:912-966
// All use coalesced 128-bit loads, shared-memory staging and warp-shuffle reductions.
#include <cuda_runtime.h>
#include <type_traits>

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
    int j = tl;
    // batches of 8 rows per thread: all eight 128-bit loads are issued before any add
    for (; j + 7 * lanes < count; j += 8 * lanes) {
      uint4 u[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        int64_t idx = idx0 + j + r * lanes;
        if (ring > 0 && idx >= ring) idx -= ring;
        u[r] = ld_nc_128(row_ptr(src, b, h, idx) + ch * 16);
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const uint32_t w[4] = {u[r].x, u[r].y, u[r].z, u[r].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = ElemTraits<T>::unpack2(w[e]);
          acc[2 * e] += f.x;
          acc[2 * e + 1] += f.y;
        }
      }
    }
    for (; j < count; j += lanes) {
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
  __syncthreads();  // red may still be read by a previous call's final sums
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
  // fused q/k preparation of a decode step (qk_prep != 0): q and k_new are the raw
  // projection rows; each gets the Qwen3.5 RMSNorm (weights qn_w / kn_w) and the rotary
  // embedding (cos / sin of sequence b at cs + b * cs_b, rot dims) in the kernel
  int qk_prep;
  const void* qn_w;
  const void* kn_w;
  const void* cs;
  const void* sn;
  int64_t cs_b;
  int rot;
  float qk_eps;
  // routed summaries precomputed on the host (decode step: one known position); -1: on device
  int host_ns;
  int host_ids[kMaxSummaries];
};

// 128 threads: four warps of 16-key tensor-core tiles (measured faster than 256 / 512,
// where more warps mean costlier barriers and merges for the few tiles of a window).
__host__ __device__ constexpr int decode_threads(int G) { return 128; }
constexpr int kDecPitch = 256 + 16;  // staged row pitch (bytes): spreads ldmatrix / fragment rows over banks
// floats of the partial-sum region: the per-warp (o) partials, or the block-mean buffer of
// a fused close (8 floats per thread)
__host__ __device__ constexpr int decode_part_floats(int G) {
  return (decode_threads(G) / 32) * G * 128 > decode_threads(G) * 8 ? (decode_threads(G) / 32) * G * 128
                                                                     : decode_threads(G) * 8;
}
size_t decode_smem_bytes(int G, int window) {
  const int maxk = window + kMaxSummaries;
  return (size_t)2 * kDecPitch * ((maxk + 15) / 16 * 16) + (size_t)G * kDecPitch + sizeof(float) * (size_t)decode_part_floats(G) +
         sizeof(float) * (size_t)(decode_threads(G) / 32) * G * 2 + sizeof(int) * (1 + kMaxSummaries);
}

__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
               "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// D += A B for one m16n8k16 tile (A row-major 16x16, B column-major 16x8, fp32 accumulate).
template <typename T>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// Four 8x8 16-bit matrices from shared memory, transposed (lanes 8i..8i+7 give the row
// addresses of matrix i).
__device__ __forceinline__ void ldmatrix_x4_trans(const void* smem_row, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"((uint32_t)__cvta_generic_to_shared(smem_row)));
}

// One CTA per (query index, b * Hkv) serves the G query heads of a KV head.
//   1. loads: the raw window rows, the routed summary rows and the G query rows arrive in
//      shared memory in one round trip.  In a fused decode step the ring rows of
//      positions <= p - 2 are requested (bulk copies) before griddepcontrol.wait (under programmatic
//      dependent launch, while the previous kernel of the stream finishes): only the
//      immediately preceding kernel can still be running, and in a decode step the ring rows
//      it may write are those of position p - 1 (the previous step's append) at most.
//   2. each warp takes 16-key tiles in turn: S = Q K^T and O += P V on tensor cores
//      (mma.sync m16n8k16, the G heads as rows), with an online softmax (exp2 domain) that
//      keeps each head's running max, sum and output columns in registers.
//   3. the per-warp (max, sum, output) partials of each head are merged once through shared
//      memory (the online log-sum-exp merge): one thread per (head, two columns) derives
//      the rescale factors and sums the partials.
// Optionally the CTA also closes one block into the summary pool and appends the new token
// to the ring (fused decode step).
template <typename T, int G>
__global__ void __launch_bounds__(decode_threads(G)) decode_kernel(const ActiveArgs a) {
  constexpr int NT = decode_threads(G);
  constexpr int NW = NT / 32;
  extern __shared__ __align__(16) uint8_t dsm_raw[];
  const int maxk = (a.window + kMaxSummaries + 15) / 16 * 16;  // rows per K / V region (whole 16-key tiles)
  uint8_t* kv = dsm_raw;                                      // [2][maxk][kDecPitch] K rows, V rows
  uint8_t* qraw = kv + 2 * maxk * kDecPitch;                  // [G][kDecPitch] queries as loaded
  float* part = reinterpret_cast<float*>(qraw + G * kDecPitch);  // [NW][G][128] partial outputs
  float* red = part;                                          // block-mean buffer of a fused close
  float* ml = part + decode_part_floats(G);                   // [NW][G][2] partial max, sum
  int* sel = reinterpret_cast<int*>(ml + NW * G * 2);         // [1 + 16] summary count + ids

  const int t = blockIdx.x;
  const int b = blockIdx.y / a.Hkv, kvh = blockIdx.y % a.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool fused = a.knew != nullptr && a.ring > 0;
  // positions come from the host in a fused step; a device positions array is an input
  const int64_t p0 = a.positions ? -1 : a.pos0 + t;

  auto issue_rows = [&](int64_t lo, int idx_lo, int j0, int j1, int nraw) {
    const int n = j1 - j0;
#pragma unroll 1
    for (int c = threadIdx.x; c < 2 * n * 16; c += NT) {
      const int isv = c >= n * 16;
      const int e = isv ? c - n * 16 : c;
      const int j = j0 + (e >> 4), ch = e & 15;
      const uint8_t* src;
      if (a.knew && j == nraw - 1) {
        src = reinterpret_cast<const uint8_t*>(isv ? a.vnew : a.knew) +
              2 * (b * (isv ? a.vn_b : a.kn_b) + kvh * (isv ? a.vn_h : a.kn_h));
      } else {
        int idx = idx_lo + j;
        if (a.ring > 0 && idx >= (int)a.ring) idx -= (int)a.ring;
        src = row_ptr(isv ? a.v : a.k, b, kvh, idx);
      }
      cp_async_16(kv + (isv * maxk + j) * kDecPitch + ch * 16, src + ch * 16);
    }
  };
  // raw window [lo, hi]; with a fused append the newest row (p) is read from the input
  auto window_of = [&](int64_t p, int64_t& lo, int& nraw, int& idx_lo) {
    lo = max64(0, p - a.window + 1);
    if (a.ring == 0) lo = max64(lo, a.kv_pos0);
    int64_t hi = p;
    if (hi > a.kv_len - 1) hi = a.kv_len - 1;
    nraw = hi >= lo ? (int)(hi - lo + 1) : 0;
    idx_lo = a.ring > 0 ? (int)((uint64_t)lo % (uint64_t)a.ring) : (int)(lo - a.kv_pos0);
  };
  int64_t lo = 0;
  int nraw = 0, idx_lo = 0, npre = 0;
  // The pre-wait rows arrive by untiled bulk copies (one 256-byte row per instruction,
  // counted on pre_bar) instead of 16-byte cp.async: the few cp.async issued after the
  // wait then do not queue behind ~2k outstanding requests of the prefetch.
  __shared__ __align__(8) uint64_t pre_bar;
  const bool pre = fused && p0 >= 0;
  if (pre) {
    window_of(p0, lo, nraw, idx_lo);
    npre = (int)(p0 - 1 - lo);  // rows j < npre sit at positions <= p - 2
    npre = npre < 0 ? 0 : (npre > nraw ? nraw : npre);
    if (threadIdx.x == 0) {
      sm100::mbar_init(&pre_bar, 1);
      sm100::fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) sm100::mbar_arrive_expect_tx(&pre_bar, (uint32_t)npre * 512u);
#pragma unroll 1
    for (int j = threadIdx.x; j < 2 * npre; j += NT) {
      const int isv = j >= npre;
      const int jj = isv ? j - npre : j;
      int idx = idx_lo + jj;
      if (a.ring > 0 && idx >= (int)a.ring) idx -= (int)a.ring;
      sm100::bulk_copy_g2s(kv + (isv * maxk + jj) * kDecPitch, row_ptr(isv ? a.v : a.k, b, kvh, idx), 256u,
                           &pre_bar);
    }
  }
  // V rows nk .. end of the last 16-key tile are zeroed (so that P = 0 there never meets
  // stale bits); with the key count known before the wait (host-routed step) that happens
  // here, off the critical path
  const bool zero_early = pre && a.host_ns >= 0;
  if (zero_early) {
    const int nk0 = nraw + a.host_ns;
    for (int c = threadIdx.x; c < ((nk0 + 15) / 16 * 16 - nk0) * 16; c += NT)
      *reinterpret_cast<uint4*>(kv + (maxk + nk0 + (c >> 4)) * kDecPitch + (c & 15) * 16) = make_uint4(0, 0, 0, 0);
  }
  // Launched with programmatic stream serialization: wait for the previous kernel of the
  // stream (and its memory) before touching anything it may write, then let the next
  // kernel start launching.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int64_t p = a.positions ? a.positions[t] : p0;
  if (!(fused && p0 >= 0)) window_of(p, lo, nraw, idx_lo);
  issue_rows(lo, idx_lo, npre, nraw, nraw);
  // host-routed summaries of a step that closes no block: their rows load together with
  // the window rows, in the same round trip (a block closed in this step is written below
  // and may be routed, so such steps load the summaries after the close)
  const bool early_sum = a.host_ns >= 0 && a.close_block < 0;
  if (early_sum) {
#pragma unroll 1
    for (int c = threadIdx.x; c < 2 * a.host_ns * 16; c += NT) {
      const int isv = c >= a.host_ns * 16;
      const int e = isv ? c - a.host_ns * 16 : c;
      const int j = e >> 4, ch = e & 15;
      cp_async_16(kv + (isv * maxk + nraw + j) * kDecPitch + ch * 16,
                  row_ptr(isv ? a.vs : a.ks, b, kvh, a.host_ids[j]) + ch * 16);
    }
  }
  for (int c = threadIdx.x; c < G * 16; c += NT) {
    const int g = c >> 4, ch = c & 15;
    cp_async_16(qraw + g * kDecPitch + ch * 16, row_ptr(a.q, b, kvh * G + g, t) + ch * 16);
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
  for (int c = early_sum ? 2 * ns * 16 : threadIdx.x; c < 2 * ns * 16; c += NT) {
    const int isv = c >= ns * 16;
    const int e = isv ? c - ns * 16 : c;
    const int j = e >> 4, ch = e & 15;
    cp_async_16(kv + (isv * maxk + nraw + j) * kDecPitch + ch * 16, row_ptr(isv ? a.vs : a.ks, b, kvh, sel[1 + j]) + ch * 16);
  }
  cp_async_wait_all();
  if (pre) {
    // bounded wait for the bulk-copied rows: on a timeout record the failure (read back by
    // bna_take_device_error) and carry on rather than spin
    bool done = false;
    for (int it = 0; it < (1 << 24) && !done; ++it) done = sm100::mbar_try_wait(&pre_bar, 0);
    if (!done && threadIdx.x == 0) atomicCAS(&g_device_error, 0, 0x1000 | 13);
  }
  __syncthreads();
  if (a.qk_prep) {
    // warp r normalises and rotates query row r (r < G) or, for r == G, the new key row
#pragma unroll 1
    for (int r = warp; r <= G; r += NW) {
      uint8_t* row = r < G ? qraw + r * kDecPitch : kv + (nraw - 1) * kDecPitch;
      const uint8_t* wp = static_cast<const uint8_t*>(r < G ? a.qn_w : a.kn_w);
      const uint2 u = *reinterpret_cast<const uint2*>(row + 8 * lane);
      const uint2 uw = *reinterpret_cast<const uint2*>(wp + 8 * lane);
      float x[4], w[4], c[4] = {1.f, 1.f, 1.f, 1.f}, sn[4] = {0.f, 0.f, 0.f, 0.f};
      const float2 x0 = ElemTraits<T>::unpack2(u.x), x1 = ElemTraits<T>::unpack2(u.y);
      const float2 w0 = ElemTraits<T>::unpack2(uw.x), w1 = ElemTraits<T>::unpack2(uw.y);
      x[0] = x0.x; x[1] = x0.y; x[2] = x1.x; x[3] = x1.y;
      w[0] = w0.x; w[1] = w0.y; w[2] = w1.x; w[3] = w1.y;
      const int half_lanes = a.rot >> 3;
      if (lane < 2 * half_lanes) {
        const uint8_t* cb = static_cast<const uint8_t*>(a.cs) + 2 * (b * a.cs_b) + 8 * lane;
        const uint8_t* sb = static_cast<const uint8_t*>(a.sn) + 2 * (b * a.cs_b) + 8 * lane;
        const uint2 uc = *reinterpret_cast<const uint2*>(cb), us = *reinterpret_cast<const uint2*>(sb);
        const float2 c0 = ElemTraits<T>::unpack2(uc.x), c1 = ElemTraits<T>::unpack2(uc.y);
        const float2 s0 = ElemTraits<T>::unpack2(us.x), s1 = ElemTraits<T>::unpack2(us.y);
        c[0] = c0.x; c[1] = c0.y; c[2] = c1.x; c[3] = c1.y;
        sn[0] = s0.x; sn[1] = s0.y; sn[2] = s1.x; sn[3] = s1.y;
      }
      qk_row<T>(x, w, a.qk_eps, lane, half_lanes, c, sn);
      *reinterpret_cast<uint2*>(row + 8 * lane) = make_uint2(ElemTraits<T>::pack2(x[0], x[1]), ElemTraits<T>::pack2(x[2], x[3]));
    }
    __syncthreads();
  }
  if (a.knew && threadIdx.x < 32) {
    // fused append: the new token (staged as the last window row) goes to ring slot
    // p % ring; any block close above has already read the ring
    const int slot = (int)((uint64_t)p % (uint64_t)a.ring);
    const int isv = threadIdx.x >= 16;
    const int ch = threadIdx.x & 15;
    st_128(row_ptr(isv ? a.v : a.k, b, kvh, slot) + ch * 16,
           *reinterpret_cast<const uint4*>(kv + (isv * maxk + nraw - 1) * kDecPitch + ch * 16));
  }

  // Tensor-core tiles (mma.sync m16n8k16, fp32 accumulate): warp w takes the 16-key tiles
  // w, w + NW, ... of the staged keys.  S = Q K^T for its tile has the G heads as rows (padded
  // to 16) and 16 keys as columns; an online softmax (exp2 domain) per head turns it into P
  // (16-bit, in registers, already in the A-operand layout), and O += P V over the 128 value
  // columns (16 n-tiles, V fragments by ldmatrix.trans).  Rows >= G and keys >= nk are masked.
  const int gid = lane >> 2, tig = lane & 3;
  if (!zero_early) {  // rows nk .. end of the last tile (see above)
    for (int c = threadIdx.x; c < ((nk + 15) / 16 * 16 - nk) * 16; c += NT)
      *reinterpret_cast<uint4*>(kv + (maxk + nk + (c >> 4)) * kDecPitch + (c & 15) * 16) = make_uint4(0, 0, 0, 0);
    __syncthreads();
  }
  uint32_t qa[8][4];  // Q fragments for the 8 k-steps of 16 head dims (rows gid, gid + 8)
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int d = kk * 16 + tig * 2;
    qa[kk][0] = gid < G ? *reinterpret_cast<const uint32_t*>(qraw + gid * kDecPitch + 2 * d) : 0u;
    qa[kk][1] = gid + 8 < G ? *reinterpret_cast<const uint32_t*>(qraw + (gid + 8) * kDecPitch + 2 * d) : 0u;
    qa[kk][2] = gid < G ? *reinterpret_cast<const uint32_t*>(qraw + gid * kDecPitch + 2 * (d + 8)) : 0u;
    qa[kk][3] = gid + 8 < G ? *reinterpret_cast<const uint32_t*>(qraw + (gid + 8) * kDecPitch + 2 * (d + 8)) : 0u;
  }
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};  // rows gid, gid + 8
  float acc[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  const int ntiles = (nk + 15) >> 4;
#pragma unroll 1
  for (int kt = warp; kt < ntiles; kt += NW) {
    const int k0 = kt * 16;
    float sacc[2][4];  // two 8-key n-tiles
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      sacc[h][0] = sacc[h][1] = sacc[h][2] = sacc[h][3] = 0.f;
      const uint8_t* krow = kv + (k0 + h * 8 + gid) * kDecPitch;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(krow + 2 * (kk * 16 + tig * 2));
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(krow + 2 * (kk * 16 + tig * 2 + 8));
        mma_16816<T>(sacc[h], qa[kk], b0, b1);
      }
    }
    // scale, mask keys >= nk, tile max per row
    float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k0 + h * 8 + tig * 2 + (e & 1);
        const float v = key < nk ? sacc[h][e] * a.scale_log2 : -INFINITY;
        sacc[h][e] = v;
        tmax[e >> 1] = fmaxf(tmax[e >> 1], v);
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 1));
      tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 2));
    }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float mn = fmaxf(mrow[r], tmax[r]);
      corr[r] = ex2_approx(mrow[r] - mn);  // 0 when the row had no keys yet
      mrow[r] = mn;
      lrow[r] *= corr[r];
    }
    uint32_t pa[4];
    float psum[2] = {0.f, 0.f};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float p0 = ex2_approx(sacc[h][0] - mrow[0]), p1 = ex2_approx(sacc[h][1] - mrow[0]);
      const float p2 = ex2_approx(sacc[h][2] - mrow[1]), p3 = ex2_approx(sacc[h][3] - mrow[1]);
      psum[0] += p0 + p1;
      psum[1] += p2 + p3;
      pa[h * 2] = ElemTraits<T>::pack2(p0, p1);      // row gid, keys 8h + 2 tig ..
      pa[h * 2 + 1] = ElemTraits<T>::pack2(p2, p3);  // row gid + 8
    }
    // A fragment order: (row gid, k 0-7), (row gid+8, k 0-7), (row gid, k 8-15), (row gid+8, k 8-15)
    const uint32_t pfrag[4] = {pa[0], pa[1], pa[2], pa[3]};
#pragma unroll
    for (int r = 0; r < 2; ++r) lrow[r] += psum[r];
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      acc[n][0] *= corr[0];
      acc[n][1] *= corr[0];
      acc[n][2] *= corr[1];
      acc[n][3] *= corr[1];
    }
    // V fragments: ldmatrix.x4.trans over (keys k0..k0+15) x (columns 16 np .. 16 np + 15)
    const uint8_t* vbase = kv + (size_t)maxk * kDecPitch;
#pragma unroll
    for (int np = 0; np < 8; ++np) {
      const int mat = lane >> 3, rr = lane & 7;
      const uint8_t* addr = vbase + (k0 + (mat & 1) * 8 + rr) * kDecPitch + 2 * (np * 16 + (mat >> 1) * 8);
      uint32_t v0, v1, v2, v3;
      ldmatrix_x4_trans(addr, v0, v1, v2, v3);
      mma_16816<T>(acc[2 * np], pfrag, v0, v1);
      mma_16816<T>(acc[2 * np + 1], pfrag, v2, v3);
    }
  }
  // row sums across the quad
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
  }
  // partials of warp w: outputs at part[w][g][col], (max, sum) at ml[w][g]
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int g = gid + 8 * r;
    if (g < G) {
#pragma unroll
      for (int n = 0; n < 16; ++n)
        *reinterpret_cast<float2*>(part + (warp * G + g) * 128 + n * 8 + tig * 2) = make_float2(acc[n][2 * r], acc[n][2 * r + 1]);
      if (tig == 0) {
        ml[(warp * G + g) * 2] = mrow[r];
        ml[(warp * G + g) * 2 + 1] = lrow[r];
      }
    }
  }
  __syncthreads();
  // merge: thread = (head, two columns).  Each thread derives its head's global max, the
  // partials' rescale factors and the total sum itself (a few shared-memory reads and
  // nact exp2 per thread), so no second barrier and no serial per-head phase
  constexpr int NP = NW;  // partials per head
  const int nact = ntiles < NW ? ntiles : NW;  // warps that saw keys
#pragma unroll 1
  for (int r = threadIdx.x; r < G * 64; r += NT) {
    const int g = r >> 6, c = (r & 63) * 2;
    float mw[NP];
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NP; ++w) {
      mw[w] = w < nact ? ml[(w * G + g) * 2] : -INFINITY;
      M = fmaxf(M, mw[w]);
    }
    float L = 0.f, s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int w = 0; w < NP; ++w) {
      if (w < nact) {
        const float cw = mw[w] == -INFINITY ? 0.f : ex2_approx(mw[w] - M);
        L = fmaf(ml[(w * G + g) * 2 + 1], cw, L);
        const float2 f = *reinterpret_cast<const float2*>(part + (w * G + g) * 128 + c);
        s0 = fmaf(f.x, cw, s0);
        s1 = fmaf(f.y, cw, s1);
      }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    *reinterpret_cast<uint32_t*>(row_ptr(a.out, b, kvh * G + g, t) + c * 2) = ElemTraits<T>::pack2(s0 * inv, s1 * inv);
    if (a.lse && c == 0) a.lse[b * a.ls_b + (int64_t)(kvh * G + g) * a.ls_h + t] = (M + log2f(L)) * 0.6931471805599453f;
  }
}

// ------------------------------------------------------------------------------ launch probe
// An empty grid launched like the decode step (programmatic dependent launch): a chain of
// these measures the per-launch floor that a chain of decode steps cannot go below.
__global__ void launch_probe_kernel() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

int launch_probe(int ctas, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(ctas > 0 ? ctas : 1));
  cfg.blockDim = dim3(32);
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, launch_probe_kernel), "launch probe");
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
                  const bna_tensor4* vnew, int64_t close_block, int64_t close_slot, cudaStream_t stream,
                  const QKPrep* prep) {
  ActiveArgs a{};
  if (prep) {
    a.qk_prep = 1;
    a.qn_w = prep->q_weight;
    a.kn_w = prep->k_weight;
    a.cs = prep->cos;
    a.sn = prep->sin;
    a.cs_b = prep->cs_b;
    a.rot = prep->rot;
    a.qk_eps = prep->eps;
  }
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
  const size_t smem = decode_smem_bytes(a.G, window);
  dim3 grid((unsigned)a.Tq, (unsigned)(a.B * a.Hkv));
  if (grid.x == 0 || grid.y == 0) return BNA_OK;
  auto launch = [&](auto kern) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(decode_threads(a.G));
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
