// decode_tail.cu — the decoder layer after the attention, for one decode step of 1..8
// tokens, as ONE cooperative kernel: everything between this layer's attention and the
// next layer's attention.
//
//   phase 0  x2  = x + o_proj(o * sigmoid(gate))          (attention output gate, residual)
//   phase 1  act = silu(gate_proj(h)) * up_proj(h),  h = rmsnorm(x2)
//   phase 2  x3  = x2 + down_proj(act)                     (residual)
//   phase 3  qkv = [q_proj; k_proj; v_proj](rmsnorm(x3))   (the next layer's projections; optional)
//
// Each phase is a weight-streaming GEMV of the same form as gemv.cu (warp task = one output
// row or gate/up row pair over a K segment of up to 1024 columns; segments of an output meet
// in shared memory; fp32 dot products rounded where the eager layer rounds) and every
// phase's input depends on all of the previous phase's outputs, so the phases are separated
// by grid-wide barriers instead of kernel boundaries.  One CTA runs per SM (a cooperative
// launch guarantees they are co-resident), and while a phase computes, the CTA's weight
// slices of the NEXT phase stream into shared memory by cp.async, so each barrier is
// followed by compute on weights that have already arrived.
//
// The barrier is a counter plus generation word in device memory, reset by its last
// arrival, so it needs no per-launch state; calls on one device must not overlap (they
// share the words).  Every spin is bounded: on timeout the CTA records an error in the
// device error word (bna_take_device_error), raises an abort flag and returns.
#include <cuda_runtime.h>

#include <string>
#include <type_traits>

#include "common.cuh"

namespace bna {
int* device_error_word();

namespace {

constexpr int kTailThreads = 256;  // 8 warps
constexpr int kTailWarps = kTailThreads / 32;
constexpr long long kBarrierTimeoutCycles = 4000000000LL;  // ~2 s at 2 GHz

__device__ unsigned int g_tail_count = 0;
__device__ unsigned int g_tail_gen = 0;
__device__ int g_tail_abort = 0;

struct TailArgs {
  int M, H, I, nqkv, heads, head_dim;
  const uint8_t* o;       // [M, heads * head_dim] contiguous
  const uint8_t* gate;    // gate[m, h, d] at gate + m * g_tok + h * g_head + d
  int64_t g_tok, g_head;
  const uint8_t* x;       // [M, H] contiguous: the layer input (residual)
  const uint8_t* w_o;     // [H, heads * head_dim]
  const uint8_t* post_w;  // [H]
  float post_eps;
  const uint8_t* w_gu;    // [2 I, H]: gate rows, then up rows
  const uint8_t* w_d;     // [H, I]
  const uint8_t* next_w;  // [H] next layer's input norm (phase 3)
  float next_eps;
  const uint8_t* w_qkv;   // [nqkv, H] (nullptr: no phase 3)
  uint8_t* x2;            // [M, H]
  uint8_t* act;           // [M, I]
  uint8_t* x3;            // [M, H]
  uint8_t* qkv;           // [M, nqkv]
  int* err;
  uint32_t region0, region1;  // bytes of the two weight staging regions
};

// Phase p: a GEMV of n_out outputs over K columns, S segments of 4 chunks per output,
// R rows per output (2 for the gate/up pairs of SWIGLU).
struct Phase {
  const uint8_t* w;
  int64_t K, up_off;
  int n_out, S, R;
  __device__ int opc() const { return kTailWarps / S; }
  __device__ int ctasks() const { return (n_out + opc() - 1) / opc(); }
};

__device__ __forceinline__ void unpack8t(const uint4& u, float* f, bool bf) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 t = bf ? ElemTraits<__nv_bfloat16>::unpack2(w[e]) : ElemTraits<__half>::unpack2(w[e]);
    f[2 * e] = t.x;
    f[2 * e + 1] = t.y;
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack8t(const float* f) {
  return make_uint4(ElemTraits<T>::pack2(f[0], f[1]), ElemTraits<T>::pack2(f[2], f[3]),
                    ElemTraits<T>::pack2(f[4], f[5]), ElemTraits<T>::pack2(f[6], f[7]));
}

__device__ __forceinline__ void cp16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
               "l"(gsrc)
               : "memory");
}

// Stage this CTA's weight slices of phase `ph` into `dst` (slot = task, warp, row, chunk, lane).
__device__ void stage_weights(const Phase& ph, uint8_t* dst) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = (int)(ph.K >> 8);
  int k = 0;
  for (int ct = blockIdx.x; ct < ph.ctasks(); ct += gridDim.x, ++k) {
    const int ol = warp / ph.S, seg = warp - ol * ph.S;
    int o = ct * ph.opc() + ol;
    if (o >= ph.n_out) o = ph.n_out - 1;
    for (int r = 0; r < ph.R; ++r) {
      const int64_t row = (int64_t)o + (r ? ph.up_off : 0);
      for (int c = 0; c < 4; ++c) {
        const int ch = seg * 4 + c;
        if (ch < nch)
          cp16(dst + ((((size_t)k * kTailWarps + warp) * ph.R + r) * 4 + c) * 512 + lane * 16,
               ph.w + 2 * (row * ph.K + (int64_t)(ch * 32 + lane) * 8));
      }
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// Grid barrier (all CTAs co-resident).  Returns false after a timeout or an abort.
__device__ bool grid_barrier(const TailArgs& a) {
  __syncthreads();
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    volatile unsigned int* gen = &g_tail_gen;
    const unsigned int my = *gen;
    __threadfence();
    const unsigned int arrived = atomicAdd(&g_tail_count, 1u);
    if (arrived == gridDim.x - 1) {
      atomicExch(&g_tail_count, 0u);
      __threadfence();
      atomicAdd(&g_tail_gen, 1u);
    } else {
      const long long t0 = clock64();
      while (*gen == my) {
        if (*reinterpret_cast<volatile int*>(&g_tail_abort) || clock64() - t0 > kBarrierTimeoutCycles) {
          atomicExch(&g_tail_abort, 1);
          if (a.err) atomicCAS(a.err, 0, 0x2000);
          ok = 0;
          break;
        }
      }
    }
    __threadfence();
  }
  __syncthreads();
  if (!ok) asm volatile("cp.async.wait_all;" ::: "memory");  // own copies land before returning
  return ok != 0;
}

// x_in [M][K] (storage type) in shared memory from a global [M][K] source (plain, or with
// the attention gate, or Qwen3.5-RMSNorm'd with weight nw).
enum Build { B_PLAIN = 0, B_GATE = 1, B_NORM = 2 };

template <typename T>
__device__ void build_x(const TailArgs& a, int mode, const uint8_t* src, int64_t K, const uint8_t* nw, float eps,
                        uint8_t* xs, float* red) {
  constexpr bool bf = std::is_same<T, __nv_bfloat16>::value;
  const int nvec = (int)(K >> 3);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int m = 0; m < a.M; ++m) {
    float ss = 0.f;
    for (int v = tid; v < nvec; v += kTailThreads) {
      float f[8];
      // inputs written by other CTAs before a grid barrier: read through L2 (not L1)
      unpack8t(__ldcg(reinterpret_cast<const uint4*>(src + 2 * ((int64_t)m * K + v * 8))), f, bf);
      if (mode == B_GATE) {
        const int c = v * 8, h = c / a.head_dim, d = c - h * a.head_dim;
        float g[8];
        unpack8t(__ldcg(reinterpret_cast<const uint4*>(a.gate + 2 * ((int64_t)m * a.g_tok + (int64_t)h * a.g_head + d))), g, bf);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = f[e] * round_to<T>(1.f / (1.f + __expf(-g[e])));
      }
      if (mode == B_NORM) {
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
      }
      *reinterpret_cast<uint4*>(xs + 2 * ((int64_t)m * K + v * 8)) = pack8t<T>(f);
    }
    if (mode == B_NORM) {
      ss = warp_sum(ss);
      if (lane == 0) red[warp] = ss;
      __syncthreads();
      float tot = 0.f;
      for (int i = 0; i < kTailWarps; ++i) tot += red[i];
      const float r = rsqrtf(tot / (float)K + eps);
      for (int v = tid; v < nvec; v += kTailThreads) {
        uint8_t* p = xs + 2 * ((int64_t)m * K + v * 8);
        float f[8], w[8];
        unpack8t(*reinterpret_cast<const uint4*>(p), f, bf);
        unpack8t(ld_nc_128(nw + 16 * v), w, bf);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = (f[e] * r) * (1.f + w[e]);
        *reinterpret_cast<uint4*>(p) = pack8t<T>(f);
      }
      __syncthreads();
    }
  }
  __syncthreads();
}

enum Epi { E_RESID = 0, E_SWIGLU = 1, E_STORE = 2 };

// Compute this CTA's tasks of a phase from staged weights `ws` and input `xs`.
template <typename T, int MT>
__device__ void compute_phase(const TailArgs& a, const Phase& ph, const uint8_t* ws, const uint8_t* xs, int epi,
                              const uint8_t* res, uint8_t* out, int64_t out_stride, float (*part)[2][MT]) {
  constexpr bool bf = std::is_same<T, __nv_bfloat16>::value;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = (int)(ph.K >> 8);
  int k = 0;
  for (int ct = blockIdx.x; ct < ph.ctasks(); ct += gridDim.x, ++k) {
    const int ol = warp / ph.S, seg = warp - ol * ph.S;
    float acc[2][MT];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[r][m] = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int ch = seg * 4 + c;
      if (ch < nch) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          if (r < ph.R) {
            float wf[8];
            unpack8t(*reinterpret_cast<const uint4*>(ws + ((((size_t)k * kTailWarps + warp) * ph.R + r) * 4 + c) * 512 +
                                                     lane * 16),
                     wf, bf);
#pragma unroll
            for (int m = 0; m < MT; ++m) {
              float xf[8];
              unpack8t(*reinterpret_cast<const uint4*>(xs + 2 * ((int64_t)m * ph.K + (ch * 32 + lane) * 8)), xf, bf);
#pragma unroll
              for (int e = 0; e < 8; ++e) acc[r][m] = fmaf(wf[e], xf[e], acc[r][m]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        float v = acc[r][m];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0) part[warp][r][m] = v;
      }
    __syncthreads();
    const int opc = ph.opc();
    if ((int)threadIdx.x < opc * MT) {
      const int ole = threadIdx.x / MT, m = threadIdx.x - ole * MT;
      const int oe = ct * opc + ole;
      if (oe < ph.n_out && m < a.M) {
        float y0 = 0.f, y1 = 0.f;
        for (int sg = 0; sg < ph.S; ++sg) {
          y0 += part[ole * ph.S + sg][0][m];
          y1 += part[ole * ph.S + sg][1][m];
        }
        float v;
        if (epi == E_SWIGLU) {
          const float g = round_to<T>(y0), u = round_to<T>(y1);
          v = round_to<T>(g / (1.f + __expf(-g))) * u;
        } else {
          v = round_to<T>(y0);
          if (epi == E_RESID) {
            const unsigned short rb = __ldcg(reinterpret_cast<const unsigned short*>(res + 2 * ((int64_t)m * a.H + oe)));
            v = v + ElemTraits<T>::unpack2((uint32_t)rb).x;
          }
        }
        *reinterpret_cast<uint16_t*>(out + 2 * ((int64_t)m * out_stride + oe)) =
            (uint16_t)(ElemTraits<T>::pack2(v, 0.f) & 0xFFFFu);
      }
    }
    __syncthreads();
  }
}

__device__ __forceinline__ int seg_count(int64_t K) {
  const int nch = (int)(K >> 8);
  return nch <= 4 ? 1 : (nch <= 8 ? 2 : (nch <= 16 ? 4 : 8));
}

template <typename T, int MT>
__global__ void __launch_bounds__(kTailThreads, 1) decode_tail_kernel(const TailArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float part[kTailWarps][2][MT];
  __shared__ float red[kTailWarps];
  uint8_t* r0 = smem;                 // staging region 0: o_proj, then down_proj weights
  uint8_t* r1 = smem + a.region0;     // staging region 1: gate/up, then q/k/v weights
  uint8_t* xs = r1 + a.region1;       // [MT][Kmax] input rows
  if (threadIdx.x == 0 && blockIdx.x == 0) g_tail_abort = 0;  // first barrier orders this
  const int Kq = a.heads * a.head_dim;
  const Phase p0{a.w_o, Kq, 0, a.H, seg_count(Kq), 1};
  const Phase p1{a.w_gu, a.H, a.I, a.I, seg_count(a.H), 2};
  const Phase p2{a.w_d, a.I, 0, a.H, seg_count(a.I), 1};
  const Phase p3{a.w_qkv, a.H, 0, a.nqkv, seg_count(a.H), 1};
  stage_weights(p0, r0);
  stage_weights(p1, r1);
  // phase 0: x2 = x + o_proj(o * sigmoid(gate))
  build_x<T>(a, B_GATE, a.o, Kq, nullptr, 0.f, xs, red);
  asm volatile("cp.async.wait_group 1;" ::: "memory");
  __syncthreads();
  compute_phase<T, MT>(a, p0, r0, xs, E_RESID, a.x, a.x2, a.H, part);
  stage_weights(p2, r0);  // region 0 is free again
  if (!grid_barrier(a)) return;
  // phase 1: act = swiglu(gate_up(rmsnorm(x2)))
  build_x<T>(a, B_NORM, a.x2, a.H, a.post_w, a.post_eps, xs, red);
  asm volatile("cp.async.wait_group 1;" ::: "memory");
  __syncthreads();
  compute_phase<T, MT>(a, p1, r1, xs, E_SWIGLU, nullptr, a.act, a.I, part);
  if (a.w_qkv) stage_weights(p3, r1);
  if (!grid_barrier(a)) return;
  // phase 2: x3 = x2 + down(act)
  build_x<T>(a, B_PLAIN, a.act, a.I, nullptr, 0.f, xs, red);
  if (a.w_qkv) asm volatile("cp.async.wait_group 1;" ::: "memory");
  else asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  compute_phase<T, MT>(a, p2, r0, xs, E_RESID, a.x2, a.x3, a.H, part);
  if (!a.w_qkv) return;
  if (!grid_barrier(a)) return;
  // phase 3: qkv = W_qkv rmsnorm(x3) (the next layer's input norm)
  build_x<T>(a, B_NORM, a.x3, a.H, a.next_w, a.next_eps, xs, red);
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  compute_phase<T, MT>(a, p3, r1, xs, E_STORE, nullptr, a.qkv, a.nqkv, part);
}

// bytes one CTA stages for a phase of n_out outputs over K columns (R rows each)
size_t stage_bytes(int n_out, int64_t K, int R, int grid) {
  const int nch = (int)(K >> 8);
  const int S = nch <= 4 ? 1 : (nch <= 8 ? 2 : (nch <= 16 ? 4 : 8));
  const int opc = kTailWarps / S;
  const int ctasks = (n_out + opc - 1) / opc;
  const int per = (ctasks + grid - 1) / grid;
  return (size_t)per * kTailWarps * R * 4 * 512;
}

template <typename T, int MT>
int launch_tail(TailArgs a, cudaStream_t s) {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = sms;
  const int64_t Kq = (int64_t)a.heads * a.head_dim;
  size_t reg0 = stage_bytes(a.H, Kq, 1, grid), rd = stage_bytes(a.H, a.I, 1, grid);
  if (rd > reg0) reg0 = rd;
  size_t reg1 = stage_bytes(a.I, a.H, 2, grid);
  if (a.w_qkv) {
    const size_t rq = stage_bytes(a.nqkv, a.H, 1, grid);
    if (rq > reg1) reg1 = rq;
  }
  int64_t kmax = Kq > a.H ? Kq : a.H;
  if (a.I > kmax) kmax = a.I;
  const size_t smem = reg0 + reg1 + (size_t)MT * kmax * 2;
  if (smem > 225 * 1024) return fail(BNA_UNSUPPORTED, "decode_tail: the layer's weight slices exceed shared memory (" +
                                                          std::to_string(smem) + " bytes per CTA)");
  a.region0 = (uint32_t)reg0;
  a.region1 = (uint32_t)reg1;
  auto kern = decode_tail_kernel<T, MT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "decode_tail smem attribute");
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kTailThreads, smem);
  if (e != cudaSuccess) return check_cuda(e, "decode_tail occupancy");
  if (per_sm < 1) return fail(BNA_UNSUPPORTED, "decode_tail: one CTA per SM does not fit");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kTailThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, a), "decode_tail launch");
}

template <typename T>
int launch_tail_m(const TailArgs& a, cudaStream_t s) {
  if (a.M <= 1) return launch_tail<T, 1>(a, s);
  if (a.M <= 2) return launch_tail<T, 2>(a, s);
  if (a.M <= 4) return launch_tail<T, 4>(a, s);
  return launch_tail<T, 8>(a, s);
}

bool al16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace bna

using namespace bna;

extern "C" BNA_API int bna_decode_layer_tail(
    const void* o, const void* gate, int64_t gate_tok_stride, int64_t gate_head_stride, int32_t heads,
    int32_t head_dim, const void* x, const void* w_o, const void* post_norm_weight, float post_eps,
    const void* w_gate_up, const void* w_down, int32_t hidden, int32_t intermediate, const void* next_norm_weight,
    float next_eps, const void* w_qkv, int32_t qkv_rows, void* x2, void* act, void* x3, void* qkv, int32_t tokens,
    int32_t dtype, void* stream) {
  if (tokens < 1 || tokens > 8) return fail(BNA_UNSUPPORTED, "decode_tail: 1 <= tokens <= 8");
  if (hidden <= 0 || hidden % 256 || intermediate <= 0 || intermediate % 256 || heads <= 0 || head_dim <= 0 ||
      (heads * head_dim) % 256 || head_dim % 8)
    return fail(BNA_UNSUPPORTED, "decode_tail: hidden, intermediate and heads * head_dim must be multiples of 256");
  if (hidden > 8192 || intermediate > 8192 || heads * head_dim > 8192)
    return fail(BNA_UNSUPPORTED, "decode_tail: in_features <= 8192");
  if (!o || !gate || !x || !w_o || !post_norm_weight || !w_gate_up || !w_down || !x2 || !act || !x3)
    return fail(BNA_BAD_SHAPE, "decode_tail: null pointer");
  if (w_qkv && (!next_norm_weight || !qkv || qkv_rows <= 0)) return fail(BNA_BAD_SHAPE, "decode_tail: bad next-layer arguments");
  for (const void* p : {o, gate, x, w_o, post_norm_weight, w_gate_up, w_down, next_norm_weight, w_qkv,
                        (const void*)x2, (const void*)act, (const void*)x3, (const void*)qkv})
    if (!al16(p)) return fail(BNA_BAD_STRIDE, "decode_tail: pointers must be 16-byte aligned");
  if (gate_tok_stride % 8 || gate_head_stride % 8) return fail(BNA_BAD_STRIDE, "decode_tail: gate strides must be multiples of 8");
  TailArgs a{};
  a.M = tokens; a.H = hidden; a.I = intermediate; a.nqkv = w_qkv ? qkv_rows : 0;
  a.heads = heads; a.head_dim = head_dim;
  a.o = static_cast<const uint8_t*>(o); a.gate = static_cast<const uint8_t*>(gate);
  a.g_tok = gate_tok_stride; a.g_head = gate_head_stride;
  a.x = static_cast<const uint8_t*>(x); a.w_o = static_cast<const uint8_t*>(w_o);
  a.post_w = static_cast<const uint8_t*>(post_norm_weight); a.post_eps = post_eps;
  a.w_gu = static_cast<const uint8_t*>(w_gate_up); a.w_d = static_cast<const uint8_t*>(w_down);
  a.next_w = static_cast<const uint8_t*>(next_norm_weight); a.next_eps = next_eps;
  a.w_qkv = static_cast<const uint8_t*>(w_qkv);
  a.x2 = static_cast<uint8_t*>(x2); a.act = static_cast<uint8_t*>(act); a.x3 = static_cast<uint8_t*>(x3);
  a.qkv = static_cast<uint8_t*>(qkv);
  a.err = device_error_word();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == BNA_BF16) return launch_tail_m<__nv_bfloat16>(a, s);
  if (dtype == BNA_F16) return launch_tail_m<__half>(a, s);
  return fail(BNA_BAD_DTYPE, "decode_tail: bfloat16 or float16 only");
}
