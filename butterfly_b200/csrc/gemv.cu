// gemv.cu — decode-time projections of the Qwen3.5 decoder layer around the compressed
// attention, for a handful of tokens (M <= 8): y[m, n] = sum_k W[n, k] * x_in[m, k], with the
// step before the projection fused as a prologue and the step after it as an epilogue.
//
//   prologue  NONE    x_in = x
//             NORM    x_in = rmsnorm(x [+ res])   (Qwen3.5 form; the sum is written out)
//             GATE    x_in = o * sigmoid(gate)    (attention output gate)
//   epilogue  STORE   y = round(acc)
//             RESID   y = round(res2 + round(acc)) (the decoder layer's residual add)
//             SWIGLU  y[i] = round(round(silu(round(acc[i]))) * round(acc[i + up_off]))
//
// Each prologue/epilogue does the eager ops' arithmetic, rounding to the storage type where
// the eager layer rounds.  The projection is HBM-bound (every weight byte is read once per
// call).  A warp owns one output (the gate/up row pair for SWIGLU) over one K segment of
// up to 1024 columns, lane l taking columns [8(32c + l), +8) of chunk c; it issues all its
// 128-bit weight loads before griddepcontrol.wait, so under programmatic dependent launch
// the weight stream of a projection overlaps the tail of the kernel that produces its
// input.  x_in is then built in shared memory by every CTA (it is a few KB), the dot
// products are reduced across the warp with shuffles and the K segments through shared
// memory.
#include <cuda_runtime.h>

#include <string>
#include <type_traits>

#include "common.cuh"

namespace bna {
namespace {

enum Prologue { PRO_NONE = 0, PRO_NORM = 1, PRO_GATE = 2 };
enum Epilogue { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2 };

constexpr int kGemvWarps = 8;
constexpr int kMaxM = 8;

struct GemvArgs {
  const uint8_t* x;     // [M, K] rows of x_stride (NONE / NORM), or o [M, K] contiguous (GATE)
  int64_t x_stride;
  const uint8_t* res;   // NORM: residual added before the norm (nullable)
  int64_t res_stride;
  const uint8_t* norm_w;
  float eps;
  uint8_t* sum_out;     // NORM with res: x + res written here by CTA 0 (nullable)
  int64_t sum_stride;
  const uint8_t* gate;  // GATE: gate[m, h, d] at gate + m*g_tok + h*g_head + d
  int64_t g_tok, g_head;
  int head_dim;
  const uint8_t* w;     // [N_rows, K] row-major
  int64_t K;
  int n_out;            // outputs per token (rows, or SWIGLU pairs)
  int64_t up_off;       // SWIGLU: row offset of the up rows
  const uint8_t* res2;  // RESID: residual [M, n_out] of res2_stride
  int64_t res2_stride;
  uint8_t* out;         // [M, n_out] of out_stride
  int64_t out_stride;
  int M;
};

template <typename T>
__device__ __forceinline__ float rnd(float x) {
  return ElemTraits<T>::unpack2(ElemTraits<T>::pack2(x, 0.f)).x;
}

__device__ __forceinline__ void unpack8f(const uint4& u, float* f, bool bf) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 t = bf ? ElemTraits<__nv_bfloat16>::unpack2(w[e]) : ElemTraits<__half>::unpack2(w[e]);
    f[2 * e] = t.x;
    f[2 * e + 1] = t.y;
  }
}

// Build x_in [M, K] (storage type) in shared memory.
template <typename T, int PRO>
__device__ __forceinline__ void build_input(const GemvArgs& a, uint8_t* xs, float* red) {
  constexpr bool bf = std::is_same<T, __nv_bfloat16>::value;
  const int nvec = (int)(a.K >> 3);
  const int tid = threadIdx.x, nth = blockDim.x;
  const int warp = tid >> 5, lane = tid & 31;
  for (int m = 0; m < a.M; ++m) {
    float ss = 0.f;
    for (int v = tid; v < nvec; v += nth) {
      float f[8];
      if (PRO == PRO_GATE) {
        const int c = v * 8;
        const int h = c / a.head_dim, d = c - h * a.head_dim;
        float g[8];
        unpack8f(ld_128(a.x + 2 * ((int64_t)m * a.K + c)), f, bf);
        unpack8f(ld_128(a.gate + 2 * ((int64_t)m * a.g_tok + (int64_t)h * a.g_head + d)), g, bf);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = f[e] * rnd<T>(sigmoid_fast(g[e]));
      } else {
        unpack8f(ld_128(a.x + 2 * ((int64_t)m * a.x_stride + v * 8)), f, bf);
        if (PRO == PRO_NORM && a.res) {
          float r[8];
          unpack8f(ld_128(a.res + 2 * ((int64_t)m * a.res_stride + v * 8)), r, bf);
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = rnd<T>(f[e] + r[e]);
          if (a.sum_out && blockIdx.x == 0) {
            const uint4 p = make_uint4(ElemTraits<T>::pack2(f[0], f[1]), ElemTraits<T>::pack2(f[2], f[3]),
                                       ElemTraits<T>::pack2(f[4], f[5]), ElemTraits<T>::pack2(f[6], f[7]));
            st_128(a.sum_out + 2 * ((int64_t)m * a.sum_stride + v * 8), p);
          }
        }
        if (PRO == PRO_NORM) {
#pragma unroll
          for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
        }
      }
      const uint4 p = make_uint4(ElemTraits<T>::pack2(f[0], f[1]), ElemTraits<T>::pack2(f[2], f[3]),
                                 ElemTraits<T>::pack2(f[4], f[5]), ElemTraits<T>::pack2(f[6], f[7]));
      *reinterpret_cast<uint4*>(xs + 2 * ((int64_t)m * a.K + v * 8)) = p;
    }
    if (PRO == PRO_NORM) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) red[warp] = ss;
      __syncthreads();
      float tot = 0.f;
      for (int i = 0; i < (nth >> 5); ++i) tot += red[i];
      const float r = rsqrtf(tot / (float)a.K + a.eps);
      for (int v = tid; v < nvec; v += nth) {
        uint8_t* p = xs + 2 * ((int64_t)m * a.K + v * 8);
        float f[8], w[8];
        unpack8f(*reinterpret_cast<const uint4*>(p), f, bf);
        unpack8f(ld_nc_128(a.norm_w + 16 * v), w, bf);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = (f[e] * r) * (1.f + w[e]);
        *reinterpret_cast<uint4*>(p) = make_uint4(ElemTraits<T>::pack2(f[0], f[1]), ElemTraits<T>::pack2(f[2], f[3]),
                                                  ElemTraits<T>::pack2(f[4], f[5]), ElemTraits<T>::pack2(f[6], f[7]));
      }
      __syncthreads();  // red[] reused by the next token
    }
  }
  __syncthreads();
}

// Warp task = (output, K segment of up to 4 chunks of 256 columns): S segments per output,
// 8 / S outputs per CTA.  A warp preloads its (at most 4 x R) 128-bit weight loads before the
// dependency wait, so the code each warp runs is one short straight stretch (long unrolled
// code executed once per warp is bound by instruction fetch), and every projection
// spreads over hundreds of CTAs.  The S segment partials of an output meet in shared memory.
template <typename T, int PRO, int EPI, int MT, int S>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(const GemvArgs a) {
  constexpr bool bf = std::is_same<T, __nv_bfloat16>::value;
  constexpr int R = EPI == EPI_SWIGLU ? 2 : 1;
  constexpr int OPC = kGemvWarps / S;  // outputs per CTA
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[kGemvWarps];
  __shared__ float part[kGemvWarps][R][MT];
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ol = warp / S, seg = warp - ol * S;
  const int o = blockIdx.x * OPC + ol;
  const bool active = o < a.n_out;
  const int nch = (int)(a.K >> 8);
  const int c0 = seg * 4;
  const int oc = active ? o : a.n_out - 1;  // clamp: loads stay in bounds, results dropped
  const uint8_t* wrow[R];
  wrow[0] = a.w + 2 * ((int64_t)oc * a.K);
  if (R == 2) wrow[R - 1] = a.w + 2 * (((int64_t)oc + a.up_off) * a.K);
  uint4 wv[R][4];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (c0 + c < nch) wv[r][c] = ld_nc_128(wrow[r] + 16 * ((c0 + c) * 32 + lane));
  // the input is produced by the previous kernel of the stream
  asm volatile("griddepcontrol.wait;" ::: "memory");
  build_input<T, PRO>(a, smem, red);
  float acc[R][MT];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[r][m] = 0.f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    if (c0 + c < nch) {
      float wf[R][8];
#pragma unroll
      for (int r = 0; r < R; ++r) unpack8f(wv[r][c], wf[r], bf);
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        float xf[8];
        unpack8f(*reinterpret_cast<const uint4*>(smem + 2 * ((int64_t)m * a.K + ((c0 + c) * 32 + lane) * 8)), xf, bf);
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[r][m] = fmaf(wf[r][e], xf[e], acc[r][m]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      float v = acc[r][m];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) part[warp][r][m] = v;
    }
  __syncthreads();
  // epilogue: thread = (output of this CTA, token)
  const int tid = threadIdx.x;
  if (tid >= OPC * MT) return;
  const int ole = tid / MT, m = tid - ole * MT;
  const int oe = blockIdx.x * OPC + ole;
  if (oe >= a.n_out || m >= a.M) return;
  float y[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float t = 0.f;
#pragma unroll
    for (int sg = 0; sg < S; ++sg) t += part[ole * S + sg][r][m];
    y[r] = t;
  }
  float out;
  if (EPI == EPI_SWIGLU) {
    const float g = rnd<T>(y[0]), u = rnd<T>(y[R - 1]);
    out = rnd<T>(g / (1.f + __expf(-g))) * u;
  } else {
    out = rnd<T>(y[0]);
    if (EPI == EPI_RESID) {
      const uint16_t rb = *reinterpret_cast<const uint16_t*>(a.res2 + 2 * ((int64_t)m * a.res2_stride + oe));
      out = out + ElemTraits<T>::unpack2((uint32_t)rb).x;
    }
  }
  *reinterpret_cast<uint16_t*>(a.out + 2 * ((int64_t)m * a.out_stride + oe)) =
      (uint16_t)(ElemTraits<T>::pack2(out, 0.f) & 0xFFFFu);
}

template <typename T, int PRO, int EPI, int MT, int S>
int launch_gemv_ms(const GemvArgs& a, cudaStream_t s) {
  constexpr int OPC = kGemvWarps / S;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((a.n_out + OPC - 1) / OPC));
  cfg.blockDim = dim3(kGemvWarps * 32);
  cfg.dynamicSmemBytes = (size_t)MT * a.K * 2;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto kern = gemv_kernel<T, PRO, EPI, MT, S>;
  if (cfg.dynamicSmemBytes > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cfg.dynamicSmemBytes);
    if (e != cudaSuccess) return check_cuda(e, "gemv smem attribute");
  }
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, a), "gemv launch");
}

template <typename T, int PRO, int EPI, int MT>
int launch_gemv_m(const GemvArgs& a, cudaStream_t s) {
  const int nch = (int)(a.K >> 8);
  if (nch <= 4) return launch_gemv_ms<T, PRO, EPI, MT, 1>(a, s);
  if (nch <= 8) return launch_gemv_ms<T, PRO, EPI, MT, 2>(a, s);
  if (nch <= 16) return launch_gemv_ms<T, PRO, EPI, MT, 4>(a, s);
  return launch_gemv_ms<T, PRO, EPI, MT, 8>(a, s);
}

template <typename T, int PRO, int EPI>
int launch_gemv(const GemvArgs& a, cudaStream_t s) {
  if (a.M <= 1) return launch_gemv_m<T, PRO, EPI, 1>(a, s);
  if (a.M <= 2) return launch_gemv_m<T, PRO, EPI, 2>(a, s);
  if (a.M <= 4) return launch_gemv_m<T, PRO, EPI, 4>(a, s);
  return launch_gemv_m<T, PRO, EPI, 8>(a, s);
}

template <int PRO, int EPI>
int dispatch(const GemvArgs& a, int dtype, cudaStream_t s) {
  if (dtype == BNA_BF16) return launch_gemv<__nv_bfloat16, PRO, EPI>(a, s);
  if (dtype == BNA_F16) return launch_gemv<__half, PRO, EPI>(a, s);
  return fail(BNA_BAD_DTYPE, "gemv: bfloat16 or float16 only");
}

bool a16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int check_common(const GemvArgs& a) {
  if (a.M < 1 || a.M > kMaxM) return fail(BNA_UNSUPPORTED, "gemv: 1 <= tokens <= 8");
  if (a.K <= 0 || a.K % 256 || a.K > 8192) return fail(BNA_UNSUPPORTED, "gemv: in_features must be a multiple of 256, <= 8192");
  if ((int64_t)a.M * a.K * 2 > 160 * 1024) return fail(BNA_UNSUPPORTED, "gemv: tokens * in_features too large");
  if (a.n_out <= 0) return fail(BNA_BAD_SHAPE, "gemv: out_features must be positive");
  if (!a.x || !a.w || !a.out) return fail(BNA_BAD_SHAPE, "gemv: null pointer");
  for (const void* p : {(const void*)a.x, (const void*)a.w, (const void*)a.res, (const void*)a.norm_w,
                        (const void*)a.sum_out, (const void*)a.gate})
    if (!a16(p)) return fail(BNA_BAD_STRIDE, "gemv: pointers must be 16-byte aligned");
  for (int64_t st : {a.x_stride, a.res_stride, a.sum_stride, a.g_tok, a.g_head})
    if (st % 8) return fail(BNA_BAD_STRIDE, "gemv: strides must be multiples of 8 elements");
  return BNA_OK;
}

}  // namespace
}  // namespace bna

using namespace bna;

extern "C" BNA_API int bna_gemv_rmsnorm(const void* x, int64_t x_stride, const void* res, int64_t res_stride,
                                        const void* norm_weight, float eps, void* sum_out, int64_t sum_stride,
                                        const void* w, int64_t out_features, int64_t in_features, int32_t swiglu,
                                        void* out, int64_t out_stride, int32_t tokens, int32_t dtype, void* stream) {
  GemvArgs a{};
  a.x = static_cast<const uint8_t*>(x); a.x_stride = x_stride;
  a.res = static_cast<const uint8_t*>(res); a.res_stride = res ? res_stride : 0;
  a.norm_w = static_cast<const uint8_t*>(norm_weight); a.eps = eps;
  a.sum_out = static_cast<uint8_t*>(sum_out); a.sum_stride = sum_out ? sum_stride : 0;
  a.w = static_cast<const uint8_t*>(w); a.K = in_features;
  a.out = static_cast<uint8_t*>(out); a.out_stride = out_stride; a.M = tokens;
  if (!norm_weight) return fail(BNA_BAD_SHAPE, "gemv_rmsnorm: null norm weight");
  if (sum_out && !res) return fail(BNA_BAD_SHAPE, "gemv_rmsnorm: sum_out needs a residual");
  if (in_features > 8192) return fail(BNA_UNSUPPORTED, "gemv_rmsnorm: in_features <= 8192");
  if (swiglu) {
    if (out_features % 2) return fail(BNA_BAD_SHAPE, "gemv_rmsnorm: swiglu needs an even number of rows");
    a.n_out = (int)(out_features / 2);
    a.up_off = out_features / 2;
  } else {
    a.n_out = (int)out_features;
  }
  if (int rc = check_common(a)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return swiglu ? dispatch<PRO_NORM, EPI_SWIGLU>(a, dtype, s) : dispatch<PRO_NORM, EPI_STORE>(a, dtype, s);
}

extern "C" BNA_API int bna_gemv_gated(const void* o, const void* gate, int64_t gate_tok_stride,
                                      int64_t gate_head_stride, int32_t head_dim, const void* w, int64_t out_features,
                                      int64_t in_features, const void* res, int64_t res_stride, void* out,
                                      int64_t out_stride, int32_t tokens, int32_t dtype, void* stream) {
  GemvArgs a{};
  a.x = static_cast<const uint8_t*>(o); a.x_stride = in_features;
  a.gate = static_cast<const uint8_t*>(gate); a.g_tok = gate_tok_stride; a.g_head = gate_head_stride;
  a.head_dim = head_dim;
  a.w = static_cast<const uint8_t*>(w); a.K = in_features; a.n_out = (int)out_features;
  a.res2 = static_cast<const uint8_t*>(res); a.res2_stride = res_stride;
  a.out = static_cast<uint8_t*>(out); a.out_stride = out_stride; a.M = tokens;
  if (!gate || head_dim <= 0 || head_dim % 8 || in_features % head_dim)
    return fail(BNA_BAD_SHAPE, "gemv_gated: bad gate / head_dim");
  if (int rc = check_common(a)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return res ? dispatch<PRO_GATE, EPI_RESID>(a, dtype, s) : dispatch<PRO_GATE, EPI_STORE>(a, dtype, s);
}

extern "C" BNA_API int bna_gemv(const void* x, int64_t x_stride, const void* w, int64_t out_features,
                                int64_t in_features, const void* res, int64_t res_stride, void* out, int64_t out_stride,
                                int32_t tokens, int32_t dtype, void* stream) {
  GemvArgs a{};
  a.x = static_cast<const uint8_t*>(x); a.x_stride = x_stride;
  a.w = static_cast<const uint8_t*>(w); a.K = in_features; a.n_out = (int)out_features;
  a.res2 = static_cast<const uint8_t*>(res); a.res2_stride = res_stride;
  a.out = static_cast<uint8_t*>(out); a.out_stride = out_stride; a.M = tokens;
  if (int rc = check_common(a)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return res ? dispatch<PRO_NONE, EPI_RESID>(a, dtype, s) : dispatch<PRO_NONE, EPI_STORE>(a, dtype, s);
}
