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
// call): each warp owns one output row (the gate/up pair for SWIGLU) and streams it with
// 128-bit loads, lane l taking
// columns [8(32c + l), +8) of chunk c.  All of a warp's weight loads are issued before
// griddepcontrol.wait, so under programmatic dependent launch the weight stream of a
// projection overlaps the tail of the kernel that produces its input; x_in is then built
// in shared memory by every CTA (it is a few KB) and the dot products are reduced across
// the warp with shuffles.
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
        for (int e = 0; e < 8; ++e) f[e] = f[e] * rnd<T>(1.f / (1.f + __expf(-g[e])));
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

// R rows per warp (the two rows of a SWIGLU pair when EPI == SWIGLU), NPRE chunks of 256
// columns preloaded per row before the dependency wait; further chunks are streamed.
template <typename T, int PRO, int EPI, int R, int NPRE>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(const GemvArgs a) {
  constexpr bool bf = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[kGemvWarps];
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows_per_warp = EPI == EPI_SWIGLU ? 1 : R;
  const int o0 = (blockIdx.x * kGemvWarps + warp) * rows_per_warp;  // first output of this warp
  const bool active = o0 < a.n_out;
  const int nch = (int)(a.K >> 8);
  int64_t row[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    int o = EPI == EPI_SWIGLU ? o0 : o0 + r;
    if (o >= a.n_out) o = a.n_out - 1;  // clamp: loads stay in bounds, results dropped
    row[r] = EPI == EPI_SWIGLU ? (int64_t)o + (r ? a.up_off : 0) : (int64_t)o;
  }
  uint4 wpre[R][NPRE];
  if (active) {
#pragma unroll
    for (int c = 0; c < NPRE; ++c)
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (c < nch) wpre[r][c] = ld_nc_128(a.w + 2 * (row[r] * a.K + (int64_t)(c * 32 + lane) * 8));
  }
  // the input is produced by the previous kernel of the stream
  asm volatile("griddepcontrol.wait;" ::: "memory");
  build_input<T, PRO>(a, smem, red);
  if (!active) return;
  float acc[R][kMaxM];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < kMaxM; ++m) acc[r][m] = 0.f;
  // acc[r][m] += W[row r, chunk c] . x_in[m, chunk c]
#define BNA_GEMV_CHUNK(WV, C)                                                                              \
  {                                                                                                        \
    float wf_[R][8];                                                                                       \
    _Pragma("unroll") for (int r = 0; r < R; ++r) unpack8f(WV[r], wf_[r], bf);                             \
    _Pragma("unroll") for (int m = 0; m < kMaxM; ++m) {                                                    \
      if (m < a.M) {                                                                                       \
        float xf_[8];                                                                                      \
        unpack8f(*reinterpret_cast<const uint4*>(smem + 2 * ((int64_t)m * a.K + ((C) * 32 + lane) * 8)), xf_, bf); \
        _Pragma("unroll") for (int r = 0; r < R; ++r)                                                      \
        _Pragma("unroll") for (int e = 0; e < 8; ++e) acc[r][m] = fmaf(wf_[r][e], xf_[e], acc[r][m]);      \
      }                                                                                                    \
    }                                                                                                      \
  }
#pragma unroll
  for (int c = 0; c < NPRE; ++c) {
    if (c < nch) {
      uint4 wv[R];
#pragma unroll
      for (int r = 0; r < R; ++r) wv[r] = wpre[r][c];
      BNA_GEMV_CHUNK(wv, c)
    }
  }
  for (int c0 = NPRE; c0 < nch; c0 += NPRE) {
    uint4 wb[R][NPRE];
#pragma unroll
    for (int c = 0; c < NPRE; ++c)
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (c0 + c < nch) wb[r][c] = ld_nc_128(a.w + 2 * (row[r] * a.K + (int64_t)((c0 + c) * 32 + lane) * 8));
#pragma unroll
    for (int c = 0; c < NPRE; ++c) {
      if (c0 + c < nch) {
        uint4 wv[R];
#pragma unroll
        for (int r = 0; r < R; ++r) wv[r] = wb[r][c];
        BNA_GEMV_CHUNK(wv, c0 + c)
      }
    }
  }
#undef BNA_GEMV_CHUNK
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < kMaxM; ++m)
      if (m < a.M) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[r][m] += __shfl_xor_sync(0xffffffffu, acc[r][m], o);
      }
  if (lane != 0) return;
  for (int m = 0; m < a.M; ++m) {
    if (EPI == EPI_SWIGLU) {
      const float g = rnd<T>(acc[0][m]), u = rnd<T>(acc[R - 1][m]);
      const float y = rnd<T>(g / (1.f + __expf(-g))) * u;
      *reinterpret_cast<uint16_t*>(a.out + 2 * ((int64_t)m * a.out_stride + o0)) =
          (uint16_t)(ElemTraits<T>::pack2(y, 0.f) & 0xFFFFu);
    } else {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int o = o0 + r;
        if (o >= a.n_out) break;
        float y = rnd<T>(acc[r][m]);
        if (EPI == EPI_RESID) {
          const uint16_t rb = *reinterpret_cast<const uint16_t*>(a.res2 + 2 * ((int64_t)m * a.res2_stride + o));
          y = y + ElemTraits<T>::unpack2((uint32_t)rb).x;
        }
        *reinterpret_cast<uint16_t*>(a.out + 2 * ((int64_t)m * a.out_stride + o)) =
            (uint16_t)(ElemTraits<T>::pack2(y, 0.f) & 0xFFFFu);
      }
    }
  }
}

// One output row per warp (the gate/up row pair for SWIGLU), so even the 1024-row
// projections spread over 128 CTAs; all of a row's chunks are preloaded when they fit.
template <typename T, int PRO, int EPI>
int launch_gemv(const GemvArgs& a, cudaStream_t s) {
  constexpr int R = EPI == EPI_SWIGLU ? 2 : 1;
  const int per_cta = kGemvWarps * (EPI == EPI_SWIGLU ? 1 : R);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((a.n_out + per_cta - 1) / per_cta));
  cfg.blockDim = dim3(kGemvWarps * 32);
  cfg.dynamicSmemBytes = (size_t)a.M * a.K * 2;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int nch = (int)(a.K >> 8);
  cudaError_t e;
  constexpr int kBig = R == 1 ? 16 : 8;
  auto kern = nch <= 4 ? gemv_kernel<T, PRO, EPI, R, 4>
                       : (nch <= 8 ? gemv_kernel<T, PRO, EPI, R, 8> : gemv_kernel<T, PRO, EPI, R, kBig>);
  if (cfg.dynamicSmemBytes > 48 * 1024) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cfg.dynamicSmemBytes);
    if (e != cudaSuccess) return check_cuda(e, "gemv smem attribute");
  }
  e = cudaLaunchKernelEx(&cfg, kern, a);
  return check_cuda(e, "gemv launch");
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
  if (a.K <= 0 || a.K % 256) return fail(BNA_UNSUPPORTED, "gemv: in_features must be a multiple of 256");
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
