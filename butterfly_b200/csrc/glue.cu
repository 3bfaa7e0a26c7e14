// glue.cu — the decoder-layer steps on either side of the compressed attention path,
// fused into single HBM-bound kernels.  Each one replaces a chain of eager elementwise
// ops of the Qwen3.5 decoder layer that the reference runs around its attention
// (bna/integrations/qwen_torch.py:535-573 before the attention, :1585-1591 after it; the
// norms and MLP of transformers' Qwen3_5DecoderLayer around them):
//   * rmsnorm:       [residual add +] Qwen3.5 RMSNorm  y = x * rsqrt(mean(x^2) + eps) * (1 + w)
//   * qk_norm_rope:  per-head q/k RMSNorm + partial rotary embedding (rotate-half form)
//   * gate_mul:      attention output * sigmoid(gate)
//   * swiglu:        silu(gate) * up
// Arithmetic follows the eager ops step by step: fp32 inside a norm, and after every
// elementwise op of the 16-bit storage type the value is rounded to that type, as torch
// does when it runs those ops one at a time on bf16 tensors.
#include <cuda_runtime.h>

#include <string>
#include <type_traits>

#include "common.cuh"

namespace bna {
namespace {

constexpr int kWarps = 8;  // warps per CTA of the row kernels

__device__ __forceinline__ void unpack8(const uint4& u, float* f, bool bf) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 t = bf ? ElemTraits<__nv_bfloat16>::unpack2(w[e]) : ElemTraits<__half>::unpack2(w[e]);
    f[2 * e] = t.x;
    f[2 * e + 1] = t.y;
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float* f) {
  return make_uint4(ElemTraits<T>::pack2(f[0], f[1]), ElemTraits<T>::pack2(f[2], f[3]),
                    ElemTraits<T>::pack2(f[4], f[5]), ElemTraits<T>::pack2(f[6], f[7]));
}

// ------------------------------------------------------------------------------ RMSNorm
// One warp per row; lane l holds chunks l, l+32, ... of 8 elements (NC chunks per lane).
struct NormArgs {
  const uint8_t* x;
  int64_t xs;
  const uint8_t* res;
  int64_t rs;
  const uint8_t* w;
  uint8_t* out;
  int64_t os;
  uint8_t* sum;
  int64_t ss;
  int64_t rows;
  int hidden;
  float eps;
};

template <typename T, int NC>
__global__ void __launch_bounds__(kWarps * 32) rmsnorm_kernel(const NormArgs a) {
  constexpr bool bf = std::is_same<T, __nv_bfloat16>::value;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  float v[NC * 8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * 8;
    unpack8(ld_nc_128(a.x + 2 * (row * a.xs + col)), v + c * 8, bf);
    if (a.res) {
      float r[8];
      unpack8(ld_nc_128(a.res + 2 * (row * a.rs + col)), r, bf);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[c * 8 + e] = round_to<T>(v[c * 8 + e] + r[e]);
      if (a.sum) st_128(a.sum + 2 * (row * a.ss + col), pack8<T>(v + c * 8));
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += v[c * 8 + e] * v[c * 8 + e];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)a.hidden + a.eps);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * 8;
    float w[8];
    unpack8(ld_nc_128(a.w + 2 * col), w, bf);
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = (v[c * 8 + e] * r) * (1.f + w[e]);
    st_128(a.out + 2 * (row * a.os + col), pack8<T>(y));
  }
}

// ------------------------------------------------------------------------------ q/k prep
// One warp per (token, head) row of head_dim 128: lane l holds dims 4l..4l+3 (8 bytes).
struct QKArgs {
  const uint8_t* q;
  int64_t q_tok, q_head;
  const uint8_t* k;
  int64_t k_tok, k_head;
  const uint8_t* qw;
  const uint8_t* kw;
  const uint8_t* cos;
  const uint8_t* sin;
  int64_t cs_tok;
  int rot;
  uint8_t* q_out;
  uint8_t* k_out;
  const uint8_t* v;   // optional pass-through of V rows into v_out (same layout as k_out)
  int64_t v_tok, v_head;
  uint8_t* v_out;
  int64_t tokens;
  int Hq, Hkv;
  float eps;
};

__device__ __forceinline__ void unpack4(const uint2& u, float (&f)[4], bool bf) {
  const float2 a = bf ? ElemTraits<__nv_bfloat16>::unpack2(u.x) : ElemTraits<__half>::unpack2(u.x);
  const float2 b = bf ? ElemTraits<__nv_bfloat16>::unpack2(u.y) : ElemTraits<__half>::unpack2(u.y);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}

// One 128-dim head row held by a half-warp (lane l of the half: dims 8l..8l+7): the
// Qwen3.5 RMSNorm and the rotate-half rotary embedding on the first 16 * half_lanes dims,
// with the same arithmetic as qk_row (the 16-lane reductions only differ in order).
template <typename T>
__device__ __forceinline__ void qk_row16(float (&x)[8], const float (&w)[8], float eps, int hl, int half_lanes,
                                         const float (&c)[8], const float (&s)[8]) {
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) ss += x[e] * x[e];
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss * (1.f / 128.f) + eps);
#pragma unroll
  for (int e = 0; e < 8; ++e) x[e] = round_to<T>((x[e] * r) * (1.f + w[e]));
  const bool in_rot = hl < 2 * half_lanes;
  const bool first = hl < half_lanes;
  const int lane = threadIdx.x & 31;
  const int src = in_rot ? (first ? lane + half_lanes : lane - half_lanes) : lane;
  float p[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) p[e] = __shfl_sync(0xffffffffu, x[e], src);
  if (in_rot) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float rh = first ? -p[e] : p[e];
      x[e] = round_to<T>(round_to<T>(x[e] * c[e]) + round_to<T>(rh * s[e]));
    }
  }
}

// One warp per token: its head rows two at a time (one per half-warp, 16-byte loads), all
// of the token's loads issued before any arithmetic.  Needs rot % 16 == 0.
template <typename T, int HQ, int HKV>
__global__ void __launch_bounds__(kWarps * 32) qk_norm_rope_kernel(const QKArgs a) {
  constexpr bool bf = std::is_same<T, __nv_bfloat16>::value;
  constexpr int NH = HQ + HKV;
  constexpr int NP = (NH + 1) / 2;  // row pairs
  const int lane = threadIdx.x & 31, half = lane >> 4, hl = lane & 15;
  const int64_t t = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (t >= a.tokens) return;
  uint4 raw[NP];
#pragma unroll
  for (int pr = 0; pr < NP; ++pr) {
    int h = 2 * pr + half;
    if (h >= NH) h = NH - 1;  // odd row count: the second half repeats the last row (not stored)
    const uint8_t* src = h < HQ ? a.q + 2 * (t * a.q_tok + (int64_t)h * a.q_head)
                                : a.k + 2 * (t * a.k_tok + (int64_t)(h - HQ) * a.k_head);
    raw[pr] = *reinterpret_cast<const uint4*>(src + 16 * hl);
  }
  const int half_lanes = a.rot >> 4;
  float c[8], sn[8], wq[8], wk[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) { c[e] = 1.f; sn[e] = 0.f; wk[e] = 0.f; }
  if (hl < 2 * half_lanes) {
    unpack8(*reinterpret_cast<const uint4*>(a.cos + 2 * (t * a.cs_tok) + 16 * hl), c, bf);
    unpack8(*reinterpret_cast<const uint4*>(a.sin + 2 * (t * a.cs_tok) + 16 * hl), sn, bf);
  }
  unpack8(*reinterpret_cast<const uint4*>(a.qw + 16 * hl), wq, bf);
  if (HKV) unpack8(*reinterpret_cast<const uint4*>(a.kw + 16 * hl), wk, bf);
#pragma unroll
  for (int pr = 0; pr < NP; ++pr) {
    const int h = 2 * pr + half;
    float x[8];
    unpack8(raw[pr], x, bf);
    qk_row16<T>(x, (h < HQ) ? wq : wk, a.eps, hl, half_lanes, c, sn);
    if (h < NH) {
      uint8_t* dst = h < HQ ? a.q_out + 2 * ((t * HQ + h) * 128) : a.k_out + 2 * ((t * HKV + (h - HQ)) * 128);
      *reinterpret_cast<uint4*>(dst + 16 * hl) = pack8<T>(x);
    }
  }
  if (a.v_out) {
#pragma unroll
    for (int pr = 0; pr < (HKV + 1) / 2; ++pr) {
      const int h = 2 * pr + half;
      if (h < HKV)
        *reinterpret_cast<uint4*>(a.v_out + 2 * ((t * HKV + h) * 128) + 16 * hl) =
            *reinterpret_cast<const uint4*>(a.v + 2 * (t * a.v_tok + (int64_t)h * a.v_head) + 16 * hl);
    }
  }
}

// Few tokens (decode): one warp per (token, head) row instead, so the rows of one token are
// normalised in parallel rather than one after another.
template <typename T, int HQ, int HKV>
__global__ void __launch_bounds__(kWarps * 32) qk_norm_rope_row_kernel(const QKArgs a) {
  constexpr bool bf = std::is_same<T, __nv_bfloat16>::value;
  const int lane = threadIdx.x & 31;
  const int item = blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int NH = HQ + HKV + (a.v_out ? HKV : 0);
  if (item >= (int)a.tokens * NH) return;
  const int t = item / NH, h = item - t * NH;
  if (h >= HQ + HKV) {  // V pass-through row
    const int hv = h - HQ - HKV;
    *reinterpret_cast<uint2*>(a.v_out + 2 * (((int64_t)t * HKV + hv) * 128) + 8 * lane) =
        *reinterpret_cast<const uint2*>(a.v + 2 * ((int64_t)t * a.v_tok + (int64_t)hv * a.v_head) + 8 * lane);
    return;
  }
  const bool isq = h < HQ;
  const uint8_t* src = isq ? a.q + 2 * ((int64_t)t * a.q_tok + (int64_t)h * a.q_head)
                           : a.k + 2 * ((int64_t)t * a.k_tok + (int64_t)(h - HQ) * a.k_head);
  float x[4], w[4];
  unpack4(*reinterpret_cast<const uint2*>(src + 8 * lane), x, bf);
  unpack4(*reinterpret_cast<const uint2*>((isq ? a.qw : a.kw) + 8 * lane), w, bf);
  const int half_lanes = a.rot >> 3;
  float c[4] = {1.f, 1.f, 1.f, 1.f}, sn[4] = {0.f, 0.f, 0.f, 0.f};
  if (lane < 2 * half_lanes) {
    unpack4(*reinterpret_cast<const uint2*>(a.cos + 2 * ((int64_t)t * a.cs_tok) + 8 * lane), c, bf);
    unpack4(*reinterpret_cast<const uint2*>(a.sin + 2 * ((int64_t)t * a.cs_tok) + 8 * lane), sn, bf);
  }
  qk_row<T>(x, w, a.eps, lane, half_lanes, c, sn);
  uint8_t* dst = isq ? a.q_out + 2 * (((int64_t)t * HQ + h) * 128) : a.k_out + 2 * (((int64_t)t * HKV + (h - HQ)) * 128);
  *reinterpret_cast<uint2*>(dst + 8 * lane) = make_uint2(ElemTraits<T>::pack2(x[0], x[1]), ElemTraits<T>::pack2(x[2], x[3]));
}

// ------------------------------------------------------------------------------ gate, swiglu
struct GateArgs {
  const uint8_t* o;  // [tokens, heads, dh] contiguous
  const uint8_t* g;  // token stride g_tok, head stride g_head
  int64_t g_tok, g_head;
  uint8_t* out;      // [tokens, heads * dh] contiguous
  int64_t tokens;
  int heads, dh;
};

// Thread = one 8-element vector of one token row; the grid covers all vectors once
// (32-bit index arithmetic: tokens * heads * dh / 8 < 2^31 is checked on the host).
template <typename T>
__global__ void __launch_bounds__(256) gate_mul_kernel(const GateArgs a) {
  constexpr bool bf = std::is_same<T, __nv_bfloat16>::value;
  const int per_head = a.dh >> 3;
  const int per_row = a.heads * per_head;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int)a.tokens * per_row) return;
  const int t = i / per_row;
  const int j = i - t * per_row;
  const int h = j / per_head, c = j - h * per_head;
  float o[8], g[8];
  unpack8(ld_nc_128(a.o + 16 * (int64_t)i), o, bf);
  unpack8(ld_nc_128(a.g + 2 * ((int64_t)t * a.g_tok + (int64_t)h * a.g_head + c * 8)), g, bf);
  float y[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) y[e] = o[e] * round_to<T>(sigmoid_fast(g[e]));
  st_128(a.out + 16 * (int64_t)i, pack8<T>(y));
}

struct SwigluArgs {
  const uint8_t* gu;  // row r: gate at gu + r * stride, up at + up_off
  int64_t stride, up_off;
  uint8_t* out;       // [rows, inter] contiguous
  int64_t rows;
  int inter;
};

template <typename T>
__global__ void __launch_bounds__(256) swiglu_kernel(const SwigluArgs a) {
  constexpr bool bf = std::is_same<T, __nv_bfloat16>::value;
  const int per_row = a.inter >> 3;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int)a.rows * per_row) return;
  const int r = i / per_row;
  const int c = i - r * per_row;
  const uint8_t* base = a.gu + 2 * ((int64_t)r * a.stride + c * 8);
  float g[8], u[8];
  unpack8(ld_nc_128(base), g, bf);
  unpack8(ld_nc_128(base + 2 * a.up_off), u, bf);
  float y[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) y[e] = round_to<T>(silu_fast(g[e])) * u[e];
  st_128(a.out + 16 * (int64_t)i, pack8<T>(y));
}

unsigned flat_grid(int64_t n) { return (unsigned)((n + 255) / 256); }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <typename T>
int launch_rmsnorm(const NormArgs& a, cudaStream_t s) {
  const dim3 grid((unsigned)((a.rows + kWarps - 1) / kWarps)), block(kWarps * 32);
  switch (a.hidden / 256) {
    case 1: rmsnorm_kernel<T, 1><<<grid, block, 0, s>>>(a); break;
    case 2: rmsnorm_kernel<T, 2><<<grid, block, 0, s>>>(a); break;
    case 4: rmsnorm_kernel<T, 4><<<grid, block, 0, s>>>(a); break;
    case 8: rmsnorm_kernel<T, 8><<<grid, block, 0, s>>>(a); break;
    case 10: rmsnorm_kernel<T, 10><<<grid, block, 0, s>>>(a); break;
    case 12: rmsnorm_kernel<T, 12><<<grid, block, 0, s>>>(a); break;
    case 16: rmsnorm_kernel<T, 16><<<grid, block, 0, s>>>(a); break;
    default: return fail(BNA_UNSUPPORTED, "rmsnorm: hidden must be 256 x {1,2,4,8,10,12,16}");
  }
  return check_cuda(cudaGetLastError(), "rmsnorm launch");
}

// Sum of squares of each row (fp32), one warp per row: the statistics of an RMSNorm that a
// following GEMM applies as a row scale (bna_gemm_swiglu / bna_gemm_qkv_norm_rope row_ss).
template <typename T>
__global__ void __launch_bounds__(256) row_sumsq_kernel(const uint8_t* x, int64_t xs, float* out, int64_t ld,
                                                        int64_t rows, int H) {
  constexpr bool bf = std::is_same<T, __nv_bfloat16>::value;
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const uint8_t* row = x + 2 * r * xs;
  float ss = 0.f;
  for (int c = lane * 8; c < H; c += 256) {
    float f[8];
    unpack8(ld_nc_128(row + 2 * c), f, bf);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) *reinterpret_cast<float4*>(out + r * ld) = make_float4(ss, 0.f, 0.f, 0.f);
}

}  // namespace
}  // namespace bna

using namespace bna;

extern "C" BNA_API int bna_row_sumsq(const void* x, int64_t x_stride, float* out, int64_t ld_out, int64_t rows,
                                     int32_t H, int32_t dtype, void* stream) {
  if (rows < 0 || H <= 0 || H % 8) return fail(BNA_BAD_SHAPE, "row_sumsq: rows >= 0 and H a positive multiple of 8");
  if (rows == 0) return BNA_OK;
  if (!x || !out) return fail(BNA_BAD_SHAPE, "row_sumsq: null pointer");
  if (dtype != BNA_BF16 && dtype != BNA_F16) return fail(BNA_BAD_DTYPE, "row_sumsq: bfloat16 or float16 only");
  if (x_stride % 8 || ld_out < 4 || ld_out % 4 || !aligned16(x) || !aligned16(out))
    return fail(BNA_BAD_STRIDE, "row_sumsq: 16-byte aligned rows (stride a multiple of 8 elements), ld_out a multiple of 4 floats");
  const dim3 grid((unsigned)((rows + 7) / 8)), block(256);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* xp = static_cast<const uint8_t*>(x);
  if (dtype == BNA_BF16) row_sumsq_kernel<__nv_bfloat16><<<grid, block, 0, s>>>(xp, x_stride, out, ld_out, rows, H);
  else row_sumsq_kernel<__half><<<grid, block, 0, s>>>(xp, x_stride, out, ld_out, rows, H);
  return check_cuda(cudaGetLastError(), "row_sumsq launch");
}

extern "C" BNA_API int bna_rmsnorm(const void* x, int64_t x_stride, const void* res, int64_t res_stride,
                                   const void* weight, void* out, int64_t out_stride, void* sum_out,
                                   int64_t sum_stride, int64_t rows, int32_t hidden, float eps, int32_t dtype,
                                   void* stream) {
  if (rows < 0) return fail(BNA_BAD_SHAPE, "rmsnorm: rows must be >= 0");
  if (rows == 0) return BNA_OK;
  if (!x || !weight || !out) return fail(BNA_BAD_SHAPE, "rmsnorm: null pointer");
  if (hidden <= 0 || hidden % 256) return fail(BNA_UNSUPPORTED, "rmsnorm: hidden must be a multiple of 256");
  for (int64_t st : {x_stride, out_stride, res ? res_stride : (int64_t)8, sum_out ? sum_stride : (int64_t)8})
    if (st % 8) return fail(BNA_BAD_STRIDE, "rmsnorm: row strides must be multiples of 8 elements");
  for (const void* p : {x, weight, (const void*)out, res, (const void*)sum_out})
    if (p && !aligned16(p)) return fail(BNA_BAD_STRIDE, "rmsnorm: pointers must be 16-byte aligned");
  if (sum_out && !res) return fail(BNA_BAD_SHAPE, "rmsnorm: sum_out needs a residual input");
  NormArgs a{static_cast<const uint8_t*>(x), x_stride, static_cast<const uint8_t*>(res), res_stride,
             static_cast<const uint8_t*>(weight), static_cast<uint8_t*>(out), out_stride,
             static_cast<uint8_t*>(sum_out), sum_stride, rows, hidden, eps};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == BNA_BF16) return launch_rmsnorm<__nv_bfloat16>(a, s);
  if (dtype == BNA_F16) return launch_rmsnorm<__half>(a, s);
  return fail(BNA_BAD_DTYPE, "rmsnorm: bfloat16 or float16 only");
}

extern "C" BNA_API int bna_qk_norm_rope(const void* q, int64_t q_tok_stride, int64_t q_head_stride, const void* k,
                                        int64_t k_tok_stride, int64_t k_head_stride, const void* q_weight,
                                        const void* k_weight, const void* cos, const void* sin,
                                        int64_t cs_tok_stride, int32_t rot, void* q_out, void* k_out,
                                        const void* v, int64_t v_tok_stride, int64_t v_head_stride, void* v_out,
                                        int64_t tokens, int32_t hq, int32_t hkv, int32_t head_dim, float eps,
                                        int32_t dtype, void* stream) {
  if ((v == nullptr) != (v_out == nullptr)) return fail(BNA_BAD_SHAPE, "qk_norm_rope: v and v_out go together");
  if (v && (v_tok_stride % 4 || v_head_stride % 4 || (reinterpret_cast<uintptr_t>(v) & 7) ||
            (reinterpret_cast<uintptr_t>(v_out) & 7)))
    return fail(BNA_BAD_STRIDE, "qk_norm_rope: v strides must be multiples of 4 elements, pointers 8-byte aligned");
  if (tokens < 0 || hq <= 0 || hkv < 0) return fail(BNA_BAD_SHAPE, "qk_norm_rope: bad sizes");
  if (tokens == 0) return BNA_OK;
  if (head_dim != 128) return fail(BNA_UNSUPPORTED, "qk_norm_rope: head_dim must be 128");
  if (rot < 0 || rot > head_dim || rot % 8) return fail(BNA_UNSUPPORTED, "qk_norm_rope: rotary dims must be a multiple of 8 <= head_dim");
  if (!q || !q_weight || !q_out || (hkv && (!k || !k_weight || !k_out)) || (rot && (!cos || !sin)))
    return fail(BNA_BAD_SHAPE, "qk_norm_rope: null pointer");
  for (int64_t st : {q_tok_stride, q_head_stride, k_tok_stride, k_head_stride, rot ? cs_tok_stride : (int64_t)4})
    if (st % 4) return fail(BNA_BAD_STRIDE, "qk_norm_rope: strides must be multiples of 4 elements");
  for (const void* p : {q, k, q_weight, k_weight, cos, sin, (const void*)q_out, (const void*)k_out})
    if (p && (reinterpret_cast<uintptr_t>(p) & 7)) return fail(BNA_BAD_STRIDE, "qk_norm_rope: pointers must be 8-byte aligned");
  QKArgs a{static_cast<const uint8_t*>(q), q_tok_stride, q_head_stride, static_cast<const uint8_t*>(k), k_tok_stride,
           k_head_stride, static_cast<const uint8_t*>(q_weight), static_cast<const uint8_t*>(k_weight),
           static_cast<const uint8_t*>(cos), static_cast<const uint8_t*>(sin), cs_tok_stride, rot,
           static_cast<uint8_t*>(q_out), static_cast<uint8_t*>(k_out), static_cast<const uint8_t*>(v), v_tok_stride,
           v_head_stride, static_cast<uint8_t*>(v_out), tokens, hq, hkv, eps};
  const dim3 grid((unsigned)((tokens + kWarps - 1) / kWarps)), block(kWarps * 32);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype != BNA_BF16 && dtype != BNA_F16) return fail(BNA_BAD_DTYPE, "qk_norm_rope: bfloat16 or float16 only");
  const bool bf = dtype == BNA_BF16;
  bool wide_ok = rot % 16 == 0 && q_tok_stride % 8 == 0 && q_head_stride % 8 == 0 && k_tok_stride % 8 == 0 &&
                 k_head_stride % 8 == 0 && cs_tok_stride % 8 == 0 && (!v || (v_tok_stride % 8 == 0 && v_head_stride % 8 == 0));
  for (const void* p : {q, k, q_weight, k_weight, cos, sin, v, (const void*)q_out, (const void*)k_out, (const void*)v_out})
    if (p && (reinterpret_cast<uintptr_t>(p) & 15)) wide_ok = false;
  const bool per_row = tokens <= 64 || !wide_ok;
  const dim3 grid_rows((unsigned)((tokens * (hq + hkv + (v_out ? hkv : 0)) + kWarps - 1) / kWarps));
#define BNA_QK_CASE(HQ_, HKV_)                                                                      \
  if (hq == HQ_ && hkv == HKV_) {                                                                    \
    if (per_row) {                                                                                   \
      if (bf) qk_norm_rope_row_kernel<__nv_bfloat16, HQ_, HKV_><<<grid_rows, block, 0, s>>>(a);     \
      else qk_norm_rope_row_kernel<__half, HQ_, HKV_><<<grid_rows, block, 0, s>>>(a);               \
    } else {                                                                                         \
      if (bf) qk_norm_rope_kernel<__nv_bfloat16, HQ_, HKV_><<<grid, block, 0, s>>>(a);              \
      else qk_norm_rope_kernel<__half, HQ_, HKV_><<<grid, block, 0, s>>>(a);                        \
    }                                                                                                \
    return check_cuda(cudaGetLastError(), "qk_norm_rope launch");                                    \
  }
  BNA_QK_CASE(8, 2) BNA_QK_CASE(16, 4) BNA_QK_CASE(8, 1) BNA_QK_CASE(8, 8) BNA_QK_CASE(4, 2) BNA_QK_CASE(16, 2)
  BNA_QK_CASE(32, 8) BNA_QK_CASE(16, 8) BNA_QK_CASE(32, 4) BNA_QK_CASE(24, 4) BNA_QK_CASE(4, 1) BNA_QK_CASE(2, 1)
#undef BNA_QK_CASE
  return fail(BNA_UNSUPPORTED, "qk_norm_rope: unsupported (q heads, kv heads) pair");
}

extern "C" BNA_API int bna_gate_sigmoid_mul(const void* o, const void* gate, int64_t gate_tok_stride,
                                            int64_t gate_head_stride, void* out, int64_t tokens, int32_t heads,
                                            int32_t head_dim, int32_t dtype, void* stream) {
  if (tokens < 0 || heads <= 0 || head_dim <= 0 || head_dim % 8) return fail(BNA_BAD_SHAPE, "gate_sigmoid_mul: bad sizes");
  if (tokens == 0) return BNA_OK;
  if (!o || !gate || !out) return fail(BNA_BAD_SHAPE, "gate_sigmoid_mul: null pointer");
  if (gate_tok_stride % 8 || gate_head_stride % 8) return fail(BNA_BAD_STRIDE, "gate_sigmoid_mul: gate strides must be multiples of 8");
  if (!aligned16(o) || !aligned16(gate) || !aligned16(out)) return fail(BNA_BAD_STRIDE, "gate_sigmoid_mul: pointers must be 16-byte aligned");
  GateArgs a{static_cast<const uint8_t*>(o), static_cast<const uint8_t*>(gate), gate_tok_stride, gate_head_stride,
             static_cast<uint8_t*>(out), tokens, heads, head_dim};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (tokens * heads * (int64_t)head_dim / 8 >= (int64_t)1 << 31) return fail(BNA_UNSUPPORTED, "gate_sigmoid_mul: too many elements");
  const unsigned grid = flat_grid(tokens * heads * head_dim / 8);
  if (dtype == BNA_BF16) gate_mul_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(a);
  else if (dtype == BNA_F16) gate_mul_kernel<__half><<<grid, 256, 0, s>>>(a);
  else return fail(BNA_BAD_DTYPE, "gate_sigmoid_mul: bfloat16 or float16 only");
  return check_cuda(cudaGetLastError(), "gate_sigmoid_mul launch");
}

extern "C" BNA_API int bna_swiglu(const void* gate_up, int64_t row_stride, int64_t up_offset, void* out, int64_t rows,
                                  int32_t inter, int32_t dtype, void* stream) {
  if (rows < 0 || inter <= 0 || inter % 8) return fail(BNA_BAD_SHAPE, "swiglu: bad sizes");
  if (rows == 0) return BNA_OK;
  if (!gate_up || !out) return fail(BNA_BAD_SHAPE, "swiglu: null pointer");
  if (row_stride % 8 || up_offset % 8) return fail(BNA_BAD_STRIDE, "swiglu: strides must be multiples of 8");
  if (!aligned16(gate_up) || !aligned16(out)) return fail(BNA_BAD_STRIDE, "swiglu: pointers must be 16-byte aligned");
  SwigluArgs a{static_cast<const uint8_t*>(gate_up), row_stride, up_offset, static_cast<uint8_t*>(out), rows, inter};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows * (int64_t)inter / 8 >= (int64_t)1 << 31) return fail(BNA_UNSUPPORTED, "swiglu: too many elements");
  const unsigned grid = flat_grid(rows * inter / 8);
  if (dtype == BNA_BF16) swiglu_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(a);
  else if (dtype == BNA_F16) swiglu_kernel<__half><<<grid, 256, 0, s>>>(a);
  else return fail(BNA_BAD_DTYPE, "swiglu: bfloat16 or float16 only");
  return check_cuda(cudaGetLastError(), "swiglu launch");
}
