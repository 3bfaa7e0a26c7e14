// common.cuh — small shared helpers: element types, 128-bit moves, host-side status.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string>

#include "../../include/bna_b200.h"

namespace bna {

// 2^x in one MUFU instruction (flush-to-zero, ~2 ulp); exp2(-inf) = 0.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max of three floats in one instruction (sm_100 three-input max.f32)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Two fp32 -> packed bf16x2 with round-to-nearest-even, on the integer ALU pipe (keeps the
// conversion work off the transcendental pipe that the softmax exponentials saturate).
// Inputs are finite.
__device__ __forceinline__ uint32_t pack_bf16x2_alu(float a, float b) {
  uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
  ua += 0x7FFFu + ((ua >> 16) & 1u);
  ub += 0x7FFFu + ((ub >> 16) & 1u);
  return __byte_perm(ua, ub, 0x7632);
}

template <typename T> struct ElemTraits;
template <> struct ElemTraits<__nv_bfloat16> {
  static constexpr uint32_t kUmmaFormat = 1;
  __device__ static __forceinline__ uint32_t pack2_fast(float a, float b) { return pack2(a, b); }
  __device__ static __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ static __forceinline__ float2 unpack2(uint32_t u) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&u);
    return __bfloat1622float2(h);
  }
  // element-wise product of two packed pairs, rounded once: the fp32 product of two 16-bit
  // values is exact, so this equals rounding the fp32 product
  __device__ static __forceinline__ uint32_t mul2(uint32_t a, uint32_t b) {
    __nv_bfloat162 r = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
  }
};
template <> struct ElemTraits<__half> {
  static constexpr uint32_t kUmmaFormat = 0;
  __device__ static __forceinline__ uint32_t pack2_fast(float a, float b) { return pack2(a, b); }
  __device__ static __forceinline__ uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ static __forceinline__ float2 unpack2(uint32_t u) {
    __half2 h = *reinterpret_cast<__half2*>(&u);
    return __half22float2(h);
  }
  __device__ static __forceinline__ uint32_t mul2(uint32_t a, uint32_t b) {
    __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
  }
};

// Round to the 16-bit storage type and back (what a torch op on bf16/fp16 tensors does to
// its fp32 result).
template <typename T>
__device__ __forceinline__ float round_to(float x) {
  const uint32_t p = ElemTraits<T>::pack2(x, 0.f);
  return ElemTraits<T>::unpack2(p).x;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One 128-dim head row held by a warp (lane l: dims 4l..4l+3): Qwen3.5 RMSNorm
// (x * rsqrt(mean(x^2) + eps) * (1 + w), fp32, rounded) followed by the rotary embedding in
// rotate-half form on the first 8 * half_lanes * 2 dims with cos/sin c/s (each product and
// the sum rounded to the storage type, as the eager bf16 ops).
template <typename T>
__device__ __forceinline__ void qk_row(float (&x)[4], const float (&w)[4], float eps, int lane, int half_lanes,
                                       const float (&c)[4], const float (&s)[4]) {
  const float ss = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
  const float r = rsqrtf(ss * (1.f / 128.f) + eps);
#pragma unroll
  for (int e = 0; e < 4; ++e) x[e] = round_to<T>((x[e] * r) * (1.f + w[e]));
  // rotate-half partner of dim d (d < rot): d + rot/2 for the first half, d - rot/2 after
  const bool in_rot = lane < 2 * half_lanes;
  const bool first = lane < half_lanes;
  const int src_lane = in_rot ? (first ? lane + half_lanes : lane - half_lanes) : lane;
  float p[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) p[e] = __shfl_sync(0xffffffffu, x[e], src_lane);
  if (in_rot) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float rh = first ? -p[e] : p[e];
      x[e] = round_to<T>(round_to<T>(x[e] * c[e]) + round_to<T>(rh * s[e]));
    }
  }
}

__device__ __forceinline__ uint4 ld_nc_128(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
// 1 / (1 + e^-x) from the fast exponential and the fast divide (two MUFU operations, no
// IEEE division sequence); callers round the result to 16 bits, where its few-ulp fp32
// error is invisible except at rounding ties.  Saturates to 0 below x ~ -87.
__device__ __forceinline__ float sigmoid_fast(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }
// silu(x) = x / (1 + e^-x) with the same two MUFU operations (callers round to 16 bits).
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.f + __expf(-x)); }

// Pull the 128-byte line holding p into L2 (no registers held while it is in flight).
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}
__device__ __forceinline__ uint4 ld_128(const void* p) {
  uint4 r;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ void st_128(void* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
// 256-bit global store (sm_100): one 32-byte chunk per lane halves the cache-line
// requests of row-per-lane stores compared with 16-byte stores.
__device__ __forceinline__ void st_256(void* p, const uint32_t* v) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v[0]), "r"(v[1]), "r"(v[2]),
               "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

// Fused q/k preparation of a decode step (see bna_decode_step_qk).
struct QKPrep {
  const void* q_weight;
  const void* k_weight;
  const void* cos;
  const void* sin;
  int64_t cs_b;
  int rot;
  float eps;
};

// Host-side error reporting (thread-local last error string).
void set_error(const std::string& msg);
int fail(int status, const std::string& msg);
int check_cuda(cudaError_t e, const char* what);

}  // namespace bna
