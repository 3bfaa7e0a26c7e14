// gemm_sm100.cu — projections of the Qwen3.5 decoder layer on Blackwell tensor cores, with
// the elementwise step that follows each one applied in the epilogue.
//
// Epilogues of one persistent tcgen05 GEMM (out = h . W^T, fp32 accumulation):
//
//  * SwiGLU (the MLP's gate/up projection, transformers' Qwen3_5MLP
//    down_proj(act_fn(gate_proj(x)) * up_proj(x))):
//        act[m, j] = silu(h[m,:] . Wg[j,:]) * (h[m,:] . Wu[j,:])     Wg = W[0:I], Wu = W[I:2I]
//    A tile pairs 128 gate rows with the 128 matching up rows of W, so one accumulator row
//    holds both halves of 128 output columns; the [M, 2I] gate/up product never reaches HBM.
//    The gate and up products, silu(gate) and the product are each rounded to the 16-bit
//    type, as the eager ops (SiLU from the fast exponential and divide).
//
//  * q/k norm + RoPE (the attention's merged q/k/v projection; Qwen3_5Attention.forward and
//    bna/integrations/qwen_torch.py:535-573: q_norm / k_norm per head, then the rotary
//    embedding in rotate-half form on the first `rot` dims): the output columns come in
//    128-wide head groups [q0 gate0 q1 gate1 .. | k0 k1 .. | v0 v1 ..]; query and key groups
//    are RMS-normalised (x * rsqrt(mean(x^2) + eps) * (1 + w)) and rotated in the epilogue,
//    gate and value groups are stored as computed.  Rounding follows the eager ops: the
//    projection is rounded, the norm computes in fp32 and rounds, and each rotary product and
//    the sum are rounded.
//
// The third epilogue is the residual add of
// o_proj / down_proj (out = round(round(acc) + res), optionally writing per-row partial sums
// of squares for the next RMSNorm).  The SwiGLU and q/k/v forms can fold the RMSNorm before
// them in: the A operand is then the un-normalised residual, W carries (1 + norm weight) in
// its columns, and each accumulator row is scaled by rsqrt(mean(x^2) + eps) from those sums.
//
// Tiles (default form, CTA pairs, cta_group::2): a cluster of two CTAs computes 256 rows of h
// x 256 rows of W as one M = 256, N = 256 MMA per 16-wide k-step; CTA r stages h rows
// m0 + 128 r and the r-th 128-row W box (gate rows j0.. / up rows I + j0.. for SwiGLU, rows
// n0.. / n0 + 128.. otherwise) in a 6-stage ring of 32 KB stages, so each CTA's accumulator
// holds its 128 rows x all 256 columns (both halves of 128 SwiGLU outputs).  The single-CTA
// form (BNA_GEMM_CTA_PAIR=0, kept for comparison) stages 128 rows of h and both W boxes in a
// 4-stage ring of 48 KB stages.  K advances in 64-element (128-byte) blocks.  Persistent CTAs
// (one per SM) walk the tiles with the output column tile innermost, so the CTAs in flight
// share h rows through L2.
//
// Warp roles:
//   warp 0       TMA producer (one lane; in both CTAs of a pair, whose tiles all land on the
//                leader's barrier)
//   warp 1       TMEM allocator + MMA issuer (converged warp, one elected lane issues; in a
//                pair only the leader issues, for both CTAs); accumulators double-buffered in
//                TMEM columns [0, 256) and [256, 512)
//   warps 2..    epilogue, 16 warps (8 for q/k/v): warp w reads TMEM lane quarter w % 4 (32
//                rows) and its part of the columns; its stores overlap the next tile's MMAs
// In a pair, the leader's commits arrive on both CTAs' barriers and both CTAs' epilogue warps
// arrive on the leader's accumulator-empty barrier; a cluster barrier at the end keeps either
// CTA from leaving while the other's MMAs, commits or arrivals may still reach it.
// Every wait is bounded: a timeout sets the CTA abort flag and the device error word, the
// roles wind down, in-flight copies and MMAs are drained (again with bounded waits) and the
// TMEM is freed.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <map>
#include <mutex>
#include <string>
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace bna {

int* device_error_word();  // kernels.cu

namespace {

// Epilogue warps: 16 for SwiGLU and the residual add (a quarter of a row's outputs each:
// enough warps per SM sub-partition to hide the MUFU, TMEM and load latencies), 8 for q/k/v (one 128-column head
// group each; the norm + RoPE epilogue needs 119+ registers, which 576 threads cannot hold).
__host__ __device__ constexpr int epi_warps(int epi) { return epi == 1 ? 8 : 16; }
__host__ __device__ constexpr int gemm_threads(int epi) { return 64 + 32 * epi_warps(epi); }
constexpr int kStages = 4;
constexpr uint32_t kStageBytes = 3 * 16384;  // h tile, gate tile, up tile
constexpr uint32_t kBarOff = kStages * kStageBytes;
constexpr uint32_t kNormOff = kBarOff + 256;          // q / k norm weights (2 x 128 16-bit values)
constexpr uint32_t kGemmSmem = kNormOff + 512 + 1024;  // + 1024-byte alignment slack

enum { kEpiSwiglu = 0, kEpiQKNorm = 1, kEpiResid = 2 };

struct GemmArgs {
  int M, K;
  int tiles_n, total_tiles;
  int b2;        // W row offset of the second 128-row box of a tile (I for SwiGLU, 128 otherwise)
  int tile_w;    // W rows a tile advances by (128 for SwiGLU, 256 otherwise)
  uint8_t* out;
  int64_t ldo;   // elements
  int st256;     // output base and row stride allow 32-byte stores
  int* err;
  // q/k norm + RoPE epilogue
  int q_groups;  // head groups [0, q_groups) alternate query / gate
  int k_groups;  // then k_groups key groups; the rest are values
  const uint8_t* qn_w;
  const uint8_t* kn_w;
  const uint8_t* cs;  // cos / sin of row m at cs + 2 * m * rot (rot values each)
  const uint8_t* sn;
  int rot;
  float eps;
  // residual epilogue: out = round(acc + res), res [M, N] of row stride ldr (may be out)
  const uint8_t* res;
  int64_t ldr;
  // residual epilogue: per-row partial sums of squares of the (rounded) output, [M, ss_ld]
  // fp32 with column 4 * tn + part (a quarter of a 256-column tile each); null: none
  float* ss_out;
  int ss_ld;
  // SwiGLU / q/k/v: RMSNorm folded in.  The A operand is the un-normalised residual, W carries
  // the norm weight (1 + w) per column of K, and the accumulator of row m is scaled by
  // rsqrt(sum(rs[m, 0:rs_parts]) * rs_inv_n + rs_eps) before the epilogue; null: no scaling
  const float* rs;
  int rs_parts;
  int64_t rs_ld;
  float rs_inv_n, rs_eps;
};

__device__ __forceinline__ void unpack8v(const uint4& u, float* f, bool bf) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 t = bf ? ElemTraits<__nv_bfloat16>::unpack2(w[e]) : ElemTraits<__half>::unpack2(w[e]);
    f[2 * e] = t.x;
    f[2 * e + 1] = t.y;
  }
}

__device__ __forceinline__ void store32(uint8_t* p, const uint32_t* w, bool st256) {
  if (st256) {
    st_256(p, w);
  } else {
    st_128(p, make_uint4(w[0], w[1], w[2], w[3]));
    st_128(p + 16, make_uint4(w[4], w[5], w[6], w[7]));
  }
}

// Normalised value of one rounded projection element: round(x * r * (1 + w)).
template <typename T>
__device__ __forceinline__ float qk_norm1(float x, float r, float w) {
  return round_to<T>((round_to<T>(x) * r) * (1.f + w));
}

// Epilogue of one 128-column head group of the q/k/v projection for this thread's row:
// `kind` 0 stores the rounded products, 1 / 2 normalises them (query / key norm weights)
// and rotates the first `rot` dims.  TMEM is read 32 columns per wait; stores are 32 bytes
// per thread (one full sector of the row).
template <typename T>
__device__ __forceinline__ void qkv_group_epilogue(const GemmArgs& a, uint32_t tg, uint8_t* orow, bool store,
                                                   int kind, int64_t m, const uint8_t* norm_smem, float rsc) {
  using namespace sm100;
  constexpr bool bf = std::is_same<T, __nv_bfloat16>::value;
  const bool s256 = a.st256 != 0;
  if (kind == 0) {
#pragma unroll 1
    for (int c = 0; c < 128; c += 32) {
      float x[32];
      tmem_ld16(tg + (uint32_t)c, x);
      tmem_ld16(tg + (uint32_t)(c + 16), x + 16);
      tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 32; ++e) x[e] *= rsc;
      uint32_t w[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) w[e] = ElemTraits<T>::pack2(x[2 * e], x[2 * e + 1]);
      if (store) {
        store32(orow + 2 * c, w, s256);
        store32(orow + 2 * c + 32, w + 8, s256);
      }
    }
    return;
  }
  const uint8_t* wn = norm_smem + (kind == 1 ? 0 : 256);  // this kind's norm weights (shared memory)
  const uint8_t* csr = a.cs + 2 * m * a.rot;
  const uint8_t* snr = a.sn + 2 * m * a.rot;
  // the row's rotary tables come into L1 while pass 1 runs
  for (int off = 0; off < 2 * a.rot; off += 128) {
    asm volatile("prefetch.global.L1 [%0];" ::"l"(csr + off));
    asm volatile("prefetch.global.L1 [%0];" ::"l"(snr + off));
  }
  // pass 1: sum of squares of the rounded projection
  float ss = 0.f;
#pragma unroll 1
  for (int c = 0; c < 128; c += 32) {
    float x[32];
    tmem_ld16(tg + (uint32_t)c, x);
    tmem_ld16(tg + (uint32_t)(c + 16), x + 16);
    tmem_ld_wait();
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const float v = round_to<T>(x[e] * rsc);
      ss = fmaf(v, v, ss);
    }
  }
  const float r = rsqrtf(ss * (1.f / 128.f) + a.eps);
  const int hr = a.rot >> 1;
  // pass 2a: rotary dims, in pairs of 16-column chunks (d, d + rot/2)
#pragma unroll 1
  for (int c = 0; c < hr; c += 16) {
    float x1[16], x2[16];
    tmem_ld16(tg + (uint32_t)c, x1);
    tmem_ld16(tg + (uint32_t)(c + hr), x2);
    tmem_ld_wait();
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      x1[e] *= rsc;
      x2[e] *= rsc;
    }
    uint32_t o1[8], o2[8];
#pragma unroll
    for (int hb = 0; hb < 16; hb += 8) {
      float w1[8], w2[8], c1[8], c2[8], s1[8], s2[8];
      unpack8v(*reinterpret_cast<const uint4*>(wn + 2 * (c + hb)), w1, bf);
      unpack8v(*reinterpret_cast<const uint4*>(wn + 2 * (c + hr + hb)), w2, bf);
      unpack8v(ld_nc_128(csr + 2 * (c + hb)), c1, bf);
      unpack8v(ld_nc_128(csr + 2 * (c + hr + hb)), c2, bf);
      unpack8v(ld_nc_128(snr + 2 * (c + hb)), s1, bf);
      unpack8v(ld_nc_128(snr + 2 * (c + hr + hb)), s2, bf);
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        float y1[2], y2[2];
#pragma unroll
        for (int f = 0; f < 2; ++f) {
          const float n1 = qk_norm1<T>(x1[hb + e + f], r, w1[e + f]);
          const float n2 = qk_norm1<T>(x2[hb + e + f], r, w2[e + f]);
          y1[f] = round_to<T>(round_to<T>(n1 * c1[e + f]) + round_to<T>(-n2 * s1[e + f]));
          y2[f] = round_to<T>(round_to<T>(n2 * c2[e + f]) + round_to<T>(n1 * s2[e + f]));
        }
        o1[(hb + e) >> 1] = ElemTraits<T>::pack2(y1[0], y1[1]);
        o2[(hb + e) >> 1] = ElemTraits<T>::pack2(y2[0], y2[1]);
      }
    }
    if (store) {
      store32(orow + 2 * c, o1, s256);
      store32(orow + 2 * (c + hr), o2, s256);
    }
  }
  // pass 2b: the remaining dims, normalised only
#pragma unroll 1
  for (int c = a.rot; c < 128; c += 16) {
    float x[16];
    tmem_ld16(tg + (uint32_t)c, x);
    tmem_ld_wait();
#pragma unroll
    for (int e = 0; e < 16; ++e) x[e] *= rsc;
    uint32_t o[8];
#pragma unroll
    for (int hb = 0; hb < 16; hb += 8) {
      float w[8];
      unpack8v(*reinterpret_cast<const uint4*>(wn + 2 * (c + hb)), w, bf);
#pragma unroll
      for (int e = 0; e < 8; e += 2)
        o[(hb + e) >> 1] = ElemTraits<T>::pack2(qk_norm1<T>(x[hb + e], r, w[e]), qk_norm1<T>(x[hb + e + 1], r, w[e + 1]));
    }
    if (store) store32(orow + 2 * c, o, s256);
  }
}

// Epilogue of one accumulator tile for this thread's row m: `half` selects the columns this
// warp handles (SwiGLU: one of four 32-column parts of the 128 outputs; q/k/v: one of two
// 128-column head groups), tn the tile's 256-column block.
template <typename T, int EPI>
__device__ __forceinline__ void tile_epilogue(const GemmArgs& a, uint32_t tacc, int m, int tn, int half,
                                              const uint8_t* norm_smem, const uint4* rv, float rsc) {
  using namespace sm100;
  if constexpr (EPI == kEpiSwiglu) {
    // warp part `half` (0..3) of the row: output columns [32 half, 32 half + 32)
    uint8_t* orow = a.out + 2 * ((int64_t)m * a.ldo + tn * 128);
#pragma unroll 1
    for (int c = half * 32; c < half * 32 + 32; c += 16) {
      float g[16], u[16];
      tmem_ld16(tacc + (uint32_t)c, g);
      tmem_ld16(tacc + 128u + (uint32_t)c, u);
      tmem_ld_wait();
      uint32_t w[8];
#pragma unroll
      for (int e = 0; e < 16; e += 2) {
        // gate products rounded (as a pair), silu rounded, times the rounded up products
        const float2 gr = ElemTraits<T>::unpack2(ElemTraits<T>::pack2(g[e] * rsc, g[e + 1] * rsc));
        w[e >> 1] = ElemTraits<T>::mul2(ElemTraits<T>::pack2(silu_fast(gr.x), silu_fast(gr.y)),
                                        ElemTraits<T>::pack2(u[e] * rsc, u[e + 1] * rsc));
      }
      if (m < a.M) {
        if (a.st256) {
          st_256(orow + 2 * c, w);
        } else {
          st_128(orow + 2 * c, make_uint4(w[0], w[1], w[2], w[3]));
          st_128(orow + 2 * c + 16, make_uint4(w[4], w[5], w[6], w[7]));
        }
      }
    }
  } else if constexpr (EPI == kEpiResid) {
    // warp part `half` (0..3) of the row: columns [64 half, 64 half + 64) of the tile; rv
    // holds the residual of those columns, loaded before the accumulator wait by the thread
    // that writes the sums (so in place is allowed)
    uint8_t* orow = a.out + 2 * ((int64_t)m * a.ldo + (int64_t)tn * 256 + half * 64);
    float ss = 0.f;  // sum of squares of this thread's 64 outputs (the next norm's input)
#pragma unroll
    for (int c = 0; c < 64; c += 16) {
      float x[16];
      tmem_ld16(tacc + (uint32_t)(half * 64 + c), x);
      tmem_ld_wait();
      const uint4 r0 = rv[c >> 3], r1 = rv[(c >> 3) + 1];
      const uint32_t rw[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
      uint32_t w[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        // as the eager ops: the projection rounded, then the residual added and rounded
        const float2 p2 = ElemTraits<T>::unpack2(ElemTraits<T>::pack2(x[2 * e], x[2 * e + 1]));
        const float2 r2 = ElemTraits<T>::unpack2(rw[e]);
        w[e] = ElemTraits<T>::pack2(p2.x + r2.x, p2.y + r2.y);
        const float2 o2 = ElemTraits<T>::unpack2(w[e]);
        ss = fmaf(o2.x, o2.x, ss);
        ss = fmaf(o2.y, o2.y, ss);
      }
      if (m < a.M) {
        if (a.st256) {
          st_256(orow + 2 * c, w);
        } else {
          st_128(orow + 2 * c, make_uint4(w[0], w[1], w[2], w[3]));
          st_128(orow + 2 * c + 16, make_uint4(w[4], w[5], w[6], w[7]));
        }
      }
    }
    if (a.ss_out && m < a.M) a.ss_out[(int64_t)m * a.ss_ld + 4 * tn + half] = ss;
  } else {
    const int grp = tn * 2 + half;  // 128-column head group of this warp
    const int kind = grp < a.q_groups ? ((grp & 1) ? 0 : 1) : (grp < a.q_groups + a.k_groups ? 2 : 0);
    qkv_group_epilogue<T>(a, tacc + (uint32_t)half * 128u, a.out + 2 * ((int64_t)m * a.ldo + grp * 128), m < a.M,
                          kind, m < a.M ? m : 0, norm_smem, rsc);
  }
}

// Residual epilogue: this thread's 64 residual values of tile `tile` (row m), loaded before
// the accumulator wait so their latency overlaps it.
__device__ __forceinline__ void load_residual(const GemmArgs& a, int m, int tn, int half, uint4* rv) {
  if (m < a.M) {
    const uint8_t* rrow = a.res + 2 * ((int64_t)m * a.ldr + (int64_t)tn * 256 + half * 64);
#pragma unroll
    for (int i = 0; i < 8; ++i) rv[i] = ld_128(rrow + 16 * i);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) rv[i] = make_uint4(0, 0, 0, 0);
  }
}

// Folded RMSNorm: the row scale of row m from the partial sums of squares (1 without them).
__device__ __forceinline__ float row_scale(const GemmArgs& a, int m) {
  if (!a.rs || m >= a.M) return 1.f;
  const float* p = a.rs + (int64_t)m * a.rs_ld;
  float s = 0.f;
#pragma unroll 4
  for (int i = 0; i < a.rs_parts; i += 4) {
    const float4 v = *reinterpret_cast<const float4*>(p + i);
    s += (v.x + v.y) + (v.z + v.w);
  }
  return rsqrtf(s * a.rs_inv_n + a.rs_eps);
}

template <typename T, int EPI>
__global__ void __launch_bounds__(gemm_threads(EPI), 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                      const __grid_constant__ GemmArgs a) {
  using namespace sm100;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ uint8_t gsm_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* full = bars;                  // [kStages] stage loaded
  uint64_t* empty = bars + kStages;       // [kStages] stage consumed by the MMAs
  uint64_t* accfull = bars + 2 * kStages; // [2] accumulator buffer complete
  uint64_t* accempty = accfull + 2;       // [2] accumulator buffer read out (8 epilogue warps)
  uint64_t* drain = accempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(drain + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accfull[b], 1);
      mbar_init(&accempty[b], epi_warps(EPI));
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmW);
  }
  if (EPI == kEpiQKNorm && warp == 2) {  // the q and k norm weights, once per CTA
    const uint8_t* src = lane < 16 ? a.qn_w + 16 * lane : a.kn_w + 16 * (lane - 16);
    *reinterpret_cast<uint4*>(smem + kNormOff + 16 * lane) = ld_nc_128(src);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int KB = a.K >> 6;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      for (int tile = blockIdx.x; tile < a.total_tiles && !*abort_flag; tile += gridDim.x) {
        const int m0 = (tile / a.tiles_n) * 128, j0 = (tile % a.tiles_n) * a.tile_w;
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % kStages, use = it / kStages;
          if (use > 0 && !mbar_wait(&empty[s], (uint32_t)(use - 1) & 1u, abort_flag, 20, a.err)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + (uint32_t)s * kStageBytes;
          mbar_arrive_expect_tx(&full[s], kStageBytes);
          tma_load_4d(st, &tmA, &full[s], kb * 64, m0, 0, 0);
          tma_load_4d(st + 16384, &tmW, &full[s], kb * 64, j0, 0, 0);
          tma_load_4d(st + 32768, &tmW, &full[s], kb * 64, a.b2 + j0, 0, 0);
        }
        if (!ok) break;
      }
      // drain: the last loads of each stage have landed before the CTA may exit (they have
      // long since, unless a wait above gave up)
      volatile int never_abort = 0;
      for (int d = it - 1; d >= 0 && d >= it - kStages; --d)
        mbar_wait(&full[d % kStages], (uint32_t)(d / kStages) & 1u, &never_abort, 21, a.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t fmt = ElemTraits<T>::kUmmaFormat;
    const uint32_t idesc = idesc_f16(128, 256, fmt, false);
    auto wait_all = [&](uint64_t* bar, uint32_t parity, int site) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, site, a.err)) != 0;
    };
    int it = 0, tc = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < a.total_tiles && ok; tile += gridDim.x, ++tc) {
      const int buf = tc & 1, use = tc >> 1;
      if (use > 0 && !wait_all(&accempty[buf], (uint32_t)(use - 1) & 1u, 22)) break;
      tc_fence_after();
      const uint32_t dacc = tmem + (uint32_t)buf * 256u;
      for (int kb = 0; kb < KB; ++kb, ++it) {
        const int s = it % kStages;
        if (!wait_all(&full[s], (uint32_t)(it / kStages) & 1u, 23)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t st = smem_u32(smem + (uint32_t)s * kStageBytes);
        const uint64_t da = desc_sw128(st, 16, 1024), db = desc_sw128(st + 16384, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16_ss_warp(dacc, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), idesc, (kb | kk) != 0);
        mma_commit_warp(&empty[s]);
      }
      if (ok) mma_commit_warp(&accfull[buf]);
    }
    volatile int never_abort = 0;
    mma_commit_warp(drain);
    if (lane == 0) mbar_wait(drain, 0, &never_abort, 24, a.err);
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3, half = (warp - 2) >> 2;  // TMEM lane quarter; column part
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    int tc = 0;
    for (int tile = blockIdx.x; tile < a.total_tiles; tile += gridDim.x, ++tc) {
      const int buf = tc & 1;
      const int m = (tile / a.tiles_n) * 128 + row, tn = tile % a.tiles_n;
      uint4 rv[EPI == kEpiResid ? 8 : 1];
      if constexpr (EPI == kEpiResid) load_residual(a, m, tn, half, rv);
      const float rsc = EPI == kEpiResid ? 1.f : row_scale(a, m);
      if (!mbar_wait(&accfull[buf], (uint32_t)(tc >> 1) & 1u, abort_flag, 25, a.err)) break;
      tc_fence_after();
      tile_epilogue<T, EPI>(a, tmem + lane_off + (uint32_t)buf * 256u, m, tn, half, smem + kNormOff, rv, rsc);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------- CTA-pair form
// The same GEMM on CTA pairs (clusters of 2, tcgen05 cta_group::2): a pair computes a
// 256-row x 256-column tile as one M = 256, N = 256 MMA per 16-wide k-step.  CTA r holds
// h rows m0 + 128 r and the r-th 128-row W box (gate / up rows for SwiGLU), so per k-block a
// CTA stages 32 KB instead of 48 KB: each W byte is read from shared memory once per 256
// output rows instead of once per 128.  Both CTAs' tiles land on the leader's (rank 0)
// `full` barrier; the leader's MMA warp issues for the pair and its commits arrive on the
// `empty` / `accfull` barriers of both CTAs; both CTAs' epilogue warps arrive on the
// leader's `accempty`.  Each CTA's epilogue reads its own 128 accumulator rows (all 256
// columns), exactly as in the single-CTA form.
constexpr int kPairStages = 6;
constexpr uint32_t kPairStageBytes = 2 * 16384;  // h tile, one W box
constexpr uint32_t kPairBarOff = kPairStages * kPairStageBytes;
constexpr uint32_t kPairNormOff = kPairBarOff + 256;
constexpr uint32_t kPairSmem = kPairNormOff + 512 + 1024;

template <typename T, int EPI>
__global__ void __launch_bounds__(gemm_threads(EPI), 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ GemmArgs a) {
  using namespace sm100;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ uint8_t gsm_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPairBarOff);
  uint64_t* full = bars;                       // [kPairStages] both CTAs' tiles landed (leader's copy used)
  uint64_t* empty = bars + kPairStages;        // [kPairStages] stage consumed (both CTAs)
  uint64_t* accfull = bars + 2 * kPairStages;  // [2] accumulator buffer complete (both CTAs)
  uint64_t* accempty = accfull + 2;            // [2] buffer read out by 16 epilogue warps (leader's copy)
  uint64_t* drain = accempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(drain + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = (int)(blockIdx.x >> 1), npairs = (int)(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accfull[b], 1);
      mbar_init(&accempty[b], 2 * epi_warps(EPI));
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmW);
  }
  if (EPI == kEpiQKNorm && warp == 2) {
    const uint8_t* src = lane < 16 ? a.qn_w + 16 * lane : a.kn_w + 16 * (lane - 16);
    *reinterpret_cast<uint4*>(smem + kPairNormOff + 16 * lane) = ld_nc_128(src);
  }
  tc_fence_before();
  // both CTAs' barriers are initialised before either CTA signals the other's
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int KB = a.K >> 6;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producers (both CTAs)
    if (lane == 0) {
      const uint32_t full0 = mapa_shared(smem_u32(full), 0);  // leader's full[0]
      int it = 0;
      for (int tile = pair; tile < a.total_tiles && !*abort_flag; tile += npairs) {
        const int m0 = (tile / a.tiles_n) * 256 + (int)rank * 128;
        const int w0 = (rank ? a.b2 : 0) + (tile % a.tiles_n) * a.tile_w;
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % kPairStages, use = it / kPairStages;
          if (use > 0 && !mbar_wait(&empty[s], (uint32_t)(use - 1) & 1u, abort_flag, 30, a.err)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + (uint32_t)s * kPairStageBytes;
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * kPairStageBytes);
          const uint32_t fb = full0 + (uint32_t)s * 8u;
          tma_load_4d_pair(st, &tmA, fb, kb * 64, m0, 0, 0);
          tma_load_4d_pair(st + 16384, &tmW, fb, kb * 64, w0, 0, 0);
        }
        if (!ok) break;
      }
      // the leader drains the last loads of each stage (its barrier counts both CTAs' bytes)
      if (leader) {
        volatile int never_abort = 0;
        for (int d = it - 1; d >= 0 && d >= it - kPairStages; --d)
          mbar_wait(&full[d % kPairStages], (uint32_t)(d / kPairStages) & 1u, &never_abort, 31, a.err);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (leader only)
    if (leader) {
      constexpr uint32_t fmt = ElemTraits<T>::kUmmaFormat;
      const uint32_t idesc = idesc_f16(256, 256, fmt, false);
      auto wait_all = [&](uint64_t* bar, uint32_t parity, int site) -> bool {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, site, a.err)) != 0;
      };
      int it = 0, tc = 0;
      bool ok = true;
      for (int tile = pair; tile < a.total_tiles && ok; tile += npairs, ++tc) {
        const int buf = tc & 1, use = tc >> 1;
        if (use > 0 && !wait_all(&accempty[buf], (uint32_t)(use - 1) & 1u, 32)) break;
        tc_fence_after();
        const uint32_t dacc = tmem + (uint32_t)buf * 256u;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % kPairStages;
          if (!wait_all(&full[s], (uint32_t)(it / kPairStages) & 1u, 33)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(smem + (uint32_t)s * kPairStageBytes);
          const uint64_t da = desc_sw128(st, 16, 1024), db = desc_sw128(st + 16384, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16_ss_pair_warp(dacc, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), idesc, (kb | kk) != 0);
          mma_commit_pair_both_warp(&empty[s]);
        }
        if (ok) mma_commit_pair_both_warp(&accfull[buf]);
      }
      volatile int never_abort = 0;
      mma_commit_pair_local_warp(drain);
      if (lane == 0) mbar_wait(drain, 0, &never_abort, 34, a.err);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3, half = (warp - 2) >> 2;  // TMEM lane quarter; column part
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint32_t accempty0 = mapa_shared(smem_u32(accempty), 0);
    int tc = 0;
    for (int tile = pair; tile < a.total_tiles; tile += npairs, ++tc) {
      const int buf = tc & 1;
      const int m = (tile / a.tiles_n) * 256 + (int)rank * 128 + row, tn = tile % a.tiles_n;
      uint4 rv[EPI == kEpiResid ? 8 : 1];
      if constexpr (EPI == kEpiResid) load_residual(a, m, tn, half, rv);
      const float rsc = EPI == kEpiResid ? 1.f : row_scale(a, m);
      if (!mbar_wait(&accfull[buf], (uint32_t)(tc >> 1) & 1u, abort_flag, 35, a.err)) break;
      tc_fence_after();
      tile_epilogue<T, EPI>(a, tmem + lane_off + (uint32_t)buf * 256u, m, tn, half, smem + kPairNormOff, rv, rsc);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(accempty0 + (uint32_t)buf * 8u);
    }
  }
  tc_fence_before();
  __syncthreads();
  // neither CTA leaves (or frees its TMEM) while the pair's MMAs, commits or remote arrivals
  // may still reach it
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult qr;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  }
  return fn;
}

// Row-major [rows, K] matrix (row stride ld elements) as a tensor map with 128-row x 64-column
// boxes, 128-byte swizzle (the K-major operand layout of the MMA descriptors).
int encode_rows(CUtensorMap* m, const void* base, int64_t rows, int K, int64_t ld, CUtensorMapDataType dt,
                const char* name) {
  EncodeFn enc = encode_fn();
  if (!enc) return fail(BNA_CUDA_ERROR, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[4] = {(cuuint64_t)K, (cuuint64_t)rows, 1, 1};
  cuuint64_t strides[3] = {(cuuint64_t)ld * 2, 16, 16};
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = enc(m, dt, 4, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(BNA_BAD_STRIDE, std::string(name) + ": cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return BNA_OK;
}

int sm_count(int dev) {
  static std::mutex mu;
  static std::map<int, int> cache;
  std::lock_guard<std::mutex> g(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  cache[dev] = n;
  return n;
}

}  // namespace
}  // namespace bna

using namespace bna;

namespace bna {
namespace {

// CTA-pair tiles unless BNA_GEMM_CTA_PAIR=0 (the single-CTA form, kept for comparison).
bool use_cta_pairs() {
  static const bool on = [] {
    const char* e = std::getenv("BNA_GEMM_CTA_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}

int launch_gemm(int epi, const CUtensorMap& ma, const CUtensorMap& mw, GemmArgs& a, int dtype, void* stream) {
  a.err = device_error_word();
  int dev = 0;
  cudaGetDevice(&dev);
  const int nsm = sm_count(dev);
  const bool pair = use_cta_pairs() && nsm >= 2;
  int grid;
  if (pair) {
    // a pair tile covers 256 rows; two CTAs per tile, an even grid of at most nsm CTAs
    a.total_tiles = (int)(((int64_t)a.M + 255) / 256) * a.tiles_n;
    grid = 2 * (a.total_tiles < nsm / 2 ? a.total_tiles : nsm / 2);
  } else {
    a.total_tiles = (int)(((int64_t)a.M + 127) / 128) * a.tiles_n;
    grid = a.total_tiles < nsm ? a.total_tiles : nsm;
  }
  const int smem_bytes = pair ? (int)kPairSmem : (int)kGemmSmem;
  auto launch = [&](auto kern) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, bool> done;
    {
      std::lock_guard<std::mutex> g(mu);
      bool& d = done[{reinterpret_cast<const void*>(kern), dev}];
      if (!d) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
        if (pair) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
        d = true;
      }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(gemm_threads(epi));
    cfg.dynamicSmemBytes = smem_bytes;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = 2;
    at[1].val.clusterDim.y = 1;
    at[1].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = pair ? 2 : 1;
    cudaLaunchKernelEx(&cfg, kern, ma, mw, a);
  };
  const bool bf = dtype == BNA_BF16;
  if (pair) {
    if (epi == kEpiSwiglu) bf ? launch(gemm_pair_kernel<__nv_bfloat16, kEpiSwiglu>) : launch(gemm_pair_kernel<__half, kEpiSwiglu>);
    else if (epi == kEpiQKNorm) bf ? launch(gemm_pair_kernel<__nv_bfloat16, kEpiQKNorm>) : launch(gemm_pair_kernel<__half, kEpiQKNorm>);
    else bf ? launch(gemm_pair_kernel<__nv_bfloat16, kEpiResid>) : launch(gemm_pair_kernel<__half, kEpiResid>);
  } else {
    if (epi == kEpiSwiglu) bf ? launch(gemm_sm100_kernel<__nv_bfloat16, kEpiSwiglu>) : launch(gemm_sm100_kernel<__half, kEpiSwiglu>);
    else if (epi == kEpiQKNorm) bf ? launch(gemm_sm100_kernel<__nv_bfloat16, kEpiQKNorm>) : launch(gemm_sm100_kernel<__half, kEpiQKNorm>);
    else bf ? launch(gemm_sm100_kernel<__nv_bfloat16, kEpiResid>) : launch(gemm_sm100_kernel<__half, kEpiResid>);
  }
  return check_cuda(cudaGetLastError(), pair ? "gemm_sm100 (CTA pairs) launch" : "gemm_sm100 launch");
}

int check_gemm_common(const void* h, int64_t ldh, const void* w, int64_t ldw, const void* out, int64_t ldo, int64_t M,
                      int32_t K, int32_t dtype, const char* name) {
  const std::string n(name);
  if (dtype != BNA_BF16 && dtype != BNA_F16) return fail(BNA_BAD_DTYPE, n + ": bfloat16 or float16 only");
  if (M < 0 || K <= 0) return fail(BNA_BAD_SHAPE, n + ": bad sizes");
  if (M > 0 && (!h || !w || !out)) return fail(BNA_BAD_SHAPE, n + ": null pointer");
  if (K % 64) return fail(BNA_UNSUPPORTED, n + ": K must be a multiple of 64");
  if (ldh < K || ldw < K) return fail(BNA_BAD_STRIDE, n + ": row strides below the row length");
  if (ldh % 8 || ldw % 8 || ldo % 8) return fail(BNA_BAD_STRIDE, n + ": row strides must be multiples of 8 elements");
  if ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(BNA_BAD_STRIDE, n + ": pointers must be 16-byte aligned");
  if (M >= ((int64_t)1 << 31) - 128) return fail(BNA_UNSUPPORTED, n + ": too many rows");
  return BNA_OK;
}

// Folded-RMSNorm arguments of the SwiGLU and q/k/v GEMMs (row_ss null: none).
int set_row_scale(GemmArgs& a, const float* row_ss, int64_t ld, int32_t parts, float eps, int K, const char* name) {
  if (!row_ss) return BNA_OK;
  const std::string n(name);
  if (parts <= 0 || parts % 4 || ld < parts || ld % 4 || (reinterpret_cast<uintptr_t>(row_ss) & 15))
    return fail(BNA_BAD_STRIDE, n + ": row sums of squares need a positive multiple of 4 parts, a row stride of 4 floats and 16-byte alignment");
  a.rs = row_ss;
  a.rs_ld = ld;
  a.rs_parts = parts;
  a.rs_inv_n = 1.f / (float)K;
  a.rs_eps = eps;
  return BNA_OK;
}

}  // namespace
}  // namespace bna

extern "C" BNA_API int bna_gemm_swiglu(const void* h, int64_t ldh, const void* w, int64_t ldw, void* out, int64_t ldo,
                                       int64_t M, int32_t K, int32_t inter, const float* row_ss, int64_t row_ss_ld,
                                       int32_t row_ss_parts, float norm_eps, int32_t dtype, void* stream) {
  if (int rc = check_gemm_common(h, ldh, w, ldw, out, ldo, M, K, dtype, "gemm_swiglu")) return rc;
  if (inter <= 0 || inter % 128) return fail(BNA_UNSUPPORTED, "gemm_swiglu: inter must be a positive multiple of 128");
  if (ldo < inter) return fail(BNA_BAD_STRIDE, "gemm_swiglu: output row stride below inter");
  {
    GemmArgs probe{};
    if (int rc = set_row_scale(probe, row_ss, row_ss_ld, row_ss_parts, norm_eps, K, "gemm_swiglu")) return rc;
  }
  if (M == 0) return BNA_OK;
  const CUtensorMapDataType dt = dtype == BNA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ma, mw;
  if (int rc = encode_rows(&ma, h, M, K, ldh, dt, "h")) return rc;
  if (int rc = encode_rows(&mw, w, 2 * (int64_t)inter, K, ldw, dt, "w")) return rc;
  GemmArgs a{};
  a.M = (int)M;
  a.K = K;
  a.tiles_n = inter / 128;
  a.total_tiles = (int)(((M + 127) / 128) * a.tiles_n);
  a.b2 = inter;
  a.tile_w = 128;
  a.out = static_cast<uint8_t*>(out);
  a.ldo = ldo;
  if (int rc = set_row_scale(a, row_ss, row_ss_ld, row_ss_parts, norm_eps, K, "gemm_swiglu")) return rc;
  a.st256 = ((reinterpret_cast<uintptr_t>(out) & 31) == 0 && (ldo * 2) % 32 == 0) ? 1 : 0;
  return launch_gemm(kEpiSwiglu, ma, mw, a, dtype, stream);
}

extern "C" BNA_API int bna_gemm_qkv_norm_rope(const void* h, int64_t ldh, const void* w, int64_t ldw, void* out,
                                              int64_t ldo, int64_t M, int32_t K, int32_t N, int32_t num_q_heads,
                                              int32_t num_kv_heads, const void* q_norm_w, const void* k_norm_w,
                                              const void* cos, const void* sin, int32_t rot, float eps,
                                              const float* row_ss, int64_t row_ss_ld, int32_t row_ss_parts,
                                              float norm_eps, int32_t dtype, void* stream) {
  if (int rc = check_gemm_common(h, ldh, w, ldw, out, ldo, M, K, dtype, "gemm_qkv_norm_rope")) return rc;
  if (N <= 0 || N % 256) return fail(BNA_UNSUPPORTED, "gemm_qkv_norm_rope: N must be a positive multiple of 256");
  if (ldo < N) return fail(BNA_BAD_STRIDE, "gemm_qkv_norm_rope: output row stride below N");
  if (num_q_heads <= 0 || num_kv_heads <= 0 || (2 * num_q_heads + 2 * num_kv_heads) * 128 != N)
    return fail(BNA_BAD_SHAPE, "gemm_qkv_norm_rope: N must be (2 * q heads + 2 * kv heads) * 128");
  if (rot < 0 || rot > 128 || rot % 32) return fail(BNA_UNSUPPORTED, "gemm_qkv_norm_rope: rot must be a multiple of 32 up to 128");
  if (M > 0 && (!q_norm_w || !k_norm_w || (rot > 0 && (!cos || !sin))))
    return fail(BNA_BAD_SHAPE, "gemm_qkv_norm_rope: null norm weights or rotary tables");
  if ((reinterpret_cast<uintptr_t>(q_norm_w) | reinterpret_cast<uintptr_t>(k_norm_w) | reinterpret_cast<uintptr_t>(cos) |
       reinterpret_cast<uintptr_t>(sin)) & 15)
    return fail(BNA_BAD_STRIDE, "gemm_qkv_norm_rope: norm weights and rotary tables must be 16-byte aligned");
  {
    GemmArgs probe{};
    if (int rc = set_row_scale(probe, row_ss, row_ss_ld, row_ss_parts, norm_eps, K, "gemm_qkv_norm_rope")) return rc;
  }
  if (M == 0) return BNA_OK;
  const CUtensorMapDataType dt = dtype == BNA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ma, mw;
  if (int rc = encode_rows(&ma, h, M, K, ldh, dt, "h")) return rc;
  if (int rc = encode_rows(&mw, w, N, K, ldw, dt, "w")) return rc;
  GemmArgs a{};
  a.M = (int)M;
  a.K = K;
  a.tiles_n = N / 256;
  a.total_tiles = (int)(((M + 127) / 128) * a.tiles_n);
  a.b2 = 128;
  a.tile_w = 256;
  a.out = static_cast<uint8_t*>(out);
  a.ldo = ldo;
  a.q_groups = 2 * num_q_heads;
  a.k_groups = num_kv_heads;
  a.qn_w = static_cast<const uint8_t*>(q_norm_w);
  a.kn_w = static_cast<const uint8_t*>(k_norm_w);
  a.cs = static_cast<const uint8_t*>(cos);
  a.sn = static_cast<const uint8_t*>(sin);
  a.rot = rot;
  a.eps = eps;
  if (int rc = set_row_scale(a, row_ss, row_ss_ld, row_ss_parts, norm_eps, K, "gemm_qkv_norm_rope")) return rc;
  a.st256 = ((reinterpret_cast<uintptr_t>(out) & 31) == 0 && (ldo * 2) % 32 == 0) ? 1 : 0;
  return launch_gemm(kEpiQKNorm, ma, mw, a, dtype, stream);
}

extern "C" BNA_API int bna_gemm_residual(const void* h, int64_t ldh, const void* w, int64_t ldw, const void* res,
                                         int64_t ldr, void* out, int64_t ldo, int64_t M, int32_t K, int32_t N,
                                         float* ss_out, int64_t ss_ld, int32_t dtype, void* stream) {
  if (int rc = check_gemm_common(h, ldh, w, ldw, out, ldo, M, K, dtype, "gemm_residual")) return rc;
  if (N <= 0 || N % 256) return fail(BNA_UNSUPPORTED, "gemm_residual: N must be a positive multiple of 256");
  if (ldo < N || ldr < N) return fail(BNA_BAD_STRIDE, "gemm_residual: output / residual row stride below N");
  if (M > 0 && !res) return fail(BNA_BAD_SHAPE, "gemm_residual: null residual");
  if (ldr % 8 || (reinterpret_cast<uintptr_t>(res) & 15)) return fail(BNA_BAD_STRIDE, "gemm_residual: residual must be 16-byte aligned with a row stride of 8 elements");
  if (res != out || ldr != ldo) {
    // the residual is read by the thread that writes the same element; any other overlap races
    const uintptr_t r0 = reinterpret_cast<uintptr_t>(res), o0 = reinterpret_cast<uintptr_t>(out);
    const uintptr_t r1 = r0 + 2 * (uintptr_t)((M - 1) * ldr + N), o1 = o0 + 2 * (uintptr_t)((M - 1) * ldo + N);
    if (M > 0 && r0 < o1 && o0 < r1) return fail(BNA_BAD_SHAPE, "gemm_residual: residual overlaps the output other than in place");
  }
  if (ss_out && (ss_ld < 4 * (N / 256) || ss_ld % 4 || (reinterpret_cast<uintptr_t>(ss_out) & 15)))
    return fail(BNA_BAD_STRIDE, "gemm_residual: ss_out needs a row stride of at least 4 * N / 256 floats, a multiple of 4, 16-byte aligned");
  if (M == 0) return BNA_OK;
  const CUtensorMapDataType dt = dtype == BNA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ma, mw;
  if (int rc = encode_rows(&ma, h, M, K, ldh, dt, "h")) return rc;
  if (int rc = encode_rows(&mw, w, N, K, ldw, dt, "w")) return rc;
  GemmArgs a{};
  a.M = (int)M;
  a.K = K;
  a.tiles_n = N / 256;
  a.b2 = 128;
  a.tile_w = 256;
  a.out = static_cast<uint8_t*>(out);
  a.ldo = ldo;
  a.res = static_cast<const uint8_t*>(res);
  a.ldr = ldr;
  a.ss_out = ss_out;
  a.ss_ld = (int)ss_ld;
  a.st256 = ((reinterpret_cast<uintptr_t>(out) & 31) == 0 && (ldo * 2) % 32 == 0) ? 1 : 0;
  return launch_gemm(kEpiResid, ma, mw, a, dtype, stream);
}
