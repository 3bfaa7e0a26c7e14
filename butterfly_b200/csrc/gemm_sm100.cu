// gemm_sm100.cu — the Qwen3.5 MLP's gate/up projection with SwiGLU in the epilogue, on
// Blackwell tensor cores.
//
//   act[m, j] = silu(h[m,:] . Wg[j,:]) * (h[m,:] . Wu[j,:])       Wg = W[0:I], Wu = W[I:2I]
//
// It replaces the merged gate/up GEMM followed by the SwiGLU kernel of the fused decoder
// layer (transformers' Qwen3_5MLP: down_proj(act_fn(gate_proj(x)) * up_proj(x))): the
// [M, 2I] gate/up product never reaches HBM.  Rounding follows the eager ops: the gate and
// up products are rounded to the 16-bit type, silu(gate) is rounded, and so is the product.
//
// Tiles: 128 rows of h x (128 gate rows + the 128 matching up rows of W), so one
// M = 128, N = 256 accumulator holds both halves of 128 output columns.  K advances in
// 64-element (128-byte) blocks: per block TMA loads a 16 KB h tile and two 16 KB W tiles
// (gate rows j0.., up rows I + j0..) into one 4-stage ring; placed back to back, the two W
// tiles form the 256-row K-major B operand.  Persistent CTAs (one per SM) walk the tiles
// with the output column tile innermost, so the CTAs in flight share h rows through L2.
//
// Warp roles (320 threads):
//   warp 0       TMA producer (one lane)
//   warp 1       TMEM allocator + MMA issuer (converged warp, one elected lane issues);
//                accumulators double-buffered in TMEM columns [0, 256) and [256, 512)
//   warps 2..9   epilogue: warp w reads TMEM lane quarter w % 4 (32 rows) and one half of
//                the 128 output columns; its stores overlap the next tile's MMAs
// Every wait is bounded: a timeout sets the CTA abort flag and the device error word, the
// roles wind down, in-flight copies and MMAs are drained (again with bounded waits) and the
// TMEM is freed.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <map>
#include <mutex>
#include <string>
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace bna {

int* device_error_word();  // kernels.cu

namespace {

constexpr int kGemmThreads = 320;
constexpr int kStages = 4;
constexpr uint32_t kStageBytes = 3 * 16384;  // h tile, gate tile, up tile
constexpr uint32_t kBarOff = kStages * kStageBytes;
constexpr uint32_t kGemmSmem = kBarOff + 256 + 1024;  // + barriers, + 1024-byte alignment slack

struct SwigluGemmArgs {
  int M, K, I;
  int tiles_n, total_tiles;
  uint8_t* out;
  int64_t ldo;  // elements
  int st256;    // output base and row stride allow 32-byte stores
  int* err;
};

template <typename T>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_swiglu_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                       const __grid_constant__ SwigluGemmArgs a) {
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
      mbar_init(&accempty[b], 8);
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
        const int m0 = (tile / a.tiles_n) * 128, j0 = (tile % a.tiles_n) * 128;
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
          tma_load_4d(st + 32768, &tmW, &full[s], kb * 64, a.I + j0, 0, 0);
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
    const int q = warp & 3, half = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    int tc = 0;
    for (int tile = blockIdx.x; tile < a.total_tiles; tile += gridDim.x, ++tc) {
      const int buf = tc & 1;
      if (!mbar_wait(&accfull[buf], (uint32_t)(tc >> 1) & 1u, abort_flag, 25, a.err)) break;
      tc_fence_after();
      const int m = (tile / a.tiles_n) * 128 + row, j0 = (tile % a.tiles_n) * 128;
      const uint32_t tacc = tmem + lane_off + (uint32_t)buf * 256u;
      uint8_t* orow = a.out + 2 * ((int64_t)m * a.ldo + j0);
#pragma unroll 1
      for (int c = half * 64; c < half * 64 + 64; c += 16) {
        float g[16], u[16];
        tmem_ld16(tacc + (uint32_t)c, g);
        tmem_ld16(tacc + 128u + (uint32_t)c, u);
        tmem_ld_wait();
        uint32_t w[8];
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const float g0 = round_to<T>(g[e]), g1 = round_to<T>(g[e + 1]);
          const float s0 = round_to<T>(g0 / (1.f + __expf(-g0))), s1 = round_to<T>(g1 / (1.f + __expf(-g1)));
          w[e >> 1] = ElemTraits<T>::mul2(ElemTraits<T>::pack2(s0, s1),
                                          ElemTraits<T>::pack2(u[e], u[e + 1]));
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

extern "C" BNA_API int bna_gemm_swiglu(const void* h, int64_t ldh, const void* w, int64_t ldw, void* out, int64_t ldo,
                                       int64_t M, int32_t K, int32_t inter, int32_t dtype, void* stream) {
  if (dtype != BNA_BF16 && dtype != BNA_F16) return fail(BNA_BAD_DTYPE, "gemm_swiglu: bfloat16 or float16 only");
  if (M < 0 || K <= 0 || inter <= 0) return fail(BNA_BAD_SHAPE, "gemm_swiglu: bad sizes");
  if (M == 0) return BNA_OK;
  if (!h || !w || !out) return fail(BNA_BAD_SHAPE, "gemm_swiglu: null pointer");
  if (K % 64 || inter % 128) return fail(BNA_UNSUPPORTED, "gemm_swiglu: K must be a multiple of 64, inter of 128");
  if (ldh < K || ldw < K || ldo < inter) return fail(BNA_BAD_STRIDE, "gemm_swiglu: row strides below the row length");
  if (ldh % 8 || ldw % 8 || ldo % 8) return fail(BNA_BAD_STRIDE, "gemm_swiglu: row strides must be multiples of 8 elements");
  if ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(BNA_BAD_STRIDE, "gemm_swiglu: pointers must be 16-byte aligned");
  if (M >= ((int64_t)1 << 31) - 128) return fail(BNA_UNSUPPORTED, "gemm_swiglu: too many rows");
  const CUtensorMapDataType dt = dtype == BNA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ma, mw;
  if (int rc = encode_rows(&ma, h, M, K, ldh, dt, "h")) return rc;
  if (int rc = encode_rows(&mw, w, 2 * (int64_t)inter, K, ldw, dt, "w")) return rc;
  SwigluGemmArgs a{};
  a.M = (int)M;
  a.K = K;
  a.I = inter;
  a.tiles_n = inter / 128;
  const int64_t tiles = ((M + 127) / 128) * a.tiles_n;
  if (tiles >= ((int64_t)1 << 31)) return fail(BNA_UNSUPPORTED, "gemm_swiglu: too many tiles");
  a.total_tiles = (int)tiles;
  a.out = static_cast<uint8_t*>(out);
  a.ldo = ldo;
  a.st256 = ((reinterpret_cast<uintptr_t>(out) & 31) == 0 && (ldo * 2) % 32 == 0) ? 1 : 0;
  a.err = device_error_word();
  int dev = 0;
  cudaGetDevice(&dev);
  const int nsm = sm_count(dev);
  const int grid = a.total_tiles < nsm ? a.total_tiles : nsm;
  auto launch = [&](auto kern) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, bool> done;
    {
      std::lock_guard<std::mutex> g(mu);
      bool& d = done[{reinterpret_cast<const void*>(kern), dev}];
      if (!d) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem);
        d = true;
      }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = kGemmSmem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, ma, mw, a);
  };
  if (dtype == BNA_BF16) launch(gemm_swiglu_kernel<__nv_bfloat16>);
  else launch(gemm_swiglu_kernel<__half>);
  return check_cuda(cudaGetLastError(), "gemm_swiglu launch");
}
