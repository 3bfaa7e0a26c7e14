// prefill_sm100.cu — compressed Butterfly prefill attention on Blackwell tensor cores.
//
// Semantics (bna/torch/attention_wayfinder_permute.py:1046-1122): every query at
// position q attends, with one softmax over the union, to the raw keys
// [max(0, q-W+1), q] and to the cursor-packed routed block summaries of its block
// (partner / sink / far-local blocks that end before the block's raw-window start).
// GQA: the G = Hq/Hkv query heads of a KV head share its keys.
//
// Work unit = (batch b, KV head, query tile of QT = 128/G positions).  Its 128 MMA rows
// are the G heads x QT positions (M = 128).  The keys of the tile are one contiguous
// slice of NR = round_up(W - 1 + QT, 16) raw positions starting at q0 - (W - 1), plus
// a 16-row tile holding the block's routed summaries (zero rows where unused):
//   S  = Q . [K_slice ; K_sum]^T   two tcgen05.mma chains into one TMEM tile (N = NR, 16)
//   P  = masked softmax(S) (exp2, fp32 row sums), stored bf16/f16 to smem (SW128 K-major)
//   O  = P . [V_slice ; V_sum]      tcgen05.mma with V as an MN-major operand
// Loads: Q, K, V by TMA (128-byte swizzle, zero fill outside the tensor) into a
// 2-stage ring; summaries by the producer warp with 128-bit loads.
//
// Warp roles (192 threads, one CTA per SM, persistent over units):
//   warp 0      producer: TMA issue + summary rows
//   warp 1      TMEM allocator + single-thread MMA issuer
//   warps 2..5  softmax + epilogue (thread = TMEM lane = MMA row)
// TMEM: S double buffer at columns [0,128) and [128,256), O at [256,384).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "route.cuh"
#include "sm100.cuh"

namespace bna {

struct PrefillArgs {
  int B, Hq, Hkv, G, Tq;
  int QT, NR, ntiles, total_units, stages;
  int q_tmajor;  // Q tile rows ordered (position, head) instead of (head, position)
  int64_t q_pos0, kv_pos0, total_len;
  int window;
  float scale_log2;
  bna_route route;
  const void* ksum;
  const void* vsum;
  int64_t ks_b, ks_h, ks_n, vs_b, vs_h, vs_n;
  void* out;
  int64_t os_b, os_h, os_t;
  float* lse;
  int64_t ls_b, ls_h;
  int* err;  // device error word
};

struct PrefillSmem {
  uint32_t q, kv_half, k, v, ks, vs, stage, p, p_bytes, bars, total;
  __host__ __device__ PrefillSmem(int NR, int stages) {
    q = 0;                        // 2 halves x 128 rows x 128 B
    kv_half = (uint32_t)NR * 128;  // one 64-column half of a K or V slice
    k = 32768;
    v = k + 2 * kv_half;
    ks = v + 2 * kv_half;          // 2 halves x 16 rows x 128 B
    vs = ks + 4096;
    stage = vs + 4096;
    p = stage * stages;
    p_bytes = ((NR + 16 + 63) / 64) * 16384;
    bars = p + p_bytes;
    total = bars + 256 + 1024;  // + alignment slack
  }
};

namespace {

constexpr float kLn2 = 0.6931471805599453f;

template <typename T>
__global__ void __launch_bounds__(192, 1)
    prefill_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const PrefillArgs a) {
  using namespace sm100;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const PrefillSmem L(a.NR, a.stages);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* full = bars;        // [2] TMA + summaries landed
  uint64_t* empty = bars + 2;   // [2] stage consumed by PV
  uint64_t* sfull = bars + 4;   // [2] S tile ready in TMEM
  uint64_t* pfull = bars + 6;   // P written to smem (128 arrivals)
  uint64_t* ofull = bars + 7;   // O ready in TMEM
  uint64_t* drain = bars + 8;   // MMA drain at exit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 10);

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&full[s], 2);
      mbar_init(&empty[s], 1);
      mbar_init(&sfull[s], 1);
    }
    mbar_init(pfull, 128);
    mbar_init(ofull, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int NR = a.NR, QT = a.QT, G = a.G, S = a.stages;
  const int BS = a.route.block_size;
  auto stage_ptr = [&](int s) { return smem + (uint32_t)s * L.stage; };

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    int i = 0;
    for (int u = blockIdx.x; u < a.total_units; u += gridDim.x, ++i) {
      const int s = i % S;
      const uint32_t ph = (uint32_t)(i / S) & 1u;
      if (i >= S && !mbar_wait(&empty[s], ph ^ 1u, abort_flag, 1, a.err)) break;
      const int t = u % a.ntiles, rest = u / a.ntiles, kvh = rest % a.Hkv, b = rest / a.Hkv;
      const int qs = t * QT;
      const int64_t qg = a.q_pos0 + qs;
      const int kidx = (int)(qg - (a.window - 1) - a.kv_pos0);
      uint8_t* st = stage_ptr(s);
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[s], 32768u + 4u * L.kv_half);
        if (a.q_tmajor) {
          tma_load_4d(st + L.q, &tmQ, &full[s], 0, kvh * G, qs, b);
          tma_load_4d(st + L.q + 16384, &tmQ, &full[s], 64, kvh * G, qs, b);
        } else {
          tma_load_4d(st + L.q, &tmQ, &full[s], 0, qs, kvh * G, b);
          tma_load_4d(st + L.q + 16384, &tmQ, &full[s], 64, qs, kvh * G, b);
        }
        tma_load_4d(st + L.k, &tmK, &full[s], 0, kidx, kvh, b);
        tma_load_4d(st + L.k + L.kv_half, &tmK, &full[s], 64, kidx, kvh, b);
        tma_load_4d(st + L.v, &tmV, &full[s], 0, kidx, kvh, b);
        tma_load_4d(st + L.v + L.kv_half, &tmV, &full[s], 64, kidx, kvh, b);
      }
      int ids[kMaxSummaries];
      const int blk = (int)(qg / BS);
      const int ns = prefill_summaries(a.route, blk, a.window, a.route.neighbors, ids);
      const uint8_t* kbase = reinterpret_cast<const uint8_t*>(a.ksum) + 2 * (b * a.ks_b + kvh * a.ks_h);
      const uint8_t* vbase = reinterpret_cast<const uint8_t*>(a.vsum) + 2 * (b * a.vs_b + kvh * a.vs_h);
#pragma unroll 4
      for (int c = lane; c < 256; c += 32) {
        const int r = c >> 4, ch = c & 15, half = ch >> 3, cc = ch & 7;
        uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
        if (r < ns) {
          kv = ld_nc_128(kbase + 2 * (ids[r] * a.ks_n) + ch * 16);
          vv = ld_nc_128(vbase + 2 * (ids[r] * a.vs_n) + ch * 16);
        }
        const uint32_t off = half * 2048 + r * 128 + ((cc ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(st + L.ks + off) = kv;
        *reinterpret_cast<uint4*>(st + L.vs + off) = vv;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t fmt = ElemTraits<T>::kUmmaFormat;
      const uint32_t id_qk = idesc_f16(128, NR, fmt, false);
      const uint32_t id_qs = idesc_f16(128, 16, fmt, false);
      const uint32_t id_pv = idesc_f16(128, 128, fmt, true);
      const uint32_t sP = smem_u32(smem + L.p);
      int n = 0;
      for (int u = blockIdx.x; u < a.total_units; u += gridDim.x) ++n;
      bool ok = true;
      auto issue_qk = [&](int i) -> bool {
        const int s = i % S;
        if (!mbar_wait(&full[s], (uint32_t)(i / S) & 1u, abort_flag, 2, a.err)) return false;
        tc_fence_after();
        const uint32_t base = smem_u32(stage_ptr(s));
        const uint32_t dS = tmem + (uint32_t)(i & 1) * 128u;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t kin = (uint32_t)(kk & 3) * 32u;
          const uint64_t aq = desc_sw128(base + L.q + (kk >> 2) * 16384u + kin, 16, 1024);
          const uint64_t bk = desc_sw128(base + L.k + (kk >> 2) * L.kv_half + kin, 16, 1024);
          const uint64_t bs = desc_sw128(base + L.ks + (kk >> 2) * 2048u + kin, 16, 1024);
          mma_f16_ss(dS, aq, bk, id_qk, kk > 0);
          mma_f16_ss(dS + (uint32_t)NR, aq, bs, id_qs, kk > 0);
        }
        mma_commit(&sfull[i & 1]);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int s = j % S;
        if (!mbar_wait(pfull, (uint32_t)j & 1u, abort_flag, 3, a.err)) return false;
        tc_fence_after();
        const uint32_t base = smem_u32(stage_ptr(s));
        const int nks = (NR + 16) / 16;
        for (int ks = 0; ks < nks; ++ks) {
          const uint64_t ap = desc_sw128(sP + (ks >> 2) * 16384u + (uint32_t)(ks & 3) * 32u, 16, 1024);
          const uint64_t bv = (ks * 16 < NR) ? desc_sw128(base + L.v + (uint32_t)ks * 2048u, L.kv_half, 1024)
                                             : desc_sw128(base + L.vs, 2048, 1024);
          mma_f16_ss(tmem + 256u, ap, bv, id_pv, ks > 0);
        }
        mma_commit(ofull);
        mma_commit(&empty[s]);
        return true;
      };
      for (int i = 0; i < n && ok; ++i) {
        ok = issue_qk(i);
        if (ok && i > 0) ok = issue_pv(i - 1);
      }
      if (ok && n > 0) issue_pv(n - 1);
      // Drain: every MMA issued above has completed once this commit arrives.
      volatile int never_abort = 0;
      mma_commit(drain);
      mbar_wait(drain, 0, &never_abort, 6, a.err);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(quad * 32) << 16);
    uint8_t* sP = smem + L.p;
    const int g = a.q_tmajor ? (row % G) : (row / QT);
    const int qi = a.q_tmajor ? (row / G) : (row % QT);
    int i = 0;
    for (int u = blockIdx.x; u < a.total_units; u += gridDim.x, ++i) {
      if (!mbar_wait(&sfull[i & 1], (uint32_t)(i >> 1) & 1u, abort_flag, 4, a.err)) break;
      tc_fence_after();
      const int t = u % a.ntiles, rest = u / a.ntiles, kvh = rest % a.Hkv, b = rest / a.Hkv;
      const int qs = t * QT;
      const int qloc = qs + qi;
      const bool valid_row = qloc < a.Tq;
      const int64_t qglob = a.q_pos0 + qloc;
      const int64_t kstart = a.q_pos0 + qs - (a.window - 1);
      int ids[kMaxSummaries];
      const int ns = prefill_summaries(a.route, (int)((a.q_pos0 + qs) / BS), a.window, a.route.neighbors, ids);
      const int lo = (int)(max64(0, qglob - a.window + 1) - kstart);
      const int hi = (int)(qglob - kstart);
      const uint32_t sAddr = lane_addr + (uint32_t)(i & 1) * 128u;

      float m = -INFINITY;
      for (int c0 = 0; c0 < NR; c0 += 16) {
        float x[16];
        tmem_ld16(sAddr + c0, x);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (c0 + j >= lo && c0 + j <= hi) m = fmaxf(m, x[j]);
      }
      {
        float x[16];
        tmem_ld16(sAddr + NR, x);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (j < ns) m = fmaxf(m, x[j]);
      }
      const float mb = valid_row ? m * a.scale_log2 : 0.f;
      float l = 0.f;
      for (int c0 = 0; c0 < NR + 16; c0 += 16) {
        float x[16];
        tmem_ld16(sAddr + c0, x);
        tmem_ld_wait();
        uint32_t pk[8];
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          float p0, p1;
          const int c = c0 + j;
          bool v0, v1;
          if (c0 < NR) {
            v0 = c >= lo && c <= hi;
            v1 = c + 1 >= lo && c + 1 <= hi;
          } else {
            v0 = j < ns;
            v1 = j + 1 < ns;
          }
          v0 = v0 && valid_row;
          v1 = v1 && valid_row;
          p0 = v0 ? exp2f(fmaf(x[j], a.scale_log2, -mb)) : 0.f;
          p1 = v1 ? exp2f(fmaf(x[j + 1], a.scale_log2, -mb)) : 0.f;
          l += p0 + p1;
          pk[j >> 1] = ElemTraits<T>::pack2(p0, p1);
        }
        const int half = c0 >> 6, cc = (c0 & 63) >> 3;
        uint8_t* base = sP + half * 16384 + row * 128;
        *reinterpret_cast<uint4*>(base + ((cc ^ (row & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *reinterpret_cast<uint4*>(base + (((cc + 1) ^ (row & 7)) << 4)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(pfull);
      if (!mbar_wait(ofull, (uint32_t)i & 1u, abort_flag, 5, a.err)) break;
      tc_fence_after();
      const float inv = (valid_row && l > 0.f) ? 1.f / l : 0.f;
      uint8_t* orow = reinterpret_cast<uint8_t*>(a.out) +
                      2 * (b * a.os_b + (int64_t)(kvh * G + g) * a.os_h + (int64_t)qloc * a.os_t);
      for (int c0 = 0; c0 < 128; c0 += 16) {
        float x[16];
        tmem_ld16(lane_addr + 256u + c0, x);
        tmem_ld_wait();
        if (valid_row) {
          uint32_t pk[8];
#pragma unroll
          for (int j = 0; j < 16; j += 2) pk[j >> 1] = ElemTraits<T>::pack2(x[j] * inv, x[j + 1] * inv);
          st_128(orow + c0 * 2, make_uint4(pk[0], pk[1], pk[2], pk[3]));
          st_128(orow + c0 * 2 + 16, make_uint4(pk[4], pk[5], pk[6], pk[7]));
        }
      }
      if (valid_row && a.lse)
        a.lse[b * a.ls_b + (int64_t)(kvh * G + g) * a.ls_h + qloc] = (mb + log2f(l)) * kLn2;
      tc_fence_before();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

// ----------------------------------------------------------------------------- host
int* device_error_word();  // kernels.cu
using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;

static EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  }
  return fn;
}

// Tensor map over a [d0,d1,d2,d3] view with d3 innermost; `order` lists which of d0..d2
// become tensor-map dimensions 1..3 (dimension 0 is always d3 = head_dim).
static int encode_map(CUtensorMap* m, const bna_tensor4* t, CUtensorMapDataType dt, const int order[3],
                      const uint32_t box[3], const char* name) {
  EncodeFn enc = get_encode();
  if (!enc) return fail(BNA_CUDA_ERROR, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[4];
  cuuint64_t strides[3];
  cuuint32_t boxd[4] = {64, box[0], box[1], box[2]};
  cuuint32_t es[4] = {1, 1, 1, 1};
  dims[0] = (cuuint64_t)t->size[3];
  for (int i = 0; i < 3; ++i) {
    const int d = order[i];
    dims[i + 1] = (cuuint64_t)t->size[d];
    int64_t st = t->stride[d] * 2;
    if (t->size[d] == 1) st = 16;  // unused dimension: any legal stride
    if (st <= 0 || (st % 16) != 0) return fail(BNA_BAD_STRIDE, std::string(name) + ": strides must be 16-byte multiples");
    strides[i] = (cuuint64_t)st;
  }
  if ((reinterpret_cast<uintptr_t>(t->data) & 15) != 0) return fail(BNA_BAD_STRIDE, std::string(name) + ": data not 16-byte aligned");
  CUresult r = enc(m, dt, 4, t->data, dims, strides, boxd, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(BNA_BAD_STRIDE, std::string(name) + ": cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return BNA_OK;
}

int launch_prefill(const bna_tensor4* q, const bna_tensor4* k, const bna_tensor4* v, const bna_tensor4* ks,
                   const bna_tensor4* vs, bna_tensor4* out, float* lse, int64_t ls_b, int64_t ls_h, int dtype,
                   const bna_route* route, int window, int64_t q_pos0, int64_t kv_pos0, int64_t total_len,
                   float scale, cudaStream_t stream) {
  PrefillArgs a{};
  a.B = (int)q->size[0];
  a.Hq = (int)q->size[1];
  a.Tq = (int)q->size[2];
  a.Hkv = (int)k->size[1];
  a.G = a.Hq / a.Hkv;
  a.QT = 128 / a.G;
  a.NR = ((window - 1 + a.QT) + 15) / 16 * 16;
  if (a.NR + 16 > 256)
    return fail(BNA_UNSUPPORTED, "window too large for one tensor-core key tile (need W - 1 + 128/G + 16 <= 256)");
  if (route->block_size % a.QT != 0 || q_pos0 % route->block_size != 0)
    return fail(BNA_UNSUPPORTED, "block_size must be a multiple of 128/G and q_pos0 a multiple of block_size");
  a.ntiles = (a.Tq + a.QT - 1) / a.QT;
  a.total_units = a.B * a.Hkv * a.ntiles;
  if (a.total_units == 0) return BNA_OK;
  a.q_pos0 = q_pos0;
  a.kv_pos0 = kv_pos0;
  a.total_len = total_len;
  a.window = window;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.route = *route;
  a.ksum = ks->data;
  a.vsum = vs->data;
  a.ks_b = ks->stride[0]; a.ks_h = ks->stride[1]; a.ks_n = ks->stride[2];
  a.vs_b = vs->stride[0]; a.vs_h = vs->stride[1]; a.vs_n = vs->stride[2];
  a.out = out->data;
  a.os_b = out->stride[0]; a.os_h = out->stride[1]; a.os_t = out->stride[2];
  a.lse = lse;
  a.ls_b = ls_b;
  a.ls_h = ls_h;
  a.err = device_error_word();

  int dev = 0, nsm = 0, max_smem = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  a.stages = 2;
  if ((int)PrefillSmem(a.NR, 2).total > max_smem) a.stages = 1;
  const uint32_t smem = PrefillSmem(a.NR, a.stages).total;
  if ((int)smem > max_smem) return fail(BNA_UNSUPPORTED, "prefill tile does not fit in shared memory");

  const CUtensorMapDataType dt = dtype == BNA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap mq, mk, mv;
  // Q: tile rows (head, position) if positions are the outer stride, else (position, head).
  a.q_tmajor = (q->size[2] > 1 && q->size[1] > 1 && q->stride[1] < q->stride[2]) ? 1 : 0;
  int rc;
  if (a.q_tmajor) {
    const int oq[3] = {1, 2, 0};
    const uint32_t bq[3] = {(uint32_t)a.G, (uint32_t)a.QT, 1};
    rc = encode_map(&mq, q, dt, oq, bq, "q");
  } else {
    const int oq[3] = {2, 1, 0};
    const uint32_t bq[3] = {(uint32_t)a.QT, (uint32_t)a.G, 1};
    rc = encode_map(&mq, q, dt, oq, bq, "q");
  }
  if (rc) return rc;
  const int okv[3] = {2, 1, 0};
  const uint32_t bkv[3] = {(uint32_t)a.NR, 1, 1};
  if ((rc = encode_map(&mk, k, dt, okv, bkv, "k"))) return rc;
  if ((rc = encode_map(&mv, v, dt, okv, bkv, "v"))) return rc;

  const int grid = a.total_units < nsm ? a.total_units : nsm;
  if (dtype == BNA_BF16) {
    auto kern = prefill_sm100_kernel<__nv_bfloat16>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<grid, 192, smem, stream>>>(mq, mk, mv, a);
  } else {
    auto kern = prefill_sm100_kernel<__half>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<grid, 192, smem, stream>>>(mq, mk, mv, a);
  }
  return check_cuda(cudaGetLastError(), "prefill_sm100_kernel launch");
}

}  // namespace bna
