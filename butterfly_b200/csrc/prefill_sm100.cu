// prefill_sm100.cu — compressed Butterfly prefill attention on Blackwell tensor cores.
//
// Semantics (bna/torch/attention_wayfinder_permute.py:1046-1122): every query at
// position q attends, with one softmax over the union, to the raw keys
// [max(0, q-W+1), q] and to the cursor-packed routed block summaries of its block
// (partner / sink / far-local blocks that end before the block's raw-window start).
// GQA: the G = Hq/Hkv query heads of a KV head share its keys.
//
// Work unit = (batch b, KV head, query tile of QT = 128/G positions).  Its 128 MMA rows
// are the G heads x QT positions (M = 128).  The keys of a unit are the NR =
// round_up(W - 1 + QT, 16) raw positions starting at q0 - (W - 1), then a 16-row tile of
// the block's routed summaries (zero rows where unused):
//   S = Q . [K_window ; K_sum]^T     tcgen05.mma chains into TMEM (fp32)
//   P = masked softmax(S)            exp2 domain, fp32 row sums; P written back as 16-bit
//                                    values into the S columns of TMEM
//   O = P . [V_window ; V_sum]       tcgen05.mma with A = P from TMEM, V an MN-major operand
//
// Sliding window.  Each CTA processes a contiguous range of units; consecutive units of
// one (b, KV head) advance by QT positions, so K and V live in shared-memory rings of
// R = NR + 2 QT rows and a unit loads only its QT new rows (a whole window only when a run
// of one (b, KV head) starts).  Q streams through a ring of QS tiles.  All loads are TMA
// (128-byte swizzle, zero fill outside the tensor); summary rows are copied by the producer
// warps with cp.async whose completion arrives on the same barrier as the TMA bytes.
//
// Warp roles (608 threads, one CTA per SM):
//   warp 0        Q + K producer        warp 18        V producer
//   warp 1        TMEM allocator + MMA issuer: the whole warp runs the issue code with
//                 warp-uniform operands and one elected lane issues each tcgen05.mma
//   warps 2..17   softmax/epilogue: all 16 warps work on every unit; the four warps of a
//                 TMEM lane quarter split its columns in 8-column chunks, and while the
//                 tensor pipe computes unit i's P.V they run unit i-1's epilogue
// TMEM (512 columns): two S/P tiles at [0, 256) (unit parity) and two O tiles at [256, 512).
#include <map>
#include <mutex>
#include <type_traits>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "route.cuh"
#include "sm100.cuh"

namespace bna {

struct PrefillArgs {
  int B, Hq, Hkv, G, Tq;
  int QT, NR, ntiles, total_units, QS;
  int q_tmajor;  // Q tile rows ordered (position, head) instead of (head, position)
  int64_t q_pos0, kv_pos0, total_len;
  int q_pos0_i, kidx0, blk0, tiles_per_block;  // 32-bit forms of the position math
  int window;
  float scale_log2;
  bna_route route;
  const void* ksum;
  const void* vsum;
  int64_t ks_b, ks_h, ks_n, vs_b, vs_h, vs_n;
  void* out;
  int64_t os_b, os_h, os_t;
  int o_st256;  // output base and strides are 32-byte multiples: 256-bit stores
  float* lse;
  int64_t ls_b, ls_h;
  // optional output gate (the attention output gate of a gated q_proj): when non-null the
  // kernel writes round(O) * round(sigmoid(gate)) instead of O; element strides like out
  const void* gate;
  int64_t gs_b, gs_h, gs_t;
  int* err;         // device error word
  uint64_t* trace;  // optional timeline: [cta][unit < 64][16] globaltimer stamps
};

// Shared-memory plan (1024-byte aligned regions).
//   q      QS tiles x 2 halves x 128 rows x 128 B
//   kslot  kKSlots slots; a slot holds a tile's NR window rows followed by its 16 summary
//          rows, so one MMA of N = NR + 16 covers both (2 halves x (NR + 16) rows x 128 B)
//   vring  V window rows as a ring of R = NR + 2 QT rows (2 halves)
//   vsum   3 slots x 2 halves x 16 V summary rows x 128 B
constexpr int kKSlots = 2;
struct PrefillSmem {
  uint32_t R, q, kslot, kslot_half, kslot_size, ring_half, vring, vsum, xchg, bars, total;
  __host__ __device__ PrefillSmem(int NR, int QT, int QS) {
    R = (uint32_t)(NR + 2 * QT);        // V ring rows (multiple of 16)
    q = 0;
    kslot = (uint32_t)QS * 32768;
    kslot_half = (uint32_t)(NR + 16) * 128;  // multiple of 1024 (NR is a multiple of 16)
    kslot_size = 2 * kslot_half;
    ring_half = R * 128;                // one 64-column half of the V ring
    vring = kslot + kKSlots * kslot_size;
    vsum = vring + 2 * ring_half;
    xchg = vsum + 3 * 4096;             // [2 (max, sum)][2 tile parities][4 column quarters][128] floats
    bars = xchg + 8192;
    total = bars + 512 + 1024;          // + alignment slack
  }
};

namespace {

constexpr float kLn2 = 0.6931471805599453f;
constexpr int kThreads = 608;  // 19 warps
constexpr int kVWarp = 18;     // V producer

// Route of a query block, out of line: producers call it once per block (every few tiles),
// and one shared copy keeps the hot loops small in the instruction cache.
__device__ __noinline__ int prefill_summaries_ool(const bna_route& r, int blk, int window, int* ids) {
  return prefill_summaries(r, blk, window, r.neighbors, ids);
}

template <typename T, int NR_, bool GATED>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const __grid_constant__ PrefillArgs a) {
  using namespace sm100;
  // programmatic dependent launch: wait for the previous kernel of the stream (and its
  // memory), then let the next one start launching
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int QT = a.QT, G = a.G, QS = a.QS;
  const PrefillSmem L(NR_, QT, QS);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* qfull = bars;        // [4] Q tile of unit i landed (slot i % QS)
  uint64_t* kfull = bars + 4;    // [kKSlots] K window + summary rows of unit i landed (slot i % kKSlots)
  uint64_t* vfull = bars + 7;    // [3] new V rows + V summary tile of unit i landed
  uint64_t* qkdone = bars + 10;  // [4] QK(i) complete (ring i % 4)
  uint64_t* pvdone = bars + 14;  // [4] PV(i) complete: O ready, V rows / summary tile free
  uint64_t* sfull = bars + 18;   // [2] per S/P tile (unit parity): S ready in TMEM
  uint64_t* pfull = bars + 20;   // [2] per S/P tile: P stored in TMEM (512 arrivals)
  uint64_t* drain = bars + 22;   // MMA drain at exit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 23);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 24);
  uint32_t* unit_meta = reinterpret_cast<uint32_t*>(bars + 25);  // [8] (unit << 8) | summary count
  float* xchg = reinterpret_cast<float*>(smem + L.xchg);

  if (threadIdx.x == 0) {
    for (int s = 0; s < 4; ++s) {
      mbar_init(&qfull[s], 1);
      mbar_init(&qkdone[s], 1);
      mbar_init(&pvdone[s], 1);
    }
    // TMA expect-tx arrival + producer arrival + 32 cp.async arrivals
    for (int s = 0; s < kKSlots; ++s) mbar_init(&kfull[s], 34);
    for (int s = 0; s < 3; ++s) mbar_init(&vfull[s], 34);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sfull[s], 1);
      mbar_init(&pfull[s], 512);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    for (int k = 0; k < 8; ++k) unit_meta[k] = 0xFFFFFFFFu;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
  }
  if (warp == kVWarp && lane == 0) prefetch_tmap(&tmV);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  constexpr int NK_ = NR_ + 16;  // keys per unit (raw window + summary rows)
  constexpr int NR = NR_;
  const int R = (int)L.R;
  // this CTA's contiguous range of units
  const int u_begin = (int)((int64_t)blockIdx.x * a.total_units / gridDim.x);
  const int n_units = (int)((int64_t)(blockIdx.x + 1) * a.total_units / gridDim.x) - u_begin;
  auto stamp = [&](int i, int ev) {
    if (a.trace && i < 64) a.trace[((int64_t)blockIdx.x * 64 + i) * 16 + ev] = globaltimer();
  };
  // ring row where unit i's key window starts (advances QT per unit, mod R)
  auto roff = [&](int i) { return (int)(((int64_t)i * QT) % R); };

  if (warp == 0 || warp == kVWarp) {
    // ------------------------------------------------------------------ producers
    // Warp 0: Q tiles (ring of QS) and K slots (kKSlots); warp kVWarp: the V ring.  Per unit
    // the producer also gathers the routed-summary rows: behind the window rows of the K
    // slot, and into a 16-row V summary tile (slot i % 3).
    const bool isv = warp == kVWarp;
    const uint8_t* sumbase = reinterpret_cast<const uint8_t*>(isv ? a.vsum : a.ksum);
    const int64_t sb_ = isv ? a.vs_b : a.ks_b, sh_ = isv ? a.vs_h : a.ks_h, sn_ = isv ? a.vs_n : a.ks_n;
    // (t, kvh, b) of the current unit are advanced incrementally; the route is recomputed
    // only when the block changes (every tiles_per_block units)
    int ids[kMaxSummaries];
    int ns = 0, route_blk = -1;
    int t = 0, kvh = 0, b = 0;
    if (n_units > 0) {
      t = u_begin % a.ntiles;
      const int rest = u_begin / a.ntiles;
      kvh = rest % a.Hkv;
      b = rest / a.Hkv;
    }
    for (int i = 0; i < n_units; ++i) {
      if (i > 0 && ++t == a.ntiles) {
        t = 0;
        if (++kvh == a.Hkv) {
          kvh = 0;
          ++b;
        }
      }
      const int qs = t * QT;
      const int blk = a.blk0 + t / a.tiles_per_block;
      if (blk != route_blk) {
        ns = prefill_summaries(a.route, blk, a.window, a.route.neighbors, ids);
        route_blk = blk;
      }
      uint64_t* fb;
      uint8_t* sumt;     // summary rows: row r of half h at sumt + h * sum_half + r * 128
      uint32_t sum_half;
      if (!isv) {
        // Q slot i % QS is free once QK(i - QS) completed and K slot i % kKSlots once
        // QK(i - kKSlots) did; a commit covers every earlier MMA, so one wait does both
        const int dq = i - (QS < kKSlots ? QS : kKSlots);
        if (dq >= 0 && !mbar_wait(&qkdone[dq & 3], (uint32_t)(dq >> 2) & 1u, abort_flag, 1, a.err)) break;
        uint8_t* kd = smem + L.kslot + (uint32_t)(i % kKSlots) * L.kslot_size;
        fb = &kfull[i % kKSlots];
        if (lane == 0) {
          stamp(i, 0);
          uint8_t* qd = smem + L.q + (uint32_t)(i % QS) * 32768u;
          uint64_t* qb = &qfull[i % QS];
          mbar_arrive_expect_tx(qb, 32768u);
          if (a.q_tmajor) {
            tma_load_4d(qd, &tmQ, qb, 0, kvh * G, qs, b);
            tma_load_4d(qd + 16384, &tmQ, qb, 64, kvh * G, qs, b);
          } else {
            tma_load_4d(qd, &tmQ, qb, 0, qs, kvh * G, b);
            tma_load_4d(qd + 16384, &tmQ, qb, 64, qs, kvh * G, b);
          }
          // the whole window (keys before position 0 read as zeros and are masked)
          mbar_arrive_expect_tx(fb, (uint32_t)NR * 256u);
          tma_load_4d(kd, &tmK, fb, 0, a.kidx0 + qs, kvh, b);
          tma_load_4d(kd + L.kslot_half, &tmK, fb, 64, a.kidx0 + qs, kvh, b);
          stamp(i, 1);
        }
        sumt = kd + (uint32_t)NR * 128u;
        sum_half = L.kslot_half;
      } else {
        // V ring rows and summary tile i % 3 are free once PV(i - 3) completed; a new run
        // rewrites a whole window: PV(i - 1)
        const bool run_start = i == 0 || t == 0;
        const int dep = run_start ? i - 1 : i - 3;
        if (dep >= 0 && !mbar_wait(&pvdone[dep & 3], (uint32_t)(dep >> 2) & 1u, abort_flag, 10, a.err)) break;
        fb = &vfull[i % 3];
        if (lane == 0) {
          const int rows = run_start ? NR : QT;
          const int idx0 = a.kidx0 + qs + (run_start ? 0 : NR - QT);
          const int row0 = run_start ? roff(i) : (roff(i) + NR - QT) % R;
          mbar_arrive_expect_tx(fb, (uint32_t)rows * 256u);
          for (int c = 0; c < rows; c += 16) {
            int rr = row0 + c;
            if (rr >= R) rr -= R;
            uint8_t* dst = smem + L.vring + (uint32_t)rr * 128u;
            tma_load_4d(dst, &tmV, fb, 0, idx0 + c, kvh, b);
            tma_load_4d(dst + L.ring_half, &tmV, fb, 64, idx0 + c, kvh, b);
          }
        }
        sumt = smem + L.vsum + (uint32_t)(i % 3) * 4096u;
        sum_half = 2048;
      }
      // summary rows: cp.async straight into the swizzled rows, completion counted on the
      // unit's barrier (32 lanes x .noinc); rows past the valid ones are zeroed directly.
      // Summary rows start on an 8-row boundary, so the swizzle phase is r & 7.
      const uint8_t* base = sumbase + 2 * (b * sb_ + kvh * sh_);
#pragma unroll 1
      for (int j = 0; j < 8; ++j) {
        const int c = lane + 32 * j, r = c >> 4, ch = c & 15, half = ch >> 3, cc = ch & 7;
        uint8_t* dst = sumt + half * sum_half + r * 128 + ((cc ^ (r & 7)) << 4);
        if (r < ns) cp_async_16_sm(dst, base + 2 * (ids[r] * sn_) + ch * 16);
        else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
      }
      cp_async_mbar_arrive_noinc(fb);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        stamp(i, isv ? 15 : 2);
        if (!isv) *reinterpret_cast<volatile uint32_t*>(unit_meta + (i & 7)) = ((uint32_t)i << 8) | (uint32_t)ns;
        mbar_arrive(fb);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp issues (converged, warp-uniform operands; one elected lane per MMA) in a
    // fixed order QK(0), QK(1), PV(0), QK(2), PV(1), ...  Waits are taken by every lane and
    // combined with a vote, so the branches stay warp-uniform.
    {
      constexpr uint32_t fmt = ElemTraits<T>::kUmmaFormat;
      const uint32_t id_qk = idesc_f16(128, NK_, fmt, false);
      const uint32_t id_pv = idesc_f16(128, 128, fmt, true);
      const int n = n_units;
      auto wait_all = [&](uint64_t* bar, uint32_t parity, int site) -> bool {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, site, a.err)) != 0;
      };
      auto issue_qk = [&](int i) {
        const int g = i & 1;
        tc_fence_after();
        fence_proxy_async_smem();  // summary rows arrived through cp.async (generic proxy)
        if (lane == 0) stamp(i, 3);
        // S[128 x NK] = Q[128 x 128] . [window rows | summary rows]^T: one MMA per 16-wide
        // k-step; k-step kk adds (kk & 3) * 32 B inside the swizzle atom and the half offset
        // for kk >= 4 (descriptor start addresses count 16-byte units)
        const uint64_t dq0 = desc_sw128(smem_u32(smem + L.q + (uint32_t)(i % QS) * 32768u), 16, 1024);
        const uint64_t dk0 = desc_sw128(smem_u32(smem + L.kslot + (uint32_t)(i % kKSlots) * L.kslot_size), 16, 1024);
        const uint64_t kh = L.kslot_half >> 4;
        const uint32_t dS = tmem + (uint32_t)g * 128u;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t kin = (uint64_t)((kk & 3) * 2);
          mma_f16_ss_warp(dS, dq0 + kin + (kk >= 4 ? 1024u : 0u), dk0 + kin + (kk >= 4 ? kh : 0), id_qk, kk > 0);
        }
        mma_commit_warp(&sfull[g]);
        mma_commit_warp(&qkdone[i & 3]);
      };
      auto issue_pv = [&](int i) {
        const int g = i & 1;
        tc_fence_after();
        fence_proxy_async_smem();
        if (lane == 0) stamp(i, 4);
        const uint32_t vs = smem_u32(smem + L.vsum + (uint32_t)(i % 3) * 4096u);
        const uint32_t aP = tmem + (uint32_t)g * 128u;
        const uint32_t dO = tmem + 256u + (uint32_t)g * 128u;
        const int r0 = roff(i);
        const uint64_t dv0 = desc_sw128(smem_u32(smem + L.vring), L.ring_half, 1024);  // + row * 128 B
#pragma unroll
        for (int ks = 0; ks < NR / 16; ++ks) {
          int row = r0 + ks * 16;
          if (row >= R) row -= R;
          mma_f16_ts_warp(dO, aP + (uint32_t)ks * 8u, dv0 + (uint64_t)(row * 8), id_pv, ks > 0);
        }
        mma_f16_ts_warp(dO, aP + (uint32_t)(NR / 16) * 8u, desc_sw128(vs, 2048, 1024), id_pv, 1);
        mma_commit_warp(&pvdone[i & 3]);
      };
      for (int p = -2; p < n; ++p) {
        if (p >= 0) {  // PV(p): P(p) stored by its group, V rows and summaries landed
          if (!wait_all(&pfull[p & 1], (uint32_t)(p >> 1) & 1u, 7)) break;
          if (!wait_all(&vfull[p % 3], (uint32_t)(p / 3) & 1u, 7)) break;
          issue_pv(p);
        }
        const int j = p + 2;
        if (j < n) {  // QK(j): S/P tile of PV(j - 2) free, Q and K landed
          if (j >= 2 && !wait_all(&pvdone[(j - 2) & 3], (uint32_t)((j - 2) >> 2) & 1u, 8)) break;
          if (!wait_all(&qfull[j % QS], (uint32_t)(j / QS) & 1u, 8)) break;
          if (!wait_all(&kfull[j % kKSlots], (uint32_t)(j / kKSlots) & 1u, 8)) break;
          issue_qk(j);
        }
      }
      volatile int never_abort = 0;
      mma_commit_warp(drain);
      if (lane == 0) mbar_wait(drain, 0, &never_abort, 6, a.err);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    // All 16 warps work on every unit.  Warp w may read TMEM lane quarter w % 4 (its rows);
    // the four warps of a quarter split the row's columns: S in 8-column chunks, O in 32
    // columns each.  The warps of one SM sub-partition thus run the same code together.
    // Row maxima are exchanged through shared memory under a 128-thread named barrier per
    // quarter; the epilogue of unit i - 1 runs after the softmax of unit i, so the P.V
    // product of a unit overlaps the next unit's softmax.
    constexpr int NCH = NK_ / 8;          // 8-column S chunks
    constexpr int MC = (NCH + 3) / 4;     // most chunks of one column quarter
    const int sw = warp - 2;
    const int cq = sw >> 2;               // column quarter
    const int quad = warp & 3;            // TMEM lane quarter this warp may access
    const int row = quad * 32 + lane;
    const int chb = cq * NCH / 4, chn = (cq + 1) * NCH / 4 - chb;  // my S chunks
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int g = a.q_tmajor ? (row % G) : (row / QT);
    const int qi = a.q_tmajor ? (row / G) : (row % QT);
    float* pmax = xchg;                   // [2][4][128]
    float* psum = xchg + 1024;            // [2][4][128]
    const uint32_t bar_id = 1u + (uint32_t)quad;
    const float sl2 = a.scale_log2;
    // epilogue state of the previous unit
    int e_b = 0, e_kvh = 0, e_qloc = 0;
    bool e_valid = false;
    float e_mb = 0.f;
    auto epilogue = [&](int i) -> bool {
      // gate values of this row's 32 output columns (pulled into L2 a unit earlier), read
      // into registers per 16 columns at the store
      const bool gated = GATED && e_valid;
      const uint8_t* gp = nullptr;
      if (gated)
        gp = reinterpret_cast<const uint8_t*>(a.gate) +
             2 * (e_b * a.gs_b + (int64_t)(e_kvh * G + g) * a.gs_h + (int64_t)e_qloc * a.gs_t) + cq * 64;
      if (!mbar_wait(&pvdone[i & 3], (uint32_t)(i >> 2) & 1u, abort_flag, 5, a.err)) return false;
      if (row == 0 && cq == 0) stamp(i, 7);
      tc_fence_after();
      const float* ps = psum + (i & 1) * 512 + row;
      const float l = (ps[0] + ps[128]) + (ps[256] + ps[384]);
      const float inv = (e_valid && l > 0.f) ? 1.f / l : 0.f;
      float o[32];
      const uint32_t tO = tmem + lane_off + 256u + (uint32_t)(i & 1) * 128u + (uint32_t)cq * 32u;
      tmem_ld16(tO, o);
      tmem_ld16(tO + 16, o + 16);
      tmem_ld_wait();
      if (e_valid) {
        uint8_t* orow = reinterpret_cast<uint8_t*>(a.out) +
                        2 * (e_b * a.os_b + (int64_t)(e_kvh * G + g) * a.os_h + (int64_t)e_qloc * a.os_t) + cq * 64;
#pragma unroll
        for (int c0 = 0; c0 < 32; c0 += 16) {
          uint32_t w[8];
          uint4 gv[2] = {};
          if (gated) {
            gv[0] = ld_nc_128(gp + c0 * 2);
            gv[1] = ld_nc_128(gp + c0 * 2 + 16);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            w[j] = ElemTraits<T>::pack2_fast(o[c0 + 2 * j] * inv, o[c0 + 2 * j + 1] * inv);
            if (gated) {  // as the eager ops: round(round(O) * round(sigmoid(gate)))
              const uint32_t gw = j % 4 == 0 ? gv[j / 4].x : j % 4 == 1 ? gv[j / 4].y : j % 4 == 2 ? gv[j / 4].z : gv[j / 4].w;
              const float2 gg = ElemTraits<T>::unpack2(gw);
              w[j] = ElemTraits<T>::mul2(w[j], ElemTraits<T>::pack2(sigmoid_fast(gg.x), sigmoid_fast(gg.y)));
            }
          }
          if (a.o_st256) {
            st_256(orow + c0 * 2, w);
          } else {
            st_128(orow + c0 * 2, make_uint4(w[0], w[1], w[2], w[3]));
            st_128(orow + c0 * 2 + 16, make_uint4(w[4], w[5], w[6], w[7]));
          }
        }
        if (a.lse && cq == 0)
          a.lse[e_b * a.ls_b + (int64_t)(e_kvh * G + g) * a.ls_h + e_qloc] = (e_mb + log2f(l)) * kLn2;
      }
      if (row == 0 && cq == 0) stamp(i, 8);
      tc_fence_before();
      return true;
    };
    bool ok = true;
    for (int i = 0; i < n_units && ok; ++i) {
      const int u = u_begin + i;
      const int t = u % a.ntiles, rest = u / a.ntiles, kvh = rest % a.Hkv, b = rest / a.Hkv;
      const int qs = t * QT;
      const int qloc = qs + qi;
      const bool valid_row = qloc < a.Tq;
      if (GATED && valid_row)  // the gate row this unit's epilogue reads, one unit from now
        prefetch_l2(reinterpret_cast<const uint8_t*>(a.gate) +
                    2 * (b * a.gs_b + (int64_t)(kvh * G + g) * a.gs_h + (int64_t)qloc * a.gs_t) + cq * 64);
      // positions fit in 32 bits (checked on the host); no 64-bit division on this path
      const int qglob = a.q_pos0_i + qloc;
      const int kstart = a.q_pos0_i + qs - (a.window - 1);
      const int lo = max(0, qglob - a.window + 1) - kstart;
      const int hi = qglob - kstart;
      if (!mbar_wait(&sfull[i & 1], (uint32_t)(i >> 1) & 1u, abort_flag, 4, a.err)) break;
      // routed-summary count of this unit, published by the producer (tagged word)
      int ns = 0;
      {
        const volatile uint32_t* slot = unit_meta + (i & 7);
        uint32_t w = *slot;
        for (int spin = 0; (w >> 8) != (uint32_t)i && spin < (1 << 22); ++spin) w = *slot;
        if ((w >> 8) == (uint32_t)i) {
          ns = (int)(w & 0xFFu);
        } else {
          // The producer never published this unit's count: record the failure (the host
          // sees it through bna_take_device_error), wind the CTA down through the abort
          // flag, and keep this unit's control flow uniform with no summary keys.
          *abort_flag = 1;
          atomicCAS(a.err, 0, 0x1000 | 9);
        }
      }
      if (row == 0 && cq == 0) stamp(i, 5);
      tc_fence_after();
      const uint32_t wlo = valid_row ? (uint32_t)lo : 1u;
      const uint32_t wspan = valid_row ? (uint32_t)(hi - lo) : 0u;
      const int nsv = valid_row ? ns : 0;
      const uint32_t tS = tmem + lane_off + (uint32_t)(i & 1) * 128u;

      // my S chunks in registers; masked entries become -inf
      float x[MC * 8];
#pragma unroll
      for (int j = 0; j < MC; ++j)
        if (j < chn) tmem_ld8(tS + (uint32_t)(chb + j) * 8u, x + j * 8);
      tmem_ld_wait();
      float mp[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int j = 0; j < MC; ++j) {
        if (j < chn) {
          const int c0 = (chb + j) * 8;  // chunks never straddle the window / summary boundary
          if (c0 < NR_) {
            const uint32_t d0 = (uint32_t)c0 - wlo;
#pragma unroll
            for (int e = 0; e < 8; ++e) x[j * 8 + e] = (d0 + (uint32_t)e <= wspan) ? x[j * 8 + e] : -INFINITY;
          } else {
            const int s0 = c0 - NR_;
#pragma unroll
            for (int e = 0; e < 8; ++e) x[j * 8 + e] = (s0 + e < nsv) ? x[j * 8 + e] : -INFINITY;
          }
#pragma unroll
          for (int e = 0; e < 8; e += 4) {
            mp[0] = fmax3(mp[0], x[j * 8 + e], x[j * 8 + e + 1]);
            mp[1] = fmax3(mp[1], x[j * 8 + e + 2], x[j * 8 + e + 3]);
          }
        }
      }
      pmax[(i & 1) * 512 + cq * 128 + row] = fmaxf(mp[0], mp[1]);
      named_bar_sync(bar_id, 128);
      const float* pm = pmax + (i & 1) * 512 + row;
      const float m = fmaxf(fmaxf(pm[0], pm[128]), fmaxf(pm[256], pm[384]));
      const float mb = m > -INFINITY ? m * sl2 : 0.f;
      float lp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < MC; ++j) {
        if (j < chn) {
          uint32_t pk[4];
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            const float p0 = ex2_approx(fmaf(x[j * 8 + e], sl2, -mb));
            const float p1 = ex2_approx(fmaf(x[j * 8 + e + 1], sl2, -mb));
            lp[e >> 1] += p0 + p1;
            pk[e >> 1] = ElemTraits<T>::pack2_fast(p0, p1);
          }
          tmem_st4(tS + (uint32_t)(chb + j) * 4u, pk);  // P column = S column / 2
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&pfull[i & 1]);
      if (row == 0 && cq == 0) stamp(i, 6);
      psum[(i & 1) * 512 + cq * 128 + row] = (lp[0] + lp[1]) + (lp[2] + lp[3]);
      // output of the previous unit (its partial sums were published before this unit's
      // max-exchange barrier)
      if (i > 0) ok = epilogue(i - 1);
      e_b = b;
      e_kvh = kvh;
      e_qloc = qloc;
      e_valid = valid_row;
      e_mb = mb;
    }
    // the last unit's partial sums: every thread of the quarter must have written them
    named_bar_sync(bar_id, 128);
    if (ok && n_units > 0) epilogue(n_units - 1);
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
namespace staged {
int launch_prefill_staged(const bna_tensor4*, const bna_tensor4*, const bna_tensor4*, const bna_tensor4*,
                          const bna_tensor4*, bna_tensor4*, float*, int64_t, int64_t, int, const bna_route*, int, int64_t,
                          int64_t, int64_t, float, cudaStream_t);
}

// Optional prefill timeline buffer (device, >= grid * 64 * 16 uint64), set by
// bna_set_prefill_trace; nullptr disables the stamps.
static uint64_t* g_prefill_trace = nullptr;
void set_prefill_trace(uint64_t* p) { g_prefill_trace = p; }
// Per-device limits and per-(kernel, device) shared-memory opt-in, looked up once: they
// are host-side costs on every call otherwise.
struct DeviceLimits {
  int nsm, max_smem;
};
static DeviceLimits device_limits(int dev) {
  static std::mutex mu;
  static std::map<int, DeviceLimits> cache;
  std::lock_guard<std::mutex> g(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  DeviceLimits d{0, 0};
  cudaDeviceGetAttribute(&d.nsm, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&d.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cache[dev] = d;
  return d;
}
static void set_smem_limit_once(const void* fn, int dev, int smem) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;  // largest limit set so far
  std::lock_guard<std::mutex> g(mu);
  int& cur = done[{fn, dev}];
  if (cur >= smem) return;
  cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cur = smem;
}

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
                   float scale, cudaStream_t stream, const bna_tensor4* gate) {
  PrefillArgs a{};
  if (gate) {
    a.gate = gate->data;
    a.gs_b = gate->stride[0]; a.gs_h = gate->stride[1]; a.gs_t = gate->stride[2];
  }
  a.B = (int)q->size[0];
  a.Hq = (int)q->size[1];
  a.Tq = (int)q->size[2];
  a.Hkv = (int)k->size[1];
  a.G = a.Hq / a.Hkv;
  a.QT = 128 / a.G;
  a.NR = ((window - 1 + a.QT) + 15) / 16 * 16;
  if (a.NR + 16 > 256)
    return fail(BNA_UNSUPPORTED, "window too large for one tensor-core key tile (need W - 1 + 128/G + 16 <= 256)");
  if (total_len >= (int64_t)1 << 30 || kv_pos0 + k->size[2] >= (int64_t)1 << 30)
    return fail(BNA_UNSUPPORTED, "sequences of 2^30 tokens or more");
  if (route->block_size % a.QT != 0 || q_pos0 % route->block_size != 0)
    return fail(BNA_UNSUPPORTED, "block_size must be a multiple of 128/G and q_pos0 a multiple of block_size");
  a.ntiles = (a.Tq + a.QT - 1) / a.QT;
  a.total_units = a.B * a.Hkv * a.ntiles;
  if (a.total_units == 0) return BNA_OK;
  a.q_pos0 = q_pos0;
  a.kv_pos0 = kv_pos0;
  a.total_len = total_len;
  a.window = window;
  a.q_pos0_i = (int)q_pos0;
  a.kidx0 = (int)(q_pos0 - (window - 1) - kv_pos0);
  a.blk0 = (int)(q_pos0 / route->block_size);
  a.tiles_per_block = route->block_size / a.QT;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.route = *route;
  a.ksum = ks->data;
  a.vsum = vs->data;
  a.ks_b = ks->stride[0]; a.ks_h = ks->stride[1]; a.ks_n = ks->stride[2];
  a.vs_b = vs->stride[0]; a.vs_h = vs->stride[1]; a.vs_n = vs->stride[2];
  a.out = out->data;
  a.os_b = out->stride[0]; a.os_h = out->stride[1]; a.os_t = out->stride[2];
  a.o_st256 = (reinterpret_cast<uintptr_t>(out->data) % 32 == 0) && (a.os_b * 2) % 32 == 0 &&
              (a.os_h * 2) % 32 == 0 && (a.os_t * 2) % 32 == 0;
  a.lse = lse;
  a.ls_b = ls_b;
  a.ls_h = ls_h;
  a.err = device_error_word();
  a.trace = g_prefill_trace;


  int dev = 0;
  cudaGetDevice(&dev);
  const DeviceLimits lim = device_limits(dev);
  const int nsm = lim.nsm, max_smem = lim.max_smem;
  a.QS = 3;
  if ((int)PrefillSmem(a.NR, a.QT, 3).total > max_smem) a.QS = 2;
  const uint32_t smem = PrefillSmem(a.NR, a.QT, a.QS).total;
  if ((int)smem > max_smem) {  // rings too large for this shape: stage-based variant
    if (gate) return fail(BNA_UNSUPPORTED, "the gated epilogue needs the ring-based kernel (window too large)");
    return staged::launch_prefill_staged(q, k, v, ks, vs, out, lse, ls_b, ls_h, dtype, route, window, q_pos0, kv_pos0,
                                         total_len, scale, stream);
  }

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
  const uint32_t bk[3] = {(uint32_t)a.NR, 1, 1};  // a tile's whole key window
  const uint32_t bv[3] = {16, 1, 1};              // V ring loads in 16-row boxes
  if ((rc = encode_map(&mk, k, dt, okv, bk, "k"))) return rc;
  if ((rc = encode_map(&mv, v, dt, okv, bv, "v"))) return rc;

  const int grid = a.total_units < nsm ? a.total_units : nsm;
  auto launch = [&](auto kern) {
    set_smem_limit_once(reinterpret_cast<const void*>(kern), dev, (int)smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, mq, mk, mv, a);
  };
#define BNA_PREFILL_CASE(NRV)                                          \
  case NRV:                                                            \
    if (gate) {                                                        \
      if (dtype == BNA_BF16) launch(prefill_sm100_kernel<__nv_bfloat16, NRV, true>); \
      else launch(prefill_sm100_kernel<__half, NRV, true>);            \
    } else {                                                           \
      if (dtype == BNA_BF16) launch(prefill_sm100_kernel<__nv_bfloat16, NRV, false>); \
      else launch(prefill_sm100_kernel<__half, NRV, false>);           \
    }                                                                  \
    break;
  switch (a.NR) {
    BNA_PREFILL_CASE(16) BNA_PREFILL_CASE(32) BNA_PREFILL_CASE(48) BNA_PREFILL_CASE(64)
    BNA_PREFILL_CASE(80) BNA_PREFILL_CASE(96) BNA_PREFILL_CASE(112) BNA_PREFILL_CASE(128)
    BNA_PREFILL_CASE(144) BNA_PREFILL_CASE(160) BNA_PREFILL_CASE(176) BNA_PREFILL_CASE(192)
    BNA_PREFILL_CASE(208) BNA_PREFILL_CASE(224) BNA_PREFILL_CASE(240)
    default:
      return fail(BNA_UNSUPPORTED, "unsupported key-slice width");
  }
#undef BNA_PREFILL_CASE
  return check_cuda(cudaGetLastError(), "prefill_sm100_kernel launch");
}

}  // namespace bna
