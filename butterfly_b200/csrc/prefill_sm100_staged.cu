// prefill_sm100_staged.cu — stage-based variant of the tcgen05 prefill kernel, used for
// shapes whose sliding-window rings do not fit in shared memory (e.g. G = 1 with W = 64:
// a 192-row window plus two 128-row advances per ring).  Each unit loads its whole key
// window into a 2-deep stage ring; otherwise the algorithm is the one of prefill_sm100.cu.
//
// (Original header of the shared design follows.)
//
// Semantics (bna/torch/attention_wayfinder_permute.py:1046-1122): every query at
// position q attends, with one softmax over the union, to the raw keys
// [max(0, q-W+1), q] and to the cursor-packed routed block summaries of its block
// (partner / sink / far-local blocks that end before the block's raw-window start).
// GQA: the G = Hq/Hkv query heads of a KV head share its keys.
//
// Work unit = (batch b, KV head, query tile of QT = 128/G positions).  Its 128 MMA rows
// are the G heads x QT positions (M = 128).  The keys of a unit are one contiguous slice
// of NR = round_up(W - 1 + QT, 16) raw positions starting at q0 - (W - 1), followed by 16
// rows holding the block's routed summaries (zero rows where unused), so
//   S = Q . [K_slice ; K_sum]^T            one tcgen05.mma chain, N = NR + 16, fp32 in TMEM
//   P = masked softmax(S)                  exp2 domain, fp32 row sums; P stored as 16-bit
//                                          values back into the S columns of TMEM
//   O = P . [V_slice ; V_sum]              tcgen05.mma with A = P read from TMEM and V an
//                                          MN-major shared-memory operand
// Loads: Q, K, V slices by TMA (128-byte swizzle, zero fill outside the tensor) into a
// 2-stage ring; the summary rows by the producer warp with 128-bit loads written into the
// same swizzled tiles.
//
// Warp roles (320 threads, one CTA per SM, persistent over units):
//   warp 0       producer: TMA issue + summary rows
//   warp 1       TMEM allocator + single-thread MMA issuer
//   warps 2..5   softmax/epilogue group 0 (even local units)
//   warps 6..9   softmax/epilogue group 1 (odd local units)
// The two groups ping-pong so one group's softmax overlaps the other's MMAs and loads.
// TMEM (512 columns): group g's S/P tile at [128g, 128g+128), its O tile at 256 + 128g.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "route.cuh"
#include "sm100.cuh"

namespace bna {
namespace staged {

struct PrefillArgs {
  int B, Hq, Hkv, G, Tq;
  int QT, NR, ntiles, total_units, stages;
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
  float* lse;
  int64_t ls_b, ls_h;
  int* err;         // device error word
  uint64_t* trace;  // optional timeline: [cta][unit < 64][16] globaltimer stamps
};

struct PrefillSmem {
  uint32_t q, kv_rows, kv_half, k, v, stage, xchg, bars, total;
  __host__ __device__ PrefillSmem(int NR, int stages) {
    q = 0;                              // 2 halves x 128 rows x 128 B
    kv_rows = (uint32_t)NR + 16;        // raw slice + summary rows
    kv_half = kv_rows * 128;            // one 64-column half of a K or V tile
    k = 32768;
    v = k + 2 * kv_half;
    stage = v + 2 * kv_half;
    xchg = stage * stages;      // 4 x 256 floats of row max / sum exchange
    bars = xchg + 4096;
    total = bars + 256 + 1024;  // + alignment slack
  }
};

namespace {

constexpr float kLn2 = 0.6931471805599453f;
constexpr int kThreads = 608;  // 19 warps
constexpr int kVWarp = 18;    // producer of the V part of each stage

template <typename T, int NR_>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const __grid_constant__ PrefillArgs a) {
  using namespace sm100;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const PrefillSmem L(a.NR, a.stages);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* full = bars;        // [2] Q + K part of a stage landed (TMA bytes + summary rows)
  uint64_t* empty = bars + 2;   // [2] Q + K part consumed (QK done)
  uint64_t* sfull = bars + 4;   // [2] per group: S ready in TMEM
  uint64_t* pfull = bars + 6;   // [2] per group: P stored in TMEM (256 arrivals)
  uint64_t* ofull = bars + 8;   // [2] per group: O ready in TMEM
  uint64_t* drain = bars + 10;  // MMA drain at exit
  uint64_t* vfull = bars + 11;  // [2] V part of a stage landed
  uint64_t* vempty = bars + 13; // [2] V part consumed (PV done)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 16);
  uint32_t* unit_meta = reinterpret_cast<uint32_t*>(bars + 17);  // [8] (unit << 8) | summary count
  float* xchg = reinterpret_cast<float*>(smem + L.xchg);         // [2 groups][2 halves][256]

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&full[s], 2);
      mbar_init(&empty[s], 1);
      mbar_init(&vfull[s], 2);
      mbar_init(&vempty[s], 1);
      mbar_init(&sfull[s], 1);
      mbar_init(&pfull[s], 256);
      mbar_init(&ofull[s], 1);
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

  constexpr int NK_ = NR_ + 16;  // keys per unit (raw slice + summary rows)
  const int NR = NR_, QT = a.QT, G = a.G, S = a.stages;
  const int NK = NK_;
  auto stamp = [&](int i, int ev) {
    if (a.trace && i < 64) a.trace[((int64_t)blockIdx.x * 64 + i) * 16 + ev] = globaltimer();
  };
  const int BS = a.route.block_size;
  auto stage_ptr = [&](int s) { return smem + (uint32_t)s * L.stage; };

  if (warp == 0 || warp == kVWarp) {
    // ------------------------------------------------------------------ producers
    // Warp 0 fills the Q + K part of each stage, warp kVWarp the V part.  Both append the
    // unit's routed-summary rows (zero rows past the valid ones) to their K / V tile.
    // Software-pipelined by one unit: the route and the summary-row loads of unit i+1 are
    // issued before waiting for unit i's stage, so their latency is off the critical path.
    const bool isv = warp == kVWarp;
    const uint8_t* sumbase = reinterpret_cast<const uint8_t*>(isv ? a.vsum : a.ksum);
    const int64_t sb_ = isv ? a.vs_b : a.ks_b, sh_ = isv ? a.vs_h : a.ks_h, sn_ = isv ? a.vs_n : a.ks_n;
    uint64_t* fullb = isv ? vfull : full;
    uint64_t* emptyb = isv ? vempty : empty;
    const uint32_t tile_off = isv ? L.v : L.k;
    uint4 cur[8], nxt[8];
    int ns_cur = 0, ns_nxt = 0;
    auto fetch = [&](int u, uint4* regs) -> int {
      const int t = u % a.ntiles, rest = u / a.ntiles, kvh = rest % a.Hkv, b = rest / a.Hkv;
      int ids[kMaxSummaries];
      const int ns = prefill_summaries(a.route, a.blk0 + t / a.tiles_per_block, a.window, a.route.neighbors, ids);
      const uint8_t* base = sumbase + 2 * (b * sb_ + kvh * sh_);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = lane + 32 * j, r = c >> 4, ch = c & 15;
        regs[j] = make_uint4(0, 0, 0, 0);
        if (r < ns) regs[j] = ld_nc_128(base + 2 * (ids[r] * sn_) + ch * 16);
      }
      return ns;
    };
    if ((int)blockIdx.x < a.total_units) ns_cur = fetch(blockIdx.x, cur);
    int i = 0;
    for (int u = blockIdx.x; u < a.total_units; u += gridDim.x, ++i) {
      const int s = i % S;
      const uint32_t ph = (uint32_t)(i / S) & 1u;
      const int t = u % a.ntiles, rest = u / a.ntiles, kvh = rest % a.Hkv, b = rest / a.Hkv;
      const int qs = t * QT;
      const int kidx = a.kidx0 + qs;
      if (u + (int)gridDim.x < a.total_units) ns_nxt = fetch(u + gridDim.x, nxt);
      if (i >= S && !mbar_wait(&emptyb[s], ph ^ 1u, abort_flag, isv ? 10 : 1, a.err)) break;
      if (lane == 0) stamp(i, isv ? 14 : 0);
      uint8_t* st = stage_ptr(s);
      if (lane == 0) {
        if (!isv) {
          mbar_arrive_expect_tx(&full[s], 32768u + 2u * (uint32_t)NR * 128u);
          if (a.q_tmajor) {
            tma_load_4d(st + L.q, &tmQ, &full[s], 0, kvh * G, qs, b);
            tma_load_4d(st + L.q + 16384, &tmQ, &full[s], 64, kvh * G, qs, b);
          } else {
            tma_load_4d(st + L.q, &tmQ, &full[s], 0, qs, kvh * G, b);
            tma_load_4d(st + L.q + 16384, &tmQ, &full[s], 64, qs, kvh * G, b);
          }
          tma_load_4d(st + L.k, &tmK, &full[s], 0, kidx, kvh, b);
          tma_load_4d(st + L.k + L.kv_half, &tmK, &full[s], 64, kidx, kvh, b);
        } else {
          mbar_arrive_expect_tx(&vfull[s], 2u * (uint32_t)NR * 128u);
          tma_load_4d(st + L.v, &tmV, &vfull[s], 0, kidx, kvh, b);
          tma_load_4d(st + L.v + L.kv_half, &tmV, &vfull[s], 64, kidx, kvh, b);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = lane + 32 * j, r = c >> 4, ch = c & 15, half = ch >> 3, cc = ch & 7;
        const int row = NR + r;
        const uint32_t off = half * L.kv_half + row * 128 + ((cc ^ (row & 7)) << 4);
        *reinterpret_cast<uint4*>(st + tile_off + off) = cur[j];
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        stamp(i, isv ? 15 : 2);
        if (!isv) *reinterpret_cast<volatile uint32_t*>(unit_meta + (i & 7)) = ((uint32_t)i << 8) | (uint32_t)ns_cur;
        mbar_arrive(&fullb[s]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) cur[j] = nxt[j];
      ns_cur = ns_nxt;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t fmt = ElemTraits<T>::kUmmaFormat;
      const uint32_t id_qk = idesc_f16(128, NK, fmt, false);
      const uint32_t id_pv = idesc_f16(128, 128, fmt, true);
      int n = 0;
      for (int u = blockIdx.x; u < a.total_units; u += gridDim.x) ++n;
      bool ok = true;
      auto issue_qk = [&](int i) -> bool {
        const int s = i % S, g = i & 1;
        // S/P tile of group g was last read by PV(i - 2): wait for it before overwriting.
        if (i >= 2 && !mbar_wait(&ofull[g], (uint32_t)((i - 2) >> 1) & 1u, abort_flag, 7, a.err)) return false;
        if (!mbar_wait(&full[s], (uint32_t)(i / S) & 1u, abort_flag, 2, a.err)) return false;
        stamp(i, 3);
        tc_fence_after();
        const uint32_t base = smem_u32(stage_ptr(s));
        const uint32_t dS = tmem + (uint32_t)g * 128u;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t kin = (uint32_t)(kk & 3) * 32u;
          const uint64_t aq = desc_sw128(base + L.q + (kk >> 2) * 16384u + kin, 16, 1024);
          const uint64_t bk = desc_sw128(base + L.k + (kk >> 2) * L.kv_half + kin, 16, 1024);
          mma_f16_ss(dS, aq, bk, id_qk, kk > 0);
        }
        mma_commit(&sfull[g]);
        mma_commit(&empty[s]);
        return true;
      };
      auto issue_pv = [&](int i) -> bool {
        const int s = i % S, g = i & 1;
        if (!mbar_wait(&pfull[g], (uint32_t)(i >> 1) & 1u, abort_flag, 3, a.err)) return false;
        if (!mbar_wait(&vfull[s], (uint32_t)(i / S) & 1u, abort_flag, 9, a.err)) return false;
        stamp(i, 4);
        tc_fence_after();
        const uint32_t base = smem_u32(stage_ptr(s));
        const uint32_t aP = tmem + (uint32_t)g * 128u;
        const uint32_t dO = tmem + 256u + (uint32_t)g * 128u;
        for (int ks = 0; ks < NK / 16; ++ks) {
          const uint64_t bv = desc_sw128(base + L.v + (uint32_t)ks * 2048u, L.kv_half, 1024);
          mma_f16_ts(dO, aP + (uint32_t)ks * 8u, bv, id_pv, ks > 0);
        }
        mma_commit(&ofull[g]);
        mma_commit(&vempty[s]);
        return true;
      };
      // Issue whichever is ready: PV(j) once group j&1 stored P(j); QK(j) once unit j's
      // stage landed and PV(j-2) (same S/P tile) completed.  PV is preferred.  With one
      // stage, QK(j) also needs PV(j-1) issued (the stage is shared).
      int next_qk = 0, next_pv = 0, seen_full = 0, seen_v = 0;
      int64_t last = clock64();
      uint32_t spins = 0;
      while (next_pv < n && ok) {
        bool progressed = false;
        if (next_pv < next_qk && mbar_test_wait(&pfull[next_pv & 1], (uint32_t)(next_pv >> 1) & 1u) &&
            mbar_test_wait(&vfull[next_pv % S], (uint32_t)(next_pv / S) & 1u)) {
          ok = issue_pv(next_pv++);
          progressed = true;
        }
        if (!progressed && next_pv < n && seen_v < next_pv + 1 &&
            mbar_test_wait(&vfull[next_pv % S], (uint32_t)(next_pv / S) & 1u)) {
          stamp(next_pv, 1);
          seen_v = next_pv + 1;
        }
        if (!progressed && next_qk < n && seen_full < next_qk + 1 &&
            mbar_test_wait(&full[next_qk % S], (uint32_t)(next_qk / S) & 1u)) {
          stamp(next_qk, 12);
          seen_full = next_qk + 1;
        }
        if (progressed) {
        } else if (next_qk < n && next_qk < next_pv + 2 &&
                   (next_qk < 2 || mbar_test_wait(&ofull[next_qk & 1], (uint32_t)((next_qk - 2) >> 1) & 1u)) &&
                   mbar_test_wait(&full[next_qk % S], (uint32_t)(next_qk / S) & 1u)) {
          ok = issue_qk(next_qk++);
          progressed = true;
        }
        if (progressed) {
          spins = 0;
          last = clock64();
        } else if ((++spins & 255) == 0) {
          if (*abort_flag) break;
          if (clock64() - last > kWaitTimeoutCycles) {
            *abort_flag = 1;
            if (a.err) atomicCAS(a.err, 0, 0x1000 | 8);
            break;
          }
        }
      }
      volatile int never_abort = 0;
      mma_commit(drain);
      mbar_wait(drain, 0, &never_abort, 6, a.err);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    // Group grp handles local units i with i % 2 == grp.  Its 8 warps pair up per TMEM lane
    // quarter: half 0 takes S columns [0, kHalf0) and O columns [0, 64), half 1 the rest.
    // The two threads of a row exchange partial max / sum through shared memory, synced
    // by a 64-thread named barrier per (group, quarter).
    constexpr int kHalf0 = ((NK_ / 16 + 1) / 2) * 16;
    const int gw = warp - 2;
    const int grp = gw >> 3;
    const int half = (gw >> 2) & 1;
    const int quad = warp & 3;  // TMEM lane quarter this warp may access
    const int row = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tS = tmem + lane_off + (uint32_t)grp * 128u;
    const uint32_t tO = tmem + lane_off + 256u + (uint32_t)grp * 128u;
    const int g = a.q_tmajor ? (row % G) : (row / QT);
    const int qi = a.q_tmajor ? (row / G) : (row % QT);
    float* xm = xchg + (grp * 2 + half) * 256;        // my partial max [0,128) / sum [128,256)
    float* xo = xchg + (grp * 2 + (half ^ 1)) * 256;  // partner's
    const uint32_t bar_id = 1u + (uint32_t)(grp * 4 + quad);
    const float sl2 = a.scale_log2;
    int i = 0;
    for (int u = blockIdx.x; u < a.total_units; u += gridDim.x, ++i) {
      if ((i & 1) != grp) continue;
      const uint32_t par = (uint32_t)(i >> 1) & 1u;
      const int t = u % a.ntiles, rest = u / a.ntiles, kvh = rest % a.Hkv, b = rest / a.Hkv;
      const int qs = t * QT;
      const int qloc = qs + qi;
      const bool valid_row = qloc < a.Tq;
      // positions fit in 32 bits (checked on the host); no 64-bit division on this path
      const int qglob = a.q_pos0_i + qloc;
      const int kstart = a.q_pos0_i + qs - (a.window - 1);
      const int lo = max(0, qglob - a.window + 1) - kstart;
      const int hi = qglob - kstart;
      if (row == 0 && half == 0) stamp(i, 13);
      if (!mbar_wait(&sfull[grp], par, abort_flag, 4, a.err)) break;
      // routed-summary count of this unit, published by the producer (tagged word)
      int ns = 0;
      {
        const volatile uint32_t* slot = unit_meta + (i & 7);
        uint32_t w = *slot;
        for (int spin = 0; (w >> 8) != (uint32_t)i && spin < (1 << 22); ++spin) w = *slot;
        ns = (int)(w & 0xFFu);
      }
      if (row == 0 && half == 0) stamp(i, 5);
      tc_fence_after();
      const uint32_t wlo = valid_row ? (uint32_t)lo : 1u;
      const uint32_t wspan = valid_row ? (uint32_t)(hi - lo) : 0u;
      const int nsv = valid_row ? ns : 0;

      // S columns of my half in registers; masked entries become -inf.
      constexpr int kMaxCols = kHalf0 > NK_ - kHalf0 ? kHalf0 : NK_ - kHalf0;
      const int cbeg = half ? kHalf0 : 0;
      float x[kMaxCols];
      float mp[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (half == 0) {
#pragma unroll
        for (int c0 = 0; c0 < kHalf0; c0 += 16) tmem_ld16(tS + c0, x + c0);
      } else {
#pragma unroll
        for (int c0 = kHalf0; c0 < NK_; c0 += 16) tmem_ld16(tS + c0, x + (c0 - kHalf0));
      }
      tmem_ld_wait();
#pragma unroll
      for (int k = 0; k < kMaxCols; ++k) {
        const int c = cbeg + k;  // uniform per warp
        if (c < NK_) {
          const bool v = c < NR_ ? ((uint32_t)c - wlo <= wspan) : (c - NR_ < nsv);
          x[k] = v ? x[k] : -INFINITY;
          mp[k & 3] = fmaxf(mp[k & 3], x[k]);
        }
      }
      float m = fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3]));
      xm[row] = m;
      named_bar_sync(bar_id, 64);
      m = fmaxf(m, xo[row]);
      const float mb = m > -INFINITY ? m * sl2 : 0.f;
      if (row == 0 && half == 0) stamp(i, 10);
      float lp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k0 = 0; k0 < kMaxCols; k0 += 16) {
        const int c0 = cbeg + k0;
        if (c0 < NK_ && (half == 1 || c0 < kHalf0)) {
          uint32_t pk[8];
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            const float p0 = ex2_approx(fmaf(x[k0 + j], sl2, -mb));
            const float p1 = ex2_approx(fmaf(x[k0 + j + 1], sl2, -mb));
            lp[(j >> 1) & 3] += p0 + p1;
            pk[j >> 1] = ElemTraits<T>::pack2_fast(p0, p1);
          }
          tmem_st8(tS + (uint32_t)(c0 >> 1), pk);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&pfull[grp]);
      if (row == 0 && half == 0) stamp(i, 6);
      float l = (lp[0] + lp[1]) + (lp[2] + lp[3]);
      xm[128 + row] = l;
      named_bar_sync(bar_id, 64);
      l += xo[128 + row];

      if (!mbar_wait(&ofull[grp], par, abort_flag, 5, a.err)) break;
      if (row == 0 && half == 0) stamp(i, 7);
      tc_fence_after();
      const float inv = (valid_row && l > 0.f) ? 1.f / l : 0.f;
      uint8_t* orow = reinterpret_cast<uint8_t*>(a.out) +
                      2 * (b * a.os_b + (int64_t)(kvh * G + g) * a.os_h + (int64_t)qloc * a.os_t) + half * 128;
      {
        float o[64];
#pragma unroll
        for (int c0 = 0; c0 < 64; c0 += 16) tmem_ld16(tO + half * 64 + c0, o + c0);
        tmem_ld_wait();
        if (valid_row) {
#pragma unroll
          for (int c0 = 0; c0 < 64; c0 += 8) {
            uint4 w;
            w.x = ElemTraits<T>::pack2_fast(o[c0] * inv, o[c0 + 1] * inv);
            w.y = ElemTraits<T>::pack2_fast(o[c0 + 2] * inv, o[c0 + 3] * inv);
            w.z = ElemTraits<T>::pack2_fast(o[c0 + 4] * inv, o[c0 + 5] * inv);
            w.w = ElemTraits<T>::pack2_fast(o[c0 + 6] * inv, o[c0 + 7] * inv);
            st_128(orow + c0 * 2, w);
          }
        }
      }
      if (valid_row && a.lse && half == 0)
        a.lse[b * a.ls_b + (int64_t)(kvh * G + g) * a.ls_h + qloc] = (mb + log2f(l)) * kLn2;
      if (row == 0 && half == 0) stamp(i, 8);
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
}  // namespace staged
int* device_error_word();  // kernels.cu
namespace staged {

// Optional prefill timeline buffer (device, >= grid * 64 * 16 uint64), set by
// bna_set_prefill_trace; nullptr disables the stamps.
static uint64_t* g_prefill_trace = nullptr;
void set_prefill_trace(uint64_t* p) { g_prefill_trace = p; }
using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;

static EncodeFn get_encode_staged() {
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
  EncodeFn enc = get_encode_staged();
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

int launch_prefill_staged(const bna_tensor4* q, const bna_tensor4* k, const bna_tensor4* v, const bna_tensor4* ks,
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
  a.lse = lse;
  a.ls_b = ls_b;
  a.ls_h = ls_h;
  a.err = device_error_word();
  a.trace = g_prefill_trace;


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
  auto launch = [&](auto kern) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<grid, kThreads, smem, stream>>>(mq, mk, mv, a);
  };
#define BNA_PREFILL_CASE(NRV)                                          \
  case NRV:                                                            \
    if (dtype == BNA_BF16) launch(prefill_sm100_kernel<__nv_bfloat16, NRV>); \
    else launch(prefill_sm100_kernel<__half, NRV>);                    \
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

}  // namespace staged
}  // namespace bna
