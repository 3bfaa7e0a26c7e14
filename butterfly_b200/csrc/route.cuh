// route.cuh — block routing and summary selection, shared by host and device code.
//
// Restates, in closed form, the row construction of build_block_butterfly_layout
// (bna/torch/attention_wayfinder_permute.py:630-652) with the partner rules of
// bna/topology/butterfly.py:77-141, and the summary-slot filter of
// _compressed_butterfly_block_index_tensors (:952-964) / _active_ (:1005-1017):
//   row  = ordered-unique [b, b-1 .. b-lwb (stop below 0), partner(bit) for each bit, sinks]
//   slot = each row entry n with n < b and (n+1)*BS <= cutoff, in row order, cursor-packed,
//          at most max_degree of them (and n < num_summary_limit for cache reads).
#pragma once
#include <stdint.h>
#include "../../include/bna_b200.h"

#if defined(__CUDACC__)
#define BNA_HD __host__ __device__ __forceinline__
#else
#define BNA_HD inline
#endif

namespace bna {

constexpr int kMaxSummaries = 16;
constexpr int kMaxPartners = 8;

BNA_HD int bit_reverse(int value, int width) {
  int out = 0;
  for (int i = 0; i < width; ++i) out = (out << 1) | ((value >> i) & 1);
  return out;
}

// butterfly_partner_bits (butterfly.py:77-105), k-th bit.
BNA_HD int partner_bit(const bna_route& r, int k) {
  if (r.rule == BNA_RULE_BENES) {
    int base = r.stage_count <= 1 ? 0 : r.stage_idx % r.stage_count;
    int phase = (base + k) % r.stage_count;
    if (r.width <= 1) return 0;
    return phase < r.width ? phase : 2 * r.width - 2 - phase;
  }
  return (r.stage_idx + k) % r.width;
}

// butterfly_partner_block (butterfly.py:108-141); -1 for "None".
BNA_HD int partner_block(const bna_route& r, int b, int bit) {
  int w = r.width;
  if (bit < 0 || bit >= (w > 1 ? w : 1)) return -1;
  int p;
  switch (r.rule) {
    case BNA_RULE_CAUSAL_SHIFT: p = b - (1 << bit); break;
    case BNA_RULE_XOR:
    case BNA_RULE_BENES: p = b ^ (1 << bit); break;
    default: p = bit_reverse(bit_reverse(b, w) ^ (1 << bit), w); break;
  }
  if (p < 0 || p >= r.num_blocks || p > b) return -1;
  return p;
}

// Visit the ordered-unique neighbour row of block b; f(n) returns false to stop.
template <class F>
BNA_HD void for_each_neighbor(const bna_route& r, int b, const int32_t* table, F&& f) {
  if (table) {
    const int32_t* row = table + (int64_t)b * r.max_degree;
    for (int i = 0; i < r.max_degree; ++i) {
      int n = row[i];
      if (n < 0) continue;
      if (!f(n)) return;
    }
    return;
  }
  // self and locals: the contiguous range [b - nloc, b]
  int nloc = r.local_window_blocks < b ? r.local_window_blocks : b;
  if (!f(b)) return;
  for (int o = 1; o <= nloc; ++o)
    if (!f(b - o)) return;
  int partners[kMaxPartners];
  int np = 0;
  int pc = r.partner_count < kMaxPartners ? r.partner_count : kMaxPartners;
  if (r.width > 0) {
    for (int k = 0; k < pc; ++k) {
      int p = partner_block(r, b, partner_bit(r, k));
      if (p < 0) continue;
      bool dup = (p >= b - nloc && p <= b);
      for (int j = 0; j < np; ++j) dup = dup || (partners[j] == p);
      if (dup) continue;
      partners[np++] = p;
      if (!f(p)) return;
    }
  }
  int ns = r.sink_count < r.num_blocks ? r.sink_count : r.num_blocks;
  for (int s = 0; s < ns; ++s) {
    bool dup = (s >= b - nloc && s <= b);
    for (int j = 0; j < np; ++j) dup = dup || (partners[j] == s);
    if (dup) continue;
    if (!f(s)) return;
  }
}

// Cursor-packed valid summary blocks of block b for a raw-window start `cutoff`.
BNA_HD int select_summaries(const bna_route& r, int b, int64_t cutoff, int num_summary_limit,
                            const int32_t* table, int* out) {
  int cnt = 0;
  int cap = r.max_degree < kMaxSummaries ? r.max_degree : kMaxSummaries;
  for_each_neighbor(r, b, table, [&](int n) -> bool {
    if (n >= b) return true;
    if ((int64_t)(n + 1) * r.block_size > cutoff) return true;
    if (n >= num_summary_limit) return true;
    out[cnt++] = n;
    return cnt < cap;
  });
  return cnt;
}

BNA_HD int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

// Prefill: block b's summaries; cutoff = max(0, b*BS - W + 1) (:940).
BNA_HD int prefill_summaries(const bna_route& r, int b, int window, const int32_t* table, int* out) {
  int64_t cutoff = max64(0, (int64_t)b * r.block_size - window + 1);
  return select_summaries(r, b, cutoff, r.num_blocks, table, out);
}

// Active row at position p: block = min(p / BS, N - 1); cutoff = max(0, p - W + 1) (:996-997).
BNA_HD int active_block(const bna_route& r, int64_t p) {
  // positions below 2^31 (always, in practice) take the 32-bit division
  const int bs = r.block_size > 0 ? r.block_size : 1;
  int64_t blk = (p >= 0 && p < 0x7FFFFFFF) ? (int64_t)((int)p / bs) : p / bs;
  if (blk < 0) blk = 0;
  if (blk > r.num_blocks - 1) blk = r.num_blocks - 1;
  return (int)(blk < 0 ? 0 : blk);
}

BNA_HD int active_summaries(const bna_route& r, int64_t p, int window, int num_summary_limit,
                            const int32_t* table, int* out) {
  int b = active_block(r, p);
  return select_summaries(r, b, max64(0, p - window + 1), num_summary_limit, table, out);
}

}  // namespace bna
