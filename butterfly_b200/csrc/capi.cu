// capi.cu — the extern "C" boundary (include/bna_b200.h): argument validation, status
// codes with a thread-local message, route construction and selection dumps, and
// dispatch to the kernels.  No entry point allocates device memory.
#include <cuda_runtime.h>

#include <cmath>
#include <string>

#include "common.cuh"
#include "route.cuh"

namespace bna {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }
int fail(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}
int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return BNA_OK;
  return fail(BNA_CUDA_ERROR, std::string(what) + ": " + cudaGetErrorString(e));
}

int launch_prefill(const bna_tensor4*, const bna_tensor4*, const bna_tensor4*, const bna_tensor4*,
                   const bna_tensor4*, bna_tensor4*, float*, int64_t, int64_t, int, const bna_route*, int,
                   int64_t, int64_t, int64_t, float, cudaStream_t, const bna_tensor4* = nullptr);
int launch_compress(const bna_tensor4*, bna_tensor4*, int, int, int64_t, int, int64_t, int64_t, int64_t,
                    cudaStream_t, const bna_tensor4*, bna_tensor4*);
int launch_append(bna_tensor4*, bna_tensor4*, const bna_tensor4*, const bna_tensor4*, int64_t, int64_t,
                  cudaStream_t);
int launch_active(const bna_tensor4*, const bna_tensor4*, const bna_tensor4*, const bna_tensor4*,
                  const bna_tensor4*, bna_tensor4*, float*, int64_t, int64_t, int, const bna_route*, int,
                  const int64_t*, int64_t, int64_t, int64_t, int64_t, int, float, const bna_tensor4*,
                  const bna_tensor4*, int64_t, int64_t, cudaStream_t, const QKPrep* = nullptr);
int launch_selection_dump(const bna_route*, int, int32_t*, int32_t*, cudaStream_t);
int take_device_error(int, int32_t*);
int launch_probe(int, cudaStream_t);
void set_prefill_trace(uint64_t*);

// ---------------------------------------------------------------- validation helpers
static bool null4(const bna_tensor4* t) { return t == nullptr || t->data == nullptr; }

static int check_rows(const bna_tensor4* t, const char* name, int64_t dh) {
  if (null4(t)) return fail(BNA_BAD_SHAPE, std::string(name) + " is null");
  for (int i = 0; i < 4; ++i)
    if (t->size[i] < 0) return fail(BNA_BAD_SHAPE, std::string(name) + " has a negative size");
  if (t->size[3] != dh) return fail(BNA_BAD_SHAPE, std::string(name) + ": head_dim mismatch");
  if (t->stride[3] != 1) return fail(BNA_BAD_STRIDE, std::string(name) + ": head_dim must be contiguous");
  for (int i = 0; i < 3; ++i)
    if (t->size[i] > 1 && (t->stride[i] % 8) != 0)
      return fail(BNA_BAD_STRIDE, std::string(name) + ": strides must be multiples of 8 elements (16 bytes)");
  if ((reinterpret_cast<uintptr_t>(t->data) & 15) != 0)
    return fail(BNA_BAD_STRIDE, std::string(name) + ": data pointer must be 16-byte aligned");
  return BNA_OK;
}

static int check_dtype(int dtype) {
  if (dtype != BNA_BF16 && dtype != BNA_F16) return fail(BNA_BAD_DTYPE, "only bfloat16 and float16 are supported");
  return BNA_OK;
}

static int check_route(const bna_route* r) {
  if (!r) return fail(BNA_BAD_SHAPE, "route is null");
  if (r->block_size <= 0 || r->num_blocks <= 0) return fail(BNA_BAD_SHAPE, "block_size and num_blocks must be positive");
  if (r->max_degree < 1 || r->max_degree > kMaxSummaries)
    return fail(BNA_UNSUPPORTED, "max_degree must be in [1, 16]");
  if (r->partner_count < 0 || r->partner_count > kMaxPartners)
    return fail(BNA_UNSUPPORTED, "partner_count must be in [0, 8]");
  if (r->rule < 0 || r->rule > 3) return fail(BNA_UNSUPPORTED, "unknown partner rule");
  if (r->local_window_blocks < 0 || r->sink_count < 0) return fail(BNA_BAD_SHAPE, "negative local window / sink count");
  return BNA_OK;
}

static int width_of(int n) {
  if (n <= 1) return 1;
  int w = 0;
  while ((1LL << w) < n) ++w;
  return w;
}

}  // namespace bna

using namespace bna;

extern "C" {

const char* bna_last_error(void) { return g_last_error.c_str(); }
const char* bna_version(void) { return "bna_b200 0.1.0 (sm_100a)"; }

int bna_take_device_error(int device, int32_t* code_out) {
  if (!code_out) return fail(BNA_BAD_SHAPE, "code_out is null");
  return take_device_error(device, code_out);
}

int bna_set_prefill_trace(void* device_buffer) {
  set_prefill_trace(static_cast<uint64_t*>(device_buffer));
  return BNA_OK;
}

int bna_route_init(bna_route* r, int32_t seq_len, int32_t block_size, int32_t layer_idx, int32_t lwb,
                   int32_t sink_count, int32_t partner_count, int32_t rule) {
  if (!r) return fail(BNA_BAD_SHAPE, "route is null");
  if (seq_len <= 0) return fail(BNA_BAD_SHAPE, "seq_len must be positive");
  if (block_size <= 0) return fail(BNA_BAD_SHAPE, "block_size must be positive");
  if (lwb < 0) return fail(BNA_BAD_SHAPE, "local_window_blocks must be >= 0");
  if (sink_count < 0) return fail(BNA_BAD_SHAPE, "sink_count must be >= 0");
  if (partner_count < 0) return fail(BNA_BAD_SHAPE, "partner_count must be >= 0");
  if (rule < 0 || rule > 3) return fail(BNA_UNSUPPORTED, "unknown partner rule");
  if (partner_count > kMaxPartners) return fail(BNA_UNSUPPORTED, "partner_count above 8");
  if (layer_idx < 0) return fail(BNA_BAD_SHAPE, "layer_idx must be >= 0");
  bna_route x{};
  x.block_size = block_size;
  x.num_blocks = (int32_t)(((int64_t)seq_len + block_size - 1) / block_size);
  x.rule = rule;
  x.width = width_of(x.num_blocks);
  x.stage_count = rule == BNA_RULE_BENES ? (2 * x.width - 2 > 1 ? 2 * x.width - 2 : 1) : x.width;
  x.stage_idx = layer_idx % x.stage_count;
  x.partner_count = partner_count;
  x.local_window_blocks = lwb;
  x.sink_count = sink_count;
  x.neighbors = nullptr;
  x.max_degree = 1;
  int maxd = 1;
  for (int b = 0; b < x.num_blocks; ++b) {
    int n = 0;
    for_each_neighbor(x, b, nullptr, [&](int) -> bool { ++n; return true; });
    if (n > maxd) maxd = n;
  }
  x.max_degree = maxd;
  *r = x;
  if (maxd > kMaxSummaries) return fail(BNA_UNSUPPORTED, "more than 16 neighbours per block row");
  return BNA_OK;
}

int bna_block_neighbors_host(const bna_route* r, int32_t* out) {
  if (int rc = check_route(r)) return rc;
  if (!out) return fail(BNA_BAD_SHAPE, "out is null");
  for (int b = 0; b < r->num_blocks; ++b) {
    int32_t* row = out + (int64_t)b * r->max_degree;
    int n = 0;
    for_each_neighbor(*r, b, r->neighbors, [&](int v) -> bool {
      if (n < r->max_degree) row[n++] = v;
      return true;
    });
    for (int i = n; i < r->max_degree; ++i) row[i] = -1;
  }
  return BNA_OK;
}

int bna_prefill_selection_host(const bna_route* r, int32_t seq_len, int32_t window, int32_t* local_start,
                               int32_t* summary_idx, int32_t* summary_count) {
  if (int rc = check_route(r)) return rc;
  if (seq_len <= 0) return fail(BNA_BAD_SHAPE, "T must be positive");
  if (window <= 0) return fail(BNA_BAD_SHAPE, "local_window_tokens must be positive");
  for (int b = 0; b < r->num_blocks; ++b) {
    int ids[kMaxSummaries];
    const int n = prefill_summaries(*r, b, window, r->neighbors, ids);
    if (local_start) local_start[b] = (int32_t)max64(0, (int64_t)b * r->block_size - window + 1);
    if (summary_idx)
      for (int i = 0; i < r->max_degree; ++i) summary_idx[(int64_t)b * r->max_degree + i] = i < n ? ids[i] : -1;
    if (summary_count) summary_count[b] = n;
  }
  return BNA_OK;
}

int bna_active_selection_host(const bna_route* r, int32_t window, const int64_t* positions, int32_t n,
                              int32_t limit, int32_t* block, int32_t* local_start, int32_t* summary_idx,
                              int32_t* summary_count) {
  if (int rc = check_route(r)) return rc;
  if (window <= 0) return fail(BNA_BAD_SHAPE, "local_window_tokens must be positive");
  if (n > 0 && !positions) return fail(BNA_BAD_SHAPE, "positions is null");
  for (int i = 0; i < n; ++i) {
    int ids[kMaxSummaries];
    const int64_t p = positions[i];
    const int c = active_summaries(*r, p, window, limit, r->neighbors, ids);
    if (block) block[i] = active_block(*r, p);
    if (local_start) local_start[i] = (int32_t)max64(0, p - window + 1);
    if (summary_idx)
      for (int j = 0; j < r->max_degree; ++j) summary_idx[(int64_t)i * r->max_degree + j] = j < c ? ids[j] : -1;
    if (summary_count) summary_count[i] = c;
  }
  return BNA_OK;
}

int bna_prefill_selection_device(const bna_route* r, int32_t seq_len, int32_t window, int32_t* summary_idx,
                                 int32_t* summary_count, void* stream) {
  if (int rc = check_route(r)) return rc;
  if (seq_len <= 0 || window <= 0) return fail(BNA_BAD_SHAPE, "T and window must be positive");
  if (!summary_idx || !summary_count) return fail(BNA_BAD_SHAPE, "output is null");
  return launch_selection_dump(r, window, summary_idx, summary_count, (cudaStream_t)stream);
}

static int check_compress(const bna_tensor4* x, bna_tensor4* out, int32_t dtype, int32_t block_size, int32_t n_blocks,
                          int64_t valid_len, int64_t ring, int64_t slot0) {
  if (int rc = check_dtype(dtype)) return rc;
  if (null4(x) || null4(out)) return fail(BNA_BAD_SHAPE, "null tensor");
  const int64_t dh = x->size[3];
  if (dh % 8 != 0 || dh < 8 || dh > 1024 || 128 % (dh / 8) != 0)
    return fail(BNA_UNSUPPORTED, "head_dim must be 8 * a divisor of 128 (<= 1024)");
  if (int rc = check_rows(x, "x", dh)) return rc;
  if (int rc = check_rows(out, "out", dh)) return rc;
  if (block_size <= 0 || n_blocks < 0 || valid_len < 0 || ring < 0 || slot0 < 0)
    return fail(BNA_BAD_SHAPE, "block_size must be positive; counts non-negative");
  if (out->size[0] != x->size[0] || out->size[1] != x->size[1]) return fail(BNA_BAD_SHAPE, "x/out batch or head mismatch");
  if (slot0 + n_blocks > out->size[2]) return fail(BNA_CAPACITY, "summary output too small for the requested blocks");
  if (ring == 0 && valid_len > x->size[2]) return fail(BNA_BAD_SHAPE, "valid_len exceeds x's length");
  if (ring > 0 && ring > x->size[2]) return fail(BNA_BAD_SHAPE, "ring exceeds x's length");
  if (ring == 0 && (int64_t)n_blocks * block_size < valid_len) return fail(BNA_BAD_SHAPE, "n_blocks do not cover valid_len");
  return BNA_OK;
}

int bna_compress_blocks(const bna_tensor4* x, bna_tensor4* out, int32_t dtype, int32_t block_size, int64_t pos0,
                        int32_t n_blocks, int64_t valid_len, int64_t ring, int64_t slot0, void* stream) {
  if (int rc = check_compress(x, out, dtype, block_size, n_blocks, valid_len, ring, slot0)) return rc;
  return launch_compress(x, out, dtype, block_size, pos0, n_blocks, valid_len, ring, slot0, (cudaStream_t)stream,
                         nullptr, nullptr);
}

int bna_compress_kv_blocks(const bna_tensor4* k, const bna_tensor4* v, bna_tensor4* k_out, bna_tensor4* v_out,
                           int32_t dtype, int32_t block_size, int64_t pos0, int32_t n_blocks, int64_t valid_len,
                           int64_t ring, int64_t slot0, void* stream) {
  if (int rc = check_compress(k, k_out, dtype, block_size, n_blocks, valid_len, ring, slot0)) return rc;
  if (int rc = check_compress(v, v_out, dtype, block_size, n_blocks, valid_len, ring, slot0)) return rc;
  for (int i = 0; i < 4; ++i)
    if (k->size[i] != v->size[i] || k_out->size[i] != v_out->size[i]) return fail(BNA_BAD_SHAPE, "k and v shapes differ");
  return launch_compress(k, k_out, dtype, block_size, pos0, n_blocks, valid_len, ring, slot0, (cudaStream_t)stream,
                         v, v_out);
}

static int prefill_impl(const bna_tensor4* q, const bna_tensor4* k, const bna_tensor4* v,
                        const bna_tensor4* k_sum, const bna_tensor4* v_sum, bna_tensor4* out, float* lse,
                        int64_t lse_stride_b, int64_t lse_stride_h, int32_t dtype, const bna_route* route,
                        int32_t window, int64_t q_pos0, int64_t kv_pos0, int64_t total_len, float scale,
                        void* stream, const bna_tensor4* gate) {
  if (int rc = check_dtype(dtype)) return rc;
  if (int rc = check_route(route)) return rc;
  if (null4(q) || null4(k) || null4(v) || null4(k_sum) || null4(v_sum) || null4(out))
    return fail(BNA_BAD_SHAPE, "null tensor");
  const int64_t dh = q->size[3];
  if (dh != 128) return fail(BNA_UNSUPPORTED, "prefill kernel requires head_dim 128");
  const char* names[6] = {"q", "k", "v", "k_summary", "v_summary", "out"};
  const bna_tensor4* ts[6] = {q, k, v, k_sum, v_sum, out};
  for (int i = 0; i < 6; ++i)
    if (int rc = check_rows(ts[i], names[i], dh)) return rc;
  const int64_t B = q->size[0], Hq = q->size[1], Tq = q->size[2], Hkv = k->size[1];
  if (k->size[0] != B || v->size[0] != B) return fail(BNA_BAD_SHAPE, "q, k, v batch size mismatch");
  if (v->size[1] != Hkv || v->size[2] != k->size[2]) return fail(BNA_BAD_SHAPE, "k and v shape mismatch");
  if (Hkv <= 0 || Hq % Hkv != 0) return fail(BNA_BAD_SHAPE, "num query heads must be a multiple of num kv heads");
  const int64_t G = Hq / Hkv;
  if (G != 1 && G != 2 && G != 4 && G != 8) return fail(BNA_UNSUPPORTED, "GQA group size must be 1, 2, 4 or 8");
  if (out->size[0] != B || out->size[1] != Hq || out->size[2] != Tq) return fail(BNA_BAD_SHAPE, "out shape mismatch");
  if (window <= 0) return fail(BNA_BAD_SHAPE, "local_window_tokens must be positive");
  if (total_len <= 0 || q_pos0 < 0 || kv_pos0 < 0 || q_pos0 + Tq > total_len)
    return fail(BNA_BAD_SHAPE, "query range outside the sequence");
  if (kv_pos0 > q_pos0 - (window - 1) && kv_pos0 > 0)
    return fail(BNA_BAD_SHAPE, "keys must start at least W-1 positions before the first query (halo)");
  if (kv_pos0 + k->size[2] < q_pos0 + Tq) return fail(BNA_BAD_SHAPE, "keys must cover every query position");
  const int64_t N = (total_len + route->block_size - 1) / route->block_size;
  if (N != route->num_blocks) return fail(BNA_BAD_SHAPE, "route.num_blocks does not match total_len");
  if (k_sum->size[0] != B || k_sum->size[1] != Hkv || k_sum->size[2] < N || v_sum->size[2] < N || v_sum->size[1] != Hkv)
    return fail(BNA_BAD_SHAPE, "summary tensors must be [B, Hkv, >= num_blocks, dh]");
  if (B * Hkv * ((Tq * G + 127) / 128) > (int64_t)1 << 31) return fail(BNA_UNSUPPORTED, "problem too large");
  if (!(scale > 0.f) || !std::isfinite(scale)) return fail(BNA_BAD_SHAPE, "scale must be positive");
  if (gate) {
    if (null4(gate)) return fail(BNA_BAD_SHAPE, "null gate tensor");
    if (int rc = check_rows(gate, "gate", dh)) return rc;
    if (gate->size[0] != B || gate->size[1] != Hq || gate->size[2] != Tq)
      return fail(BNA_BAD_SHAPE, "gate shape must equal out shape");
  }
  return launch_prefill(q, k, v, k_sum, v_sum, out, lse, lse_stride_b, lse_stride_h, dtype, route, window, q_pos0,
                        kv_pos0, total_len, scale, (cudaStream_t)stream, gate);
}

int bna_prefill_attention(const bna_tensor4* q, const bna_tensor4* k, const bna_tensor4* v,
                          const bna_tensor4* k_sum, const bna_tensor4* v_sum, bna_tensor4* out, float* lse,
                          int64_t lse_stride_b, int64_t lse_stride_h, int32_t dtype, const bna_route* route,
                          int32_t window, int64_t q_pos0, int64_t kv_pos0, int64_t total_len, float scale,
                          void* stream) {
  return prefill_impl(q, k, v, k_sum, v_sum, out, lse, lse_stride_b, lse_stride_h, dtype, route, window, q_pos0,
                      kv_pos0, total_len, scale, stream, nullptr);
}

int bna_prefill_attention_gated(const bna_tensor4* q, const bna_tensor4* k, const bna_tensor4* v,
                                const bna_tensor4* k_sum, const bna_tensor4* v_sum, const bna_tensor4* gate,
                                bna_tensor4* out, float* lse, int64_t lse_stride_b, int64_t lse_stride_h,
                                int32_t dtype, const bna_route* route, int32_t window, int64_t q_pos0,
                                int64_t kv_pos0, int64_t total_len, float scale, void* stream) {
  if (!gate) return fail(BNA_BAD_SHAPE, "null gate tensor");
  return prefill_impl(q, k, v, k_sum, v_sum, out, lse, lse_stride_b, lse_stride_h, dtype, route, window, q_pos0,
                      kv_pos0, total_len, scale, stream, gate);
}

static int check_active_common(const bna_tensor4* q, const bna_tensor4* k, const bna_tensor4* v,
                               const bna_tensor4* k_sum, const bna_tensor4* v_sum, const bna_tensor4* out,
                               int32_t dtype, const bna_route* route, int32_t window) {
  if (int rc = check_dtype(dtype)) return rc;
  if (int rc = check_route(route)) return rc;
  if (null4(q) || null4(k) || null4(v) || null4(k_sum) || null4(v_sum) || null4(out))
    return fail(BNA_BAD_SHAPE, "null tensor");
  const int64_t dh = q->size[3];
  if (dh != 128) return fail(BNA_UNSUPPORTED, "decode kernel requires head_dim 128");
  const char* names[6] = {"q", "k", "v", "k_summary", "v_summary", "out"};
  const bna_tensor4* ts[6] = {q, k, v, k_sum, v_sum, out};
  for (int i = 0; i < 6; ++i)
    if (int rc = check_rows(ts[i], names[i], dh)) return rc;
  const int64_t B = q->size[0], Hq = q->size[1], Hkv = k->size[1];
  if (k->size[0] != B || v->size[0] != B || k_sum->size[0] != B || v_sum->size[0] != B)
    return fail(BNA_BAD_SHAPE, "q, k, v batch size mismatch");
  if (v->size[1] != Hkv || k_sum->size[1] != Hkv || v_sum->size[1] != Hkv)
    return fail(BNA_BAD_SHAPE, "k/v/summary head counts differ");
  if (Hkv <= 0 || Hq % Hkv != 0 || Hq / Hkv > 16) return fail(BNA_BAD_SHAPE, "bad GQA head counts");
  if (out->size[0] != B || out->size[1] != Hq || out->size[2] != q->size[2]) return fail(BNA_BAD_SHAPE, "out shape mismatch");
  if (window <= 0) return fail(BNA_BAD_SHAPE, "local_window_tokens must be positive");
  if (window > 128) return fail(BNA_UNSUPPORTED, "decode kernel supports local windows up to 128 tokens");
  return BNA_OK;
}

int bna_active_attention(const bna_tensor4* q, const bna_tensor4* k, const bna_tensor4* v,
                         const bna_tensor4* k_sum, const bna_tensor4* v_sum, bna_tensor4* out, float* lse,
                         int64_t lse_stride_b, int64_t lse_stride_h, int32_t dtype, const bna_route* route,
                         int32_t window, const int64_t* positions, int64_t pos0, int64_t kv_pos0, int64_t ring,
                         int32_t num_summary_limit, float scale, void* stream) {
  if (int rc = check_active_common(q, k, v, k_sum, v_sum, out, dtype, route, window)) return rc;
  if (ring < 0 || kv_pos0 < 0) return fail(BNA_BAD_SHAPE, "ring and kv_pos0 must be >= 0");
  if (ring > k->size[2]) return fail(BNA_BAD_SHAPE, "ring exceeds k's length");
  if (num_summary_limit > k_sum->size[2] || num_summary_limit > v_sum->size[2])
    return fail(BNA_BAD_SHAPE, "num_summary_limit exceeds the summary tensors");
  const int64_t kv_len = ring > 0 ? INT64_MAX / 4 : kv_pos0 + k->size[2];
  return launch_active(q, k, v, k_sum, v_sum, out, lse, lse_stride_b, lse_stride_h, dtype, route, window, positions,
                       pos0, kv_pos0, ring, kv_len, num_summary_limit, scale, nullptr, nullptr, -1, -1,
                       (cudaStream_t)stream);
}

int bna_cache_append(bna_tensor4* ring_k, bna_tensor4* ring_v, const bna_tensor4* src_k, const bna_tensor4* src_v,
                     int32_t dtype, int64_t pos0, int64_t ring, void* stream) {
  if (int rc = check_dtype(dtype)) return rc;
  if (null4(ring_k) || null4(ring_v) || null4(src_k) || null4(src_v)) return fail(BNA_BAD_SHAPE, "null tensor");
  const int64_t dh = src_k->size[3];
  if (dh % 8 != 0 || dh > 1024) return fail(BNA_UNSUPPORTED, "head_dim must be a multiple of 8");
  const char* names[4] = {"ring_k", "ring_v", "k", "v"};
  const bna_tensor4* ts[4] = {ring_k, ring_v, src_k, src_v};
  for (int i = 0; i < 4; ++i)
    if (int rc = check_rows(ts[i], names[i], dh)) return rc;
  for (int i = 0; i < 2; ++i)
    if (ring_k->size[i] != src_k->size[i] || ring_v->size[i] != src_v->size[i] || src_k->size[i] != src_v->size[i])
      return fail(BNA_BAD_SHAPE, "cache / input batch or head mismatch");
  if (src_k->size[2] != src_v->size[2]) return fail(BNA_BAD_SHAPE, "k and v lengths differ");
  if (ring <= 0 || ring > ring_k->size[2] || ring > ring_v->size[2]) return fail(BNA_BAD_SHAPE, "bad ring size");
  if (src_k->size[2] > ring) return fail(BNA_CAPACITY, "chunk longer than the ring");
  if (pos0 < 0) return fail(BNA_BAD_SHAPE, "pos0 must be >= 0");
  return launch_append(ring_k, ring_v, src_k, src_v, pos0, ring, (cudaStream_t)stream);
}

static int decode_step_impl(const bna_tensor4* q, const bna_tensor4* k_new, const bna_tensor4* v_new, bna_tensor4* ring_k,
                    bna_tensor4* ring_v, bna_tensor4* sum_k, bna_tensor4* sum_v, bna_tensor4* out, float* lse,
                    int64_t lse_stride_b, int64_t lse_stride_h, int32_t dtype, const bna_route* route, int32_t window,
                    int64_t pos, int64_t ring, int64_t close_block, int64_t close_slot, int32_t num_summary_limit,
                    float scale, void* stream, const QKPrep* prep) {
  if (int rc = check_active_common(q, ring_k, ring_v, sum_k, sum_v, out, dtype, route, window)) return rc;
  if (null4(k_new) || null4(v_new)) return fail(BNA_BAD_SHAPE, "null new token");
  if (int rc = check_rows(k_new, "k_new", 128)) return rc;
  if (int rc = check_rows(v_new, "v_new", 128)) return rc;
  if (q->size[2] != 1 || k_new->size[2] != 1 || v_new->size[2] != 1)
    return fail(BNA_BAD_SHAPE, "decode step takes exactly one token per sequence");
  if (k_new->size[0] != q->size[0] || k_new->size[1] != ring_k->size[1] || v_new->size[1] != ring_k->size[1])
    return fail(BNA_BAD_SHAPE, "new token shape mismatch");
  if (ring <= 0 || ring > ring_k->size[2] || ring > ring_v->size[2]) return fail(BNA_BAD_SHAPE, "bad ring size");
  if (ring < window) return fail(BNA_CAPACITY, "ring shorter than the local window");
  if (pos < 0) return fail(BNA_BAD_SHAPE, "pos must be >= 0");
  if (close_block >= 0) {
    if (close_slot < 0 || close_slot >= sum_k->size[2] || close_slot >= sum_v->size[2])
      return fail(BNA_CAPACITY, "summary capacity exhausted");
    if ((close_block + 1) * route->block_size > pos + 1 || pos + 1 - close_block * route->block_size > ring)
      return fail(BNA_BAD_SHAPE, "closed block is not inside the ring tail");
  }
  if (num_summary_limit > sum_k->size[2]) return fail(BNA_BAD_SHAPE, "num_summary_limit exceeds the summary pool");
  return launch_active(q, ring_k, ring_v, sum_k, sum_v, out, lse, lse_stride_b, lse_stride_h, dtype, route, window,
                       nullptr, pos, 0, ring, pos + 1, num_summary_limit, scale, k_new, v_new, close_block, close_slot,
                       (cudaStream_t)stream, prep);
}


int bna_decode_step(const bna_tensor4* q, const bna_tensor4* k_new, const bna_tensor4* v_new, bna_tensor4* ring_k,
                    bna_tensor4* ring_v, bna_tensor4* sum_k, bna_tensor4* sum_v, bna_tensor4* out, float* lse,
                    int64_t lse_stride_b, int64_t lse_stride_h, int32_t dtype, const bna_route* route, int32_t window,
                    int64_t pos, int64_t ring, int64_t close_block, int64_t close_slot, int32_t num_summary_limit,
                    float scale, void* stream) {
  return decode_step_impl(q, k_new, v_new, ring_k, ring_v, sum_k, sum_v, out, lse, lse_stride_b, lse_stride_h, dtype,
                          route, window, pos, ring, close_block, close_slot, num_summary_limit, scale, stream, nullptr);
}

int bna_decode_step_qk(const bna_tensor4* q_raw, const bna_tensor4* k_raw, const bna_tensor4* v_new,
                       bna_tensor4* ring_k, bna_tensor4* ring_v, bna_tensor4* sum_k, bna_tensor4* sum_v,
                       bna_tensor4* out, float* lse, int64_t lse_stride_b, int64_t lse_stride_h, int32_t dtype,
                       const bna_route* route, int32_t window, int64_t pos, int64_t ring, int64_t close_block,
                       int64_t close_slot, int32_t num_summary_limit, float scale, const void* q_norm_weight,
                       const void* k_norm_weight, const void* cos, const void* sin, int64_t cs_batch_stride,
                       int32_t rot, float eps, void* stream) {
  if (!q_norm_weight || !k_norm_weight) return fail(BNA_BAD_SHAPE, "decode_step_qk: null norm weight");
  if (rot < 0 || rot > 128 || rot % 8) return fail(BNA_UNSUPPORTED, "decode_step_qk: rotary dims must be a multiple of 8 <= 128");
  if (rot && (!cos || !sin)) return fail(BNA_BAD_SHAPE, "decode_step_qk: null cos / sin");
  for (const void* p : {q_norm_weight, k_norm_weight, cos, sin})
    if (p && (reinterpret_cast<uintptr_t>(p) & 7)) return fail(BNA_BAD_STRIDE, "decode_step_qk: pointers must be 8-byte aligned");
  if (cs_batch_stride % 4) return fail(BNA_BAD_STRIDE, "decode_step_qk: cos/sin batch stride must be a multiple of 4");
  QKPrep prep{q_norm_weight, k_norm_weight, cos, sin, cs_batch_stride, rot, eps};
  return decode_step_impl(q_raw, k_raw, v_new, ring_k, ring_v, sum_k, sum_v, out, lse, lse_stride_b, lse_stride_h,
                          dtype, route, window, pos, ring, close_block, close_slot, num_summary_limit, scale, stream,
                          &prep);
}

}  // extern "C"

extern "C" BNA_API int bna_launch_probe(int32_t ctas, void* stream) {
  return bna::launch_probe(ctas, static_cast<cudaStream_t>(stream));
}
