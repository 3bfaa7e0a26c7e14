// static_scratch.cu — prefill attention for callers that cannot allocate device memory.
//
// Some hosts of this library cannot call cudaMalloc at all: code running inside a
// graph-captured or allocator-owned region of another framework, plugins whose host
// forbids device allocations after start-up, or embedded runtimes with a fixed memory
// plan.  The regular prefill path needs two scratch buffers between its two kernels
// (the K and V block means that the attention kernel routes to), which the caller
// normally allocates.  This entry point instead keeps those block means in a file-scope
// device array, so the caller supplies only q, k, v and the output.  The array is
// reserved on a device when this library's device code is loaded there: with CUDA's
// default lazy module loading that is the first call on the device (which is also why
// that call must come before any stream capture); with CUDA_MODULE_LOADING=EAGER it is
// when the library is loaded.
//
// Limits and sharing rules:
//   * kScratchBytes (8 MiB) bounds 2 * B * Hkv * ceil(T / block_size) * head_dim * 2 bytes
//     (K and V means): e.g. B * Hkv * num_blocks <= 16384 at head_dim 128.  Larger
//     problems are rejected with BNA_CAPACITY.
//   * Every GPU that loads the library holds the 8 MiB until the process exits.
//   * All calls share the one array and it keeps the last call's contents.  Every block
//     mean a call reads is written earlier in the same call, so nothing needs clearing,
//     but calls whose work overlaps on the GPU (different streams, or different host
//     threads on one device) race on the array and must be serialised by the caller.
//   * The first call on each device looks up the array's device address with that device
//     current (cudaGetSymbolAddress); make that first call outside any stream capture.
//     The address is kept for the life of the process: do not use this entry point on a
//     device after cudaDeviceReset (or any other teardown of its primary context).
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "common.cuh"

namespace {

constexpr size_t kScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_prefill_scratch[kScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (host code must not use the
// symbol itself: on the host it names a stand-in, not device memory).
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return bna::check_cuda(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return bna::fail(BNA_UNSUPPORTED, "device index above 63");
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_prefill_scratch);
    if (e != cudaSuccess) return bna::check_cuda(e, "cudaGetSymbolAddress(static prefill scratch)");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return BNA_OK;
}

}  // namespace

extern "C" BNA_API int bna_prefill_attention_static_scratch(
    const bna_tensor4* q, const bna_tensor4* k, const bna_tensor4* v, bna_tensor4* out, float* lse,
    int64_t lse_stride_b, int64_t lse_stride_h, int32_t dtype, const bna_route* route, int32_t window,
    float scale, void* stream) {
  if (!q || !k || !v || !out || !route) return bna::fail(BNA_BAD_SHAPE, "null argument");
  if (route->block_size <= 0) return bna::fail(BNA_BAD_SHAPE, "block_size must be positive");
  const int64_t B = k->size[0], Hkv = k->size[1], T = k->size[2], dh = k->size[3];
  if (B < 0 || Hkv < 0 || T <= 0 || dh <= 0) return bna::fail(BNA_BAD_SHAPE, "bad k shape");
  const int64_t N = (T + route->block_size - 1) / route->block_size;
  // Everything the launched kernels would reject is checked first, so a rejected call
  // launches nothing and leaves the scratch untouched.
  if (dh != 128) return bna::fail(BNA_UNSUPPORTED, "head_dim must be 128");
  if (route->num_blocks != N) return bna::fail(BNA_BAD_SHAPE, "route num_blocks does not match ceil(T / block_size)");
  for (int d = 0; d < 4; ++d)
    if (v->size[d] != k->size[d]) return bna::fail(BNA_BAD_SHAPE, "k and v shapes differ");
  if (q->size[0] != B || q->size[2] != T || q->size[3] != dh || q->size[1] <= 0 || Hkv <= 0 ||
      q->size[1] % Hkv != 0)
    return bna::fail(BNA_BAD_SHAPE, "q must be [B, Hq, T, head_dim] with Hq a multiple of Hkv");
  for (int d = 0; d < 4; ++d)
    if (out->size[d] != q->size[d]) return bna::fail(BNA_BAD_SHAPE, "out must have q's shape");
  if (window <= 0) return bna::fail(BNA_BAD_SHAPE, "window must be positive");
  const int64_t one = B * Hkv * N * dh * 2;  // bytes of one [B, Hkv, N, dh] 16-bit tensor
  const int64_t one_aligned = (one + 255) / 256 * 256;
  if (2 * one_aligned > (int64_t)kScratchBytes)
    return bna::fail(BNA_CAPACITY, "problem needs " + std::to_string(2 * one_aligned) +
                                       " bytes of block means; the static scratch holds " +
                                       std::to_string(kScratchBytes));
  void* base = nullptr;
  if (int rc = scratch_for_current_device(&base)) return rc;
  bna_tensor4 ks{}, vs{};
  ks.data = base;
  vs.data = static_cast<unsigned char*>(base) + one_aligned;
  for (bna_tensor4* t : {&ks, &vs}) {
    t->size[0] = B; t->size[1] = Hkv; t->size[2] = N; t->size[3] = dh;
    t->stride[3] = 1; t->stride[2] = dh; t->stride[1] = N * dh; t->stride[0] = Hkv * N * dh;
  }
  // The same validated public entry points the allocating path uses, on scratch views.
  if (int rc = bna_compress_kv_blocks(k, v, &ks, &vs, dtype, route->block_size, 0, (int32_t)N, T, 0, 0, stream))
    return rc;
  return bna_prefill_attention(q, k, v, &ks, &vs, out, lse, lse_stride_b, lse_stride_h, dtype, route, window, 0, 0,
                               T, scale, stream);
}
