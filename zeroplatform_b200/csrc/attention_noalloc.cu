// attention_noalloc.cu -- paged decode attention for callers that must not allocate device memory.
//
// zcu_paged_attention_noalloc runs the same paged-attention kernel as zcu_paged_attention, but its split-K
// scratch (the per-split partial results and the arrival counters that pick the CTA which merges them) lives
// in one fixed array compiled into this library instead of a workspace the library allocates on demand.
// It is for callers that cannot call cudaMalloc at the point where they run attention: a serving process
// that has handed all free HBM to its KV page pool (so a late allocation would fail or fragment it), or a
// host runtime whose decode loop forbids device allocation after start-up because cudaMalloc and cudaFree
// can synchronise the whole device and stall every stream on it.
//
// Limits and sharing:
//   * the array holds kScratchBytes = 1 MiB: 8,192 int32 arrival counters (one per sequence x query head)
//     followed by the split partials, batch * hq * splits * (hd + 2) floats; a request that needs more is
//     rejected with kTooLarge and a message, and nothing is launched;
//   * every GPU that loads the library holds the array until the process exits;
//   * all calls on a device share it, so two calls whose kernels overlap on the GPU (different streams, no
//     ordering between them) race; calls on one stream are ordered and safe;
//   * the array keeps what the last call left; the counters must start at zero, so each call clears them
//     (cudaMemsetAsync on the same stream) before its launch.
// Set-up: the first call on each device looks the array's device address up with cudaGetSymbolAddress
// (with that device current) and caches it.
// Nothing in this file calls cudaMalloc, cudaFree or an allocating library routine.

#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/zero_tensor_cuda.h"
#include "common.cuh"
#include "kernels.h"

namespace zc {

// Message for zc_cuda_last_error() on the calling thread (defined with the other entry points in capi.cu).
void set_last_error(const std::string& msg);

namespace {

constexpr size_t kScratchBytes = 1u << 20;
constexpr size_t kCounterInts = 8192;
constexpr size_t kPartialFloats = (kScratchBytes - kCounterInts * sizeof(int)) / sizeof(float);
constexpr int kMaxDevices = 64;

// Counters first (int32), then partials (fp32); both views are 256-byte aligned.
static __device__ __align__(256) float g_attn_scratch[kScratchBytes / sizeof(float)];

std::mutex g_mu;
void* g_addr[kMaxDevices] = {};

// Host code never passes g_attn_scratch itself to a kernel: in host code that name is a host-side shadow, not
// a device address.  The device address comes from cudaGetSymbolAddress, once per device.
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    set_last_error("zcu_paged_attention_noalloc: no usable current device");
    return kCudaError;
  }
  std::lock_guard<std::mutex> g(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      set_last_error(std::string("zcu_paged_attention_noalloc: cudaGetSymbolAddress failed: ") +
                     cudaGetErrorString(e));
      return kCudaError;
    }
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return kOk;
}

}  // namespace
}  // namespace zc

extern "C" int32_t zcu_paged_attention_noalloc(const float* q, const void* k_pool, const void* v_pool, int32_t kv_dtype,
                                               const int32_t* page_table, const int32_t* ctx_len, float* out,
                                               int32_t batch, int32_t hq, int32_t hkv, int32_t hd, int32_t page_size,
                                               int32_t max_pages, int32_t num_pages, int64_t page_stride,
                                               int64_t slot_stride, int64_t head_stride, float scale, int32_t max_ctx,
                                               void* stream) {
  using namespace zc;
  set_last_error("");
  if (num_pages <= 0 || batch <= 0 || hq <= 0) {
    set_last_error("zcu_paged_attention_noalloc: batch, hq and num_pages must be positive");
    return kBadArgument;
  }
  PagedAttnArgs a{};
  a.q = q;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.page_table = page_table;
  a.ctx_len = ctx_len;
  a.out = out;
  a.batch = batch;
  a.hq = hq;
  a.hkv = hkv;
  a.hd = hd;
  a.page_size = page_size;
  a.max_pages = max_pages;
  a.num_pages = num_pages;
  a.page_stride = page_stride;
  a.slot_stride = slot_stride;
  a.head_stride = head_stride;
  a.scale = scale;
  a.kv_half = kv_dtype == 1;
  a.max_ctx = max_ctx;
  if (const int rc = paged_attention_check(a)) {
    set_last_error(rc == kUnsupported ? "zcu_paged_attention_noalloc: head size must be 8, 16, 32, 64, 128 or 256"
                                      : "zcu_paged_attention_noalloc: null pointer, or batch/hq/hkv/page_size/"
                                        "max_pages not positive, or hq not a multiple of hkv");
    return rc;
  }
  a.splits = paged_attention_choose_splits(batch, hkv, max_ctx, page_size);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (a.splits > 1) {
    const size_t partials = paged_attention_workspace_floats(batch, hq, hd, a.splits);
    const size_t counters = (size_t)batch * hq;
    if (partials > kPartialFloats || counters > kCounterInts) {
      set_last_error("zcu_paged_attention_noalloc: this shape needs " + std::to_string(partials) +
                     " partial floats and " + std::to_string(counters) + " counters of scratch; the fixed scratch " +
                     "holds " + std::to_string(kPartialFloats) + " and " + std::to_string(kCounterInts));
      return kTooLarge;
    }
    void* base = nullptr;
    const int rc = scratch_for_current_device(&base);
    if (rc != kOk) return rc;
    int* ctr = static_cast<int*>(base);
    if (cudaMemsetAsync(ctr, 0, counters * sizeof(int), s) != cudaSuccess) {
      set_last_error(std::string("zcu_paged_attention_noalloc: clearing the counters failed: ") +
                     cudaGetErrorString(cudaGetLastError()));
      return kCudaError;
    }
    a.counters = ctr;
    a.workspace = reinterpret_cast<float*>(static_cast<char*>(base) + kCounterInts * sizeof(int));
  }
  const int rc = paged_attention(a, s);
  if (rc != kOk) set_last_error("zcu_paged_attention_noalloc: launch failed or shape unsupported");
  return rc;
}
