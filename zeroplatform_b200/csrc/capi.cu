// capi.cu -- extern "C" entry points of libzero_tensor.so (declared in include/zero_tensor.h and
// include/zero_tensor_cuda.h).
//
// Host-pointer entries (zc_*) follow the ZeroTensor native-bridge contract
// (ZeroTensor/src/ZeroTensor.Core/Native/ZeroTensorNativeBridge.cs:93-389): synchronous, caller-owned
// host buffers, 0 = handled.  Each host thread gets its own non-blocking CUDA stream and grow-only
// device staging buffers per device, so concurrent callers (Parallel.For workers) never share state.
// Device-pointer entries (zcu_*) only enqueue work on the caller's stream.

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "../../include/zero_tensor.h"
#include "../../include/zero_tensor_cuda.h"
#include "allreduce_p2p.h"
#include "common.cuh"
#include "kernels.h"

namespace {

using namespace zc;

thread_local std::string t_last_error;

int fail(int code, const char* what) {
  t_last_error = what;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  char buf[256];
  std::snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
  t_last_error = buf;
  return kCudaError;
}

#define ZC_CUDA(call)                                   \
  do {                                                  \
    cudaError_t e_ = (call);                            \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
  } while (0)

#define ZC_RC(call)                                              \
  do {                                                           \
    int rc_ = (call);                                            \
    if (rc_ != kOk) {                                            \
      if (t_last_error.empty()) t_last_error = #call " failed"; \
      return rc_;                                                \
    }                                                            \
  } while (0)

// Per-thread, per-device staging context for the host-pointer entries.  Contexts live until the process
// exits (the driver releases their memory); freeing them from thread-exit destructors could run after
// the CUDA runtime has been torn down.
struct HostCtx {
  int device = -1;
  cudaStream_t stream = nullptr;
  void* buf[8] = {};
  size_t cap[8] = {};
  // Registered-weight calls: x and y pass through pinned host buffers mapped into the device's address space
  // (copied by kernels, no DMA set-up), and the fetch -> GEMV -> store sequence of each registered tensor is
  // replayed as one CUDA graph.  Graphs name the staging buffers, so any reallocation drops them all.
  void* pin[2] = {};  // [0] x, [1] y (host pointers; the device uses the same addresses)
  size_t pin_cap[2] = {};
  std::map<uint64_t, cudaGraphExec_t> graphs;  // registration id -> fetch x, GEMV, store y
};

void drop_graphs(HostCtx* c) {
  for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second);
  c->graphs.clear();
}
thread_local std::vector<HostCtx*> t_ctx;

int host_ctx(HostCtx** out) {
  int dev = 0;
  ZC_CUDA(cudaGetDevice(&dev));
  for (HostCtx* c : t_ctx)
    if (c->device == dev) {
      *out = c;
      return kOk;
    }
  HostCtx* c = new HostCtx();
  c->device = dev;
  ZC_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
  t_ctx.push_back(c);
  *out = c;
  return kOk;
}

int staging(HostCtx* c, int slot, size_t bytes, void** p) {
  if (bytes == 0) bytes = 16;
  if (c->cap[slot] < bytes) {
    drop_graphs(c);
    if (c->buf[slot]) {
      ZC_CUDA(cudaStreamSynchronize(c->stream));
      ZC_CUDA(cudaFree(c->buf[slot]));
      c->buf[slot] = nullptr;
      c->cap[slot] = 0;
    }
    size_t cap = std::max(bytes, c->cap[slot] * 2);
    if (cudaMalloc(&c->buf[slot], cap) != cudaSuccess) {
      cudaGetLastError();
      return fail(kOutOfMemory, "device staging allocation failed");
    }
    c->cap[slot] = cap;
  }
  *p = c->buf[slot];
  return kOk;
}

// Pinned, device-mapped host buffer `slot` of at least `bytes` (grow-only).
int pinned(HostCtx* c, int slot, size_t bytes, void** p) {
  if (bytes == 0) bytes = 16;
  if (c->pin_cap[slot] < bytes) {
    drop_graphs(c);
    if (c->pin[slot]) {
      ZC_CUDA(cudaStreamSynchronize(c->stream));
      ZC_CUDA(cudaFreeHost(c->pin[slot]));
      c->pin[slot] = nullptr;
      c->pin_cap[slot] = 0;
    }
    const size_t cap = std::max(bytes, c->pin_cap[slot] * 2);
    if (cudaHostAlloc(&c->pin[slot], cap, cudaHostAllocMapped) != cudaSuccess) {
      cudaGetLastError();
      c->pin[slot] = nullptr;
      return fail(kOutOfMemory, "pinned staging allocation failed");
    }
    c->pin_cap[slot] = cap;
  }
  *p = c->pin[slot];
  return kOk;
}

int finish(HostCtx* c) {
  ZC_CUDA(cudaGetLastError());
  ZC_CUDA(cudaStreamSynchronize(c->stream));
  return kOk;
}

// Library-owned device scratch, one set of slots per (device, stream): calls on one stream are ordered,
// so they may share it; calls on different streams never do.  Slots: 0 attention split partials,
// 1 attention arrival counters (zeroed at allocation, left zeroed by every launch), 2 fp16 activations of
// the tensor-core GEMM.  A call that has to grow a slot allocates, which is not allowed while the stream
// is being captured into a CUDA graph: make one call of the same shape before capturing.
struct StreamScratch {
  void* buf[4] = {};
  size_t cap[4] = {};
};
std::mutex g_ws_mu;
std::map<std::pair<int, cudaStream_t>, StreamScratch> g_ws;

int stream_scratch(cudaStream_t s, int slot, size_t bytes, bool zeroed, void** out) {
  int dev = 0;
  ZC_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> g(g_ws_mu);
  StreamScratch& w = g_ws[{dev, s}];
  if (bytes == 0) bytes = 16;
  if (w.cap[slot] < bytes) {
    if (w.buf[slot]) {
      ZC_CUDA(cudaStreamSynchronize(s));
      ZC_CUDA(cudaFree(w.buf[slot]));
      w.buf[slot] = nullptr;
      w.cap[slot] = 0;
    }
    if (cudaMalloc(&w.buf[slot], bytes) != cudaSuccess) {
      cudaGetLastError();
      return fail(kOutOfMemory, "workspace allocation failed");
    }
    if (zeroed) ZC_CUDA(cudaMemsetAsync(w.buf[slot], 0, bytes, s));
    w.cap[slot] = bytes;
  }
  *out = w.buf[slot];
  return kOk;
}

int attn_workspace(cudaStream_t s, size_t floats, size_t counters, float** ws, int** ctr) {
  void *a, *b;
  ZC_RC(stream_scratch(s, 0, floats * sizeof(float), false, &a));
  ZC_RC(stream_scratch(s, 1, counters * sizeof(int), true, &b));
  *ws = static_cast<float*>(a);
  *ctr = static_cast<int*>(b);
  return kOk;
}

// Per-device status word written by kernels whose bounded waits expired (0 = healthy).
std::mutex g_status_mu;
std::map<int, int*> g_status;

int device_status_ptr(int** out) {
  int dev = 0;
  ZC_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> g(g_status_mu);
  int*& p = g_status[dev];
  if (!p) {
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) {
      cudaGetLastError();
      p = nullptr;
      return fail(kOutOfMemory, "status word allocation failed");
    }
    ZC_CUDA(cudaMemset(p, 0, sizeof(int)));
  }
  *out = p;
  return kOk;
}

int attention_device(const PagedAttnArgs& in, cudaStream_t s) {
  PagedAttnArgs a = in;
  int splits = paged_attention_choose_splits(a.batch, a.hkv, a.max_ctx, a.page_size);
  a.splits = splits;
  a.workspace = nullptr;
  a.counters = nullptr;
  if (splits > 1) {
    ZC_RC(attn_workspace(s, paged_attention_workspace_floats(a.batch, a.hq, a.hd, splits),
                         (size_t)a.batch * a.hq, &a.workspace, &a.counters));
  }
  return paged_attention(a, s);
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Weights registered with zc_register_weights: host pointer -> device-resident SoA copy.
struct Registered {
  uint64_t id = 0;  // unique per registration (keys the per-thread replay graphs)
  int qtype = 0;
  size_t n = 0, k = 0;
  int device = -1;
  void* qs = nullptr;
  void* d = nullptr;
};
std::mutex g_reg_mu;
std::map<std::pair<const uint8_t*, int>, Registered> g_reg;  // (host pointer, device)
uint64_t g_reg_next_id = 1;

bool find_registered(const uint8_t* w, int qtype, size_t n, size_t k, Registered* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> g(g_reg_mu);
  auto it = g_reg.find({w, dev});
  if (it == g_reg.end() || it->second.qtype != qtype || it->second.n != n || it->second.k != k) return false;
  *out = it->second;
  return true;
}

int gemv_host(int qtype, const uint8_t* w, const float* x, float* y, size_t n, size_t k) {
  if (!w || !x || !y) return fail(kBadArgument, "null pointer");
  if (k == 0 || k % QK) return fail(kBadArgument, "k_cols must be a positive multiple of 32");
  if (n == 0) return kOk;
  if (n > 0x7fffffff || k > 0x7fffffff) return fail(kUnsupported, "dimension too large");
  HostCtx* c = nullptr;
  ZC_RC(host_ctx(&c));
  Registered reg;
  if (find_registered(w, qtype, n, k, &reg)) {  // resident weights: only x and y cross PCIe
    void *d_x, *d_y, *h_x, *h_y;
    ZC_RC(staging(c, 3, k * sizeof(float), &d_x));
    ZC_RC(staging(c, 4, n * sizeof(float), &d_y));
    ZC_RC(pinned(c, 0, k * sizeof(float), &h_x));
    ZC_RC(pinned(c, 1, n * sizeof(float), &h_y));
    std::memcpy(h_x, x, k * sizeof(float));
    // fetch x over the bus, the GEMV (its weight loads start while x is in flight), store y over the bus
    auto enqueue = [&]() -> int {
      ZC_RC(copy_words(h_x, d_x, k * sizeof(float), c->stream));
      if (qtype == 8)
        ZC_RC(gemv_q8_0((const int8_t*)reg.qs, (const uint16_t*)reg.d, (const float*)d_x, (float*)d_y, (int)n,
                        (int)k, 0, c->stream));
      else
        ZC_RC(gemv_q4_0((const uint8_t*)reg.qs, (const uint16_t*)reg.d, (const float*)d_x, (float*)d_y, (int)n,
                        (int)k, 0, c->stream));
      return copy_words(d_y, h_y, n * sizeof(float), c->stream);
    };
    auto it = c->graphs.find(reg.id);
    if (it != c->graphs.end()) {
      ZC_CUDA(cudaGraphLaunch(it->second, c->stream));
    } else {
      ZC_RC(enqueue());  // first call of this tensor on this thread: run directly, then record the graph
      ZC_RC(finish(c));
      if (c->graphs.size() >= 256) drop_graphs(c);
      cudaGraph_t g = nullptr;
      cudaGraphExec_t ge = nullptr;
      ZC_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
      const int rc = enqueue();
      const cudaError_t ec = cudaStreamEndCapture(c->stream, &g);
      if (rc != kOk) {
        if (g) cudaGraphDestroy(g);
        return rc;
      }
      ZC_CUDA(ec);
      const cudaError_t ei = cudaGraphInstantiate(&ge, g, 0);
      cudaGraphDestroy(g);
      ZC_CUDA(ei);
      c->graphs[reg.id] = ge;
    }
    ZC_RC(finish(c));
    std::memcpy(y, h_y, n * sizeof(float));
    return kOk;
  }
  const size_t nb = n * (k / QK);
  const size_t aos_bytes = nb * (qtype == 8 ? Q8_BLOCK_BYTES : Q4_BLOCK_BYTES);
  const size_t qs_bytes = qtype == 8 ? n * k : n * k / 2;
  void *d_aos, *d_qs, *d_d, *d_x, *d_y;
  ZC_RC(staging(c, 0, aos_bytes, &d_aos));
  ZC_RC(staging(c, 1, qs_bytes, &d_qs));
  ZC_RC(staging(c, 2, nb * 2, &d_d));
  ZC_RC(staging(c, 3, k * sizeof(float), &d_x));
  ZC_RC(staging(c, 4, n * sizeof(float), &d_y));
  ZC_CUDA(cudaMemcpyAsync(d_aos, w, aos_bytes, cudaMemcpyHostToDevice, c->stream));
  ZC_CUDA(cudaMemcpyAsync(d_x, x, k * sizeof(float), cudaMemcpyHostToDevice, c->stream));
  if (qtype == 8) {
    ZC_RC(repack_q8_0((const uint8_t*)d_aos, (int8_t*)d_qs, (uint16_t*)d_d, n, k, c->stream));
    ZC_RC(gemv_q8_0((const int8_t*)d_qs, (const uint16_t*)d_d, (const float*)d_x, (float*)d_y, (int)n, (int)k, 0,
                    c->stream));
  } else {
    ZC_RC(repack_q4_0((const uint8_t*)d_aos, (uint8_t*)d_qs, (uint16_t*)d_d, n, k, c->stream));
    ZC_RC(gemv_q4_0((const uint8_t*)d_qs, (const uint16_t*)d_d, (const float*)d_x, (float*)d_y, (int)n, (int)k, 0,
                    c->stream));
  }
  ZC_CUDA(cudaMemcpyAsync(y, d_y, n * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
  return finish(c);
}

}  // namespace

namespace zc {
void set_last_error(const std::string& msg) { t_last_error = msg; }
}  // namespace zc

extern "C" {

// ------------------------------------------------------------------------------------------
// Reference bridge ABI (include/zero_tensor.h)
// ------------------------------------------------------------------------------------------
uint32_t zc_version(void) { return (0u << 16) | (1u << 8) | 0u; }

int32_t zc_is_simd_supported(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return 0;
  }
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return major == 10 ? 1 : 0;
}

const char* zc_cuda_last_error(void) { return t_last_error.c_str(); }

int32_t zc_gemv_q8_0(const uint8_t* w, const float* x, float* y, size_t n_rows, size_t k_cols) {
  t_last_error.clear();
  return gemv_host(8, w, x, y, n_rows, k_cols);
}

int32_t zc_gemv_q4_0(const uint8_t* w, const float* x, float* y, size_t n_rows, size_t k_cols) {
  t_last_error.clear();
  return gemv_host(4, w, x, y, n_rows, k_cols);
}

int32_t zc_register_weights(int32_t ggml_type, const uint8_t* w, size_t n_rows, size_t k_cols) {
  t_last_error.clear();
  const int qtype = ggml_type == 8 ? 8 : (ggml_type == 2 ? 4 : 0);
  if (!qtype) return fail(kUnsupported, "only Q8_0 (8) and Q4_0 (2) tensors can be registered");
  if (!w || n_rows == 0 || k_cols == 0 || k_cols % QK) return fail(kBadArgument, "bad weight tensor");
  if (n_rows > 0x7fffffff || k_cols > 0x7fffffff) return fail(kUnsupported, "dimension too large");
  int dev = 0;
  ZC_CUDA(cudaGetDevice(&dev));
  zc_unregister_weights(w);
  HostCtx* c = nullptr;
  ZC_RC(host_ctx(&c));
  const size_t nb = n_rows * (k_cols / QK);
  const size_t aos_bytes = nb * (qtype == 8 ? Q8_BLOCK_BYTES : Q4_BLOCK_BYTES);
  Registered r;
  r.qtype = qtype;
  r.n = n_rows;
  r.k = k_cols;
  r.device = dev;
  if (cudaMalloc(&r.qs, qtype == 8 ? n_rows * k_cols : n_rows * k_cols / 2) != cudaSuccess ||
      cudaMalloc(&r.d, nb * 2) != cudaSuccess) {
    cudaGetLastError();
    if (r.qs) cudaFree(r.qs);
    return fail(kOutOfMemory, "device allocation for registered weights failed");
  }
  void* d_aos;
  int rc = staging(c, 0, aos_bytes, &d_aos);
  if (rc == kOk && cudaMemcpyAsync(d_aos, w, aos_bytes, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
    rc = cuda_fail(cudaGetLastError(), "cudaMemcpyAsync(weights)");
  if (rc == kOk)
    rc = qtype == 8 ? repack_q8_0((const uint8_t*)d_aos, (int8_t*)r.qs, (uint16_t*)r.d, n_rows, k_cols, c->stream)
                    : repack_q4_0((const uint8_t*)d_aos, (uint8_t*)r.qs, (uint16_t*)r.d, n_rows, k_cols, c->stream);
  if (rc == kOk) rc = finish(c);
  if (rc != kOk) {
    cudaFree(r.qs);
    cudaFree(r.d);
    return rc;
  }
  std::lock_guard<std::mutex> g(g_reg_mu);
  r.id = g_reg_next_id++;
  g_reg[{w, dev}] = r;
  return kOk;
}

int32_t zc_unregister_weights(const uint8_t* w) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return kCudaError;
  }
  Registered r;
  {
    std::lock_guard<std::mutex> g(g_reg_mu);
    auto it = g_reg.find({w, dev});
    if (it == g_reg.end()) return kNotHandled;
    r = it->second;
    g_reg.erase(it);
  }
  cudaDeviceSynchronize();  // no call may still be reading the copy
  cudaFree(r.qs);
  cudaFree(r.d);
  return kOk;
}

int32_t zc_gemm_f32(size_t m, size_t n, size_t k, float alpha, const float* a, intptr_t rsa, intptr_t csa,
                    const float* b, intptr_t rsb, intptr_t csb, float beta, float* c, intptr_t rsc, intptr_t csc,
                    int32_t parallel) {
  (void)parallel;
  t_last_error.clear();
  if (!a || !b || !c) return fail(kBadArgument, "null pointer");
  if (m == 0 || n == 0) return kOk;
  if (m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff) return fail(kUnsupported, "dimension too large");
  HostCtx* cx = nullptr;
  ZC_RC(host_ctx(&cx));
  // Pack the strided operands row-major on the host, run the GEMM, scatter C back.
  std::vector<float> ha(m * k), hb(k * n), hc(m * n);
  for (size_t i = 0; i < m; ++i)
    for (size_t p = 0; p < k; ++p) ha[i * k + p] = a[(intptr_t)i * rsa + (intptr_t)p * csa];
  for (size_t p = 0; p < k; ++p)
    for (size_t j = 0; j < n; ++j) hb[p * n + j] = b[(intptr_t)p * rsb + (intptr_t)j * csb];
  if (beta != 0.f)
    for (size_t i = 0; i < m; ++i)
      for (size_t j = 0; j < n; ++j) hc[i * n + j] = c[(intptr_t)i * rsc + (intptr_t)j * csc];
  void *da, *db, *dc;
  ZC_RC(staging(cx, 0, ha.size() * 4, &da));
  ZC_RC(staging(cx, 1, hb.size() * 4, &db));
  ZC_RC(staging(cx, 2, hc.size() * 4, &dc));
  ZC_CUDA(cudaMemcpyAsync(da, ha.data(), ha.size() * 4, cudaMemcpyHostToDevice, cx->stream));
  ZC_CUDA(cudaMemcpyAsync(db, hb.data(), hb.size() * 4, cudaMemcpyHostToDevice, cx->stream));
  if (beta != 0.f) ZC_CUDA(cudaMemcpyAsync(dc, hc.data(), hc.size() * 4, cudaMemcpyHostToDevice, cx->stream));
  ZC_RC(sgemm((int)m, (int)n, (int)k, alpha, (const float*)da, (const float*)db, beta, (float*)dc, cx->stream));
  ZC_CUDA(cudaMemcpyAsync(hc.data(), dc, hc.size() * 4, cudaMemcpyDeviceToHost, cx->stream));
  ZC_RC(finish(cx));
  for (size_t i = 0; i < m; ++i)
    for (size_t j = 0; j < n; ++j) c[(intptr_t)i * rsc + (intptr_t)j * csc] = hc[i * n + j];
  return kOk;
}

// TensorOps.FlashAttentionCpu's native dispatch (TensorOps.Neural.cs:1062-1080): q [batch][sq][d], k [kv batch][sk][d],
// v [kv batch][sk][dv], out [batch][sq][dv], kv batch of b = is_gqa ? (b / hq) * hkv + (b % hq) / group : b.  The ABI
// carries no mask extent, so the managed code's mask broadcast (batch b reads mask block b % (mask length / sq*sk))
// cannot be reproduced here: a call with a mask, or with a shape outside the kernel's (dv != d, d not 16 / 32 / 64 /
// 128, a grouped batch that is not a multiple of hq), returns -1 and the managed FlashAttention runs.
int32_t zc_flash_attention_f32(size_t batch, size_t sq, size_t sk, size_t d, size_t dv, float scale, int32_t is_gqa,
                               size_t hq, size_t hkv, size_t group, const float* q, const float* k, const float* v,
                               const float* mask, float* out) {
  t_last_error.clear();
  if (mask) {
    t_last_error = "zc_flash_attention_f32: an additive mask is not handled (the ABI carries no mask extent)";
    return kNotHandled;
  }
  if (!q || !k || !v || !out) return fail(kBadArgument, "null pointer");
  if (batch == 0 || sq == 0) return kOk;
  if (dv != d || (d != 16 && d != 32 && d != 64 && d != 128)) {
    t_last_error = "zc_flash_attention_f32: head sizes outside 16 / 32 / 64 / 128 (or dv != d) are not handled";
    return kNotHandled;
  }
  size_t seqs = batch, heads = 1, groups = 1, kv_heads = 1;
  if (is_gqa) {
    if (hq == 0 || hkv == 0 || group == 0 || hq != hkv * group || batch % hq) {
      t_last_error = "zc_flash_attention_f32: grouped batch does not split into hq heads";
      return kNotHandled;
    }
    seqs = batch / hq;
    heads = hq;
    groups = group;
    kv_heads = hkv;
  }
  if (seqs > 65535 || heads > 65535 || sq > 0x7fffffffu || sk > 0x7fffffffu || sq * d > (1ull << 40)) {
    t_last_error = "zc_flash_attention_f32: dimensions beyond the launch grid are not handled";
    return kNotHandled;
  }
  const size_t q_floats = batch * sq * d;
  const size_t kv_floats = seqs * kv_heads * sk * d;
  if (sk == 0) {  // no keys: every row's sum is 0 and the output is zeros (FlashAttentionComputeRow)
    std::memset(out, 0, q_floats * sizeof(float));
    return kOk;
  }
  HostCtx* c = nullptr;
  ZC_RC(host_ctx(&c));
  void *dq, *dk, *dv_, *dctx, *dpt, *dout;
  ZC_RC(staging(c, 0, q_floats * 4, &dq));
  ZC_RC(staging(c, 1, kv_floats * 4, &dk));
  ZC_RC(staging(c, 2, kv_floats * 4, &dv_));
  ZC_RC(staging(c, 3, sq * 4, &dctx));
  ZC_RC(staging(c, 4, 16, &dpt));
  ZC_RC(staging(c, 5, q_floats * 4, &dout));
  const std::vector<int32_t> ctx(sq, (int32_t)sk);
  const int32_t page0 = 0;
  ZC_CUDA(cudaMemcpyAsync(dq, q, q_floats * 4, cudaMemcpyHostToDevice, c->stream));
  ZC_CUDA(cudaMemcpyAsync(dk, k, kv_floats * 4, cudaMemcpyHostToDevice, c->stream));
  ZC_CUDA(cudaMemcpyAsync(dv_, v, kv_floats * 4, cudaMemcpyHostToDevice, c->stream));
  ZC_CUDA(cudaMemcpyAsync(dctx, ctx.data(), sq * 4, cudaMemcpyHostToDevice, c->stream));
  ZC_CUDA(cudaMemcpyAsync(dpt, &page0, 4, cudaMemcpyHostToDevice, c->stream));
  PrefillAttnArgs a{};
  a.q = (const float*)dq;
  a.k = dk;
  a.v = dv_;
  a.page_table = (const int32_t*)dpt;
  a.ctx_len = (const int32_t*)dctx;
  a.out = (float*)dout;
  a.rows = (int)sq;
  a.seqs = (int)seqs;
  a.hq = (int)heads;
  a.group = (int)groups;
  a.hd = (int)d;
  a.page_size = (int)sk;  // one page holds a kv batch's sk keys
  a.max_pages = 1;
  a.num_pages = 1;
  a.page_stride = 0;
  a.slot_stride = (long long)d;
  a.head_stride = (long long)(sk * d);
  a.kv_seq_stride = (long long)(kv_heads * sk * d);
  a.q_row_stride = (long long)d;
  a.q_head_stride = (long long)(sq * d);
  a.q_seq_stride = (long long)(heads * sq * d);
  a.pt_seq_stride = 0;
  a.ctx_seq_stride = 0;
  a.out_row_stride = a.q_row_stride;
  a.out_head_stride = a.q_head_stride;
  a.out_seq_stride = a.q_seq_stride;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.kv_half = 0;
  ZC_RC(prefill_attention(a, c->stream));
  ZC_CUDA(cudaMemcpyAsync(out, dout, q_floats * 4, cudaMemcpyDeviceToHost, c->stream));
  return finish(c);
}

int32_t zc_rmsnorm_f32(size_t n, const float* x, const float* w, float* dst, float eps) {
  t_last_error.clear();
  if (!x || !w || !dst) return fail(kBadArgument, "null pointer");
  if (n == 0) return kOk;
  if (n > 0x7fffffff) return fail(kUnsupported, "dimension too large");
  HostCtx* c = nullptr;
  ZC_RC(host_ctx(&c));
  void *dx, *dw, *dy;
  ZC_RC(staging(c, 0, n * 4, &dx));
  ZC_RC(staging(c, 1, n * 4, &dw));
  ZC_RC(staging(c, 2, n * 4, &dy));
  ZC_CUDA(cudaMemcpyAsync(dx, x, n * 4, cudaMemcpyHostToDevice, c->stream));
  ZC_CUDA(cudaMemcpyAsync(dw, w, n * 4, cudaMemcpyHostToDevice, c->stream));
  ZC_RC(rmsnorm((const float*)dx, (const float*)dw, (float*)dy, 1, (int)n, eps, c->stream));
  ZC_CUDA(cudaMemcpyAsync(dst, dy, n * 4, cudaMemcpyDeviceToHost, c->stream));
  return finish(c);
}

static int32_t unary_host(size_t n, const float* a, const float* b, float* dst, int op) {
  t_last_error.clear();
  if (!a || !dst || (op == 1 && !b)) return fail(kBadArgument, "null pointer");
  if (n == 0) return kOk;
  HostCtx* c = nullptr;
  ZC_RC(host_ctx(&c));
  void *da, *db, *dy;
  ZC_RC(staging(c, 0, n * 4, &da));
  ZC_RC(staging(c, 1, n * 4, &db));
  ZC_RC(staging(c, 2, n * 4, &dy));
  ZC_CUDA(cudaMemcpyAsync(da, a, n * 4, cudaMemcpyHostToDevice, c->stream));
  if (op == 1) {
    ZC_CUDA(cudaMemcpyAsync(db, b, n * 4, cudaMemcpyHostToDevice, c->stream));
    ZC_RC(swiglu((const float*)da, (const float*)db, (float*)dy, n, c->stream));
  } else {
    ZC_RC(silu((const float*)da, (float*)dy, n, c->stream));
  }
  ZC_CUDA(cudaMemcpyAsync(dst, dy, n * 4, cudaMemcpyDeviceToHost, c->stream));
  return finish(c);
}

int32_t zc_silu_f32(size_t n, const float* src, float* dst) { return unary_host(n, src, nullptr, dst, 0); }

int32_t zc_swiglu_f32(size_t n, const float* gate, const float* up, float* dst) {
  return unary_host(n, gate, up, dst, 1);
}

int32_t zc_rope_f32(size_t num_heads, size_t seq_len, size_t head_dim, size_t pos_offset, float theta_base,
                    float* x) {
  t_last_error.clear();
  if (!x) return fail(kBadArgument, "null pointer");
  if (head_dim == 0 || (head_dim & 1)) return fail(kBadArgument, "head_dim must be even");
  const size_t n = num_heads * seq_len * head_dim;
  if (n == 0) return kOk;
  HostCtx* c = nullptr;
  ZC_RC(host_ctx(&c));
  void* dx;
  ZC_RC(staging(c, 0, n * 4, &dx));
  ZC_CUDA(cudaMemcpyAsync(dx, x, n * 4, cudaMemcpyHostToDevice, c->stream));
  ZC_RC(rope_tensorops((float*)dx, (int)num_heads, (int)seq_len, (int)head_dim, (int)pos_offset, theta_base,
                       c->stream));
  ZC_CUDA(cudaMemcpyAsync(x, dx, n * 4, cudaMemcpyDeviceToHost, c->stream));
  return finish(c);
}

int32_t zc_paged_attention_f32(size_t hq, size_t hkv, size_t hd, size_t block_size, size_t ctx_len, float scale,
                               const float* q, const float* k_cache, const float* v_cache, const int32_t* block_table,
                               float* out) {
  t_last_error.clear();
  if (!q || !out) return fail(kBadArgument, "null pointer");
  if (hq == 0 || hkv == 0 || hq % hkv || hd == 0 || block_size == 0) return fail(kBadArgument, "bad head geometry");
  if (hq > 4096 || hd > 4096 || block_size > 65536 || ctx_len > (1u << 28))
    return fail(kUnsupported, "dimension too large");
  if (ctx_len > 0 && (!k_cache || !v_cache || !block_table)) return fail(kBadArgument, "null pointer");
  HostCtx* c = nullptr;
  ZC_RC(host_ctx(&c));
  const size_t nlb = (ctx_len + block_size - 1) / block_size;
  const size_t blk_floats = block_size * hkv * hd;
  // Gather the referenced blocks into a compact device pool (logical order), so that only the pages
  // the table names cross PCIe; the ABI does not carry the pool's extent.
  int32_t max_id = -1;
  for (size_t i = 0; i < nlb; ++i) {
    if (block_table[i] < 0) return fail(kBadArgument, "negative block id");
    max_id = std::max(max_id, block_table[i]);
  }
  void *dq, *dk, *dv, *dpt, *dctx, *dout;
  ZC_RC(staging(c, 0, hq * hd * 4, &dq));
  ZC_RC(staging(c, 1, std::max<size_t>(nlb, 1) * blk_floats * 4, &dk));
  ZC_RC(staging(c, 2, std::max<size_t>(nlb, 1) * blk_floats * 4, &dv));
  ZC_RC(staging(c, 3, std::max<size_t>(nlb, 1) * 4 + 4, &dpt));
  ZC_RC(staging(c, 4, 16, &dctx));
  ZC_RC(staging(c, 5, hq * hd * 4, &dout));
  std::vector<int32_t> ident(std::max<size_t>(nlb, 1));
  for (size_t i = 0; i < ident.size(); ++i) ident[i] = (int32_t)i;
  const int32_t ctx32 = (int32_t)ctx_len;
  ZC_CUDA(cudaMemcpyAsync(dq, q, hq * hd * 4, cudaMemcpyHostToDevice, c->stream));
  for (size_t i = 0; i < nlb; ++i) {
    const size_t src = (size_t)block_table[i] * blk_floats;
    ZC_CUDA(cudaMemcpyAsync((float*)dk + i * blk_floats, k_cache + src, blk_floats * 4, cudaMemcpyHostToDevice,
                            c->stream));
    ZC_CUDA(cudaMemcpyAsync((float*)dv + i * blk_floats, v_cache + src, blk_floats * 4, cudaMemcpyHostToDevice,
                            c->stream));
  }
  ZC_CUDA(cudaMemcpyAsync(dpt, ident.data(), ident.size() * 4, cudaMemcpyHostToDevice, c->stream));
  ZC_CUDA(cudaMemcpyAsync(dctx, &ctx32, 4, cudaMemcpyHostToDevice, c->stream));
  PagedAttnArgs a{};
  a.q = (const float*)dq;
  a.k_pool = dk;
  a.v_pool = dv;
  a.page_table = (const int32_t*)dpt;
  a.ctx_len = (const int32_t*)dctx;
  a.out = (float*)dout;
  a.batch = 1;
  a.hq = (int)hq;
  a.hkv = (int)hkv;
  a.hd = (int)hd;
  a.page_size = (int)block_size;
  a.max_pages = (int)std::max<size_t>(nlb, 1);
  a.num_pages = (int)std::max<size_t>(nlb, 1);
  a.page_stride = (long long)blk_floats;
  a.slot_stride = (long long)(hkv * hd);
  a.head_stride = (long long)hd;
  a.scale = scale;
  a.kv_half = 0;
  a.max_ctx = (int)ctx_len;
  int rc = attention_device(a, c->stream);
  if (rc != kOk) {
    if (t_last_error.empty()) t_last_error = "paged attention: unsupported head_dim or layout";
    cudaStreamSynchronize(c->stream);
    return rc;
  }
  ZC_CUDA(cudaMemcpyAsync(out, dout, hq * hd * 4, cudaMemcpyDeviceToHost, c->stream));
  (void)max_id;
  return finish(c);
}

int32_t zc_dot_i8(size_t n, const int8_t* a, const int8_t* b, int32_t* out) {
  t_last_error.clear();
  // an empty managed array pinned with `fixed` arrives as a null pointer
  if (!out || (n > 0 && (!a || !b))) return fail(kBadArgument, "null pointer");
  HostCtx* c = nullptr;
  ZC_RC(host_ctx(&c));
  void *da, *db, *dr;
  ZC_RC(staging(c, 0, n, &da));
  ZC_RC(staging(c, 1, n, &db));
  ZC_RC(staging(c, 2, 16, &dr));
  if (n) {
    ZC_CUDA(cudaMemcpyAsync(da, a, n, cudaMemcpyHostToDevice, c->stream));
    ZC_CUDA(cudaMemcpyAsync(db, b, n, cudaMemcpyHostToDevice, c->stream));
  }
  ZC_RC(dot_i8((const int8_t*)da, (const int8_t*)db, n, (int32_t*)dr, c->stream));
  ZC_CUDA(cudaMemcpyAsync(out, dr, 4, cudaMemcpyDeviceToHost, c->stream));
  return finish(c);
}

// ------------------------------------------------------------------------------------------
// Device-pointer extension (include/zero_tensor_cuda.h)
// ------------------------------------------------------------------------------------------
int32_t zcu_quantize_q8_0(const float* src, uint8_t* blocks, size_t n, void* stream) {
  return quantize_q8_0(src, blocks, n, as_stream(stream));
}

int32_t zcu_quantize_q4_0(const float* src, uint8_t* blocks, size_t n, void* stream) {
  return quantize_q4_0(src, blocks, n, as_stream(stream));
}

int32_t zcu_q8_0_repack(const uint8_t* aos, int8_t* qs, uint16_t* d, size_t n_rows, size_t k_cols, void* stream) {
  return repack_q8_0(aos, qs, d, n_rows, k_cols, as_stream(stream));
}

int32_t zcu_q4_0_repack(const uint8_t* aos, uint8_t* qs, uint16_t* d, size_t n_rows, size_t k_cols, void* stream) {
  return repack_q4_0(aos, qs, d, n_rows, k_cols, as_stream(stream));
}

int32_t zcu_gemv_q8_0(const int8_t* qs, const uint16_t* d, const float* x, float* y, size_t n_rows, size_t k_cols,
                      int32_t accumulate, void* stream) {
  if (n_rows > 0x7fffffff || k_cols > 0x7fffffff) return kUnsupported;
  return gemv_q8_0(qs, d, x, y, (int)n_rows, (int)k_cols, accumulate, as_stream(stream));
}

int32_t zcu_gemv_q4_0(const uint8_t* qs, const uint16_t* d, const float* x, float* y, size_t n_rows, size_t k_cols,
                      int32_t accumulate, void* stream) {
  if (n_rows > 0x7fffffff || k_cols > 0x7fffffff) return kUnsupported;
  return gemv_q4_0(qs, d, x, y, (int)n_rows, (int)k_cols, accumulate, as_stream(stream));
}

int32_t zcu_gemm_q8_0(const int8_t* qs, const uint16_t* d, const float* x, float* y, size_t m, size_t n_rows,
                      size_t k_cols, int32_t accumulate, void* stream) {
  t_last_error.clear();
  if (m > 0x7fffffff || n_rows > 0x7fffffff || k_cols > 0x7fffffff) return fail(kUnsupported, "dimension too large");
  if (m == 0 || n_rows == 0) return kOk;
  cudaStream_t s = as_stream(stream);
  void* ws;
  int* status;
  const size_t bytes = gemm_q8_0_workspace_bytes((int)m, (int)n_rows, (int)k_cols);
  ZC_RC(stream_scratch(s, 2, bytes, false, &ws));
  ZC_RC(device_status_ptr(&status));
  return gemm_q8_0_tc(qs, d, x, y, (int)m, (int)n_rows, (int)k_cols, accumulate, ws, bytes, status, s);
}

int32_t zcu_gemm_q4_0(const uint8_t* qs, const uint16_t* d, const float* x, float* y, size_t m, size_t n_rows,
                      size_t k_cols, int32_t accumulate, void* stream) {
  t_last_error.clear();
  if (m > 0x7fffffff || n_rows > 0x7fffffff || k_cols > 0x7fffffff) return fail(kUnsupported, "dimension too large");
  if (m == 0 || n_rows == 0) return kOk;
  cudaStream_t s = as_stream(stream);
  void* ws;
  int* status;
  const size_t bytes = gemm_q8_0_workspace_bytes((int)m, (int)n_rows, (int)k_cols);
  ZC_RC(stream_scratch(s, 2, bytes, false, &ws));
  ZC_RC(device_status_ptr(&status));
  return gemm_q4_0_tc(qs, d, x, y, (int)m, (int)n_rows, (int)k_cols, accumulate, ws, bytes, status, s);
}

int32_t zcu_sample(float* logits, int32_t rows, int32_t vocab, const int32_t* past, const int32_t* past_len,
                   int32_t past_cap, const zcu_sampling_config* cfg, const float* uniforms, int32_t* out,
                   int32_t* cand_idx, float* cand_p, int32_t* n_cand, int32_t cand_cap, void* stream) {
  t_last_error.clear();
  if (!cfg) return fail(kBadArgument, "null sampling config");
  if (cfg->top_k < 0) return fail(kBadArgument, "top_k must be >= 0");
  if ((cand_idx || cand_p) && cand_cap <= 0) return fail(kBadArgument, "cand_cap must be positive");
  const SampleConfig c{cfg->temperature, cfg->top_p, cfg->min_p, cfg->top_k, cfg->repetition_penalty};
  const int rc = sample_rows(logits, rows, vocab, past, past_len, past_cap, c, uniforms, out, cand_idx, cand_p, n_cand,
                             cand_cap, as_stream(stream));
  if (rc != kOk) return fail(rc, rc == kBadArgument ? "null buffer or non-positive rows / vocab (a non-greedy config "
                                                      "needs uniforms)"
                                                    : "sampler launch failed");
  return kOk;
}

float zcu_sample_uniform(uint64_t seed, uint64_t i) { return splitmix_uniform(seed + i); }

int32_t zcu_peer_wait_selftest(int32_t ranks, int32_t wait_ms, uint32_t* seen) {
  t_last_error.clear();
  unsigned int st[16] = {};
  std::string err;
  const int rc = arp_wait_selftest(ranks, wait_ms, st, &err);
  if (rc < 0) return fail(rc, err.c_str());
  if (seen) std::memcpy(seen, st, sizeof(st));
  return rc;
}

int32_t zcu_device_status(int32_t reset) {
  int* p = nullptr;
  if (device_status_ptr(&p) != kOk) return kCudaError;
  int v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return cuda_fail(cudaGetLastError(), "reading the device status word");
  if (reset && v) cudaMemset(p, 0, sizeof(int));
  const int g = gemv_wait_status(reset);
  if (g < 0) return g;
  return v ? v : g;
}

int32_t zcu_paged_attention(const float* q, const void* k_pool, const void* v_pool, int32_t kv_dtype,
                            const int32_t* page_table, const int32_t* ctx_len, float* out, int32_t batch, int32_t hq,
                            int32_t hkv, int32_t hd, int32_t page_size, int32_t max_pages, int32_t num_pages,
                            int64_t page_stride, int64_t slot_stride, int64_t head_stride, float scale,
                            int32_t max_ctx, void* stream) {
  t_last_error.clear();
  if (num_pages <= 0) return fail(kBadArgument, "num_pages must be positive");
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
  if (const int rc = paged_attention_check(a))
    return fail(rc, rc == kUnsupported ? "head size must be 8, 16, 32, 64, 128 or 256"
                                       : "null pointer, or batch/hq/hkv/page_size/max_pages not positive, "
                                         "or hq not a multiple of hkv");
  return attention_device(a, as_stream(stream));
}

int32_t zcu_rmsnorm(const float* x, const float* w, float* out, int32_t rows, int32_t n, float eps, void* stream) {
  return rmsnorm(x, w, out, rows, n, eps, as_stream(stream));
}

int32_t zcu_swiglu(const float* gate, const float* up, float* out, size_t n, void* stream) {
  return swiglu(gate, up, out, n, as_stream(stream));
}

int32_t zcu_rope(float* x, int32_t rows, int32_t heads, int32_t hd, const int32_t* pos, int32_t pos0,
                 const float* cos_t, const float* sin_t, int32_t max_pos, void* stream) {
  return rope(x, rows, heads, hd, pos, pos0, cos_t, sin_t, max_pos, as_stream(stream));
}

int32_t zcu_embed_q8_0(const int8_t* qs, const uint16_t* d, const int32_t* tokens, int32_t n_tokens, int32_t vocab,
                       int32_t dim, float* out, void* stream) {
  return embed_q8_0(qs, d, tokens, n_tokens, vocab, dim, out, as_stream(stream));
}

}  // extern "C"
