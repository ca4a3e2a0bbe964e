// collective.cu -- NCCL communicator for the tensor-parallel and expert-parallel paths.
//
// libnccl is bound at run time with dlopen, not linked: a process that already loaded NCCL (PyTorch loads its
// own copy with libtorch_cuda) must use that same copy, or two NCCL versions would share one process.  The
// lookup order is: an NCCL already in the process (RTLD_NOLOAD on its soname), then $ZCU_NCCL_LIBRARY, then
// the dynamic linker's search for libnccl.so.2.  Only the types come from nccl.h.
//
// Every collective of a communicator is issued on the caller's stream; NCCL calls may be captured into a CUDA
// graph.  wait() replaces cudaStreamSynchronize on paths that contain collectives: it polls the stream and
// the communicator's asynchronous error, and after `timeout_ms` aborts the communicator so that a rank whose
// peer has died returns an error instead of blocking for ever.

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include "../../include/zero_tensor_cuda.h"
#include "collective.h"
#include "common.cuh"

namespace zc {

// Message for zc_cuda_last_error() on the calling thread (capi.cu).
void set_last_error(const std::string& msg);

namespace {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  ncclResult_t (*GetVersion)(int*) = nullptr;
  void* handle = nullptr;
  std::string error;
};

std::mutex g_api_mu;
NcclApi* g_api = nullptr;

template <class F>
bool bind(void* h, const char* name, F& fn) {
  fn = reinterpret_cast<F>(dlsym(h, name));
  return fn != nullptr;
}

const NcclApi* api(std::string* err) {
  std::lock_guard<std::mutex> g(g_api_mu);
  if (g_api) {
    if (!g_api->handle && err) *err = g_api->error;
    return g_api->handle ? g_api : nullptr;
  }
  g_api = new NcclApi();
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (!h) {
    const char* env = std::getenv("ZCU_NCCL_LIBRARY");
    if (env && *env) h = dlopen(env, RTLD_NOW | RTLD_GLOBAL);
  }
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) {
    const char* e = dlerror();
    g_api->error = std::string("libnccl.so.2 could not be loaded: ") + (e ? e : "unknown");
    if (err) *err = g_api->error;
    return nullptr;
  }
  bool ok = bind(h, "ncclGetUniqueId", g_api->GetUniqueId) && bind(h, "ncclCommInitRank", g_api->CommInitRank) &&
            bind(h, "ncclCommDestroy", g_api->CommDestroy) && bind(h, "ncclCommAbort", g_api->CommAbort) &&
            bind(h, "ncclCommGetAsyncError", g_api->CommGetAsyncError) &&
            bind(h, "ncclAllReduce", g_api->AllReduce) && bind(h, "ncclAllGather", g_api->AllGather) &&
            bind(h, "ncclSend", g_api->Send) && bind(h, "ncclRecv", g_api->Recv) &&
            bind(h, "ncclGroupStart", g_api->GroupStart) && bind(h, "ncclGroupEnd", g_api->GroupEnd) &&
            bind(h, "ncclGetErrorString", g_api->GetErrorString) && bind(h, "ncclGetVersion", g_api->GetVersion);
  if (!ok) {
    g_api->error = "libnccl.so.2 lacks a required symbol";
    if (err) *err = g_api->error;
    return nullptr;
  }
  g_api->handle = h;
  return g_api;
}

std::string nccl_msg(const NcclApi* a, const char* what, ncclResult_t r) {
  return std::string(what) + ": " + (a && a->GetErrorString ? a->GetErrorString(r) : "nccl error");
}

}  // namespace

struct Comm {
  ncclComm_t comm = nullptr;
  int rank = 0, size = 1;
  bool aborted = false;
};

int comm_unique_id(void* out, size_t cap, std::string* err) {
  if (!out || cap < sizeof(ncclUniqueId)) {
    if (err) *err = "the unique-id buffer must hold 128 bytes";
    return kBadArgument;
  }
  const NcclApi* a = api(err);
  if (!a) return kUnsupported;
  ncclUniqueId id;
  const ncclResult_t r = a->GetUniqueId(&id);
  if (r != ncclSuccess) {
    if (err) *err = nccl_msg(a, "ncclGetUniqueId", r);
    return kCudaError;
  }
  std::memcpy(out, &id, sizeof(id));
  return kOk;
}

int comm_create(int size, int rank, const void* id, Comm** out, std::string* err) {
  if (size < 1 || rank < 0 || rank >= size || !out || (size > 1 && !id)) {
    if (err) *err = "bad communicator rank/size/id";
    return kBadArgument;
  }
  Comm* c = new Comm();
  c->rank = rank;
  c->size = size;
  if (size > 1) {
    const NcclApi* a = api(err);
    if (!a) {
      delete c;
      return kUnsupported;
    }
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    const ncclResult_t r = a->CommInitRank(&c->comm, size, uid, rank);
    if (r != ncclSuccess) {
      if (err) *err = nccl_msg(a, "ncclCommInitRank", r);
      delete c;
      return kCudaError;
    }
  }
  *out = c;
  return kOk;
}

void comm_destroy(Comm* c) {
  if (!c) return;
  if (c->comm) {
    const NcclApi* a = api(nullptr);
    if (a) (c->aborted ? a->CommAbort : a->CommDestroy)(c->comm);
  }
  delete c;
}

int comm_rank(const Comm* c) { return c ? c->rank : 0; }
int comm_size(const Comm* c) { return c ? c->size : 1; }

int comm_allreduce_sum_f32(Comm* c, float* buf, size_t count, cudaStream_t s, std::string* err) {
  if (!c || c->size == 1 || count == 0) return kOk;
  const NcclApi* a = api(err);
  if (!a) return kUnsupported;
  const ncclResult_t r = a->AllReduce(buf, buf, count, ncclFloat32, ncclSum, c->comm, s);
  if (r != ncclSuccess) {
    if (err) *err = nccl_msg(a, "ncclAllReduce", r);
    return kCudaError;
  }
  return kOk;
}

int comm_allgather_bytes(Comm* c, const void* send, void* recv, size_t bytes, cudaStream_t s, std::string* err) {
  if (!c || bytes == 0) return kOk;
  if (c->size == 1) {
    if (send != recv && cudaMemcpyAsync(recv, send, bytes, cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
      if (err) *err = "allgather copy failed";
      return kCudaError;
    }
    return kOk;
  }
  const NcclApi* a = api(err);
  if (!a) return kUnsupported;
  const ncclResult_t r = a->AllGather(send, recv, bytes, ncclUint8, c->comm, s);
  if (r != ncclSuccess) {
    if (err) *err = nccl_msg(a, "ncclAllGather", r);
    return kCudaError;
  }
  return kOk;
}

int comm_alltoallv_bytes(Comm* c, const void* send, const size_t* send_bytes, const size_t* send_off, void* recv,
                         const size_t* recv_bytes, const size_t* recv_off, cudaStream_t s, std::string* err) {
  if (!c) return kBadArgument;
  if (c->size == 1) {
    if (send_bytes[0] && cudaMemcpyAsync(static_cast<char*>(recv) + recv_off[0],
                                         static_cast<const char*>(send) + send_off[0], send_bytes[0],
                                         cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
      if (err) *err = "all-to-all local copy failed";
      return kCudaError;
    }
    return kOk;
  }
  const NcclApi* a = api(err);
  if (!a) return kUnsupported;
  ncclResult_t r = a->GroupStart();
  for (int p = 0; p < c->size && r == ncclSuccess; ++p) {
    if (send_bytes[p])
      r = a->Send(static_cast<const char*>(send) + send_off[p], send_bytes[p], ncclUint8, p, c->comm, s);
    if (r == ncclSuccess && recv_bytes[p])
      r = a->Recv(static_cast<char*>(recv) + recv_off[p], recv_bytes[p], ncclUint8, p, c->comm, s);
  }
  const ncclResult_t r2 = a->GroupEnd();
  if (r != ncclSuccess || r2 != ncclSuccess) {
    if (err) *err = nccl_msg(a, "all-to-all send/recv", r != ncclSuccess ? r : r2);
    return kCudaError;
  }
  return kOk;
}

int comm_wait(Comm* c, cudaStream_t s, int timeout_ms, std::string* err) {
  if (!c || c->size == 1) {
    const cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
      if (err) *err = std::string("cudaStreamSynchronize: ") + cudaGetErrorString(e);
      return kCudaError;
    }
    return kOk;
  }
  const NcclApi* a = api(err);
  const auto t0 = std::chrono::steady_clock::now();
  for (unsigned it = 0;; ++it) {
    const cudaError_t e = cudaStreamQuery(s);
    if (e == cudaSuccess) return kOk;
    if (e != cudaErrorNotReady) {
      if (err) *err = std::string("stream error: ") + cudaGetErrorString(e);
      return kCudaError;
    }
    ncclResult_t ae = ncclSuccess;
    if (a && a->CommGetAsyncError(c->comm, &ae) == ncclSuccess && ae != ncclSuccess && ae != ncclInProgress) {
      if (err) *err = nccl_msg(a, "communicator failed", ae);
      c->aborted = true;
      a->CommAbort(c->comm);
      c->comm = nullptr;
      return kCudaError;
    }
    const auto ms =
        std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if (timeout_ms > 0 && ms > timeout_ms) {
      if (err) *err = "collective did not complete within " + std::to_string(timeout_ms) + " ms (peer lost?)";
      if (a) a->CommAbort(c->comm);
      c->aborted = true;
      c->comm = nullptr;
      return kCudaError;
    }
    if (it > 64) std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

bool comm_usable(const Comm* c) { return c && (c->size == 1 || c->comm != nullptr); }

}  // namespace zc

extern "C" int32_t zcu_nccl_unique_id(uint8_t* out, size_t cap) {
  std::string err;
  const int rc = zc::comm_unique_id(out, cap, &err);
  zc::set_last_error(rc == zc::kOk ? std::string() : "zcu_nccl_unique_id: " + err);
  return rc;
}
