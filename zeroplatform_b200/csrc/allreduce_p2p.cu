// allreduce_p2p.cu -- one-shot all-reduce of the residual stream over NVLink peer memory (tensor parallelism).
//
// Every rank owns a receive area in its own HBM: two buffers (alternating with the all-reduce's parity), each
// holding one slot of `cap` floats per rank, plus one epoch flag per rank.  The areas are mapped into every peer
// with CUDA IPC, so a kernel reaches a peer's memory with ordinary loads and stores over NVLink (no TMA, no
// multicast).
//
//   push   each CTA stores its share of this rank's partial x[0, n) into slot[my rank] of every rank's
//          buffer (its own included); the last CTA to finish (arrival counter) publishes the new epoch into
//          every rank's flag[my rank] with a system-scope release
//   reduce every CTA waits (bounded) until all flags of its own area carry at least the epoch, then
//          x[i] = sum over ranks r = 0 .. W-1 of slot[r][i] -- the same order on every rank, so all ranks hold
//          bit-identical sums
//
// The epoch lives on the device (one counter per rank, advanced by the reduce kernel), so the pair can be
// captured in a CUDA graph and replayed.  Buffer reuse: all-reduce e writes buffer e % 2; before any rank
// pushes e + 2 into that buffer it has finished reduce e + 1, which waited for every peer's push e + 1, which
// each peer issued only after its own reduce e -- the last reader of buffer e % 2.  Waits are bounded: after
// 10 s (or a poll limit) the kernel records an error code in the status word and returns.  Callers keep the
// ranks' host threads in step around slow host work (graph capture) with a collective barrier, so a wait only
// covers the peers' kernel progress.

#include <cuda_runtime.h>

#include <algorithm>
#include <string>
#include <vector>

#include "allreduce_p2p.h"
#include "collective.h"
#include "common.cuh"

namespace zc {

namespace {

constexpr uint64_t AR_WAIT_NS = 10000000000ull;  // 10 s: peers run on other hosts threads and may lag
constexpr uint32_t AR_WAIT_POLLS = 1u << 30;

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct PeerPtrs {
  float* data[ARP_MAX_RANKS];          // each rank's receive area (two buffers of W slots)
  unsigned int* flag[ARP_MAX_RANKS];   // each rank's flags [W]
};

// The all-reduce pair is launched without programmatic dependent launch and never triggers its dependents early:
// a push starts only after everything before it in the stream has completed, and nothing after a reduce starts
// before it has completed, so the epoch and the arrival counters are never read and written by overlapping grids.
// The fused pair (arp_push_partials + arp_reduce_rmsnorm_h) is launched with programmatic dependent launch and
// waits (griddepcontrol.wait) before any read.  The push triggers its dependent first: the reduce's grid is
// launched only once every CTA of the push is resident, so its spinning CTAs never keep the push's CTAs off the
// SMs.  The reduce never triggers: like the plain pair, nothing after it starts before it has completed and
// advanced the epoch.
//
// Push: slot[me] of every rank's current buffer = sum over s < splits of src[s * stride + i] (+ resid[i]); the
// last CTA to finish publishes the new epoch into every rank's flag[me].
template <bool PDL>
__global__ void arp_push_kernel(const float* __restrict__ src, int splits, size_t stride,
                                const float* __restrict__ resid, size_t n, size_t cap, PeerPtrs peers, int W, int me,
                                const unsigned int* __restrict__ epoch, unsigned int* __restrict__ arrivals) {
  if (PDL) {
    pdl_trigger();
    pdl_wait();
  }
  __shared__ int last;
  const unsigned int e = *reinterpret_cast<const volatile unsigned int*>(epoch) + 1;
  const size_t buf = (size_t)(e & 1) * W * cap;
  const size_t n4 = n / 4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    float4 v = reinterpret_cast<const float4*>(src)[i];
    for (int sp = 1; sp < splits; ++sp) {
      const float4 u = reinterpret_cast<const float4*>(src + (size_t)sp * stride)[i];
      v.x += u.x;
      v.y += u.y;
      v.z += u.z;
      v.w += u.w;
    }
    if (resid) {  // y += W x on the rank that carries the residual: the sum of the splits, then the add
      const float4 u = reinterpret_cast<const float4*>(resid)[i];
      v.x = u.x + v.x;
      v.y = u.y + v.y;
      v.z = u.z + v.z;
      v.w = u.w + v.w;
    }
    for (int r = 0; r < W; ++r) reinterpret_cast<float4*>(peers.data[r] + buf + (size_t)me * cap)[i] = v;
  }
  for (size_t i = n4 * 4 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float v = src[i];
    for (int sp = 1; sp < splits; ++sp) v += src[(size_t)sp * stride + i];
    if (resid) v = resid[i] + v;
    for (int r = 0; r < W; ++r) peers.data[r][buf + (size_t)me * cap + i] = v;
  }
  // the last CTA publishes the epoch once every CTA's stores are visible system-wide
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(arrivals, 1u) == gridDim.x - 1;
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence_system();
    *arrivals = 0;
    for (int r = 0; r < W; ++r) st_release_sys(peers.flag[r] + me, e);
  }
}

// Thread 0 of the calling CTA waits (bounded) until every rank's flag in this rank's area carries at least the
// epoch e; returns 0 (and records the failure) when the wait ran out.
__device__ __forceinline__ int wait_flags(const unsigned int* flags, int W, unsigned int e, unsigned int* state,
                                          int* status, uint64_t wait_ns) {
  const uint64_t t0 = now_ns();
  for (int r = 0; r < W; ++r) {
    uint32_t polls = 0;
    // a peer may already have published e + 1 (it finished this all-reduce and pushed the next one into the
    // other buffer), so wait for "at least e", wrap-around safe
    while ((int)(ld_acquire_sys(flags + r) - e) < 0) {
      if (++polls > AR_WAIT_POLLS || now_ns() - t0 > wait_ns) {
        atomicExch(status, 21);
        // what the wait saw, for the host's error message: the epoch it needed and every rank's flag
        state[4] = e;
        for (int q = 0; q < W; ++q) state[5 + q] = flags[q];
        return 0;
      }
    }
  }
  return 1;
}

// The last CTA to leave advances the epoch (every CTA has read it by then).
__device__ __forceinline__ void depart(unsigned int* epoch, unsigned int* departures, unsigned int e) {
  __shared__ int last;
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(departures, 1u) == gridDim.x - 1;
  __syncthreads();
  if (last && threadIdx.x == 0) {
    *departures = 0;
    *epoch = e;
  }
}

// One CTA per row: x[row] = sum over ranks r = 0 .. W-1 of slot[r][row] (the same order on every rank), then
// out[row] = RmsNorm(x[row]) * w as fp16 hi / lo pairs [hi dim | lo dim] (the operand of the tensor-core GEMM
// that follows) -- the computation of rmsnorm_kernel<__half> on the reduced row.
__global__ void arp_reduce_rmsnorm_kernel(float* __restrict__ x, int dim, size_t cap, const float* __restrict__ area,
                                          const unsigned int* __restrict__ flags, int W, unsigned int* __restrict__ epoch,
                                          unsigned int* __restrict__ departures, int* __restrict__ status,
                                          const float* __restrict__ w, float eps, __half* __restrict__ out) {
  pdl_wait();
  __shared__ int ok;
  __shared__ float red[32];
  const unsigned int e = *reinterpret_cast<volatile unsigned int*>(epoch) + 1;
  if (threadIdx.x == 0) ok = wait_flags(flags, W, e, epoch, status, AR_WAIT_NS);
  __syncthreads();
  if (ok) {
    const float* buf = area + (size_t)(e & 1) * W * cap + (size_t)blockIdx.x * dim;
    float* xr = x + (size_t)blockIdx.x * dim;
    float ss = 0.f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
      float v = __ldcv(buf + i);
      for (int r = 1; r < W; ++r) v += __ldcv(buf + (size_t)r * cap + i);
      xr[i] = v;
      ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
      v = warp_sum(v);
      if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float inv = 1.0f / (float)sqrt((double)(red[0] / (float)dim + eps));
    __half* orow = out + (size_t)blockIdx.x * 2 * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) store_hl(orow + i, (size_t)dim, xr[i] * inv * w[i]);
  }
  depart(epoch, departures, e);
}

__global__ void arp_reduce_kernel(float* __restrict__ x, size_t n, size_t cap, const float* __restrict__ area,
                                  const unsigned int* __restrict__ flags, int W, unsigned int* __restrict__ epoch,
                                  unsigned int* __restrict__ departures, int* __restrict__ status, uint64_t wait_ns) {
  __shared__ int ok;
  const unsigned int e = *reinterpret_cast<volatile unsigned int*>(epoch) + 1;
  if (threadIdx.x == 0) ok = wait_flags(flags, W, e, epoch, status, wait_ns);
  __syncthreads();
  if (ok) {
    const float* buf = area + (size_t)(e & 1) * W * cap;
    const size_t n4 = n / 4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
      float4 s = __ldcv(reinterpret_cast<const float4*>(buf) + i);
      for (int r = 1; r < W; ++r) {
        const float4 v = __ldcv(reinterpret_cast<const float4*>(buf + (size_t)r * cap) + i);
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
      reinterpret_cast<float4*>(x)[i] = s;
    }
    for (size_t i = n4 * 4 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
      float s = __ldcv(buf + i);
      for (int r = 1; r < W; ++r) s += __ldcv(buf + (size_t)r * cap + i);
      x[i] = s;
    }
  }
  depart(epoch, departures, e);
}

}  // namespace

struct P2pAllReduce {
  int W = 1, me = 0;
  size_t cap = 0;                 // floats per slot
  float* area = nullptr;          // own receive area: 2 * W * cap floats
  unsigned int* flags = nullptr;  // own flags [W]
  unsigned int* state = nullptr;  // epoch, push arrivals, reduce departures, diagnostics of a timed-out wait
  int* status = nullptr;
  PeerPtrs peers{};
  std::vector<void*> opened;      // IPC mappings of the peers' allocations
  void* own_alloc = nullptr;
};

int arp_create(Comm* comm, size_t cap_floats, int* status, P2pAllReduce** out, std::string* err) {
  const int W = comm_size(comm), me = comm_rank(comm);
  if (W < 2 || W > ARP_MAX_RANKS || cap_floats == 0 || !out) {
    if (err) *err = "peer all-reduce needs 2 .. 8 ranks";
    return kUnsupported;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  P2pAllReduce* A = new P2pAllReduce();
  A->W = W;
  A->me = me;
  A->cap = (cap_floats + 3) / 4 * 4;
  A->status = status;
  // one allocation: [area: 2 * W * cap floats][flags: W uint32] (256-byte aligned pieces)
  const size_t area_bytes = 2 * (size_t)W * A->cap * sizeof(float);
  const size_t total = area_bytes + 256;
  auto fail = [&](const std::string& m) {
    if (err) *err = m;
    for (void* p : A->opened) cudaIpcCloseMemHandle(p);
    if (A->own_alloc) cudaFree(A->own_alloc);
    if (A->state) cudaFree(A->state);
    delete A;
    cudaGetLastError();
    return kCudaError;
  };
  if (cudaMalloc(&A->own_alloc, total) != cudaSuccess) return fail("peer all-reduce: allocation failed");
  if (cudaMemset(A->own_alloc, 0, total) != cudaSuccess) return fail("peer all-reduce: memset failed");
  // state: [0] epoch, [1] push arrivals, [2] reduce departures, [4] epoch a timed-out wait needed, [5..] flags
  if (cudaMalloc(&A->state, 16 * sizeof(unsigned int)) != cudaSuccess ||
      cudaMemset(A->state, 0, 16 * sizeof(unsigned int)) != cudaSuccess)
    return fail("peer all-reduce: state allocation failed");
  A->area = static_cast<float*>(A->own_alloc);
  A->flags = reinterpret_cast<unsigned int*>(static_cast<char*>(A->own_alloc) + area_bytes);
  // exchange IPC handles (all ranks) through the communicator
  cudaIpcMemHandle_t mine;
  if (cudaIpcGetMemHandle(&mine, A->own_alloc) != cudaSuccess) return fail("cudaIpcGetMemHandle failed");
  void* dbuf = nullptr;
  if (cudaMalloc(&dbuf, (size_t)(W + 1) * sizeof(mine)) != cudaSuccess) return fail("handle buffer allocation failed");
  std::vector<cudaIpcMemHandle_t> all(W);
  std::string e2;
  int rc = cudaMemcpy(dbuf, &mine, sizeof(mine), cudaMemcpyHostToDevice) == cudaSuccess ? kOk : kCudaError;
  if (rc == kOk) rc = comm_allgather_bytes(comm, dbuf, static_cast<char*>(dbuf) + sizeof(mine), sizeof(mine), 0, &e2);
  if (rc == kOk && cudaDeviceSynchronize() != cudaSuccess) rc = kCudaError;
  if (rc == kOk &&
      cudaMemcpy(all.data(), static_cast<char*>(dbuf) + sizeof(mine), W * sizeof(mine), cudaMemcpyDeviceToHost) !=
          cudaSuccess)
    rc = kCudaError;
  cudaFree(dbuf);
  if (rc != kOk) return fail("exchanging IPC handles failed: " + e2);
  for (int r = 0; r < W; ++r) {
    char* base = nullptr;
    if (r == me) {
      base = static_cast<char*>(A->own_alloc);
    } else {
      void* p = nullptr;
      if (cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
        return fail("cudaIpcOpenMemHandle failed (no peer access between these GPUs?)");
      A->opened.push_back(p);
      base = static_cast<char*>(p);
    }
    A->peers.data[r] = reinterpret_cast<float*>(base);
    A->peers.flag[r] = reinterpret_cast<unsigned int*>(base + area_bytes);
  }
  *out = A;
  return kOk;
}

void arp_destroy(P2pAllReduce* A) {
  if (!A) return;
  for (void* p : A->opened) cudaIpcCloseMemHandle(p);
  if (A->own_alloc) cudaFree(A->own_alloc);
  if (A->state) cudaFree(A->state);
  delete A;
}

size_t arp_capacity(const P2pAllReduce* A) { return A ? A->cap : 0; }

std::string arp_describe(const P2pAllReduce* A) {
  if (!A) return "";
  unsigned int st[16] = {};
  if (cudaMemcpy(st, A->state, sizeof(st), cudaMemcpyDeviceToHost) != cudaSuccess) return "(state unreadable)";
  std::string m = "peer all-reduce rank " + std::to_string(A->me) + ": epoch " + std::to_string(st[0]);
  if (st[4]) {
    m += ", a wait needed epoch " + std::to_string(st[4]) + " and saw flags";
    for (int q = 0; q < A->W; ++q) m += " " + std::to_string(st[5 + q]);
  }
  return m;
}

static int push_grid(size_t n) { return (int)std::min<size_t>((n / 4 + 255) / 256 + 1, 148 * 2); }

int arp_allreduce_sum(P2pAllReduce* A, float* x, size_t n, cudaStream_t s) {
  if (!A || n > A->cap) return kTooLarge;
  if (n == 0) return kOk;
  const int grid = push_grid(n);
  arp_push_kernel<false><<<grid, 256, 0, s>>>(x, 1, 0, (const float*)nullptr, n, A->cap, A->peers, A->W, A->me,
                                              A->state, A->state + 1);
  if (cudaPeekAtLastError() != cudaSuccess) return kCudaError;
  arp_reduce_kernel<<<grid, 256, 0, s>>>(x, n, A->cap, A->area, A->flags, A->W, A->state, A->state + 2, A->status,
                                         AR_WAIT_NS);
  return cudaPeekAtLastError() == cudaSuccess ? kOk : kCudaError;
}

int arp_wait_selftest(int W, int wait_ms, unsigned int* seen, std::string* err) {
  if (W < 2 || W > ARP_MAX_RANKS || wait_ms < 1 || wait_ms > 5000 || !seen) {
    if (err) *err = "peer wait self-test: W must be 2 .. 8, wait_ms 1 .. 5000";
    return kBadArgument;
  }
  constexpr size_t cap = 256;
  const size_t area_bytes = 2 * (size_t)W * cap * sizeof(float);
  // one allocation: [area][flags: 16 words][state: 16 words][status: 4 words][x: cap floats]
  const size_t total = area_bytes + 64 + 64 + 16 + cap * sizeof(float);
  char* base = nullptr;
  if (cudaMalloc(&base, total) != cudaSuccess) {
    cudaGetLastError();
    if (err) *err = "peer wait self-test: allocation failed";
    return kOutOfMemory;
  }
  float* area = reinterpret_cast<float*>(base);
  unsigned int* flags = reinterpret_cast<unsigned int*>(base + area_bytes);
  unsigned int* state = reinterpret_cast<unsigned int*>(base + area_bytes + 64);
  int* status = reinterpret_cast<int*>(base + area_bytes + 128);
  float* x = reinterpret_cast<float*>(base + area_bytes + 144);
  int rc = cudaMemset(base, 0, total) == cudaSuccess ? kOk : kCudaError;
  const unsigned int one = 1;  // rank 0 has published epoch 1; no peer ever does
  if (rc == kOk && cudaMemcpy(flags, &one, sizeof(one), cudaMemcpyHostToDevice) != cudaSuccess) rc = kCudaError;
  int code = 0;
  if (rc == kOk) {
    arp_reduce_kernel<<<1, 256>>>(x, cap, cap, area, flags, W, state, state + 2, status,
                                  (uint64_t)wait_ms * 1000000ull);
    if (cudaDeviceSynchronize() != cudaSuccess) rc = kCudaError;
  }
  if (rc == kOk && (cudaMemcpy(&code, status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess ||
                    cudaMemcpy(seen, state, 16 * sizeof(unsigned int), cudaMemcpyDeviceToHost) != cudaSuccess))
    rc = kCudaError;
  cudaFree(base);
  if (rc != kOk) {
    if (err) *err = std::string("peer wait self-test: ") + cudaGetErrorString(cudaGetLastError());
    return rc;
  }
  return code;
}

int arp_push_partials(P2pAllReduce* A, const float* part, int splits, size_t n, const float* resid, cudaStream_t s) {
  if (!A || n > A->cap) return kTooLarge;
  if (!part || splits < 1) return kBadArgument;
  if (n == 0) return kOk;
  return launch_pdl(arp_push_kernel<true>, dim3(push_grid(n)), dim3(256), 0, s, part, splits, n, resid, n, A->cap,
                    A->peers, A->W, A->me, (const unsigned int*)A->state, A->state + 1) == cudaSuccess
             ? kOk
             : kCudaError;
}

int arp_reduce_rmsnorm_h(P2pAllReduce* A, float* x, const float* w, float eps, __half* out, int rows, int dim,
                         cudaStream_t s) {
  if (!A || (size_t)rows * dim > A->cap) return kTooLarge;
  if (!x || !w || !out || rows <= 0 || dim <= 0) return kBadArgument;
  const int threads = dim >= 1024 ? 512 : (dim >= 256 ? 256 : 128);
  return launch_pdl(arp_reduce_rmsnorm_kernel, dim3(rows), dim3(threads), 0, s, x, dim, A->cap,
                    (const float*)A->area, (const unsigned int*)A->flags, A->W, A->state, A->state + 2, A->status, w,
                    eps, out) == cudaSuccess
             ? kOk
             : kCudaError;
}

}  // namespace zc
