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

// Both kernels are launched without programmatic dependent launch and never trigger their dependents early:
// a push starts only after everything before it in the stream has completed, and nothing after a reduce starts
// before it has completed, so the epoch and the arrival counters are never read and written by overlapping grids.
__global__ void arp_push_kernel(const float* __restrict__ x, size_t n, size_t cap, PeerPtrs peers, int W, int me,
                                const unsigned int* __restrict__ epoch, unsigned int* __restrict__ arrivals) {
  __shared__ int last;
  const unsigned int e = *epoch + 1;
  const size_t buf = (size_t)(e & 1) * W * cap;
  const size_t n4 = n / 4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(x)[i];
    for (int r = 0; r < W; ++r) reinterpret_cast<float4*>(peers.data[r] + buf + (size_t)me * cap)[i] = v;
  }
  for (size_t i = n4 * 4 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    for (int r = 0; r < W; ++r) peers.data[r][buf + (size_t)me * cap + i] = x[i];
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

__global__ void arp_reduce_kernel(float* __restrict__ x, size_t n, size_t cap, const float* __restrict__ area,
                                  const unsigned int* __restrict__ flags, int W, unsigned int* __restrict__ epoch,
                                  unsigned int* __restrict__ departures, int* __restrict__ status) {
  __shared__ int ok, last;
  const unsigned int e = *epoch + 1;
  if (threadIdx.x == 0) {
    ok = 1;
    const uint64_t t0 = now_ns();
    for (int r = 0; r < W && ok; ++r) {
      uint32_t polls = 0;
      // a peer may already have published e + 1 (it finished this all-reduce and pushed the next one into the
      // other buffer), so wait for "at least e", wrap-around safe
      while ((int)(ld_acquire_sys(flags + r) - e) < 0) {
        if (++polls > AR_WAIT_POLLS || now_ns() - t0 > AR_WAIT_NS) {
          ok = 0;
          atomicExch(status, 21);
          // what the wait saw, for the host's error message: the epoch it needed and every rank's flag
          epoch[4] = e;
          for (int q = 0; q < W; ++q) epoch[5 + q] = flags[q];
          break;
        }
      }
    }
  }
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
  // the last CTA to leave advances the epoch (every CTA has read it by then)
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(departures, 1u) == gridDim.x - 1;
  __syncthreads();
  if (last && threadIdx.x == 0) {
    *departures = 0;
    *epoch = e;
  }
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

int arp_allreduce_sum(P2pAllReduce* A, float* x, size_t n, cudaStream_t s) {
  if (!A || n > A->cap) return kTooLarge;
  if (n == 0) return kOk;
  const int threads = 256;
  const int grid = (int)std::min<size_t>((n / 4 + threads - 1) / threads + 1, 148 * 2);
  arp_push_kernel<<<grid, threads, 0, s>>>(x, n, A->cap, A->peers, A->W, A->me, A->state, A->state + 1);
  if (cudaPeekAtLastError() != cudaSuccess) return kCudaError;
  arp_reduce_kernel<<<grid, threads, 0, s>>>(x, n, A->cap, A->area, A->flags, A->W, A->state, A->state + 2, A->status);
  return cudaPeekAtLastError() == cudaSuccess ? kOk : kCudaError;
}

}  // namespace zc
