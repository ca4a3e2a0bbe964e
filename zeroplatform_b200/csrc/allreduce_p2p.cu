// allreduce_p2p.cu -- one-shot all-reduce of the residual stream over NVLink peer memory (tensor parallelism).
//
// Every rank owns a receive area in its own HBM: two buffers (alternating with the all-reduce's parity), each
// holding one slot of `cap` elements per rank.  The areas are mapped into every peer with CUDA IPC, so a kernel
// reaches a peer's memory with ordinary loads and stores over NVLink (no TMA, no multicast).
//
//   push   each thread stores its elements of this rank's partial into slot[my rank] of every rank's current
//          buffer (its own included) as 8-byte words {value, epoch}: the value travels with the number of the
//          all-reduce it belongs to, in one store
//   reduce every thread polls (bounded) its elements of every rank's slot until each word carries the current
//          epoch, then x[i] = sum over ranks r = 0 .. W-1 of slot[r][i] -- the same order on every rank, so all
//          ranks hold bit-identical sums
//
// No fence, arrival counter or flag round is needed: an aligned 8-byte store reaches the reader whole, so a word
// holds either an older epoch's value or the current one.  (A flag protocol -- push, system-scope fence, arrival
// counter, per-rank flag -- measured ~17 us per 512 KB all-reduce on two GPUs with the ranks' compute removed;
// this one ~9 us.)  The epoch lives on the device (one counter per rank, advanced by the reduce kernel's last CTA),
// so the pair can be captured in a CUDA graph and replayed.  Buffer reuse: all-reduce e writes buffer e % 2;
// before any rank pushes e + 2 into that buffer it has finished reduce e + 1, which waited for every peer's push
// e + 1, which each peer issued only after its own reduce e -- the last reader of buffer e % 2 -- so while reduce
// e reads buffer e % 2 its words carry e or an earlier epoch.  Epochs are 32-bit and compared for equality: a word
// last written exactly 2^32 all-reduces earlier (possible only for elements beyond the n of every call in
// between) would pass for a fresh one.  Waits are bounded: after 10 s the kernel records an error code in the
// status word and returns, and later reduces then stop waiting.  Callers keep the ranks' host threads in step
// around slow host work (graph capture) with a collective barrier, so a wait only covers the peers' kernel
// progress.

#include <cuda_runtime.h>

#include <algorithm>
#include <string>
#include <vector>

#include "allreduce_p2p.h"
#include "collective.h"
#include "common.cuh"

namespace zc {

namespace {

constexpr uint64_t AR_WAIT_NS = 10000000000ull;  // 10 s: peers run on other hosts' threads and may lag

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

struct PeerPtrs {
  uint2* data[ARP_MAX_RANKS];  // each rank's receive area (two buffers of W slots of {value, epoch} words)
};

// The plain pair (arp_allreduce_sum) is launched without programmatic dependent launch: a push starts only after
// everything before it in the stream has completed, and nothing after a reduce starts before it has completed.
// The fused pair (arp_push_partials + arp_reduce_rmsnorm_h) is launched with programmatic dependent launch and
// waits (griddepcontrol.wait) before any read.  The push triggers its dependent first: the reduce's grid is
// launched only once every CTA of the push is resident, so its polling CTAs never keep the push's CTAs off the
// SMs.  The reduce never triggers: nothing after it starts before it has completed and advanced the epoch, so the
// epoch and the departure counter are never read and written by overlapping grids.

__device__ __forceinline__ void st_ll(uint2* p, float v, unsigned int e) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(e) : "memory");
}
__device__ __forceinline__ uint2 ld_ll(const uint2* p) {
  uint2 r;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p) : "memory");
  return r;
}

// Push: slot[me] of every rank's current buffer = {sum over s < splits of src[s * stride + i] (+ resid[i]), epoch}.
template <bool PDL>
__global__ void arp_push_kernel(const float* __restrict__ src, int splits, size_t stride,
                                const float* __restrict__ resid, size_t n, size_t cap, PeerPtrs peers, int W, int me,
                                const unsigned int* __restrict__ epoch) {
  if (PDL) {
    pdl_trigger();
    pdl_wait();
  }
  const unsigned int e = *reinterpret_cast<const volatile unsigned int*>(epoch) + 1;
  const size_t slot = ((size_t)(e & 1) * W + me) * cap;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float v = src[i];
    for (int sp = 1; sp < splits; ++sp) v += src[(size_t)sp * stride + i];
    if (resid) v = resid[i] + v;
    for (int r = 0; r < W; ++r) st_ll(peers.data[r] + slot + i, v, e);
  }
}

// Element i of every rank's slot for epoch e, summed in rank order; the value arrives with its epoch in one
// 8-byte store, so a thread polls its own elements (bounded) and no flag or fence is needed.  Returns false when
// the wait ran out.
__device__ __forceinline__ bool ll_sum(const uint2* buf, size_t cap, int W, unsigned int e, size_t i, float* out,
                                       uint64_t t0, uint64_t wait_ns) {
  float v = 0.f;
  if (t0 == 0) return false;
  for (int r = 0; r < W; ++r) {
    const uint2* p = buf + (size_t)r * cap + i;
    uint2 w = ld_ll(p);
    uint32_t polls = 0;
    while (w.y != e) {
      if ((++polls & 63) == 0 && now_ns() - t0 > wait_ns) return false;
      w = ld_ll(p);
    }
    v = r == 0 ? __uint_as_float(w.x) : v + __uint_as_float(w.x);
  }
  *out = v;
  return true;
}

// A wait ran out: record the code once, with the epoch needed and each rank's epoch word at element 0.
__device__ __forceinline__ void ll_fail(const uint2* buf, size_t cap, int W, unsigned int e, unsigned int* state,
                                        int* status) {
  if (atomicExch(status, 21) == 21) return;
  state[4] = e;
  for (int q = 0; q < W; ++q) state[5 + q] = ld_ll(buf + (size_t)q * cap).y;
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
__global__ void arp_reduce_rmsnorm_kernel(float* __restrict__ x, int dim, size_t cap, const uint2* __restrict__ area,
                                          int W, unsigned int* __restrict__ epoch,
                                          unsigned int* __restrict__ departures, int* __restrict__ status,
                                          const float* __restrict__ w, float eps, __half* __restrict__ out) {
  pdl_wait();
  __shared__ int ok;
  __shared__ float red[32];
  const unsigned int e = *reinterpret_cast<volatile unsigned int*>(epoch) + 1;
  const uint2* buf = area + (size_t)(e & 1) * W * cap;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  const uint64_t t0 = *reinterpret_cast<volatile int*>(status) ? 0 : now_ns();  // after a failure: no waits
  float* xr = x + (size_t)blockIdx.x * dim;
  float ss = 0.f;
  bool mine = true;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    float v = 0.f;
    if (mine && ll_sum(buf, cap, W, e, (size_t)blockIdx.x * dim + i, &v, t0, AR_WAIT_NS)) {
      xr[i] = v;
      ss = fmaf(v, v, ss);
    } else {
      mine = false;
    }
  }
  if (!mine) {
    ok = 0;
    ll_fail(buf, cap, W, e, epoch, status);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (ok) {
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

__global__ void arp_reduce_kernel(float* __restrict__ x, size_t n, size_t cap, const uint2* __restrict__ area,
                                  int W, unsigned int* __restrict__ epoch,
                                  unsigned int* __restrict__ departures, int* __restrict__ status, uint64_t wait_ns) {
  const unsigned int e = *reinterpret_cast<volatile unsigned int*>(epoch) + 1;
  const uint2* buf = area + (size_t)(e & 1) * W * cap;
  const uint64_t t0 = *reinterpret_cast<volatile int*>(status) ? 0 : now_ns();  // after a failure: no waits
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float v;
    if (!ll_sum(buf, cap, W, e, i, &v, t0, wait_ns)) {
      ll_fail(buf, cap, W, e, epoch, status);
      break;
    }
    x[i] = v;
  }
  depart(epoch, departures, e);
}

}  // namespace

struct P2pAllReduce {
  int W = 1, me = 0;
  size_t cap = 0;                 // elements per slot
  uint2* area = nullptr;          // own receive area: 2 * W * cap {value, epoch} words
  unsigned int* state = nullptr;  // epoch, reduce departures, diagnostics of a timed-out wait
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
  // one allocation: the area, 2 * W * cap {value, epoch} words (epoch 0: never pushed)
  const size_t area_bytes = 2 * (size_t)W * A->cap * sizeof(uint2);
  const size_t total = area_bytes;
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
  // state: [0] epoch, [2] reduce departures, [4] epoch a timed-out wait needed, [5..] each rank's epoch word seen
  if (cudaMalloc(&A->state, 16 * sizeof(unsigned int)) != cudaSuccess ||
      cudaMemset(A->state, 0, 16 * sizeof(unsigned int)) != cudaSuccess)
    return fail("peer all-reduce: state allocation failed");
  A->area = static_cast<uint2*>(A->own_alloc);
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
    A->peers.data[r] = reinterpret_cast<uint2*>(base);
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
    m += ", a wait needed epoch " + std::to_string(st[4]) + " and saw, per rank, epochs";
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
                                              A->state);
  if (cudaPeekAtLastError() != cudaSuccess) return kCudaError;
  arp_reduce_kernel<<<grid, 256, 0, s>>>(x, n, A->cap, A->area, A->W, A->state, A->state + 2, A->status,
                                         AR_WAIT_NS);
  return cudaPeekAtLastError() == cudaSuccess ? kOk : kCudaError;
}

int arp_wait_selftest(int W, int wait_ms, unsigned int* seen, std::string* err) {
  if (W < 2 || W > ARP_MAX_RANKS || wait_ms < 1 || wait_ms > 5000 || !seen) {
    if (err) *err = "peer wait self-test: W must be 2 .. 8, wait_ms 1 .. 5000";
    return kBadArgument;
  }
  constexpr size_t cap = 256;
  const size_t area_bytes = 2 * (size_t)W * cap * sizeof(uint2);
  // one allocation: [area][state: 16 words][status: 4 words][x: cap floats]
  const size_t total = area_bytes + 64 + 16 + cap * sizeof(float);
  char* base = nullptr;
  if (cudaMalloc(&base, total) != cudaSuccess) {
    cudaGetLastError();
    if (err) *err = "peer wait self-test: allocation failed";
    return kOutOfMemory;
  }
  uint2* area = reinterpret_cast<uint2*>(base);
  unsigned int* state = reinterpret_cast<unsigned int*>(base + area_bytes);
  int* status = reinterpret_cast<int*>(base + area_bytes + 64);
  float* x = reinterpret_cast<float*>(base + area_bytes + 80);
  int rc = cudaMemset(base, 0, total) == cudaSuccess ? kOk : kCudaError;
  // rank 0 has pushed epoch 1 (buffer 1, slot 0: value 0, epoch 1 in every element); no peer ever does
  std::vector<uint2> r0(cap, make_uint2(0u, 1u));
  if (rc == kOk && cudaMemcpy(area + (size_t)W * cap, r0.data(), cap * sizeof(uint2), cudaMemcpyHostToDevice) !=
                       cudaSuccess)
    rc = kCudaError;
  int code = 0;
  if (rc == kOk) {
    arp_reduce_kernel<<<1, 256>>>(x, cap, cap, area, W, state, state + 2, status, (uint64_t)wait_ms * 1000000ull);
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
                    A->peers, A->W, A->me, (const unsigned int*)A->state) == cudaSuccess
             ? kOk
             : kCudaError;
}

int arp_reduce_rmsnorm_h(P2pAllReduce* A, float* x, const float* w, float eps, __half* out, int rows, int dim,
                         cudaStream_t s) {
  if (!A || (size_t)rows * dim > A->cap) return kTooLarge;
  if (!x || !w || !out || rows <= 0 || dim <= 0) return kBadArgument;
  const int threads = dim >= 1024 ? 512 : (dim >= 256 ? 256 : 128);
  return launch_pdl(arp_reduce_rmsnorm_kernel, dim3(rows), dim3(threads), 0, s, x, dim, A->cap,
                    (const uint2*)A->area, A->W, A->state, A->state + 2, A->status, w, eps, out) == cudaSuccess
             ? kOk
             : kCudaError;
}

}  // namespace zc
