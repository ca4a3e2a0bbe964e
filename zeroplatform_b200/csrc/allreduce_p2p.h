// allreduce_p2p.h -- one-shot all-reduce over NVLink peer memory (allreduce_p2p.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>

#include <string>

namespace zc {

struct Comm;
struct P2pAllReduce;

constexpr int ARP_MAX_RANKS = 8;

// Collective over the communicator's ranks (2 .. 8, one GPU each, with peer access): maps every rank's receive
// area into every other rank.  cap_floats = the largest all-reduce it will serve.  Bounded-wait failures are
// recorded in *status (device word).
int arp_create(Comm* comm, size_t cap_floats, int* status, P2pAllReduce** out, std::string* err);
void arp_destroy(P2pAllReduce* a);
size_t arp_capacity(const P2pAllReduce* a);
// The epoch and, after a timed-out wait, what it waited for and saw (for error messages).
std::string arp_describe(const P2pAllReduce* a);
// Runs the reduce kernel of this all-reduce on one GPU against a local receive area of W ranks in which only rank
// 0 has pushed (its words carry epoch 1), with a wait limit of wait_ms: the kernel's bounded wait runs out, it
// records its code (21) and returns.  Returns that code (0 would mean the wait did not run out), or < 0 when the
// test could not run; seen[0..15] receives the kernel's state words ([4] = the epoch it waited for, [5 + r] = the
// epoch of rank r's first word).
int arp_wait_selftest(int W, int wait_ms, unsigned int* seen, std::string* err);
// In-place sum of x[0, n) over all ranks (n <= capacity); two kernels on stream s, graph-capturable.
int arp_allreduce_sum(P2pAllReduce* a, float* x, size_t n, cudaStream_t s);

// The same all-reduce split around the kernels that produce and consume it (tensor-parallel decode steps):
//   arp_push_partials     this rank's term = sum over s < splits of part[s * n + i] (+ resid[i]), the split-K
//                         partials of the GEMM before it, stored straight into every rank's slot (no x round trip)
//   arp_reduce_rmsnorm_h  x[rows][dim] = sum of the ranks' terms, and out = RmsNorm(x) * w as fp16 hi / lo pairs
//                         [rows][hi dim | lo dim] for the tensor-core GEMM after it
// Every arp_push_partials must be followed by one arp_reduce_rmsnorm_h (or an arp_allreduce_sum never starts
// between them); rows * dim = n <= capacity.
int arp_push_partials(P2pAllReduce* a, const float* part, int splits, size_t n, const float* resid, cudaStream_t s);
int arp_reduce_rmsnorm_h(P2pAllReduce* a, float* x, const float* w, float eps, __half* out, int rows, int dim,
                         cudaStream_t s);

}  // namespace zc
