// allreduce_p2p.h -- one-shot all-reduce over NVLink peer memory (allreduce_p2p.cu).
#pragma once

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
// In-place sum of x[0, n) over all ranks (n <= capacity); two kernels on stream s, graph-capturable.
int arp_allreduce_sum(P2pAllReduce* a, float* x, size_t n, cudaStream_t s);

}  // namespace zc
