// collective.h -- internal communicator API (collective.cu).  A communicator of size 1 needs no NCCL: its
// collectives are no-ops or local copies, so single-GPU engines share the tensor-parallel code path.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include <string>

namespace zc {

struct Comm;

int comm_unique_id(void* out, size_t cap, std::string* err);
// Collective over all ranks (blocks until every rank has called it).  `id` is the 128-byte NCCL unique id
// created by one rank with comm_unique_id and passed to the others out of band.
int comm_create(int size, int rank, const void* id, Comm** out, std::string* err);
void comm_destroy(Comm* c);
int comm_rank(const Comm* c);
int comm_size(const Comm* c);
bool comm_usable(const Comm* c);

// In-place sum of `count` floats over all ranks, on stream s.
int comm_allreduce_sum_f32(Comm* c, float* buf, size_t count, cudaStream_t s, std::string* err);
// recv[r * bytes ...] = rank r's send[0 .. bytes) for every r.
int comm_allgather_bytes(Comm* c, const void* send, void* recv, size_t bytes, cudaStream_t s, std::string* err);
// Rank-to-rank exchange of byte ranges: send[send_off[p], +send_bytes[p]) goes to rank p, and rank p's range for
// this rank lands at recv[recv_off[p], +recv_bytes[p]).  Arrays have comm_size entries.
int comm_alltoallv_bytes(Comm* c, const void* send, const size_t* send_bytes, const size_t* send_off, void* recv,
                         const size_t* recv_bytes, const size_t* recv_off, cudaStream_t s, std::string* err);
// Waits for stream s; with peers, polls the communicator's asynchronous error and aborts it after timeout_ms.
int comm_wait(Comm* c, cudaStream_t s, int timeout_ms, std::string* err);

}  // namespace zc
