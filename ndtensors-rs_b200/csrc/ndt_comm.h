// Internal interface of the NCCL communicator (comm.cpp) used by the
// gathered block-sparse contractions (blocksparse.cpp).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <vector>

namespace ndt {

struct Comm;
// Largest communicator whose gathers write straight into every rank's output
// (one peer pointer per rank in the GEMM's arguments).
constexpr int kMaxSymRanks = 8;
int comm_rank(const Comm& c);
int comm_size(const Comm& c);
int comm_device(const Comm& c);

// In-place all-gather on the communicator's stream, after the work enqueued
// so far on `after`: rank r's `doubles_per_rank` doubles at
// buf + r * doubles_per_rank reach every rank at the same place.
void comm_allgather(Comm& c, void* buf, size_t doubles_per_rank, cudaStream_t after);
// A barrier over the communicator's ranks (an all-reduce of one word) after
// the work enqueued so far on `after`; `then` waits for it.  When it has
// completed on a rank, every rank's work enqueued before its barrier has
// completed.
void comm_barrier(Comm& c, cudaStream_t after, cudaStream_t then);
// The next of two output buffers of at least `bytes` that every rank of the
// communicator has mapped (CUDA IPC), used alternately by successive calls:
// `mine` is this rank's, peers[r] rank r's as mapped here (peers[rank] ==
// mine).  Collective the first time a size is asked for (all ranks ask for
// the same sizes in the same order).  False when the ranks cannot map each
// other's memory or there are more than kMaxSymRanks of them.
bool comm_symmetric(Comm& c, size_t bytes, cudaStream_t s, void** mine, void** peers);
// `s` waits for every transfer enqueued so far on the communicator.
void comm_join(Comm& c, cudaStream_t s);

}  // namespace ndt

struct ndt_comm;
ndt::Comm& comm_of(ndt_comm* h);
