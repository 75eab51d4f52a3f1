// Internal interface of the NCCL communicator (comm.cpp) used by the
// gathered block-sparse contractions (blocksparse.cpp).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <vector>

namespace ndt {

struct Comm;
int comm_rank(const Comm& c);
int comm_size(const Comm& c);
int comm_device(const Comm& c);

// In-place all-gather on the communicator's stream, after the work enqueued
// so far on `after`: rank r's `doubles_per_rank` doubles at
// buf + r * doubles_per_rank reach every rank at the same place.
void comm_allgather(Comm& c, void* buf, size_t doubles_per_rank, cudaStream_t after);
// `s` waits for every transfer enqueued so far on the communicator.
void comm_join(Comm& c, cudaStream_t s);

}  // namespace ndt

struct ndt_comm;
ndt::Comm& comm_of(ndt_comm* h);
