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

// One point-to-point transfer of `doubles` doubles at `ptr` to / from `peer`.
struct P2POp {
  bool send;
  int peer;
  void* ptr;
  size_t doubles;
};
// Enqueue `ops` as one NCCL group on the communicator's stream, after the
// work enqueued so far on `after`; when `then` is not null it waits for the
// group.  Sends and receives between two ranks match in the order issued.
void comm_exchange(Comm& c, const std::vector<P2POp>& ops, cudaStream_t after, cudaStream_t then);
// `s` waits for every transfer enqueued so far on the communicator.
void comm_join(Comm& c, cudaStream_t s);

}  // namespace ndt

struct ndt_comm;
ndt::Comm& comm_of(ndt_comm* h);
