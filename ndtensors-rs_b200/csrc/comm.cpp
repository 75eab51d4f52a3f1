// NCCL communicators for the multi-GPU entry points (one process per GPU).
//
// The reference has no multi-GPU path; callers of the drop-in (Julia, Rust,
// Python through the C ABI) that want a sharded block-sparse contraction
// gathered on every rank create one communicator per process:
//   rank 0:      ndt_b200_comm_unique_id(id)           (128 bytes)
//   everyone:    receive id by the caller's own means  (MPI, a TCP store, ...)
//   every rank:  comm = ndt_b200_comm_init(id, nranks, rank, &status)
// or wrap a communicator they already have (ndt_b200_comm_from_nccl).
//
// NCCL is loaded at the first communicator call with dlopen("libnccl.so.2"):
// a process that already loaded NCCL (torch does) shares that copy, and the
// library itself loads without NCCL present.  The gathers use NCCL's
// in-place all-gather (its NVLink / NVSwitch algorithms), on a stream of the
// communicator's own, ordered after the library's kernels with events.
// (Point-to-point sends straight into every block's final offset were
// measured first: NCCL gives a peer pair only a couple of channels, 120 GB/s
// on two B200s, against several hundred for the all-gather.)
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/ndtensors_capi.h"
#include "ndt_internal.h"
#include "ndt_comm.h"

namespace ndt {

namespace {

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) init_rank = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclCommCount) count = nullptr;
  decltype(&ncclCommUserRank) user_rank = nullptr;
  decltype(&ncclCommCuDevice) cu_device = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  decltype(&ncclCommGetAsyncError) async_error = nullptr;
};

std::mutex g_mu;
NcclApi* g_api = nullptr;

const NcclApi& api() {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_api) return *g_api;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!h) throw Error(ErrKind::Cuda, std::string("NCCL is not available: ") + dlerror());
  auto* a = new NcclApi();
  auto sym = [&](const char* name) {
    void* p = dlsym(h, name);
    if (!p) throw Error(ErrKind::Cuda, std::string("NCCL lacks ") + name);
    return p;
  };
  a->get_unique_id = (decltype(a->get_unique_id))sym("ncclGetUniqueId");
  a->init_rank = (decltype(a->init_rank))sym("ncclCommInitRank");
  a->destroy = (decltype(a->destroy))sym("ncclCommDestroy");
  a->count = (decltype(a->count))sym("ncclCommCount");
  a->user_rank = (decltype(a->user_rank))sym("ncclCommUserRank");
  a->cu_device = (decltype(a->cu_device))sym("ncclCommCuDevice");
  a->all_gather = (decltype(a->all_gather))sym("ncclAllGather");
  a->all_reduce = (decltype(a->all_reduce))sym("ncclAllReduce");
  a->error_string = (decltype(a->error_string))sym("ncclGetErrorString");
  a->async_error = (decltype(a->async_error))sym("ncclCommGetAsyncError");
  g_api = a;
  return *g_api;
}

void check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) {
    const char* msg = g_api && g_api->error_string ? g_api->error_string(r) : "";
    throw Error(ErrKind::Cuda, std::string("NCCL ") + what + " failed: " + msg);
  }
}

}  // namespace

// Two output buffers of every rank mapped into every rank (CUDA IPC), used
// alternately by successive gathered contractions: a contraction's kernel
// writes each output tile it computes into the current buffer of every rank.
struct SymBuffers {
  size_t bytes = 0;
  void* local[2] = {nullptr, nullptr};
  void* peer[2][kMaxSymRanks] = {};  // rank r's buffer b as mapped here (own rank: local)
  int next = 0;
};

struct Comm {
  ncclComm_t nc = nullptr;
  int rank = 0, nranks = 1, device = -1;
  bool owned = false;         // created here (destroyed on release)
  cudaStream_t stream = nullptr;  // the communicator's transfer stream
  int* dflag = nullptr;       // device word of the barrier (an all-reduce of one int)
  SymBuffers sym;
  bool sym_failed = false;    // mapping failed on some rank: gathers use the all-gather path
};

int comm_rank(const Comm& c) { return c.rank; }
int comm_size(const Comm& c) { return c.nranks; }
int comm_device(const Comm& c) { return c.device; }

void comm_allgather(Comm& c, void* buf, size_t doubles_per_rank, cudaStream_t after) {
  if (doubles_per_rank == 0) return;
  const NcclApi& a = api();
  cudaEvent_t ev;
  NDT_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  NDT_CUDA(cudaEventRecord(ev, after));
  NDT_CUDA(cudaStreamWaitEvent(c.stream, ev, 0));
  cudaEventDestroy(ev);
  double* base = (double*)buf;
  check(a.all_gather(base + (size_t)c.rank * doubles_per_rank, base, doubles_per_rank, ncclDouble, c.nc, c.stream),
        "ncclAllGather");
}

void comm_barrier(Comm& c, cudaStream_t after, cudaStream_t then) {
  const NcclApi& a = api();
  cudaEvent_t ev;
  NDT_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  NDT_CUDA(cudaEventRecord(ev, after));
  NDT_CUDA(cudaStreamWaitEvent(c.stream, ev, 0));
  check(a.all_reduce(c.dflag, c.dflag, 1, ncclInt32, ncclMax, c.nc, c.stream), "ncclAllReduce");
  NDT_CUDA(cudaEventRecord(ev, c.stream));
  NDT_CUDA(cudaStreamWaitEvent(then, ev, 0));
  cudaEventDestroy(ev);
}

namespace {

void sym_release(Comm& c) {
  for (int b = 0; b < 2; b++) {
    for (int r = 0; r < c.nranks && r < kMaxSymRanks; r++)
      if (r != c.rank && c.sym.peer[b][r]) cudaIpcCloseMemHandle(c.sym.peer[b][r]);
    if (c.sym.local[b]) cudaFree(c.sym.local[b]);
    c.sym.local[b] = nullptr;
    for (int r = 0; r < kMaxSymRanks; r++) c.sym.peer[b][r] = nullptr;
  }
  c.sym.bytes = 0;
}

}  // namespace

bool comm_symmetric(Comm& c, size_t bytes, cudaStream_t s, void** mine, void** peers) {
  if (c.nranks > kMaxSymRanks || c.sym_failed) return false;
  if (bytes > c.sym.bytes) {
    // Collective (every rank asks for the same size at the same call).  The
    // barrier and the waits make sure no rank's earlier kernel still writes
    // into the buffers being replaced.
    const NcclApi& a = api();
    comm_barrier(c, s, s);
    NDT_CUDA(cudaStreamSynchronize(c.stream));
    NDT_CUDA(cudaStreamSynchronize(s));
    sym_release(c);
    const size_t want = (bytes + (2u << 20) - 1) / (2u << 20) * (2u << 20);
    int ok = 1;
    cudaIpcMemHandle_t h[2];
    for (int b = 0; b < 2 && ok; b++) {
      if (cudaMalloc(&c.sym.local[b], want) != cudaSuccess || cudaIpcGetMemHandle(&h[b], c.sym.local[b]) != cudaSuccess) {
        cudaGetLastError();
        ok = 0;
      }
    }
    // every rank allocated and exported its buffers?  (No handle is opened
    // unless all of them exist.)
    auto all_ranks = [&](int flag) {
      NDT_CUDA(cudaMemcpy(c.dflag, &flag, sizeof(int), cudaMemcpyHostToDevice));
      check(a.all_reduce(c.dflag, c.dflag, 1, ncclInt32, ncclSum, c.nc, c.stream), "ncclAllReduce");
      NDT_CUDA(cudaStreamSynchronize(c.stream));
      int total = 0;
      NDT_CUDA(cudaMemcpy(&total, c.dflag, sizeof(int), cudaMemcpyDeviceToHost));
      return total == c.nranks;
    };
    if (!all_ranks(ok)) {
      sym_release(c);
      c.sym_failed = true;
      return false;
    }
    // every rank's two handles, then whether every rank mapped every buffer
    const size_t hb = sizeof(cudaIpcMemHandle_t) * 2;
    std::vector<char> all((size_t)c.nranks * hb);
    char* dbuf = nullptr;
    NDT_CUDA(cudaMalloc(&dbuf, all.size()));
    NDT_CUDA(cudaMemcpy(dbuf + (size_t)c.rank * hb, h, hb, cudaMemcpyHostToDevice));
    check(a.all_gather(dbuf + (size_t)c.rank * hb, dbuf, hb, ncclChar, c.nc, c.stream), "ncclAllGather");
    NDT_CUDA(cudaStreamSynchronize(c.stream));
    NDT_CUDA(cudaMemcpy(all.data(), dbuf, all.size(), cudaMemcpyDeviceToHost));
    cudaFree(dbuf);
    for (int r = 0; r < c.nranks && ok; r++) {
      for (int b = 0; b < 2 && ok; b++) {
        if (r == c.rank) {
          c.sym.peer[b][r] = c.sym.local[b];
          continue;
        }
        cudaIpcMemHandle_t ph;
        memcpy(&ph, all.data() + (size_t)r * hb + b * sizeof(cudaIpcMemHandle_t), sizeof(ph));
        if (cudaIpcOpenMemHandle(&c.sym.peer[b][r], ph, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
          cudaGetLastError();
          c.sym.peer[b][r] = nullptr;
          ok = 0;
        }
      }
    }
    if (!all_ranks(ok)) {
      sym_release(c);
      c.sym_failed = true;
      return false;
    }
    c.sym.bytes = want;
    c.sym.next = 0;
  }
  const int b = c.sym.next;
  c.sym.next ^= 1;
  *mine = c.sym.local[b];
  for (int r = 0; r < c.nranks; r++) peers[r] = c.sym.peer[b][r];
  return true;
}

void comm_join(Comm& c, cudaStream_t s) {
  cudaEvent_t ev;
  NDT_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  NDT_CUDA(cudaEventRecord(ev, c.stream));
  NDT_CUDA(cudaStreamWaitEvent(s, ev, 0));
  cudaEventDestroy(ev);
}

}  // namespace ndt

using namespace ndt;

struct ndt_comm {
  Comm c;
};

Comm& comm_of(ndt_comm* h) { return h->c; }

extern "C" {

int ndt_b200_comm_unique_id(unsigned char* id) {
  if (!id) return NDT_INVALID_ARGUMENT;
  try {
    ncclUniqueId u;
    check(api().get_unique_id(&u), "ncclGetUniqueId");
    memcpy(id, u.internal, NCCL_UNIQUE_ID_BYTES);
    return NDT_SUCCESS;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return NDT_INTERNAL_ERROR;
  }
}

static ndt_comm* finish_comm(Comm c, int* status) {
  NDT_CUDA(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking));
  NDT_CUDA(cudaMalloc(&c.dflag, sizeof(int)));
  NDT_CUDA(cudaMemset(c.dflag, 0, sizeof(int)));
  *status = NDT_SUCCESS;
  return new ndt_comm{c};
}

ndt_comm* ndt_b200_comm_init(const unsigned char* id, int nranks, int rank, int* status) {
  if (!status) return nullptr;
  if (!id || nranks < 1 || rank < 0 || rank >= nranks) {
    set_last_error("ndt_b200_comm_init: need an id and 0 <= rank < nranks");
    *status = NDT_INVALID_ARGUMENT;
    return nullptr;
  }
  try {
    Comm c;
    c.device = current_device();
    ctx(c.device);
    ncclUniqueId u;
    memcpy(u.internal, id, NCCL_UNIQUE_ID_BYTES);
    check(api().init_rank(&c.nc, nranks, u, rank), "ncclCommInitRank");
    c.rank = rank;
    c.nranks = nranks;
    c.owned = true;
    return finish_comm(c, status);
  } catch (const std::exception& e) {
    set_last_error(e.what());
    *status = NDT_INTERNAL_ERROR;
    return nullptr;
  }
}

ndt_comm* ndt_b200_comm_from_nccl(void* nccl_comm, int* status) {
  if (!status) return nullptr;
  if (!nccl_comm) {
    set_last_error("ndt_b200_comm_from_nccl: NULL communicator");
    *status = NDT_INVALID_ARGUMENT;
    return nullptr;
  }
  try {
    const NcclApi& a = api();
    Comm c;
    c.nc = (ncclComm_t)nccl_comm;
    check(a.count(c.nc, &c.nranks), "ncclCommCount");
    check(a.user_rank(c.nc, &c.rank), "ncclCommUserRank");
    check(a.cu_device(c.nc, &c.device), "ncclCommCuDevice");
    if (c.device != current_device())
      throw Error(ErrKind::InvalidArgument, "the communicator's device is not the current device");
    ctx(c.device);
    c.owned = false;
    return finish_comm(c, status);
  } catch (const Error& e) {
    set_last_error(e.what());
    *status = e.kind == ErrKind::InvalidArgument ? NDT_INVALID_ARGUMENT : NDT_INTERNAL_ERROR;
    return nullptr;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    *status = NDT_INTERNAL_ERROR;
    return nullptr;
  }
}

int ndt_b200_comm_rank(const ndt_comm* c) { return c ? c->c.rank : -1; }
int ndt_b200_comm_size(const ndt_comm* c) { return c ? c->c.nranks : 0; }

void ndt_b200_comm_release(ndt_comm* c) {
  if (!c) return;
  if (c->c.stream) {
    cudaStreamSynchronize(c->c.stream);
    cudaStreamDestroy(c->c.stream);
  }
  cudaDeviceSynchronize();  // no kernel of this process still writes into the mapped buffers
  sym_release(c->c);
  if (c->c.dflag) cudaFree(c->c.dflag);
  if (c->c.owned && c->c.nc && g_api) g_api->destroy(c->c.nc);
  delete c;
}

}  // extern "C"
