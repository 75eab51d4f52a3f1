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

struct Comm {
  ncclComm_t nc = nullptr;
  int rank = 0, nranks = 1, device = -1;
  bool owned = false;         // created here (destroyed on release)
  cudaStream_t stream = nullptr;  // the communicator's transfer stream
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
  if (c->c.owned && c->c.nc && g_api) g_api->destroy(c->c.nc);
  delete c;
}

}  // extern "C"
