// Per-device context: streams, stream-ordered device pool, pinned host cache.
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>

#include "ndt_internal.h"

namespace ndt {

static thread_local std::string g_last_error;
void set_last_error(const std::string& msg) { g_last_error = msg; }
const char* last_error() { return g_last_error.c_str(); }

void throw_cuda(cudaError_t e, const char* what, const char* file, int line) {
  char buf[512];
  snprintf(buf, sizeof(buf), "CUDA error %s (%s) in %s at %s:%d", cudaGetErrorName(e),
           cudaGetErrorString(e), what, file, line);
  throw Error(ErrKind::Cuda, buf);
}

static std::mutex g_mu;
static int g_ndev = -1;

bool device_available() {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_ndev < 0) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
      n = 0;
      cudaGetLastError();  // clear the sticky "no device" error
    }
    g_ndev = n;
  }
  return g_ndev > 0;
}

int current_device() {
  if (!device_available())
    throw Error(ErrKind::Cuda, "no CUDA device is visible: this library computes on B200 GPUs only");
  int d = 0;
  NDT_CUDA(cudaGetDevice(&d));
  return d;
}

static std::map<int, DeviceCtx*> g_ctx;

DeviceCtx& ctx(int device) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_ctx.find(device);
  if (it != g_ctx.end()) return *it->second;
  DeviceCtx* c = new DeviceCtx();
  c->device = device;
  int prev = 0;
  NDT_CUDA(cudaGetDevice(&prev));
  NDT_CUDA(cudaSetDevice(device));
  NDT_CUDA(cudaStreamCreateWithFlags(&c->compute, cudaStreamNonBlocking));
  c->own_compute = c->compute;
  NDT_CUDA(cudaStreamCreateWithFlags(&c->upload, cudaStreamNonBlocking));
  NDT_CUDA(cudaStreamCreateWithFlags(&c->download, cudaStreamNonBlocking));
  NDT_CUDA(cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device));
  int optin = 0;
  NDT_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
  c->smem_optin = (size_t)optin;
  NDT_CUDA(cudaSetDevice(prev));
  g_ctx[device] = c;
  return *c;
}

DeviceCtx& ctx() { return ctx(current_device()); }

// Keep freed device memory in the device's default pool for reuse instead of
// releasing it at every synchronisation point.  Set on the library's first
// allocation on a device (not when its context is created), so a caller that
// only uses the allocation-free entry point leaves the pool's release
// threshold as it found it.
static void tune_pool(DeviceCtx& c) {
  if (c.pool_tuned.load(std::memory_order_acquire)) return;
  std::lock_guard<std::mutex> lk(g_mu);
  if (c.pool_tuned.load(std::memory_order_relaxed)) return;
  cudaMemPool_t pool;
  NDT_CUDA(cudaDeviceGetDefaultMemPool(&pool, c.device));
  uint64_t thresh = UINT64_MAX;
  NDT_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thresh));
  c.pool_tuned.store(true, std::memory_order_release);
}

void* pool_alloc(size_t bytes, cudaStream_t s) {
  DeviceCtx& c = ctx();
  tune_pool(c);
  void* p = nullptr;
  NDT_CUDA(cudaMallocAsync(&p, bytes ? bytes : 16, s));
  return p;
}

void settle_for_caller(int device) {
  DeviceCtx& c = ctx(device);
  if (!c.external_stream) NDT_CUDA(cudaStreamSynchronize(c.compute));
}

void* dev_alloc(size_t bytes, int device) {
  DeviceCtx& c = ctx(device);
  tune_pool(c);
  void* p = nullptr;
  size_t b = bytes ? bytes : 16;
  NDT_CUDA(cudaMallocAsync(&p, b, c.compute));
  return p;
}

void ensure_dynamic_smem(const void* func, size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, size_t> done;
  const int dev = current_device();
  std::lock_guard<std::mutex> lk(mu);
  size_t& have = done[{dev, func}];
  if (bytes > have) {
    NDT_CUDA(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    have = bytes;
  }
}

void dev_free(void* p, int device) {
  if (!p) return;
  DeviceCtx& c = ctx(device);
  cudaFreeAsync(p, c.compute);
}

// ---- pinned host cache: exact-size buckets rounded to 64 KiB --------------
static std::mutex g_pin_mu;
static std::multimap<size_t, void*> g_pin_free;
static const size_t kPinMin = 1 << 16;

static size_t pin_round(size_t b) { return (b + kPinMin - 1) / kPinMin * kPinMin; }

void* pinned_alloc(size_t bytes, bool* pinned) {
  size_t b = bytes ? bytes : 16;
  if (b < kPinMin || !device_available()) {
    *pinned = false;
    void* p = malloc(b);
    if (!p) throw Error(ErrKind::Panic, "host allocation failed");
    return p;
  }
  size_t r = pin_round(b);
  {
    std::lock_guard<std::mutex> lk(g_pin_mu);
    auto it = g_pin_free.find(r);
    if (it != g_pin_free.end()) {
      void* p = it->second;
      g_pin_free.erase(it);
      *pinned = true;
      return p;
    }
  }
  void* p = nullptr;
  if (cudaMallocHost(&p, r) != cudaSuccess) {
    cudaGetLastError();
    *pinned = false;
    p = malloc(b);
    if (!p) throw Error(ErrKind::Panic, "host allocation failed");
    return p;
  }
  *pinned = true;
  return p;
}

void pinned_free(void* p, size_t bytes, bool pinned) {
  if (!p) return;
  if (!pinned) {
    free(p);
    return;
  }
  std::lock_guard<std::mutex> lk(g_pin_mu);
  g_pin_free.emplace(pin_round(bytes ? bytes : 16), p);
}

void empty_caches() {
  {
    std::lock_guard<std::mutex> lk(g_pin_mu);
    for (auto& kv : g_pin_free) cudaFreeHost(kv.second);
    g_pin_free.clear();
  }
  std::lock_guard<std::mutex> lk(g_mu);
  for (auto& kv : g_ctx) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(kv.first);
    cudaStreamSynchronize(kv.second->compute);
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, kv.first) == cudaSuccess) cudaMemPoolTrimTo(pool, 0);
    cudaSetDevice(prev);
  }
}

static std::atomic<uint64_t> g_launches{0};
uint64_t launch_count() { return g_launches.load(std::memory_order_relaxed); }
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

}  // namespace ndt
