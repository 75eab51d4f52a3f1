// Storage and dense tensor value type.
//
// Mirrors the observable semantics of the reference's Tensor<ElT, Dense>
// (crates/ndtensors/src/tensor.rs:21-90) and CpuBuffer (storage/buffer.rs:71-160):
//   * storage holds max(1, prod(shape)) elements (tensor.rs:45-54, :75-90);
//   * clones share storage and copy on write (Rc::make_mut, buffer.rs:157-159);
//   * data() is a host pointer valid until the next mutation or release.
// The difference is placement: the authoritative copy lives in device memory
// once a kernel produced it, and the host mirror is filled on demand.
#include <cstring>

#include "ndt_internal.h"

namespace ndt {

size_t prod(const std::vector<size_t>& v) {
  size_t p = 1;
  for (size_t x : v) p *= x;
  return p;
}
size_t prod_max1(const std::vector<size_t>& v) {
  size_t p = prod(v);
  return p < 1 ? 1 : p;
}
std::vector<size_t> col_major_strides(const std::vector<size_t>& shape) {
  std::vector<size_t> s(shape.size());
  size_t st = 1;
  for (size_t i = 0; i < shape.size(); i++) {
    s[i] = st;
    st *= shape[i];
  }
  return s;
}

Storage::~Storage() {
  if (dev) {
    try {
      dev_free(dev, device);
    } catch (...) {
    }
  }
  if (host) pinned_free(host, bytes(), host_pinned);
}

static void host_fill(DType dt, void* p, size_t n, double re, double im) {
  if (dt == DType::F64) {
    double* d = (double*)p;
    for (size_t i = 0; i < n; i++) d[i] = re;
  } else {
    double* d = (double*)p;
    for (size_t i = 0; i < n; i++) {
      d[2 * i] = re;
      d[2 * i + 1] = im;
    }
  }
}

void* Storage::host_read() {
  if (host_valid) return host;
  if (!host) host = pinned_alloc(bytes(), &host_pinned);
  if (uniform) {
    host_fill(dt, host, len, fill_re, fill_im);
  } else if (dev_valid) {
    // Read on the download stream once the compute stream's work so far is
    // done, and wait for this copy only: the compute stream stays free, so
    // another host thread's upload and kernels overlap this read.
    DeviceCtx& c = ctx(device);
    cudaEvent_t ready, done;
    NDT_CUDA(cudaEventCreateWithFlags(&ready, cudaEventDisableTiming));
    NDT_CUDA(cudaEventCreateWithFlags(&done, cudaEventDisableTiming));
    NDT_CUDA(cudaEventRecord(ready, c.compute));
    NDT_CUDA(cudaStreamWaitEvent(c.download, ready, 0));
    NDT_CUDA(cudaMemcpyAsync(host, dev, bytes(), cudaMemcpyDeviceToHost, c.download));
    NDT_CUDA(cudaEventRecord(done, c.download));
    NDT_CUDA(cudaEventSynchronize(done));
    cudaEventDestroy(ready);
    cudaEventDestroy(done);
  } else {
    memset(host, 0, bytes());
  }
  host_valid = true;
  return host;
}

void* Storage::host_write() {
  host_read();
  dev_valid = false;
  uniform = false;
  return host;
}

const void* Storage::dev_read() {
  int d = current_device();
  if (device < 0) device = d;
  if (device != d)
    throw Error(ErrKind::InvalidArgument, "tensor lives on another device than the current one");
  DeviceCtx& c = ctx(device);
  if (dev_valid && !host_external) return dev;
  if (!dev) dev = dev_alloc(bytes(), device);
  if (uniform) {
    fill_device(dt, dev, len, fill_re, fill_im, c.compute);
  } else if (host_valid) {
    NDT_CUDA(cudaMemcpyAsync(dev, host, bytes(), cudaMemcpyHostToDevice, c.compute));
    if (!host_pinned) NDT_CUDA(cudaStreamSynchronize(c.compute));
  } else {
    NDT_CUDA(cudaMemsetAsync(dev, 0, bytes(), c.compute));
  }
  dev_valid = true;
  return dev;
}

void* Storage::dev_overwrite() {
  int d = current_device();
  if (device < 0) device = d;
  if (device != d)
    throw Error(ErrKind::InvalidArgument, "tensor lives on another device than the current one");
  if (!dev) dev = dev_alloc(bytes(), device);
  dev_valid = true;
  host_valid = false;
  uniform = false;
  host_external = false;
  return dev;
}

void* Storage::dev_write() {
  void* p = const_cast<void*>(dev_read());
  uniform = false;
  host_valid = false;
  return p;
}

void Storage::set_uniform(double re, double im) {
  uniform = true;
  fill_re = re;
  fill_im = im;
  host_valid = false;
  dev_valid = false;
  host_external = false;
}

std::shared_ptr<Storage> Storage::clone() const {
  auto s = std::make_shared<Storage>(dt, len);
  if (uniform) {
    s->set_uniform(fill_re, fill_im);
    return s;
  }
  if (dev_valid && !host_external) {
    s->device = device;
    DeviceCtx& c = ctx(device);
    s->dev = dev_alloc(bytes(), device);
    NDT_CUDA(cudaMemcpyAsync(s->dev, dev, bytes(), cudaMemcpyDeviceToDevice, c.compute));
    s->dev_valid = true;
    return s;
  }
  if (host_valid) {
    s->host = pinned_alloc(bytes(), &s->host_pinned);
    memcpy(s->host, host, bytes());
    s->host_valid = true;
    return s;
  }
  s->set_uniform(0.0, 0.0);
  return s;
}

void Dense::make_unique() {
  if (st && st.use_count() > 1) st = st->clone();
}

Dense make_uniform(DType dt, const std::vector<size_t>& shape, double re, double im) {
  Dense t;
  t.dt = dt;
  t.shape = shape;
  t.st = std::make_shared<Storage>(dt, prod_max1(shape));
  t.st->set_uniform(re, im);
  return t;
}

Dense make_from_host(DType dt, const void* data, size_t len, const std::vector<size_t>& shape) {
  Dense t;
  t.dt = dt;
  t.shape = shape;
  t.st = std::make_shared<Storage>(dt, len);
  Storage& s = *t.st;
  if (device_available()) {
    // Upload straight from the caller's buffer on the upload stream.  The
    // call returns once the copy has completed, so the caller may reuse its
    // buffer at once, and every kernel enqueued afterwards sees the data
    // without a stream dependency: the compute stream never waits on an
    // upload, and one host thread's kernels and read-back do not queue
    // behind another thread's upload.
    int d = current_device();
    DeviceCtx& c = ctx(d);
    s.device = d;
    void* p = pool_alloc(s.bytes(), c.upload);
    s.dev = p;
    cudaEvent_t ev;
    NDT_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    NDT_CUDA(cudaMemcpyAsync(p, data, s.bytes(), cudaMemcpyHostToDevice, c.upload));
    NDT_CUDA(cudaEventRecord(ev, c.upload));
    NDT_CUDA(cudaEventSynchronize(ev));
    cudaEventDestroy(ev);
    s.dev_valid = true;
  } else {
    // No device: keep a host copy so that handle bookkeeping still works;
    // every computation on it reports that no CUDA device is present.
    s.host = pinned_alloc(s.bytes(), &s.host_pinned);
    memcpy(s.host, data, s.bytes());
    s.host_valid = true;
  }
  return t;
}

Dense make_from_device(DType dt, const void* dptr, size_t len, const std::vector<size_t>& shape) {
  Dense t = make_empty_device(dt, shape);
  if (t.st->len != len) throw Error(ErrKind::ShapeMismatch, "length does not match shape");
  DeviceCtx& c = ctx(t.st->device);
  NDT_CUDA(cudaMemcpyAsync(t.st->dev, dptr, t.st->bytes(), cudaMemcpyDeviceToDevice, c.compute));
  // Return once the caller's buffer has been read (as from_data does), so it
  // may be reused or freed from any stream.
  settle_for_caller(t.st->device);
  return t;
}

Dense make_empty_device(DType dt, const std::vector<size_t>& shape) {
  Dense t;
  t.dt = dt;
  t.shape = shape;
  t.st = std::make_shared<Storage>(dt, prod_max1(shape));
  t.st->dev_overwrite();
  return t;
}

}  // namespace ndt
