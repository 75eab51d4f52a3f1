// C ABI: dense tensors.
//
// The ndt_tensor_f64_* functions reproduce crates/ndtensors-capi/src/lib.rs
// of the reference: argument checks first (NULL status -> NULL result, NULL
// inputs -> NDT_INVALID_ARGUMENT), then the operation; a TensorError maps to
// the per-function code the reference uses, and what would be a Rust panic
// (caught there by catch_unwind) maps to NDT_INTERNAL_ERROR.
#include <chrono>
#include <cmath>
#include <cstring>
#include <mutex>
#include <random>

#include "../../include/ndtensors_capi.h"
#include "ndt_internal.h"

using namespace ndt;

namespace {

NdtHandle* H(const void* p) { return (NdtHandle*)p; }

// TensorError -> `code`; panic / CUDA failure -> NDT_INTERNAL_ERROR.
int map_error(const Error& e, int code) {
  set_last_error(e.what());
  switch (e.kind) {
    case ErrKind::Panic:
    case ErrKind::Cuda:
      return NDT_INTERNAL_ERROR;
    case ErrKind::InvalidArgument:
      return NDT_INVALID_ARGUMENT;
    default:
      return code;
  }
}

std::vector<size_t> shape_of(const size_t* shape, size_t ndim) {
  return ndim ? std::vector<size_t>(shape, shape + ndim) : std::vector<size_t>();
}

std::vector<int32_t> labels_of(const long* l, size_t n) {
  std::vector<int32_t> v(n);
  for (size_t i = 0; i < n; i++) v[i] = (int32_t)l[i];  // `as i32` truncation (lib.rs:654-655)
  return v;
}

// Host-side generator for rand / randn: SplitMix64 (Steele, Lea & Flood 2014)
// with Box-Muller for normals.  The reference draws from rand's thread RNG,
// which no caller can reproduce either; the distributions match.
struct Rng {
  uint64_t s;
  std::mutex mu;
  Rng() { s = (uint64_t)std::chrono::high_resolution_clock::now().time_since_epoch().count() ^ 0x9E3779B97F4A7C15ULL; }
  uint64_t next() {
    uint64_t z = (s += 0x9E3779B97F4A7C15ULL);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
  }
  double uniform() { return (double)(next() >> 11) * (1.0 / 9007199254740992.0); }
};
Rng& rng() {
  static Rng r;
  return r;
}

template <class F>
void* create(const size_t* shape, size_t ndim, int* status, F&& make) {
  if (!status) return nullptr;
  if (!shape && ndim > 0) {
    *status = NDT_INVALID_ARGUMENT;
    return nullptr;
  }
  try {
    NdtHandle* h = new NdtHandle{make(shape_of(shape, ndim))};
    *status = NDT_SUCCESS;
    return h;
  } catch (const Error& e) {
    *status = map_error(e, NDT_INTERNAL_ERROR);
  } catch (const std::exception& e) {
    set_last_error(e.what());
    *status = NDT_INTERNAL_ERROR;
  } catch (...) {
    *status = NDT_INTERNAL_ERROR;
  }
  return nullptr;
}

Dense random_tensor(const std::vector<size_t>& shape, bool normal) {
  size_t n = prod_max1(shape);
  std::vector<double> v(n);
  Rng& r = rng();
  std::lock_guard<std::mutex> lk(r.mu);
  if (!normal) {
    for (size_t i = 0; i < n; i++) v[i] = r.uniform();
  } else {
    for (size_t i = 0; i < n; i += 2) {
      double u1 = r.uniform(), u2 = r.uniform();
      if (u1 < 1e-300) u1 = 1e-300;
      double rad = std::sqrt(-2.0 * std::log(u1)), th = 6.283185307179586 * u2;
      v[i] = rad * std::cos(th);
      if (i + 1 < n) v[i + 1] = rad * std::sin(th);
    }
  }
  return make_from_host(DType::F64, v.data(), n, shape);
}

void* from_data_impl(DType dt, const double* data, size_t len, const size_t* shape, size_t ndim, int* status) {
  if (!status) return nullptr;
  if (!data || (!shape && ndim > 0)) {
    *status = NDT_INVALID_ARGUMENT;
    return nullptr;
  }
  try {
    std::vector<size_t> sh = shape_of(shape, ndim);
    if (len != prod_max1(sh)) {  // Tensor::from_vec (tensor.rs:75-90)
      *status = NDT_SHAPE_MISMATCH;
      return nullptr;
    }
    NdtHandle* h = new NdtHandle{make_from_host(dt, data, len, sh)};
    *status = NDT_SUCCESS;
    return h;
  } catch (const Error& e) {
    *status = map_error(e, NDT_INTERNAL_ERROR);
  } catch (...) {
    *status = NDT_INTERNAL_ERROR;
  }
  return nullptr;
}

void* from_device_impl(DType dt, const double* dptr, size_t len, const size_t* shape, size_t ndim, int* status) {
  if (!status) return nullptr;
  if (!dptr || (!shape && ndim > 0)) {
    *status = NDT_INVALID_ARGUMENT;
    return nullptr;
  }
  try {
    std::vector<size_t> sh = shape_of(shape, ndim);
    if (len != prod_max1(sh)) {
      *status = NDT_SHAPE_MISMATCH;
      return nullptr;
    }
    NdtHandle* h = new NdtHandle{make_from_device(dt, dptr, len, sh)};
    *status = NDT_SUCCESS;
    return h;
  } catch (const Error& e) {
    *status = map_error(e, NDT_INTERNAL_ERROR);
  } catch (...) {
    *status = NDT_INTERNAL_ERROR;
  }
  return nullptr;
}

size_t ndim_impl(const void* t) { return t ? H(t)->t.ndim() : 0; }
size_t len_impl(const void* t) { return t ? H(t)->t.len() : 0; }
int shape_impl(const void* t, size_t* out) {
  if (!t || !out) return NDT_INVALID_ARGUMENT;
  const Dense& d = H(t)->t;
  for (size_t i = 0; i < d.ndim(); i++) out[i] = d.shape[i];
  return NDT_SUCCESS;
}
const double* data_impl(const void* t) {
  if (!t) return nullptr;
  try {
    return (const double*)H(t)->t.st->host_read();
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return nullptr;
  }
}
double* data_mut_impl(void* t) {
  if (!t) return nullptr;
  try {
    Dense& d = H(t)->t;
    d.make_unique();
    double* p = (double*)d.st->host_write();
    d.st->host_external = true;
    return p;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return nullptr;
  }
}

// Read one element (two doubles for complex) without downloading the tensor.
void read_elem(const Dense& d, size_t i, double* out) {
  Storage& s = *d.st;
  size_t w = d.dt == DType::F64 ? 1 : 2;
  if (s.uniform) {
    out[0] = s.fill_re;
    if (w == 2) out[1] = s.fill_im;
    return;
  }
  if (s.host_valid) {
    memcpy(out, (const double*)s.host + i * w, w * 8);
    return;
  }
  if (s.dev_valid) {
    DeviceCtx& c = ctx(s.device);
    NDT_CUDA(cudaMemcpyAsync(out, (const double*)s.dev + i * w, w * 8, cudaMemcpyDeviceToHost, c.compute));
    NDT_CUDA(cudaStreamSynchronize(c.compute));
    return;
  }
  memset(out, 0, w * 8);
}

void write_elem(Dense& d, size_t i, const double* v) {
  d.make_unique();
  Storage& s = *d.st;
  size_t w = d.dt == DType::F64 ? 1 : 2;
  if (!s.uniform && s.dev_valid && !s.host_external) {
    DeviceCtx& c = ctx(s.device);
    NDT_CUDA(cudaMemcpyAsync((double*)s.dev + i * w, v, w * 8, cudaMemcpyHostToDevice, c.compute));
    NDT_CUDA(cudaStreamSynchronize(c.compute));
    if (s.host_valid) memcpy((double*)s.host + i * w, v, w * 8);
    return;
  }
  double* h = (double*)s.host_write();
  memcpy(h + i * w, v, w * 8);
}

int get_linear_impl(const void* t, size_t i, double* out) {
  if (!t || !out) return NDT_INVALID_ARGUMENT;
  try {
    const Dense& d = H(t)->t;
    if (i >= d.len()) return NDT_INDEX_OUT_OF_BOUNDS;
    read_elem(d, i, out);
    return NDT_SUCCESS;
  } catch (const Error& e) {
    return map_error(e, NDT_INTERNAL_ERROR);
  } catch (...) {
    return NDT_INTERNAL_ERROR;
  }
}

int set_linear_impl(void* t, size_t i, const double* v) {
  if (!t) return NDT_INVALID_ARGUMENT;
  try {
    Dense& d = H(t)->t;
    if (i >= d.len()) return NDT_INDEX_OUT_OF_BOUNDS;
    write_elem(d, i, v);
    return NDT_SUCCESS;
  } catch (const Error& e) {
    return map_error(e, NDT_INTERNAL_ERROR);
  } catch (...) {
    return NDT_INTERNAL_ERROR;
  }
}

int fill_impl(void* t, double re, double im) {
  if (!t) return NDT_INVALID_ARGUMENT;
  try {
    Dense& d = H(t)->t;
    if (d.st.use_count() > 1) d.st = std::make_shared<Storage>(d.dt, d.len());
    d.st->set_uniform(re, im);
    return NDT_SUCCESS;
  } catch (...) {
    return NDT_INTERNAL_ERROR;
  }
}

void* permutedims_impl(const void* t, const size_t* perm, size_t ndim, int* status) {
  if (!status) return nullptr;
  if (!t || !perm) {
    *status = NDT_INVALID_ARGUMENT;
    return nullptr;
  }
  try {
    std::vector<size_t> p(perm, perm + ndim);
    NdtHandle* h = new NdtHandle{permutedims(H(t)->t, p)};
    *status = NDT_SUCCESS;
    return h;
  } catch (const Error& e) {
    *status = map_error(e, NDT_INVALID_PERMUTATION);
  } catch (const std::exception& e) {
    set_last_error(e.what());
    *status = NDT_INTERNAL_ERROR;
  } catch (...) {
    *status = NDT_INTERNAL_ERROR;
  }
  return nullptr;
}

void* contract_impl(const void* a, const long* la, size_t na, const void* b, const long* lb, size_t nb, int* status,
                    ContractSemantics sem) {
  if (!status) return nullptr;
  if (!a || !b || !la || !lb) {
    *status = NDT_INVALID_ARGUMENT;
    return nullptr;
  }
  try {
    NdtHandle* h = new NdtHandle{contract(H(a)->t, labels_of(la, na), H(b)->t, labels_of(lb, nb), sem)};
    *status = NDT_SUCCESS;
    return h;
  } catch (const Error& e) {
    *status = map_error(e, NDT_SHAPE_MISMATCH);
  } catch (const std::exception& e) {
    set_last_error(e.what());
    *status = NDT_INTERNAL_ERROR;
  } catch (...) {
    *status = NDT_INTERNAL_ERROR;
  }
  return nullptr;
}

void* contract_shard_impl(const void* a, const long* la, size_t na, const void* b, const long* lb, size_t nb,
                          long axis_label, int rank, int nranks, int* status) {
  if (!status) return nullptr;
  if (!a || !b || (!la && na) || (!lb && nb) || nranks < 1 || rank < 0 || rank >= nranks) {
    set_last_error("contract_gemm_shard: NULL argument or rank outside [0, nranks)");
    *status = NDT_INVALID_ARGUMENT;
    return nullptr;
  }
  try {
    NdtHandle* h = new NdtHandle{contract_gemm_shard(H(a)->t, labels_of(la, na), H(b)->t, labels_of(lb, nb),
                                                     (int32_t)axis_label, rank, nranks)};
    *status = NDT_SUCCESS;
    return h;
  } catch (const Error& e) {
    *status = map_error(e, NDT_SHAPE_MISMATCH);
  } catch (const std::exception& e) {
    set_last_error(e.what());
    *status = NDT_INTERNAL_ERROR;
  } catch (...) {
    *status = NDT_INTERNAL_ERROR;
  }
  return nullptr;
}

const double* device_ptr_impl(const void* t) {
  if (!t) return nullptr;
  try {
    Storage& st = *H(t)->t.st;
    const double* p = (const double*)st.dev_read();
    settle_for_caller(st.device);
    return p;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return nullptr;
  }
}

double* device_ptr_mut_impl(void* t) {
  if (!t) return nullptr;
  try {
    Dense& d = H(t)->t;
    d.make_unique();  // copy on write, as data_mut
    double* p = (double*)d.st->dev_write();
    settle_for_caller(d.st->device);
    return p;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return nullptr;
  }
}

}  // namespace

extern "C" {

// ------------------------------------------------------------------ f64
ndt_tensor_f64* ndt_tensor_f64_zeros(const size_t* shape, size_t ndim, int* status) {
  return (ndt_tensor_f64*)create(shape, ndim, status,
                                 [](const std::vector<size_t>& s) { return make_uniform(DType::F64, s, 0.0, 0.0); });
}
ndt_tensor_f64* ndt_tensor_f64_ones(const size_t* shape, size_t ndim, int* status) {
  return (ndt_tensor_f64*)create(shape, ndim, status,
                                 [](const std::vector<size_t>& s) { return make_uniform(DType::F64, s, 1.0, 0.0); });
}
ndt_tensor_f64* ndt_tensor_f64_rand(const size_t* shape, size_t ndim, int* status) {
  return (ndt_tensor_f64*)create(shape, ndim, status,
                                 [](const std::vector<size_t>& s) { return random_tensor(s, false); });
}
ndt_tensor_f64* ndt_tensor_f64_randn(const size_t* shape, size_t ndim, int* status) {
  return (ndt_tensor_f64*)create(shape, ndim, status,
                                 [](const std::vector<size_t>& s) { return random_tensor(s, true); });
}
ndt_tensor_f64* ndt_tensor_f64_from_data(const double* data, size_t len, const size_t* shape, size_t ndim,
                                         int* status) {
  return (ndt_tensor_f64*)from_data_impl(DType::F64, data, len, shape, ndim, status);
}
void ndt_tensor_f64_release(ndt_tensor_f64* t) { delete H(t); }
ndt_tensor_f64* ndt_tensor_f64_clone(const ndt_tensor_f64* src) {
  if (!src) return nullptr;
  try {
    return (ndt_tensor_f64*)new NdtHandle{H(src)->t};
  } catch (...) {
    return nullptr;
  }
}
size_t ndt_tensor_f64_ndim(const ndt_tensor_f64* t) { return ndim_impl(t); }
size_t ndt_tensor_f64_len(const ndt_tensor_f64* t) { return len_impl(t); }
int ndt_tensor_f64_shape(const ndt_tensor_f64* t, size_t* out) { return shape_impl(t, out); }
const double* ndt_tensor_f64_data(const ndt_tensor_f64* t) { return data_impl(t); }
double* ndt_tensor_f64_data_mut(ndt_tensor_f64* t) { return data_mut_impl(t); }
int ndt_tensor_f64_get_linear(const ndt_tensor_f64* t, size_t index, double* out) {
  return get_linear_impl(t, index, out);
}
int ndt_tensor_f64_set_linear(ndt_tensor_f64* t, size_t index, double value) {
  return set_linear_impl(t, index, &value);
}
int ndt_tensor_f64_fill(ndt_tensor_f64* t, double value) { return fill_impl(t, value, 0.0); }
ndt_tensor_f64* ndt_tensor_f64_permutedims(const ndt_tensor_f64* t, const size_t* perm, size_t ndim, int* status) {
  return (ndt_tensor_f64*)permutedims_impl(t, perm, ndim, status);
}
ndt_tensor_f64* ndt_tensor_f64_contract(const ndt_tensor_f64* a, const long* la, size_t na, const ndt_tensor_f64* b,
                                        const long* lb, size_t nb, int* status) {
  return (ndt_tensor_f64*)contract_impl(a, la, na, b, lb, nb, status, ContractSemantics::Naive);
}
ndt_tensor_f64* ndt_tensor_f64_contract_gemm(const ndt_tensor_f64* a, const long* la, size_t na,
                                             const ndt_tensor_f64* b, const long* lb, size_t nb, int* status) {
  return (ndt_tensor_f64*)contract_impl(a, la, na, b, lb, nb, status, ContractSemantics::Gemm);
}
ndt_tensor_f64* ndt_tensor_f64_contract_gemm_shard(const ndt_tensor_f64* a, const long* la, size_t na,
                                                   const ndt_tensor_f64* b, const long* lb, size_t nb, long axis_label,
                                                   int rank, int nranks, int* status) {
  return (ndt_tensor_f64*)contract_shard_impl(a, la, na, b, lb, nb, axis_label, rank, nranks, status);
}

void ndt_tensor_f64_contract_vjp(const ndt_tensor_f64* a, const long* la, size_t na, const ndt_tensor_f64* b,
                                 const long* lb, size_t nb, const ndt_tensor_f64* grad, ndt_tensor_f64** ga,
                                 ndt_tensor_f64** gb, int* status) {
  if (!status) return;
  if (!a || !b || !grad || !la || !lb || !ga || !gb) {
    *status = NDT_INVALID_ARGUMENT;
    return;
  }
  try {
    Dense da, db;
    contract_vjp(H(a)->t, labels_of(la, na), H(b)->t, labels_of(lb, nb), H(grad)->t, &da, &db);
    *ga = (ndt_tensor_f64*)new NdtHandle{da};
    *gb = (ndt_tensor_f64*)new NdtHandle{db};
    *status = NDT_SUCCESS;
  } catch (const Error& e) {
    int code = map_error(e, NDT_SHAPE_MISMATCH);
    *ga = nullptr;
    *gb = nullptr;
    *status = code;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    *ga = nullptr;
    *gb = nullptr;
    *status = NDT_INTERNAL_ERROR;
  } catch (...) {
    *ga = nullptr;
    *gb = nullptr;
    *status = NDT_INTERNAL_ERROR;
  }
}

void ndt_tensor_f64_contract_jvp(const ndt_tensor_f64* a, const long* la, size_t na, const ndt_tensor_f64* b,
                                 const long* lb, size_t nb, const ndt_tensor_f64* ta, const ndt_tensor_f64* tb,
                                 ndt_tensor_f64** primal_out, ndt_tensor_f64** tangent_out, int* status) {
  if (!status) return;
  if (!a || !b || !la || !lb || !primal_out || !tangent_out) {
    *status = NDT_INVALID_ARGUMENT;
    return;
  }
  std::vector<int32_t> l1 = labels_of(la, na), l2 = labels_of(lb, nb);
  Dense primal, tangent;
  bool have_tangent = false;
  // contract_jvp (naive.rs:550-583); on a TensorError the reference returns
  // NDT_SHAPE_MISMATCH without writing the out-pointers (lib.rs:864-880).
  try {
    primal = contract(H(a)->t, l1, H(b)->t, l2, ContractSemantics::Naive);
    if (ta && tb) {
      Dense d1 = contract(H(ta)->t, l1, H(b)->t, l2, ContractSemantics::Naive);
      Dense d2 = contract(H(a)->t, l1, H(tb)->t, l2, ContractSemantics::Naive);
      tangent = add(d1, d2);
      have_tangent = true;
    } else if (ta) {
      tangent = contract(H(ta)->t, l1, H(b)->t, l2, ContractSemantics::Naive);
      have_tangent = true;
    } else if (tb) {
      tangent = contract(H(a)->t, l1, H(tb)->t, l2, ContractSemantics::Naive);
      have_tangent = true;
    }
  } catch (const Error& e) {
    int code = map_error(e, NDT_SHAPE_MISMATCH);
    if (code == NDT_INTERNAL_ERROR) {
      *primal_out = nullptr;
      *tangent_out = nullptr;
    }
    *status = code;
    return;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    *primal_out = nullptr;
    *tangent_out = nullptr;
    *status = NDT_INTERNAL_ERROR;
    return;
  }
  *primal_out = (ndt_tensor_f64*)new NdtHandle{primal};
  *tangent_out = have_tangent ? (ndt_tensor_f64*)new NdtHandle{tangent} : nullptr;
  *status = NDT_SUCCESS;
}

// ------------------------------------------------------------------ c64
ndt_tensor_c64* ndt_tensor_c64_zeros(const size_t* shape, size_t ndim, int* status) {
  return (ndt_tensor_c64*)create(shape, ndim, status,
                                 [](const std::vector<size_t>& s) { return make_uniform(DType::C128, s, 0.0, 0.0); });
}
ndt_tensor_c64* ndt_tensor_c64_ones(const size_t* shape, size_t ndim, int* status) {
  return (ndt_tensor_c64*)create(shape, ndim, status,
                                 [](const std::vector<size_t>& s) { return make_uniform(DType::C128, s, 1.0, 0.0); });
}
ndt_tensor_c64* ndt_tensor_c64_from_data(const double* data, size_t len, const size_t* shape, size_t ndim,
                                         int* status) {
  return (ndt_tensor_c64*)from_data_impl(DType::C128, data, len, shape, ndim, status);
}
void ndt_tensor_c64_release(ndt_tensor_c64* t) { delete H(t); }
ndt_tensor_c64* ndt_tensor_c64_clone(const ndt_tensor_c64* src) {
  if (!src) return nullptr;
  try {
    return (ndt_tensor_c64*)new NdtHandle{H(src)->t};
  } catch (...) {
    return nullptr;
  }
}
size_t ndt_tensor_c64_ndim(const ndt_tensor_c64* t) { return ndim_impl(t); }
size_t ndt_tensor_c64_len(const ndt_tensor_c64* t) { return len_impl(t); }
int ndt_tensor_c64_shape(const ndt_tensor_c64* t, size_t* out) { return shape_impl(t, out); }
const double* ndt_tensor_c64_data(const ndt_tensor_c64* t) { return data_impl(t); }
double* ndt_tensor_c64_data_mut(ndt_tensor_c64* t) { return data_mut_impl(t); }
int ndt_tensor_c64_get_linear(const ndt_tensor_c64* t, size_t index, double* re, double* im) {
  if (!re || !im) return NDT_INVALID_ARGUMENT;
  double v[2];
  int st = get_linear_impl(t, index, v);
  if (st == NDT_SUCCESS) {
    *re = v[0];
    *im = v[1];
  }
  return st;
}
int ndt_tensor_c64_set_linear(ndt_tensor_c64* t, size_t index, double re, double im) {
  double v[2] = {re, im};
  return set_linear_impl(t, index, v);
}
int ndt_tensor_c64_fill(ndt_tensor_c64* t, double re, double im) { return fill_impl(t, re, im); }
ndt_tensor_c64* ndt_tensor_c64_permutedims(const ndt_tensor_c64* t, const size_t* perm, size_t ndim, int* status) {
  return (ndt_tensor_c64*)permutedims_impl(t, perm, ndim, status);
}
ndt_tensor_c64* ndt_tensor_c64_contract(const ndt_tensor_c64* a, const long* la, size_t na, const ndt_tensor_c64* b,
                                        const long* lb, size_t nb, int* status) {
  return (ndt_tensor_c64*)contract_impl(a, la, na, b, lb, nb, status, ContractSemantics::Naive);
}
ndt_tensor_c64* ndt_tensor_c64_contract_gemm(const ndt_tensor_c64* a, const long* la, size_t na,
                                             const ndt_tensor_c64* b, const long* lb, size_t nb, int* status) {
  return (ndt_tensor_c64*)contract_impl(a, la, na, b, lb, nb, status, ContractSemantics::Gemm);
}
ndt_tensor_c64* ndt_tensor_c64_contract_gemm_shard(const ndt_tensor_c64* a, const long* la, size_t na,
                                                   const ndt_tensor_c64* b, const long* lb, size_t nb, long axis_label,
                                                   int rank, int nranks, int* status) {
  return (ndt_tensor_c64*)contract_shard_impl(a, la, na, b, lb, nb, axis_label, rank, nranks, status);
}

// ------------------------------------------------------- device interop
ndt_tensor_f64* ndt_tensor_f64_from_device_ptr(const double* dptr, size_t len, const size_t* shape, size_t ndim,
                                               int* status) {
  return (ndt_tensor_f64*)from_device_impl(DType::F64, dptr, len, shape, ndim, status);
}
const double* ndt_tensor_f64_device_ptr(const ndt_tensor_f64* t) { return device_ptr_impl(t); }
double* ndt_tensor_f64_device_ptr_mut(ndt_tensor_f64* t) { return device_ptr_mut_impl(t); }
ndt_tensor_c64* ndt_tensor_c64_from_device_ptr(const double* dptr, size_t len, const size_t* shape, size_t ndim,
                                               int* status) {
  return (ndt_tensor_c64*)from_device_impl(DType::C128, dptr, len, shape, ndim, status);
}
const double* ndt_tensor_c64_device_ptr(const ndt_tensor_c64* t) { return device_ptr_impl(t); }
double* ndt_tensor_c64_device_ptr_mut(ndt_tensor_c64* t) { return device_ptr_mut_impl(t); }

int ndt_b200_permutedims_dev(int dtype, const void* src, void* dst, const size_t* shape, size_t ndim,
                             const size_t* perm, size_t nperm, void* stream) {
  if (!src || !dst || (!shape && ndim) || (!perm && nperm) || (dtype != 0 && dtype != 1))
    return NDT_INVALID_ARGUMENT;
  try {
    if (nperm != ndim) return NDT_INVALID_PERMUTATION;
    std::vector<char> seen(ndim, 0);
    for (size_t i = 0; i < nperm; i++) {
      if (perm[i] >= ndim || seen[perm[i]]) return NDT_INVALID_PERMUTATION;
      seen[perm[i]] = 1;
    }
    std::vector<size_t> sh(shape, shape + ndim);
    for (size_t x : sh)
      if (x == 0) return NDT_INTERNAL_ERROR;  // the reference panics on zero extents
    DType dt = dtype ? DType::C128 : DType::F64;
    cudaStream_t s = (cudaStream_t)stream;  // NULL = the legacy default stream, as in CUDA
    ctx();
    std::vector<size_t> ss = col_major_strides(sh);
    GatherDesc g;
    for (size_t i = 0; i < ndim; i++) {
      g.shape.push_back(sh[perm[i]]);
      g.src_strides.push_back((int64_t)ss[perm[i]]);
    }
    if (ndim == 0) {
      NDT_CUDA(cudaMemcpyAsync(dst, src, esize(dt), cudaMemcpyDeviceToDevice, s));
      return NDT_SUCCESS;
    }
    gather(dt, src, dst, g, s);
    return NDT_SUCCESS;
  } catch (const Error& e) {
    return map_error(e, NDT_INTERNAL_ERROR);
  } catch (...) {
    return NDT_INTERNAL_ERROR;
  }
}

int ndt_b200_gemm_dev(int dtype, long m, long n, long k, const void* A, long lda, int a_kmajor, const void* B,
                      long ldb, int b_kmajor, void* C, long ldc, int accumulate, void* stream) {
  if (!A || !B || !C || m < 0 || n < 0 || k < 0 || (dtype != 0 && dtype != 1)) return NDT_INVALID_ARGUMENT;
  try {
    cudaStream_t s = (cudaStream_t)stream;  // NULL = the legacy default stream, as in CUDA
    ctx();
    gemm(dtype ? DType::C128 : DType::F64, m, n, k, GemmOperand{A, lda, a_kmajor != 0},
         GemmOperand{B, ldb, b_kmajor != 0}, C, ldc, accumulate != 0, s);
    return NDT_SUCCESS;
  } catch (const Error& e) {
    return map_error(e, NDT_INTERNAL_ERROR);
  } catch (...) {
    return NDT_INTERNAL_ERROR;
  }
}

// ---------------------------------------------------------- control
int ndt_b200_device_available(void) { return device_available() ? 1 : 0; }

int ndt_b200_set_stream(void* stream) {
  try {
    DeviceCtx& c = ctx();
    // Finish everything queued on the old stream so that buffers freed later
    // on the new stream cannot race with it.
    NDT_CUDA(cudaStreamSynchronize(c.compute));
    c.compute = stream ? (cudaStream_t)stream : c.own_compute;
    c.external_stream = stream != nullptr;
    return NDT_SUCCESS;
  } catch (const Error& e) {
    return map_error(e, NDT_INTERNAL_ERROR);
  }
}
void* ndt_b200_get_stream(void) {
  try {
    return (void*)ctx().compute;
  } catch (...) {
    return nullptr;
  }
}
int ndt_b200_synchronize(void) {
  try {
    NDT_CUDA(cudaStreamSynchronize(ctx().compute));
    return NDT_SUCCESS;
  } catch (const Error& e) {
    return map_error(e, NDT_INTERNAL_ERROR);
  }
}
const char* ndt_b200_last_error(void) { return last_error(); }
unsigned long long ndt_b200_launch_count(void) { return (unsigned long long)launch_count(); }
void ndt_b200_empty_cache(void) {
  try {
    empty_caches();
  } catch (...) {
  }
}

}  // extern "C"
