// Elementwise device helpers: fill (lazy zeros / ones / fill), add (the
// apply_binary(+) used by contract_jvp, operations/elementwise.rs:189-210),
// scale.
#include <algorithm>

#include "ndt_internal.h"

namespace ndt {

namespace {
constexpr int kThreads = 256;

__global__ void fill_f64(double* p, int64_t n, double v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    p[i] = v;
}
__global__ void fill_c128(double2* p, int64_t n, double re, double im) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    p[i] = make_double2(re, im);
}
__global__ void add_f64(const double* a, const double* b, double* c, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    c[i] = a[i] + b[i];
}
__global__ void scale_f64(const double* a, double* c, int64_t n, double s) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    c[i] = a[i] * s;
}
__global__ void scale_c128(const double2* a, double2* c, int64_t n, double re, double im) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    double2 x = a[i];
    // (x.re + i x.im)(re + i im), same operation order as num-complex's Mul
    c[i] = make_double2(x.x * re - x.y * im, x.x * im + x.y * re);
  }
}

int grid_of(int64_t n) {
  const DeviceCtx& c = ctx();
  int64_t g = (n + kThreads - 1) / kThreads;
  return (int)std::max<int64_t>(1, std::min<int64_t>(g, (int64_t)c.sm_count * 8));
}
}  // namespace

void fill_device(DType dt, void* p, size_t n, double re, double im, cudaStream_t s) {
  if (n == 0) return;
  if (dt == DType::F64)
    fill_f64<<<grid_of(n), kThreads, 0, s>>>((double*)p, (int64_t)n, re);
  else
    fill_c128<<<grid_of(n), kThreads, 0, s>>>((double2*)p, (int64_t)n, re, im);
  count_launch();
  NDT_CUDA(cudaGetLastError());
}

void add_device(DType dt, const void* a, const void* b, void* c, size_t n, cudaStream_t s) {
  // complex addition is componentwise: treat as 2n doubles
  int64_t m = (int64_t)n * (dt == DType::F64 ? 1 : 2);
  if (m == 0) return;
  add_f64<<<grid_of(m), kThreads, 0, s>>>((const double*)a, (const double*)b, (double*)c, m);
  count_launch();
  NDT_CUDA(cudaGetLastError());
}

void scale_device(DType dt, const void* a, void* c, size_t n, double re, double im, cudaStream_t s) {
  if (n == 0) return;
  if (dt == DType::F64)
    scale_f64<<<grid_of(n), kThreads, 0, s>>>((const double*)a, (double*)c, (int64_t)n, re);
  else
    scale_c128<<<grid_of(n), kThreads, 0, s>>>((const double2*)a, (double2*)c, (int64_t)n, re, im);
  count_launch();
  NDT_CUDA(cudaGetLastError());
}

}  // namespace ndt
