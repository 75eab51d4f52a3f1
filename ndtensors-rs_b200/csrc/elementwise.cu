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

// Split-K sum: C[i + j*ldc] (+)= sum_s W[s][i + j*m], partials summed in
// split order (deterministic).  T is double or double2.
template <typename T>
__global__ void splitk_reduce_kernel(const T* __restrict__ w, int nsplit, int64_t m, int64_t n, T* c, int64_t ldc,
                                     int accumulate) {
  const int64_t mn = m * n;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < mn; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = e / m, i = e - j * m;
    T acc = w[e];
    for (int s = 1; s < nsplit; s++) {
      const T v = w[(int64_t)s * mn + e];
      if constexpr (sizeof(T) == 16) {
        acc.x += v.x;
        acc.y += v.y;
      } else {
        acc += v;
      }
    }
    T* p = c + i + j * ldc;
    if (accumulate) {
      const T o = *p;
      if constexpr (sizeof(T) == 16) {
        acc.x += o.x;
        acc.y += o.y;
      } else {
        acc += o;
      }
    }
    *p = acc;
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

void splitk_reduce(DType dt, const void* w, int nsplit, int64_t m, int64_t n, void* c, int64_t ldc, bool accumulate,
                   cudaStream_t s) {
  if (m <= 0 || n <= 0) return;
  if (dt == DType::F64)
    splitk_reduce_kernel<double><<<grid_of(m * n), kThreads, 0, s>>>((const double*)w, nsplit, m, n, (double*)c, ldc,
                                                                     accumulate ? 1 : 0);
  else
    splitk_reduce_kernel<double2><<<grid_of(m * n), kThreads, 0, s>>>((const double2*)w, nsplit, m, n, (double2*)c,
                                                                      ldc, accumulate ? 1 : 0);
  count_launch();
  NDT_CUDA(cudaGetLastError());
}

}  // namespace ndt
