// FP64 tensor-core peak microbenchmark (measurement support for the bench,
// built as its own small library, not part of the contraction ABI).
//
// The FP64 contraction kernels run on mma.sync.m16n8k8.f64 (DMMA); this
// kernel issues that instruction back to back from registers only (8
// independent accumulator chains per warp, no memory traffic) on every SM,
// which is the roofline denominator for the FP64 GEMM-shaped work.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>

namespace {

template <int K16>
__global__ void dmma_peak_kernel(double* out, int iters) {
  constexpr int NACC = 8;
  double c[NACC][4];
  double a[8], b[4];
  const int lane = threadIdx.x & 31;
  for (int i = 0; i < 8; i++) a[i] = 1e-3 * (lane + i);
  for (int i = 0; i < 4; i++) b[i] = 1e-3 * (lane - i);
  for (int j = 0; j < NACC; j++)
    for (int i = 0; i < 4; i++) c[j][i] = 0;
  for (int it = 0; it < iters; it++) {
#pragma unroll
    for (int j = 0; j < NACC; j++) {
      if constexpr (K16) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7,%8,%9,%10,%11}, "
            "{%12,%13,%14,%15}, {%0,%1,%2,%3};"
            : "+d"(c[j][0]), "+d"(c[j][1]), "+d"(c[j][2]), "+d"(c[j][3])
            : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(a[4]), "d"(a[5]), "d"(a[6]), "d"(a[7]), "d"(b[0]),
              "d"(b[1]), "d"(b[2]), "d"(b[3]));
      } else {
        asm volatile(
            "mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+d"(c[j][0]), "+d"(c[j][1]), "+d"(c[j][2]), "+d"(c[j][3])
            : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(b[0]), "d"(b[1]));
      }
    }
  }
  double s = 0;
  for (int j = 0; j < NACC; j++)
    for (int i = 0; i < 4; i++) s += c[j][i];
  out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

template <int K16>
double run(int warps, int iters, cudaStream_t s) {
  int dev = 0, nsm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  const int grid = nsm, block = 32 * warps;
  double* out = nullptr;
  if (cudaMallocAsync(&out, sizeof(double) * grid * block, s) != cudaSuccess) return -1;
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  dmma_peak_kernel<K16><<<grid, block, 0, s>>>(out, 16);
  float best = 1e30f;
  for (int r = 0; r < 5; r++) {
    cudaEventRecord(e0, s);
    dmma_peak_kernel<K16><<<grid, block, 0, s>>>(out, iters);
    cudaEventRecord(e1, s);
    cudaEventSynchronize(e1);
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    best = std::min(best, ms);
  }
  cudaFreeAsync(out, s);
  cudaStreamSynchronize(s);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (cudaGetLastError() != cudaSuccess) return -1;
  const double flop = (double)grid * warps * iters * 8.0 * 2.0 * 16 * 8 * (K16 ? 16 : 8);
  return flop / (best * 1e-3) / 1e12;
}

}  // namespace

// Best FP64 tensor rate (TFLOP/s) over m16n8k8 / m16n8k16 and 8 / 16 warps
// per SM on the current device; -1 on a CUDA error.
extern "C" __attribute__((visibility("default"))) double ndt_fp64_tensor_peak_tflops(void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  double best = -1;
  for (int w : {8, 16}) {
    best = std::max(best, run<0>(w, 4096, s));
    best = std::max(best, run<1>(w, 2048, s));
  }
  return best;
}
