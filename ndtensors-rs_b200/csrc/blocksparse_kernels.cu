// Device kernels for block-sparse storage.
//
//   bs_dense_map      packed block data <-> dense tensor (to_dense / from_dense,
//                     blocksparse_tensor.rs:290-391): one thread per packed
//                     element, the block found by binary search over the
//                     packed offsets, the dense offset from the block's start
//                     and the dense strides.
//   diag_scatter      diagonal values -> dense tensor or dense diagonal blocks
//                     (diagblocksparse_tensor.rs:399-426).
//   bs_diag_scale     out block = A block with its last axis scaled by the
//                     diagonal of the matching diag block (the fused
//                     block-sparse x diag-block-sparse contraction).
//   copy_segments     many (src, dst, bytes) copies in one launch: 64 KB
//                     work items, the segment found by binary search over
//                     the items' prefix, 16-byte vectors where a segment's
//                     addresses and length allow (assembling gathered shards
//                     into sorted block order).
#include <algorithm>
#include <cstring>

#include "ndt_internal.h"

namespace ndt {

namespace {
constexpr int kThreads = 256;

__device__ __forceinline__ int find_block(const int64_t* offs, int nblocks, int64_t e) {
  int lo = 0, hi = nblocks - 1;  // offs[b] <= e < offs[b+1]
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (offs[mid] <= e)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

template <typename T>
__global__ void dense_map_kernel(T* packed, T* dense, const int64_t* __restrict__ offs,
                                 const BsBlockDesc* __restrict__ blocks, int nblocks, int64_t total, int to_dense) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int b = find_block(offs, nblocks, e);
    const BsBlockDesc& d = blocks[b];
    int64_t r = e - offs[b], off = d.dense_base;
    for (int k = 0; k < d.ndim; k++) {
      int64_t i = r % d.shape[k];
      r /= d.shape[k];
      off += i * d.dstride[k];
    }
    if (to_dense)
      dense[off] = packed[e];
    else
      packed[e] = dense[off];
  }
}

template <typename T>
__global__ void diag_scatter_kernel(const T* __restrict__ diag, T* out, const int64_t* __restrict__ offs,
                                    const BsBlockDesc* __restrict__ blocks, int nblocks, int64_t total) {
  // element i of diagonal block b goes to out[dense_base + i * dstride[0]]
  // (dstride[0] holds the sum of the strides along every axis)
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int b = find_block(offs, nblocks, e);
    const BsBlockDesc& d = blocks[b];
    out[d.dense_base + (e - offs[b]) * d.dstride[0]] = diag[e];
  }
}

__device__ __forceinline__ double mulc(double a, double s) { return a * s; }
__device__ __forceinline__ double2 mulc(double2 a, double2 s) {
  return make_double2(a.x * s.x - a.y * s.y, a.x * s.y + a.y * s.x);
}

// One output block of the diagonal scale, reduced to what the kernel reads:
// source / output / diagonal offsets, the column length (product of all but
// the last extent), the number of columns (last extent), the diagonal length
// and the block's first global column.
struct DiagCols {
  int64_t src, out, diag, inner, ncols, ndiag, col0;
};

// One warp per output column j of a block: out[:, j] = a[:, j] * s[j] for
// j < ndiag, zero beyond (a diagonal block shorter than the axis).  The
// column is contiguous (column-major, last axis slowest), so the warp streams
// it with coalesced loads; the block is found once per column.
template <typename T>
__global__ void __launch_bounds__(kThreads) diag_scale_kernel(const T* __restrict__ a, const T* __restrict__ s,
                                                              T* __restrict__ out, const DiagCols* __restrict__ blk,
                                                              int nblocks, int64_t ncols) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = ((int64_t)gridDim.x * kThreads) >> 5;
  for (int64_t c = ((int64_t)blockIdx.x * kThreads + threadIdx.x) >> 5; c < ncols; c += nwarps) {
    int lo = 0, hi = nblocks - 1;  // largest b with col0 <= c
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (blk[mid].col0 <= c)
        lo = mid;
      else
        hi = mid - 1;
    }
    const DiagCols d = blk[lo];
    const int64_t j = c - d.col0;
    const T* src = a + d.src + j * d.inner;
    T* dst = out + d.out + j * d.inner;
    if (j < d.ndiag) {
      const T sv = s[d.diag + j];
#pragma unroll 4
      for (int64_t i = lane; i < d.inner; i += 32) dst[i] = mulc(src[i], sv);
    } else {
#pragma unroll 4
      for (int64_t i = lane; i < d.inner; i += 32) dst[i] = T{};
    }
  }
}

int grid_of(int64_t n) {
  const DeviceCtx& c = ctx();
  int64_t g = (n + kThreads - 1) / kThreads;
  return (int)std::max<int64_t>(1, std::min<int64_t>(g, (int64_t)c.sm_count * 8));
}

struct Tables {
  int64_t* offs;
  BsBlockDesc* blocks;
  void* mem;
};

Tables upload(const std::vector<int64_t>& offs, const std::vector<BsBlockDesc>& blocks, cudaStream_t s) {
  size_t b1 = offs.size() * sizeof(int64_t);
  size_t o2 = (b1 + 255) / 256 * 256;
  size_t total = o2 + blocks.size() * sizeof(BsBlockDesc);
  std::vector<char> h(total);
  memcpy(h.data(), offs.data(), b1);
  memcpy(h.data() + o2, blocks.data(), blocks.size() * sizeof(BsBlockDesc));
  void* d = nullptr;
  d = (decltype(d))pool_alloc(total, s);
  NDT_CUDA(cudaMemcpyAsync(d, h.data(), total, cudaMemcpyHostToDevice, s));
  return Tables{(int64_t*)d, (BsBlockDesc*)((char*)d + o2), d};
}
constexpr int64_t kSegChunk = 65536;  // bytes per work item

struct CopySeg {
  int64_t src, dst, bytes;  // byte offsets and length
  int64_t item0;            // first work item of the segment
};

__global__ void __launch_bounds__(kThreads) copy_segments_kernel(const char* __restrict__ src, char* __restrict__ dst,
                                                                 const CopySeg* __restrict__ segs, int nseg,
                                                                 int64_t nitems) {
  for (int64_t it = blockIdx.x; it < nitems; it += gridDim.x) {
    int lo = 0, hi = nseg - 1;  // segs[s].item0 <= it < segs[s+1].item0
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (segs[mid].item0 <= it)
        lo = mid;
      else
        hi = mid - 1;
    }
    const CopySeg sg = segs[lo];
    const int64_t b0 = (it - sg.item0) * kSegChunk;
    const int64_t b1 = min(b0 + kSegChunk, sg.bytes);
    const char* sp = src + sg.src;
    char* dp = dst + sg.dst;
    if (((sg.src | sg.dst | sg.bytes) & 15) == 0) {
      for (int64_t b = b0 + threadIdx.x * 16; b < b1; b += kThreads * 16)
        *reinterpret_cast<int4*>(dp + b) = *reinterpret_cast<const int4*>(sp + b);
    } else {
      for (int64_t b = b0 + threadIdx.x * 8; b < b1; b += kThreads * 8)
        *reinterpret_cast<double*>(dp + b) = *reinterpret_cast<const double*>(sp + b);
    }
  }
}
}  // namespace

void copy_segments(const void* src, void* dst, const std::vector<int64_t>& src_off, const std::vector<int64_t>& dst_off,
                   const std::vector<int64_t>& bytes, cudaStream_t s) {
  std::vector<CopySeg> h;
  int64_t items = 0;
  for (size_t i = 0; i < bytes.size(); i++) {
    if (bytes[i] <= 0) continue;
    if ((src_off[i] | dst_off[i] | bytes[i]) & 7) throw Error(ErrKind::Panic, "copy_segments: not 8-byte aligned");
    h.push_back(CopySeg{src_off[i], dst_off[i], bytes[i], items});
    items += (bytes[i] + kSegChunk - 1) / kSegChunk;
  }
  if (h.empty()) return;
  if ((((uintptr_t)src) | ((uintptr_t)dst)) & 15) throw Error(ErrKind::Panic, "copy_segments: base not 16-byte aligned");
  CopySeg* d = nullptr;
  const size_t tb = h.size() * sizeof(CopySeg);
  d = (decltype(d))pool_alloc(tb, s);
  NDT_CUDA(cudaMemcpyAsync(d, h.data(), tb, cudaMemcpyHostToDevice, s));
  const DeviceCtx& c = ctx();
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(items, (int64_t)c.sm_count * 8));
  copy_segments_kernel<<<grid, kThreads, 0, s>>>((const char*)src, (char*)dst, d, (int)h.size(), items);
  count_launch();
  NDT_CUDA(cudaGetLastError());
  NDT_CUDA(cudaFreeAsync(d, s));
}

void bs_dense_map(DType dt, void* packed, void* dense, const std::vector<int64_t>& offs,
                  const std::vector<BsBlockDesc>& blocks, int64_t total, bool to_dense, cudaStream_t s) {
  if (total <= 0 || blocks.empty()) return;
  Tables t = upload(offs, blocks, s);
  if (dt == DType::F64)
    dense_map_kernel<double><<<grid_of(total), kThreads, 0, s>>>((double*)packed, (double*)dense, t.offs, t.blocks,
                                                                 (int)blocks.size(), total, to_dense ? 1 : 0);
  else
    dense_map_kernel<double2><<<grid_of(total), kThreads, 0, s>>>((double2*)packed, (double2*)dense, t.offs,
                                                                  t.blocks, (int)blocks.size(), total, to_dense ? 1 : 0);
  count_launch();
  NDT_CUDA(cudaGetLastError());
  NDT_CUDA(cudaFreeAsync(t.mem, s));
}

void diag_scatter(DType dt, const void* diag, void* out, const std::vector<int64_t>& offs,
                  const std::vector<BsBlockDesc>& blocks, int64_t total, cudaStream_t s) {
  if (total <= 0 || blocks.empty()) return;
  Tables t = upload(offs, blocks, s);
  if (dt == DType::F64)
    diag_scatter_kernel<double><<<grid_of(total), kThreads, 0, s>>>((const double*)diag, (double*)out, t.offs,
                                                                    t.blocks, (int)blocks.size(), total);
  else
    diag_scatter_kernel<double2><<<grid_of(total), kThreads, 0, s>>>((const double2*)diag, (double2*)out, t.offs,
                                                                     t.blocks, (int)blocks.size(), total);
  count_launch();
  NDT_CUDA(cudaGetLastError());
  NDT_CUDA(cudaFreeAsync(t.mem, s));
}

void bs_diag_scale(DType dt, const void* a, const void* sdiag, void* out, const std::vector<int64_t>& offs,
                   const std::vector<BsBlockDesc>& blocks, int64_t total, cudaStream_t s) {
  if (total <= 0 || blocks.empty()) return;
  // blocks[b]: dense_base = source offset, dstride[0] = diagonal offset,
  // shape[0] = column length, shape[1] = columns, shape[2] = diagonal length
  std::vector<DiagCols> h(blocks.size());
  int64_t ncols = 0;
  for (size_t b = 0; b < blocks.size(); b++) {
    const BsBlockDesc& d = blocks[b];
    h[b] = DiagCols{d.dense_base, offs[b], d.dstride[0], d.shape[0], d.shape[1], d.shape[2], ncols};
    ncols += d.shape[1];
  }
  DiagCols* dt_tab = nullptr;
  const size_t bytes = h.size() * sizeof(DiagCols);
  dt_tab = (decltype(dt_tab))pool_alloc(bytes, s);
  NDT_CUDA(cudaMemcpyAsync(dt_tab, h.data(), bytes, cudaMemcpyHostToDevice, s));
  const DeviceCtx& c = ctx();
  const int64_t want = (ncols * 32 + kThreads - 1) / kThreads;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)c.sm_count * 8));
  if (dt == DType::F64)
    diag_scale_kernel<double><<<grid, kThreads, 0, s>>>((const double*)a, (const double*)sdiag, (double*)out, dt_tab,
                                                        (int)h.size(), ncols);
  else
    diag_scale_kernel<double2><<<grid, kThreads, 0, s>>>((const double2*)a, (const double2*)sdiag, (double2*)out,
                                                         dt_tab, (int)h.size(), ncols);
  count_launch();
  NDT_CUDA(cudaGetLastError());
  NDT_CUDA(cudaFreeAsync(dt_tab, s));
}

}  // namespace ndt
