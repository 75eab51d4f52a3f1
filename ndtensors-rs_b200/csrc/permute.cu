// Strided gather / permutedims on sm_100a.
//
// Replaces GenericBackend::permute_into (crates/ndtensors/src/backend/generic.rs:15-39),
// which walks the source one element at a time, with HBM-bound kernels:
//
//   plan     drop extent-1 axes, merge destination axes that are also
//            contiguous in the source (so trivially permuted axes are never
//            moved as separate axes), then classify:
//   copy     one merged axis with source stride 1: vectorised 16-byte copy
//   tiled    the source's stride-1 axis is not the destination's first axis:
//            a tile of P x Q elements is staged through shared memory.  P
//            spans a contiguous run of the source (G_in axes), Q a contiguous
//            run of the destination (G_out axes), so both the global loads and
//            the global stores are coalesced; the shared-memory row pitch is
//            odd (in elements) so that both phases are bank-conflict free.
//            CTAs are persistent and walk the tile list.
//   generic  anything else (broadcast / pinned axes without a stride-1
//            source axis, short rows): one destination element per thread.
#include <algorithm>
#include <cstdio>

#include "ndt_internal.h"

namespace ndt {

namespace {

constexpr int kMaxGroup = 8;   // axes per tile group
constexpr int kMaxOuter = 24;  // outer (tile-index) dims
constexpr int kMaxGen = 24;    // axes of the generic kernel
constexpr int kThreads = 256;

struct alignas(16) C128 {
  double re, im;
};

template <int E>
struct ElemT;
template <>
struct ElemT<8> {
  using type = double;
};
template <>
struct ElemT<16> {
  using type = C128;
};

struct TileParams {
  int P, Q;    // full tile extents (elements)
  int lds;     // shared-memory row pitch (elements), odd
  int n_gin, n_gout;
  int gin_n[kMaxGroup];       // extents (chunk for the last) of G_in axes
  int64_t gin_sdst[kMaxGroup];  // destination strides of G_in axes
  int gout_n[kMaxGroup];
  int64_t gout_ssrc[kMaxGroup];  // source strides of G_out axes
  int n_outer;
  int64_t outer_n[kMaxOuter];
  int64_t outer_ssrc[kMaxOuter];
  int64_t outer_sdst[kMaxOuter];
  int in_chunk_dim;   // outer dim index of the G_in chunk counter, or -1
  int out_chunk_dim;  // outer dim index of the G_out chunk counter, or -1
  int64_t in_total;   // full extent of the chunked G_in axis
  int64_t out_total;
  int in_inner;       // product of the full (unchunked) G_in extents
  int out_inner;
  int in_chunk, out_chunk;
  int64_t ntiles;
};

template <int E>
__global__ void __launch_bounds__(kThreads) permute_tiled_kernel(const typename ElemT<E>::type* __restrict__ src,
                                                                 typename ElemT<E>::type* __restrict__ dst,
                                                                 const __grid_constant__ TileParams tp) {
  using T = typename ElemT<E>::type;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int64_t* qoff_src = reinterpret_cast<int64_t*>(smem_raw);
  int64_t* poff_dst = qoff_src + tp.Q;
  __shared__ int64_t tile_src, tile_dst;
  __shared__ int peff_s, qeff_s;
  T* tile = reinterpret_cast<T*>(smem_raw + (((size_t)(tp.P + tp.Q) * sizeof(int64_t) + 15) & ~size_t(15)));

  // In-tile offset tables (identical for every tile).
  for (int q = threadIdx.x; q < tp.Q; q += blockDim.x) {
    int64_t off = 0;
    int r = q;
    for (int k = 0; k < tp.n_gout; k++) {
      int d = r % tp.gout_n[k];
      r /= tp.gout_n[k];
      off += (int64_t)d * tp.gout_ssrc[k];
    }
    qoff_src[q] = off;
  }
  for (int p = threadIdx.x; p < tp.P; p += blockDim.x) {
    int64_t off = 0;
    int r = p;
    for (int k = 0; k < tp.n_gin; k++) {
      int d = r % tp.gin_n[k];
      r /= tp.gin_n[k];
      off += (int64_t)d * tp.gin_sdst[k];
    }
    poff_dst[p] = off;
  }

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarp = blockDim.x >> 5;

  for (int64_t t = blockIdx.x; t < tp.ntiles; t += gridDim.x) {
    __syncthreads();  // previous tile fully written out; tables ready
    if (threadIdx.x == 0) {
      int64_t r = t, bs = 0, bd = 0;
      int peff = tp.P, qeff = tp.Q;
      for (int k = 0; k < tp.n_outer; k++) {
        int64_t d = r % tp.outer_n[k];
        r /= tp.outer_n[k];
        bs += d * tp.outer_ssrc[k];
        bd += d * tp.outer_sdst[k];
        if (k == tp.in_chunk_dim) {
          int64_t rem = tp.in_total - d * tp.in_chunk;
          if (rem < tp.in_chunk) peff = (int)(tp.in_inner * rem);
        }
        if (k == tp.out_chunk_dim) {
          int64_t rem = tp.out_total - d * tp.out_chunk;
          if (rem < tp.out_chunk) qeff = (int)(tp.out_inner * rem);
        }
      }
      tile_src = bs;
      tile_dst = bd;
      peff_s = peff;
      qeff_s = qeff;
    }
    __syncthreads();
    const int64_t bs = tile_src, bd = tile_dst;
    const int peff = peff_s, qeff = qeff_s;
    const T* s = src + bs;
    T* d = dst + bd;
    // Read phase: a warp covers 32 consecutive source elements (p) of one
    // q-row; loads are batched before the shared-memory stores.
    {
      constexpr int B = 8;
      const int nrow_chunks = (peff + 31) >> 5;
      const int items = nrow_chunks * qeff;  // (chunk, q) pairs
      for (int base = warp; base < items; base += nwarp * B) {
        T v[B];
        int pq[B];
#pragma unroll
        for (int j = 0; j < B; j++) {
          int it = base + j * nwarp;
          pq[j] = -1;
          if (it < items) {
            int q = it / nrow_chunks;
            int p = ((it - q * nrow_chunks) << 5) + lane;
            if (p < peff) {
              v[j] = s[p + qoff_src[q]];
              pq[j] = q * tp.lds + p;
            }
          }
        }
#pragma unroll
        for (int j = 0; j < B; j++)
          if (pq[j] >= 0) tile[pq[j]] = v[j];
      }
    }
    __syncthreads();
    // Write phase: a warp covers 32 consecutive destination elements (q) of
    // one p-column.
    {
      constexpr int B = 8;
      const int ncol_chunks = (qeff + 31) >> 5;
      const int items = ncol_chunks * peff;
      for (int base = warp; base < items; base += nwarp * B) {
        T v[B];
        int64_t o[B];
#pragma unroll
        for (int j = 0; j < B; j++) {
          int it = base + j * nwarp;
          o[j] = -1;
          if (it < items) {
            int p = it / ncol_chunks;
            int q = ((it - p * ncol_chunks) << 5) + lane;
            if (q < qeff) {
              v[j] = tile[q * tp.lds + p];
              o[j] = q + poff_dst[p];
            }
          }
        }
#pragma unroll
        for (int j = 0; j < B; j++)
          if (o[j] >= 0) d[o[j]] = v[j];
      }
    }
  }
}

struct GenParams {
  int nd;
  int64_t n[kMaxGen];
  int64_t ssrc[kMaxGen];
  int64_t total;
};

template <int E>
__global__ void __launch_bounds__(kThreads) permute_generic_kernel(const typename ElemT<E>::type* __restrict__ src,
                                                                   typename ElemT<E>::type* __restrict__ dst,
                                                                   const __grid_constant__ GenParams gp) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < gp.total;
       e += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = e, off = 0;
    for (int k = 0; k < gp.nd; k++) {
      int64_t dd = r % gp.n[k];
      r /= gp.n[k];
      off += dd * gp.ssrc[k];
    }
    dst[e] = src[off];
  }
}

// Contiguous copy, 16-byte vectors (both pointers 16-byte aligned).
__global__ void __launch_bounds__(kThreads) copy16_kernel(const int4* __restrict__ src, int4* __restrict__ dst,
                                                          int64_t n16) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
}
__global__ void copy8_kernel(const double* __restrict__ src, double* __restrict__ dst, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
}

struct Ax {
  int64_t n, ssrc, sdst;
};

int grid_for(int64_t work_items, int per_sm, const DeviceCtx& c) {
  int64_t g = std::min<int64_t>(work_items, (int64_t)c.sm_count * per_sm);
  return (int)std::max<int64_t>(g, 1);
}

template <int E>
void launch_tiled(const void* src, void* dst, const std::vector<Ax>& ax, int a_in, cudaStream_t s,
                  const DeviceCtx& c, bool* ok) {
  const int r = (int)ax.size();
  const int target = (E == 8) ? 64 : 32;  // P and Q targets: 512-byte runs
  TileParams tp{};
  std::vector<char> used(r, 0);
  // G_out: destination axes 0, 1, ... (never the source's stride-1 axis)
  int Q = 1, nq = 0, out_chunk_axis = -1, out_chunk = 1;
  for (int i = 0; i < r && nq < kMaxGroup; i++) {
    if (i == a_in) break;
    if ((int64_t)Q * ax[i].n <= target) {
      tp.gout_n[nq] = (int)ax[i].n;
      tp.gout_ssrc[nq] = ax[i].ssrc;
      Q *= (int)ax[i].n;
      used[i] = 1;
      nq++;
      continue;
    }
    int c = std::max(1, target / Q);
    if (c > 1) {
      tp.gout_n[nq] = c;
      tp.gout_ssrc[nq] = ax[i].ssrc;
      Q *= c;
      used[i] = 2;
      out_chunk_axis = i;
      out_chunk = c;
      nq++;
    }
    break;
  }
  // G_in: the source-contiguous run starting at the stride-1 axis
  int P = 1, np_ = 0, in_chunk_axis = -1, in_chunk = 1;
  int cur = a_in;
  int64_t run = 1;
  while (cur >= 0 && np_ < kMaxGroup) {
    if (used[cur]) break;
    if ((int64_t)P * ax[cur].n <= target) {
      tp.gin_n[np_] = (int)ax[cur].n;
      tp.gin_sdst[np_] = ax[cur].sdst;
      P *= (int)ax[cur].n;
      used[cur] = 1;
      np_++;
      run *= ax[cur].n;
      int nxt = -1;
      for (int j = 0; j < r; j++)
        if (!used[j] && ax[j].ssrc == run) {
          nxt = j;
          break;
        }
      cur = nxt;
      continue;
    }
    int c = std::max(1, target / P);
    if (c > 1) {
      tp.gin_n[np_] = c;
      tp.gin_sdst[np_] = ax[cur].sdst;
      P *= c;
      used[cur] = 2;
      in_chunk_axis = cur;
      in_chunk = c;
      np_++;
    }
    break;
  }
  tp.P = P;
  tp.Q = Q;
  tp.n_gin = np_;
  tp.n_gout = nq;
  tp.lds = (P % 2 == 0) ? P + 1 : P;
  // Outer dims: chunk counters first, then the untouched axes
  int no = 0;
  tp.in_chunk_dim = tp.out_chunk_dim = -1;
  int64_t ntiles = 1;
  auto add_outer = [&](int64_t n, int64_t ss, int64_t sd) {
    tp.outer_n[no] = n;
    tp.outer_ssrc[no] = ss;
    tp.outer_sdst[no] = sd;
    ntiles *= n;
    no++;
  };
  tp.in_inner = P / in_chunk;
  tp.out_inner = Q / out_chunk;
  if (in_chunk_axis >= 0) {
    const Ax& a = ax[in_chunk_axis];
    tp.in_chunk_dim = no;
    tp.in_total = a.n;
    tp.in_chunk = in_chunk;
    add_outer((a.n + in_chunk - 1) / in_chunk, a.ssrc * in_chunk, a.sdst * in_chunk);
  } else {
    tp.in_total = 1;
    tp.in_chunk = 1;
  }
  if (out_chunk_axis >= 0) {
    const Ax& a = ax[out_chunk_axis];
    tp.out_chunk_dim = no;
    tp.out_total = a.n;
    tp.out_chunk = out_chunk;
    add_outer((a.n + out_chunk - 1) / out_chunk, a.ssrc * out_chunk, a.sdst * out_chunk);
  } else {
    tp.out_total = 1;
    tp.out_chunk = 1;
  }
  for (int i = 0; i < r; i++) {
    if (used[i]) continue;
    if (no >= kMaxOuter) {
      *ok = false;
      return;
    }
    add_outer(ax[i].n, ax[i].ssrc, ax[i].sdst);
  }
  tp.n_outer = no;
  tp.ntiles = ntiles;
  if (P < 2 || Q < 2) {
    *ok = false;
    return;
  }
  size_t smem = (((size_t)(P + Q) * sizeof(int64_t) + 15) & ~size_t(15)) + (size_t)Q * tp.lds * E;
  if (smem > c.smem_optin) {
    *ok = false;
    return;
  }
  NDT_CUDA(cudaFuncSetAttribute(permute_tiled_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0;
  NDT_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, permute_tiled_kernel<E>, kThreads, smem));
  per_sm = std::max(1, per_sm);
  int grid = grid_for(ntiles, per_sm, c);
  using T = typename ElemT<E>::type;
  permute_tiled_kernel<E><<<grid, kThreads, smem, s>>>((const T*)src, (T*)dst, tp);
  count_launch();
  NDT_CUDA(cudaGetLastError());
  *ok = true;
}

template <int E>
void launch_generic(const void* src, void* dst, const std::vector<Ax>& ax, int64_t total, cudaStream_t s,
                    const DeviceCtx& c) {
  GenParams gp{};
  if ((int)ax.size() > kMaxGen) throw Error(ErrKind::Panic, "rank too large for the gather kernel");
  gp.nd = (int)ax.size();
  for (int i = 0; i < gp.nd; i++) {
    gp.n[i] = ax[i].n;
    gp.ssrc[i] = ax[i].ssrc;
  }
  gp.total = total;
  int grid = grid_for((total + kThreads - 1) / kThreads, 8, c);
  using T = typename ElemT<E>::type;
  permute_generic_kernel<E><<<grid, kThreads, 0, s>>>((const T*)src, (T*)dst, gp);
  count_launch();
  NDT_CUDA(cudaGetLastError());
}

}  // namespace

void gather(DType dt, const void* src, void* dst, const GatherDesc& g, cudaStream_t s) {
  const int E = (int)esize(dt);
  DeviceCtx& c = ctx();
  // Destination strides are column-major over g.shape.
  std::vector<Ax> ax;
  int64_t total = 1, sd = 1;
  for (size_t i = 0; i < g.shape.size(); i++) {
    int64_t n = (int64_t)g.shape[i];
    if (n == 0) return;  // nothing to move
    if (n > 1) ax.push_back({n, g.src_strides[i], sd});
    sd *= n;
    total *= n;
  }
  // Merge destination-adjacent axes that are also source-contiguous.
  std::vector<Ax> m;
  for (const Ax& a : ax) {
    if (!m.empty() && m.back().ssrc * m.back().n == a.ssrc) {
      m.back().n *= a.n;
      continue;
    }
    m.push_back(a);
  }
  if (m.empty()) m.push_back({1, 0, 1});
  // copy: a single source-contiguous axis
  if (m.size() == 1 && m[0].ssrc == 1) {
    size_t bytes = (size_t)total * E;
    int grid;
    if (((uintptr_t)src % 16 == 0) && ((uintptr_t)dst % 16 == 0) && bytes % 16 == 0) {
      int64_t n16 = (int64_t)(bytes / 16);
      grid = grid_for((n16 + kThreads - 1) / kThreads, 8, c);
      copy16_kernel<<<grid, kThreads, 0, s>>>((const int4*)src, (int4*)dst, n16);
    } else {
      int64_t n8 = (int64_t)(bytes / 8);
      grid = grid_for((n8 + kThreads - 1) / kThreads, 8, c);
      copy8_kernel<<<grid, kThreads, 0, s>>>((const double*)src, (double*)dst, n8);
    }
    count_launch();
    NDT_CUDA(cudaGetLastError());
    return;
  }
  int a_in = -1;
  for (size_t i = 0; i < m.size(); i++)
    if (m[i].ssrc == 1) {
      a_in = (int)i;
      break;
    }
  if (a_in > 0) {
    bool ok = false;
    if (E == 8)
      launch_tiled<8>(src, dst, m, a_in, s, c, &ok);
    else
      launch_tiled<16>(src, dst, m, a_in, s, c, &ok);
    if (ok) return;
  }
  if (E == 8)
    launch_generic<8>(src, dst, m, total, s, c);
  else
    launch_generic<16>(src, dst, m, total, s, c);
}

// permutedims.rs:198-224
static void validate_permutation(const std::vector<size_t>& perm, size_t ndim) {
  if (perm.size() != ndim) throw Error(ErrKind::InvalidPermutation, "permutation length does not match ndim");
  std::vector<char> seen(ndim, 0);
  for (size_t p : perm) {
    if (p >= ndim) throw Error(ErrKind::InvalidPermutation, "permutation index out of range");
    if (seen[p]) throw Error(ErrKind::InvalidPermutation, "duplicate index in permutation");
    seen[p] = 1;
  }
}

// permutedims.rs:51-68 (+ generic.rs:15-39 semantics, including its panic on
// a zero extent: linear_to_cartesian divides by every extent).
Dense permutedims(const Dense& t, const std::vector<size_t>& perm) {
  validate_permutation(perm, t.ndim());
  for (size_t n : t.shape)
    if (n == 0) throw Error(ErrKind::Panic, "permutedims of a tensor with a zero extent");
  std::vector<size_t> new_shape(perm.size());
  for (size_t i = 0; i < perm.size(); i++) new_shape[i] = t.shape[perm[i]];
  Dense out = make_empty_device(t.dt, new_shape);
  const void* src = t.st->dev_read();
  if (t.ndim() == 0) {
    DeviceCtx& c = ctx();
    NDT_CUDA(cudaMemcpyAsync(out.st->dev, src, esize(t.dt), cudaMemcpyDeviceToDevice, c.compute));
    return out;
  }
  std::vector<size_t> ss = col_major_strides(t.shape);
  GatherDesc g;
  g.shape = new_shape;
  g.src_strides.resize(perm.size());
  for (size_t i = 0; i < perm.size(); i++) g.src_strides[i] = (int64_t)ss[perm[i]];
  gather(t.dt, src, out.st->dev, g, ctx().compute);
  return out;
}

}  // namespace ndt
