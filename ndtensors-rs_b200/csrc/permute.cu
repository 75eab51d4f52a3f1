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
//            the global stores are coalesced (512-byte runs).  The tile
//            geometry is fixed at compile time (128 x 64 f64, 32 x 64 c128),
//            so no integer division runs per element.  CTAs are persistent
//            and double-buffered: the next tile is copied global -> shared
//            with cp.async (no register staging) while the current one is
//            written out; the odd shared-memory row pitch keeps both phases
//            bank-conflict free.
//   runs     the source's stride-1 axis is the destination's first axis:
//            contiguous runs copied in 16-byte vectors, offsets decomposed
//            once per 16 KB chunk.
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
constexpr int kWarps = kThreads / 32;

struct alignas(16) C128 {
  double re, im;
};

template <int E>
struct ElemT;
template <>
struct ElemT<8> {
  using type = double;
  // Tile extents along the source-contiguous run (TP: 1 KB source rows) and
  // the destination-contiguous run (TQ).  Two 64 KB buffers give one CTA per
  // SM; on a 16^6 tensor that is 13.8 tiles per CTA (a 1.2% tail), which
  // measured 11% faster than 64 x 64 tiles at three CTAs per SM (9.2 tiles
  // each, up to 8% tail).
  static constexpr int TP = 128;
  static constexpr int TQ = 64;
};
template <>
struct ElemT<16> {
  using type = C128;
  static constexpr int TP = 32;
  static constexpr int TQ = 64;
};

struct TileParams {
  int P, Q;  // full tile extents (elements), P <= TP, Q <= TQ
  int n_gin, n_gout;
  int gin_n[kMaxGroup];          // extents (chunk for the last) of G_in axes
  int64_t gin_sdst[kMaxGroup];   // destination strides of G_in axes
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
  int in_inner;  // product of the full (unchunked) G_in extents
  int out_inner;
  int in_chunk, out_chunk;
  int64_t ntiles;
};

template <int E>
__global__ void __launch_bounds__(kThreads) permute_tiled_kernel(const typename ElemT<E>::type* __restrict__ src,
                                                                 typename ElemT<E>::type* __restrict__ dst,
                                                                 const __grid_constant__ TileParams tp) {
  using T = typename ElemT<E>::type;
  constexpr int TP = ElemT<E>::TP, TQ = ElemT<E>::TQ;
  constexpr int LDS = TP + 1;           // odd pitch: conflict-free column reads
  constexpr int RROWS = TQ / kWarps;    // q rows per warp (read phase)
  constexpr int RCH = TP / 32;          // 32-lane chunks per row
  constexpr int WCOLS = TP / kWarps;    // p columns per warp (write phase)
  constexpr int WCH = TQ / 32;
  static_assert(TP % 32 == 0 && TQ % 32 == 0 && TP % kWarps == 0 && TQ % kWarps == 0, "tile geometry");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* tile = reinterpret_cast<T*>(smem_raw);  // two buffers of TQ * LDS elements
  __shared__ int64_t qoff_src[TQ];
  __shared__ int64_t poff_dst[TP];
  __shared__ int64_t tile_src[3], tile_dst[3];
  __shared__ int peff_s[3], qeff_s[3];

  // Programmatic dependent launch: the next kernel on the stream may be
  // scheduled as soon as this grid's CTAs start retiring (its setup overlaps
  // this grid's tail), and this grid's own setup below overlaps the previous
  // kernel; griddepcontrol.wait then holds every global access until the
  // previous grid has completed and its writes are visible.
  pdl_release();
  // In-tile offset tables, identical for every tile of the launch.
  for (int q = threadIdx.x; q < TQ; q += blockDim.x) {
    int64_t off = 0;
    int r = q;
    for (int k = 0; k < tp.n_gout; k++) {
      int d = r % tp.gout_n[k];
      r /= tp.gout_n[k];
      off += (int64_t)d * tp.gout_ssrc[k];
    }
    qoff_src[q] = off;
  }
  for (int p = threadIdx.x; p < TP; p += blockDim.x) {
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

  // Tile bases for tile t, computed by thread 0 into slot `sl`.
  auto bases = [&](int64_t t, int sl) {
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
    tile_src[sl] = bs;
    tile_dst[sl] = bd;
    peff_s[sl] = peff;
    qeff_s[sl] = qeff;
  };
  // Read phase of tile in slot `sl`: warp w copies rows q = w, w+8, ... of
  // the source run straight into shared memory (cp.async, no registers).
  auto issue_reads = [&](int b, int sl) {
    const T* s = src + tile_src[sl];
    T* buf = tile + b * (TQ * LDS);
    const int peff = peff_s[sl], qeff = qeff_s[sl];
#pragma unroll
    for (int i = 0; i < RROWS; i++) {
      const int q = warp + kWarps * i;
      const int64_t qo = qoff_src[q];
#pragma unroll
      for (int c = 0; c < RCH; c++) {
        const int p = c * 32 + lane;
        if (q < qeff && p < peff) {
          unsigned sa = (unsigned)__cvta_generic_to_shared(buf + q * LDS + p);
          if constexpr (E == 8)
            asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(sa), "l"(s + qo + p));
          else
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(s + qo + p));
        }
      }
    }
  };

  // Persistent loop.  Iteration k handles tile t_k in buffer k%2 with its
  // descriptor in slot k%3: the loads of tile t_{k+1} are in flight while
  // tile t_k is written out.  A slot is rewritten two barriers after its
  // last reader, a buffer one barrier after.
  int64_t t = blockIdx.x;
  if (threadIdx.x == 0 && t < tp.ntiles) bases(t, 0);
  pdl_wait();
  __syncthreads();  // tables and slot 0 ready
  if (t < tp.ntiles) issue_reads(0, 0);
  asm volatile("cp.async.commit_group;\n" ::);
  for (int k = 0; t < tp.ntiles; t += gridDim.x, k++) {
    const int sl = k % 3, sln = (k + 1) % 3, b = k & 1;
    const int64_t tn = t + gridDim.x;
    if (threadIdx.x == 0 && tn < tp.ntiles) bases(tn, sln);
    __syncthreads();  // slot sln ready; buffer b^1 no longer read
    if (tn < tp.ntiles) issue_reads(b ^ 1, sln);
    asm volatile("cp.async.commit_group;\n" ::);
    asm volatile("cp.async.wait_group 1;\n" ::);
    __syncthreads();  // tile t_k complete in buffer b
    // Write phase: warp w stores columns p = w, w+8, ...; 32 lanes cover 32
    // consecutive destination elements.
    const T* buf = tile + b * (TQ * LDS);
    T* d = dst + tile_dst[sl];
    const int peff = peff_s[sl], qeff = qeff_s[sl];
#pragma unroll
    for (int i = 0; i < WCOLS; i++) {
      const int p = warp + kWarps * i;
      const bool pok = p < peff;
      const int64_t po = poff_dst[p];
#pragma unroll
      for (int c = 0; c < WCH; c++) {
        const int q = c * 32 + lane;
        if (pok && q < qeff) d[po + q] = buf[q * LDS + p];
      }
    }
  }
  asm volatile("cp.async.wait_group 0;\n" ::);
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

// Run copy: the destination's first axis is the source's stride-1 axis, so
// the permute moves contiguous runs of `run_len` elements.  A work item is a
// 16 KB chunk of one run; its source / destination offsets are decomposed
// once per item over the outer axes, and each thread keeps four independent
// 16-byte loads in flight (8-byte copies when a run is not 16-byte aligned).
struct RunParams {
  int nd;
  int vec;
  int64_t n[kMaxGen], ssrc[kMaxGen], sdst[kMaxGen];
  int64_t run_bytes, chunks, items;
};
constexpr int kRunUnroll = 4;
constexpr int64_t kRunChunk = (int64_t)kThreads * kRunUnroll * 16;

__global__ void __launch_bounds__(kThreads) permute_runs_kernel(const char* __restrict__ src,
                                                                char* __restrict__ dst, int es,
                                                                const __grid_constant__ RunParams p) {
  pdl_release();
  pdl_wait();
  for (int64_t it = blockIdx.x; it < p.items; it += gridDim.x) {
    int64_t r = it / p.chunks;
    const int64_t b0 = (it - r * p.chunks) * kRunChunk;
    int64_t so = 0, dso = 0;
    for (int d = 0; d < p.nd; d++) {
      const int64_t q = r / p.n[d];
      const int64_t digit = r - q * p.n[d];
      r = q;
      so += digit * p.ssrc[d];
      dso += digit * p.sdst[d];
    }
    const char* s = src + so * es;
    char* o = dst + dso * es;
    const int64_t b1 = min(b0 + kRunChunk, p.run_bytes);
    if (p.vec) {
      int4 v[kRunUnroll];
#pragma unroll
      for (int u = 0; u < kRunUnroll; u++) {
        const int64_t b = b0 + ((int64_t)u * kThreads + threadIdx.x) * 16;
        if (b < b1) v[u] = *reinterpret_cast<const int4*>(s + b);
      }
#pragma unroll
      for (int u = 0; u < kRunUnroll; u++) {
        const int64_t b = b0 + ((int64_t)u * kThreads + threadIdx.x) * 16;
        if (b < b1) *reinterpret_cast<int4*>(o + b) = v[u];
      }
    } else {
      for (int64_t b = b0 + threadIdx.x * 8; b < b1; b += kThreads * 8)
        *reinterpret_cast<double*>(o + b) = *reinterpret_cast<const double*>(s + b);
    }
  }
}

struct Ax {
  int64_t n, ssrc, sdst;
};

void launch_runs(const void* src, void* dst, const std::vector<Ax>& ax, int es, cudaStream_t s,
                 const DeviceCtx& c) {
  RunParams p{};
  if ((int)ax.size() - 1 > kMaxGen) throw Error(ErrKind::Panic, "rank too large for the gather kernel");
  p.nd = (int)ax.size() - 1;
  bool vec = ((uintptr_t)src % 16 == 0) && ((uintptr_t)dst % 16 == 0) && (ax[0].n * es) % 16 == 0;
  int64_t nruns = 1;
  for (int i = 0; i < p.nd; i++) {
    const Ax& a = ax[i + 1];
    p.n[i] = a.n;
    p.ssrc[i] = a.ssrc;
    p.sdst[i] = a.sdst;
    vec = vec && (a.ssrc * es) % 16 == 0 && (a.sdst * es) % 16 == 0;
    nruns *= a.n;
  }
  p.vec = vec ? 1 : 0;
  p.run_bytes = ax[0].n * es;
  p.chunks = (p.run_bytes + kRunChunk - 1) / kRunChunk;
  p.items = nruns * p.chunks;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(p.items, (int64_t)c.sm_count * 64));
  launch_pdl(permute_runs_kernel, dim3(grid), dim3(kThreads), 0, s, (const char*)src, (char*)dst, es, p);
  count_launch();
  NDT_CUDA(cudaGetLastError());
}

int grid_for(int64_t work_items, int per_sm, const DeviceCtx& c) {
  int64_t g = std::min<int64_t>(work_items, (int64_t)c.sm_count * per_sm);
  return (int)std::max<int64_t>(g, 1);
}

template <int E>
void launch_tiled(const void* src, void* dst, const std::vector<Ax>& ax, int a_in, cudaStream_t s,
                  const DeviceCtx& c, bool* ok) {
  const int r = (int)ax.size();
  const int tP = ElemT<E>::TP, tQ = ElemT<E>::TQ;
  TileParams tp{};
  std::vector<char> used(r, 0);
  // G_out: destination axes 0, 1, ... (never the source's stride-1 axis)
  int Q = 1, nq = 0, out_chunk_axis = -1, out_chunk = 1;
  for (int i = 0; i < r && nq < kMaxGroup; i++) {
    if (i == a_in) break;
    if ((int64_t)Q * ax[i].n <= tQ) {
      tp.gout_n[nq] = (int)ax[i].n;
      tp.gout_ssrc[nq] = ax[i].ssrc;
      Q *= (int)ax[i].n;
      used[i] = 1;
      nq++;
      continue;
    }
    int cch = std::max(1, tQ / Q);
    if (cch > 1) {
      tp.gout_n[nq] = cch;
      tp.gout_ssrc[nq] = ax[i].ssrc;
      Q *= cch;
      used[i] = 2;
      out_chunk_axis = i;
      out_chunk = cch;
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
    if ((int64_t)P * ax[cur].n <= tP) {
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
    int cch = std::max(1, tP / P);
    if (cch > 1) {
      tp.gin_n[np_] = cch;
      tp.gin_sdst[np_] = ax[cur].sdst;
      P *= cch;
      used[cur] = 2;
      in_chunk_axis = cur;
      in_chunk = cch;
      np_++;
    }
    break;
  }
  if (P < 2 || Q < 2) {
    *ok = false;
    return;
  }
  tp.P = P;
  tp.Q = Q;
  tp.n_gin = np_;
  tp.n_gout = nq;
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
  tp.in_total = 1;
  tp.in_chunk = 1;
  tp.out_total = 1;
  tp.out_chunk = 1;
  if (in_chunk_axis >= 0) {
    const Ax& a = ax[in_chunk_axis];
    tp.in_chunk_dim = no;
    tp.in_total = a.n;
    tp.in_chunk = in_chunk;
    add_outer((a.n + in_chunk - 1) / in_chunk, a.ssrc * in_chunk, a.sdst * in_chunk);
  }
  if (out_chunk_axis >= 0) {
    const Ax& a = ax[out_chunk_axis];
    tp.out_chunk_dim = no;
    tp.out_total = a.n;
    tp.out_chunk = out_chunk;
    add_outer((a.n + out_chunk - 1) / out_chunk, a.ssrc * out_chunk, a.sdst * out_chunk);
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
  const size_t smem = 2 * (size_t)ElemT<E>::TQ * (ElemT<E>::TP + 1) * E;
  ensure_dynamic_smem((const void*)permute_tiled_kernel<E>, smem);
  int per_sm = 0;
  NDT_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, permute_tiled_kernel<E>, kThreads, smem));
  per_sm = std::max(1, per_sm);
  int grid = grid_for(ntiles, per_sm, c);
  using T = typename ElemT<E>::type;
  launch_pdl(permute_tiled_kernel<E>, dim3(grid), dim3(kThreads), smem, s, (const T*)src, (T*)dst, tp);
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
  // runs: the destination's first axis is also the source's stride-1 axis
  if (a_in == 0 && m[0].n * E >= 64) {
    launch_runs(src, dst, m, E, s, c);
    return;
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
