// FP64 tensor-core GEMM for sm_100a (DMMA: mma.sync.aligned.m16n8k8 .f64).
//
// Replaces the faer matmul calls of the reference's TTGT contraction
// (crates/ndtensors/src/contract/gemm.rs:152-159, :209-216) and the per-pair
// loop of the block-sparse contraction (contract/blocksparse.rs:144-180).
//
// sm_100a has no f64 kind for tcgen05.mma; the FP64 tensor path is the warp
// level DMMA instruction, whose measured peak on B200 is ~37 TFLOP/s (148 SMs
// x 64 FMA/clk x 1.965 GHz).  One kernel template serves
//   * dense GEMM   C[m,n] (+)= A[m,k] B[k,n]
//   * grouped GEMM over a device table of output blocks ("problems"), each
//     the sum over its matched block pairs ("segments") of A_s B_s.  A CTA
//     owns one output tile and accumulates every segment in registers, so
//     accumulation is deterministic and needs no atomics.
// Operands are staged global -> shared with cp.async in a multi-stage ring;
// shared tiles use padded pitches (4 mod 16 doubles for f64; 2 / 4 mod 8
// complex elements) so fragment loads are bank-conflict free.  Complex128
// uses the 4M real decomposition inside the kernel (Cr += Ar Br - Ai Bi,
// Ci += Ar Bi + Ai Br) on interleaved (re, im) data.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>

#include "ndt_internal.h"

namespace ndt {
namespace {

struct KArgs {
  const void* A;
  const void* B;
  void* C;
  // dense mode (tiles == nullptr)
  int64_t m, n, k, lda, ldb, ldc;
  int mtiles, ntiles_n;
  // grouped mode
  const int4* tiles;  // x = problem, y = tile m index, z = tile n index
  const GroupedProblem* probs;
  const GroupedSegment* segs;
  int accumulate;
};

__device__ __forceinline__ void cp_async8(void* smem, const void* gmem, bool pred) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  int sz = pred ? 8 : 0;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(s), "l"(gmem), "r"(sz));
}
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(sz));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void dmma(double& c0, double& c1, double& c2, double& c3, const double (&a)[4],
                                     const double (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+d"(c0), "+d"(c1), "+d"(c2), "+d"(c3)
      : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(b[0]), "d"(b[1]));
}

__device__ __forceinline__ double dneg(double x) {
  return __longlong_as_double(__double_as_longlong(x) ^ (long long)0x8000000000000000ULL);
}

// Shared-memory pitch (in elements) of an operand tile.
template <bool CPLX, bool KMAJOR, int MN, int BK>
struct Pitch {
  static constexpr int value = CPLX ? (KMAJOR ? BK + 4 : MN + 2) : (KMAJOR ? BK + 4 : MN + 4);
  static constexpr int rows = KMAJOR ? MN : BK;
  static constexpr int elems = rows * value;
};

template <bool CPLX, int BM, int BN, int BK, int WM_WARPS, int WN_WARPS, int STAGES, bool AK, bool BKM>
struct Cfg {
  static constexpr int kThreads = WM_WARPS * WN_WARPS * 32;
  static constexpr int WM = BM / WM_WARPS;  // warp tile rows
  static constexpr int WN = BN / WN_WARPS;
  static constexpr int MT = WM / 16;
  static constexpr int NT = WN / 8;
  static constexpr int ES = CPLX ? 16 : 8;
  using PA = Pitch<CPLX, AK, BM, BK>;
  using PB = Pitch<CPLX, BKM, BN, BK>;
  static constexpr int stage_elems = PA::elems + PB::elems;
  static constexpr size_t smem_bytes = (size_t)STAGES * stage_elems * ES;
};

template <bool CPLX, int BM, int BN, int BK, int WM_WARPS, int WN_WARPS, int STAGES, bool AK, bool BKM>
__global__ void __launch_bounds__(WM_WARPS* WN_WARPS * 32, 1) dmma_gemm_kernel(const __grid_constant__ KArgs args) {
  using C = Cfg<CPLX, BM, BN, BK, WM_WARPS, WN_WARPS, STAGES, AK, BKM>;
  constexpr int NTH = C::kThreads, MT = C::MT, NT = C::NT, ES = C::ES;
  constexpr int LDA = C::PA::value, LDB = C::PB::value;
  constexpr int RPL = CPLX ? 2 : 1;  // doubles per element
  extern __shared__ __align__(16) double smem[];

  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int wm0 = (warp % WM_WARPS) * C::WM;
  const int wn0 = (warp / WM_WARPS) * C::WN;

  // ---- which tile / problem
  int64_t m, n, c_off, ldc, seg_begin, seg_count;
  int64_t m0, n0;
  const char* Ab = (const char*)args.A;
  const char* Bb = (const char*)args.B;
  if (args.tiles == nullptr) {
    // dense: rasterise with groups of 8 tile-rows for L2 reuse
    int bid = blockIdx.x;
    const int GROUP = 8;
    int per_group = GROUP * args.ntiles_n;
    int grp = bid / per_group;
    int first_m = grp * GROUP;
    int gsz = min(args.mtiles - first_m, GROUP);
    int tm = first_m + (bid % per_group) % gsz;
    int tn = (bid % per_group) / gsz;
    m = args.m;
    n = args.n;
    c_off = 0;
    ldc = args.ldc;
    seg_begin = 0;
    seg_count = 1;
    m0 = (int64_t)tm * BM;
    n0 = (int64_t)tn * BN;
  } else {
    int4 td = args.tiles[blockIdx.x];
    const GroupedProblem pr = args.probs[td.x];
    m = pr.m;
    n = pr.n;
    c_off = pr.c_off;
    ldc = pr.m;
    seg_begin = pr.seg_begin;
    seg_count = pr.seg_count;
    m0 = (int64_t)td.y * BM;
    n0 = (int64_t)td.z * BN;
  }

  // ---- load iterator over (segment, k0)
  int64_t seg = seg_begin, seg_end = seg_begin + seg_count;
  int64_t a_off = 0, b_off = 0, kseg = 0, lda = 0, ldb = 0, k0 = 0;
  auto load_seg = [&](int64_t s) {
    if (args.tiles == nullptr) {
      a_off = 0;
      b_off = 0;
      kseg = args.k;
      lda = args.lda;
      ldb = args.ldb;
    } else {
      const GroupedSegment sd = args.segs[s];
      a_off = sd.a_off;
      b_off = sd.b_off;
      kseg = sd.k;
      lda = sd.lda;
      ldb = sd.ldb;
    }
  };
  int64_t total_steps = 0;
  if (args.tiles == nullptr) {
    total_steps = (args.k + BK - 1) / BK;
  } else {
    for (int64_t s = seg_begin; s < seg_end; s++) total_steps += (args.segs[s].k + BK - 1) / BK;
  }
  if (seg < seg_end) load_seg(seg);

  auto issue_load = [&](int stage) {
    double* As = smem + (size_t)stage * C::stage_elems * RPL;
    double* Bs = As + (size_t)C::PA::elems * RPL;
    const char* Ag = Ab + a_off * ES;
    const char* Bg = Bb + b_off * ES;
    // A tile: BM x BK
    static_assert((BM * BK) % NTH == 0 && (BN * BK) % NTH == 0, "tile not divisible by threads");
#pragma unroll
    for (int it = 0; it < (BM * BK) / NTH; it++) {
      const int e = tid + it * NTH;
      int r, c;  // r: row in smem, c: contiguous column in smem
      int64_t gi, gl;
      if (AK) {
        r = e / BK;
        c = e % BK;
        gi = m0 + r;
        gl = k0 + c;
      } else {
        r = e / BM;
        c = e % BM;
        gl = k0 + r;
        gi = m0 + c;
      }
      bool ok = gi < m && gl < kseg;
      const char* src = ok ? Ag + (AK ? (gl + gi * lda) : (gi + gl * lda)) * ES : Ag;
      double* dst = As + ((size_t)r * LDA + c) * RPL;
      if (CPLX)
        cp_async16(dst, src, ok);
      else
        cp_async8(dst, src, ok);
    }
    // B tile: BK x BN
#pragma unroll
    for (int it = 0; it < (BN * BK) / NTH; it++) {
      const int e = tid + it * NTH;
      int r, c;
      int64_t gj, gl;
      if (BKM) {
        r = e / BK;
        c = e % BK;
        gj = n0 + r;
        gl = k0 + c;
      } else {
        r = e / BN;
        c = e % BN;
        gl = k0 + r;
        gj = n0 + c;
      }
      bool ok = gj < n && gl < kseg;
      const char* src = ok ? Bg + (BKM ? (gl + gj * ldb) : (gj + gl * ldb)) * ES : Bg;
      double* dst = Bs + ((size_t)r * LDB + c) * RPL;
      if (CPLX)
        cp_async16(dst, src, ok);
      else
        cp_async8(dst, src, ok);
    }
  };
  auto advance = [&]() {
    k0 += BK;
    if (k0 >= kseg) {
      seg++;
      k0 = 0;
      if (seg < seg_end) load_seg(seg);
    }
  };

  double acc[MT][NT][4 * RPL];
#pragma unroll
  for (int i = 0; i < MT; i++)
#pragma unroll
    for (int j = 0; j < NT; j++)
#pragma unroll
      for (int q = 0; q < 4 * RPL; q++) acc[i][j][q] = 0.0;

  // ---- prologue
#pragma unroll
  for (int s = 0; s < STAGES - 1; s++) {
    if (seg < seg_end) {
      issue_load(s);
      advance();
    }
    cp_commit();
  }

  for (int64_t step = 0; step < total_steps; step++) {
    cp_wait<STAGES - 2>();
    __syncthreads();
    {
      int ls = (int)((step + STAGES - 1) % STAGES);
      if (seg < seg_end) {
        issue_load(ls);
        advance();
      }
      cp_commit();
    }
    const int cs = (int)(step % STAGES);
    const double* As = smem + (size_t)cs * C::stage_elems * RPL;
    const double* Bs = As + (size_t)C::PA::elems * RPL;
#pragma unroll
    for (int kk = 0; kk < BK; kk += 8) {
      double a[MT][4], b[NT][2];
      double ai[MT][4], bi[NT][2];
#pragma unroll
      for (int i = 0; i < MT; i++) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
          int row = wm0 + i * 16 + g + 8 * (q & 1);
          int col = kk + t + 4 * (q >> 1);
          int idx = AK ? row * LDA + col : col * LDA + row;
          if constexpr (CPLX) {
            double2 v = *reinterpret_cast<const double2*>(As + (size_t)idx * 2);
            a[i][q] = v.x;
            ai[i][q] = v.y;
          } else {
            a[i][q] = As[idx];
          }
        }
      }
#pragma unroll
      for (int j = 0; j < NT; j++) {
#pragma unroll
        for (int q = 0; q < 2; q++) {
          int col = wn0 + j * 8 + g;
          int kr = kk + t + 4 * q;
          int idx = BKM ? col * LDB + kr : kr * LDB + col;
          if constexpr (CPLX) {
            double2 v = *reinterpret_cast<const double2*>(Bs + (size_t)idx * 2);
            b[j][q] = v.x;
            bi[j][q] = v.y;
          } else {
            b[j][q] = Bs[idx];
          }
        }
      }
      if constexpr (!CPLX) {
#pragma unroll
        for (int i = 0; i < MT; i++)
#pragma unroll
          for (int j = 0; j < NT; j++) dmma(acc[i][j][0], acc[i][j][1], acc[i][j][2], acc[i][j][3], a[i], b[j]);
      } else {
        double nai[MT][4];
#pragma unroll
        for (int i = 0; i < MT; i++)
#pragma unroll
          for (int q = 0; q < 4; q++) nai[i][q] = dneg(ai[i][q]);
#pragma unroll
        for (int i = 0; i < MT; i++)
#pragma unroll
          for (int j = 0; j < NT; j++) {
            double* cc = acc[i][j];
            dmma(cc[0], cc[1], cc[2], cc[3], a[i], b[j]);
            dmma(cc[0], cc[1], cc[2], cc[3], nai[i], bi[j]);
            dmma(cc[RPL * 2], cc[RPL * 2 + 1], cc[RPL * 2 + 2], cc[RPL * 2 + 3], a[i], bi[j]);
            dmma(cc[RPL * 2], cc[RPL * 2 + 1], cc[RPL * 2 + 2], cc[RPL * 2 + 3], ai[i], b[j]);
          }
      }
    }
  }
  cp_wait<0>();

  // ---- epilogue: C[i + j*ldc] (+)= acc
  char* Cb = (char*)args.C + c_off * ES;
#pragma unroll
  for (int i = 0; i < MT; i++)
#pragma unroll
    for (int j = 0; j < NT; j++)
#pragma unroll
      for (int q = 0; q < 4; q++) {
        int64_t row = m0 + wm0 + i * 16 + g + 8 * (q >> 1);
        int64_t col = n0 + wn0 + j * 8 + 2 * t + (q & 1);
        if (row < m && col < n) {
          if constexpr (CPLX) {
            double2* p = reinterpret_cast<double2*>(Cb) + (row + col * ldc);
            double2 v = make_double2(acc[i][j][q], acc[i][j][4 + q]);
            if (args.accumulate) {
              double2 o = *p;
              v.x += o.x;
              v.y += o.y;
            }
            *p = v;
          } else {
            double* p = reinterpret_cast<double*>(Cb) + (row + col * ldc);
            double v = acc[i][j][q];
            if (args.accumulate) v += *p;
            *p = v;
          }
        }
      }
}

template <bool CPLX, int BM, int BN, int BK, int WMW, int WNW, int ST, bool AK, bool BKM>
void launch_cfg(const KArgs& a, int grid, cudaStream_t s) {
  using C = Cfg<CPLX, BM, BN, BK, WMW, WNW, ST, AK, BKM>;
  auto kern = dmma_gemm_kernel<CPLX, BM, BN, BK, WMW, WNW, ST, AK, BKM>;
  static bool attr = false;
  if (!attr) {
    NDT_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::smem_bytes));
    attr = true;
  }
  kern<<<grid, C::kThreads, C::smem_bytes, s>>>(a);
  count_launch();
  NDT_CUDA(cudaGetLastError());
}

// Tile configurations.  "Big": 128x128 (f64) / 64x128 (c128) per CTA, 8
// warps; "small": 64x64 (f64) / 32x64 (c128), 4 warps, for grids that would
// otherwise leave SMs idle.
template <bool CPLX, bool AK, bool BKM>
void launch(const KArgs& a, int grid, bool small, cudaStream_t s) {
  if (!CPLX) {
    if (small)
      launch_cfg<false, 64, 64, 16, 2, 2, 4, AK, BKM>(a, grid, s);
    else
      launch_cfg<false, 128, 128, 16, 2, 4, 4, AK, BKM>(a, grid, s);
  } else {
    if (small)
      launch_cfg<true, 32, 64, 16, 1, 2, 3, AK, BKM>(a, grid, s);
    else
      launch_cfg<true, 64, 128, 16, 2, 4, 3, AK, BKM>(a, grid, s);
  }
}

template <bool CPLX>
void dispatch(const KArgs& a, int grid, bool small, bool ak, bool bk, cudaStream_t s) {
  if (ak && bk)
    launch<CPLX, true, true>(a, grid, small, s);
  else if (ak && !bk)
    launch<CPLX, true, false>(a, grid, small, s);
  else if (!ak && bk)
    launch<CPLX, false, true>(a, grid, small, s);
  else
    launch<CPLX, false, false>(a, grid, small, s);
}

void tile_dims(bool cplx, bool small, int* bm, int* bn) {
  if (!cplx) {
    *bm = small ? 64 : 128;
    *bn = small ? 64 : 128;
  } else {
    *bm = small ? 32 : 64;
    *bn = small ? 64 : 128;
  }
}

}  // namespace

void gemm(DType dt, int64_t m, int64_t n, int64_t k, GemmOperand A, GemmOperand B, void* Cp, int64_t ldc,
          bool accumulate, cudaStream_t s) {
  if (m <= 0 || n <= 0) return;
  const bool cplx = dt == DType::C128;
  const DeviceCtx& c = ctx();
  // Pick the tile size that fills the SMs best (waves of one CTA per SM for
  // the big tile, ~2 per SM for the small one).
  auto waves_eff = [&](bool small) {
    int bm, bn;
    tile_dims(cplx, small, &bm, &bn);
    double tiles = (double)((m + bm - 1) / bm) * (double)((n + bn - 1) / bn);
    double slots = (double)c.sm_count * (small ? 2 : 1);
    double waves = std::ceil(tiles / slots);
    double useful = (double)m * n / ((double)((m + bm - 1) / bm) * bm * ((n + bn - 1) / bn) * bn);
    // small tiles re-read operands twice as often; weight them down a bit
    return tiles / (waves * slots) * useful * (small ? 0.9 : 1.0);
  };
  bool small = waves_eff(true) > waves_eff(false);
  int bm, bn;
  tile_dims(cplx, small, &bm, &bn);
  KArgs a{};
  a.A = A.ptr;
  a.B = B.ptr;
  a.C = Cp;
  a.m = m;
  a.n = n;
  a.k = k;
  a.lda = A.ld;
  a.ldb = B.ld;
  a.ldc = ldc;
  a.mtiles = (int)((m + bm - 1) / bm);
  a.ntiles_n = (int)((n + bn - 1) / bn);
  a.tiles = nullptr;
  a.accumulate = accumulate ? 1 : 0;
  int grid = a.mtiles * a.ntiles_n;
  if (cplx)
    dispatch<true>(a, grid, small, A.kmajor, B.kmajor, s);
  else
    dispatch<false>(a, grid, small, A.kmajor, B.kmajor, s);
}

void grouped_gemm(DType dt, const void* A, const void* B, void* Cp, bool a_kmajor, bool b_kmajor,
                  const std::vector<GroupedProblem>& probs, const std::vector<GroupedSegment>& segs,
                  const void* /*kscale*/, cudaStream_t s) {
  if (probs.empty()) return;
  const bool cplx = dt == DType::C128;
  const DeviceCtx& c = ctx();
  // Tile list: every (problem, tile) with its work (tile area x total k),
  // heaviest first so the tail of the launch is made of small tiles.
  auto build = [&](bool small, std::vector<int4>& tiles, double* eff) {
    int bm, bn;
    tile_dims(cplx, small, &bm, &bn);
    std::vector<std::pair<double, int4>> w;
    double useful = 0, padded = 0;
    for (size_t p = 0; p < probs.size(); p++) {
      const GroupedProblem& pr = probs[p];
      int64_t ktot = 0;
      for (int64_t q = pr.seg_begin; q < pr.seg_begin + pr.seg_count; q++) ktot += segs[q].k;
      int64_t mt = (pr.m + bm - 1) / bm, nt = (pr.n + bn - 1) / bn;
      useful += (double)pr.m * pr.n * ktot;
      padded += (double)mt * bm * nt * bn * ((ktot + 15) / 16 * 16);
      for (int64_t i = 0; i < mt; i++)
        for (int64_t j = 0; j < nt; j++) w.push_back({(double)ktot, make_int4((int)p, (int)i, (int)j, 0)});
    }
    std::stable_sort(w.begin(), w.end(), [](const auto& x, const auto& y) { return x.first > y.first; });
    tiles.resize(w.size());
    for (size_t i = 0; i < w.size(); i++) tiles[i] = w[i].second;
    double slots = (double)c.sm_count * (small ? 2 : 1);
    double waves = std::ceil((double)tiles.size() / slots);
    *eff = useful / padded * std::min(1.0, (double)tiles.size() / (waves * slots)) * (small ? 0.9 : 1.0);
  };
  std::vector<int4> tb, ts;
  double eb, es;
  build(false, tb, &eb);
  build(true, ts, &es);
  bool small = es > eb;
  std::vector<int4>& tiles = small ? ts : tb;
  // Device-side tables: problems, segments, tiles (one allocation).
  size_t bp = probs.size() * sizeof(GroupedProblem), bsg = segs.size() * sizeof(GroupedSegment),
         bt = tiles.size() * sizeof(int4);
  size_t off_s = (bp + 255) / 256 * 256, off_t = off_s + (bsg + 255) / 256 * 256;
  size_t total = off_t + bt;
  std::vector<char> host(total);
  memcpy(host.data(), probs.data(), bp);
  memcpy(host.data() + off_s, segs.data(), bsg);
  memcpy(host.data() + off_t, tiles.data(), bt);
  char* d = nullptr;
  NDT_CUDA(cudaMallocAsync((void**)&d, total, s));
  NDT_CUDA(cudaMemcpyAsync(d, host.data(), total, cudaMemcpyHostToDevice, s));
  KArgs a{};
  a.A = A;
  a.B = B;
  a.C = Cp;
  a.tiles = (const int4*)(d + off_t);
  a.probs = (const GroupedProblem*)d;
  a.segs = (const GroupedSegment*)(d + off_s);
  a.accumulate = 0;
  int grid = (int)tiles.size();
  if (cplx)
    dispatch<true>(a, grid, small, a_kmajor, b_kmajor, s);
  else
    dispatch<false>(a, grid, small, a_kmajor, b_kmajor, s);
  NDT_CUDA(cudaFreeAsync(d, s));
}

}  // namespace ndt
