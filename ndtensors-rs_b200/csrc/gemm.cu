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
// Operands are staged global -> shared with cp.async in a multi-stage ring.
// Each thread's copies follow a fixed pattern: a constant column within a
// shared row and a constant row step per copy, so a copy costs one pointer
// add and two compares.  f64 operands whose bases, offsets and leading
// dimensions are 16-byte aligned move as 16-byte pairs (VEC).  Shared tiles
// use padded pitches (4 mod 16 doubles for f64; 2 / 4 mod 8 complex elements
// for MN- / K-major) so the fragment loads are bank-conflict free.
// Complex128 uses the 3M real decomposition inside the kernel, on interleaved
// (re, im) data: three real tensor-core products per complex multiply-add,
// X += Ar Br, Y += Ai Bi, Z += (Ar + Ai)(Br + Bi), and Cr = X - Y,
// Ci = Z - X - Y in the epilogue (25% fewer DMMAs than the 4M form; the
// sums are formed in registers from the staged fragments).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <queue>
#include <tuple>
#include <type_traits>
#include <unordered_map>
#include <vector>

#include "ndt_internal.h"

namespace ndt {
namespace {

constexpr int kMaxPeerCopies = 7;

struct KArgs {
  const void* A;
  const void* B;
  void* C;
  // dense mode (tiles == nullptr)
  int64_t m, n, k, lda, ldb, ldc;
  int mtiles, ntiles_n;
  // grouped mode
  const int4* tiles;  // x = problem, y = tile m index, z = tile n index, w = k-steps (at least 1)
  const GroupedProblem* probs;
  const GroupedSegment* segs;
  const void* kscale;  // grouped mode: per-k scale (segments' scale_off), or null
  int kscale_real;     // complex scale values whose imaginary parts are all zero
  int accumulate;
  int ntiles;          // grouped mode: entries of `tiles`
  int* counter;        // grouped mode: [tiles reserved, CTAs done], zero at launch
  int sm_reserve;      // grouped mode: SMs to leave free of persistent CTAs
  // grouped mode: further copies of C (other ranks' output buffers mapped
  // into this process) that every tile is also written to
  int npeers;
  char* peer_c[kMaxPeerCopies];
  // grouped mode, strided operands: index runs per problem / segment
  const StridedProblem* sprobs;
  const StridedSegment* ssegs;
};

// offset of index x along its runs
__device__ __forceinline__ int64_t run_off(const IndexRuns& r, uint32_t x) {
  const uint32_t q = x / r.e0;
  return (int64_t)(x - q * r.e0) * r.s0 + (int64_t)q * r.s1;
}

__device__ __forceinline__ void cp_async8(void* smem, const void* gmem, bool pred) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  int sz = pred ? 8 : 0;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(s), "l"(gmem), "r"(sz));
}
// 16-byte copy of which only the first `bytes` (0, 8 or 16) are read; the
// rest of the 16 bytes is zero-filled.
__device__ __forceinline__ void cp_async16n(void* smem, const void* gmem, int bytes) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(bytes));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Bulk (TMA engine) copy of `bytes` (a multiple of 16, both addresses
// 16-byte aligned) from this CTA's shared memory to global memory, which may
// be another GPU's buffer mapped into this process: the engine reads the
// shared memory and sends the data while the issuing warp goes on.
__device__ __forceinline__ void bulk_store(void* gdst, const void* ssrc, unsigned bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(gdst),
               "r"((unsigned)__cvta_generic_to_shared(ssrc)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
// this thread's bulk copies have read their shared-memory source
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory"); }
// this thread's bulk copies are complete (their writes performed)
__device__ __forceinline__ void bulk_wait_done() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }
// this thread's shared-memory writes are visible to later bulk copies
__device__ __forceinline__ void fence_shared_to_bulk() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

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

template <bool CPLX, int BM, int BN, int BK, int WM_WARPS, int WN_WARPS, int STAGES, bool AK, bool BKM,
          int SCALE = 0>
struct Cfg {
  static constexpr int kThreads = WM_WARPS * WN_WARPS * 32;
  static constexpr int WM = BM / WM_WARPS;  // warp tile rows
  static constexpr int WN = BN / WN_WARPS;
  static constexpr int MT = WM / 16;
  static constexpr int NT = WN / 8;
  static constexpr int ES = CPLX ? 16 : 8;
  using PA = Pitch<CPLX, AK, BM, BK>;
  using PB = Pitch<CPLX, BKM, BN, BK>;
  // SCALE: each stage also holds the BK scale values of its k range
  static constexpr int stage_elems = PA::elems + PB::elems + (SCALE ? BK : 0);
  static constexpr size_t smem_bytes = (size_t)STAGES * stage_elems * ES;
  // complex grouped launches with peer copies of C: per column group (the
  // WM_WARPS warps holding the same columns), 8 columns of the CTA tile
  // (pitch BM + 1 elements) staged for the bulk copies to the peers
  static constexpr int push_pitch = BM + 1;
  static constexpr size_t push_bytes = CPLX ? (size_t)WN_WARPS * 8 * push_pitch * ES : 0;
};

// Copy pattern of one operand tile: ROWS x CONT elements in shared memory
// (CONT contiguous), PW elements per copy.
template <int ROWS, int CONT, int PW, int NTH>
struct CopyPlan {
  static constexpr int CW = CONT / PW;         // copies per shared row
  static constexpr int RS = NTH / CW;          // rows advanced per copy
  static constexpr int IT = ROWS * CW / NTH;   // copies per thread per stage
  static_assert(NTH % CW == 0 && (ROWS * CW) % NTH == 0, "tile not divisible by threads");
};

// VEC (f64 only): 16-byte pair copies along the contiguous index; a pair
// crossing the matrix edge copies 8 bytes and zero-fills the rest.
// SCALE (grouped only): B(k, j) is multiplied by kscale[scale_off + k] of its
// segment as its fragments leave shared memory, so a diagonal operand between
// A and B (A . diag(s) . B) costs no pass of its own over A.  1: real scale
// values (f64, or complex ones with zero imaginary parts: one multiply per
// real component), 2: complex scale values (a complex multiply).
template <bool CPLX, int BM, int BN, int BK, int WM_WARPS, int WN_WARPS, int STAGES, bool AK, bool BKM, bool VEC,
          bool GROUPED, int SCALE>
__global__ void __launch_bounds__(WM_WARPS* WN_WARPS * 32, 1) dmma_gemm_kernel(const __grid_constant__ KArgs args) {
  pdl_release();
  pdl_wait();  // before the first global access (tile tables, operands)
  static_assert(SCALE == 0 || GROUPED, "k-scaling is a grouped-mode feature");
  using C = Cfg<CPLX, BM, BN, BK, WM_WARPS, WN_WARPS, STAGES, AK, BKM, SCALE>;
  constexpr int NTH = C::kThreads, MT = C::MT, NT = C::NT, ES = C::ES;
  constexpr int LDA = C::PA::value, LDB = C::PB::value;
  constexpr int RPL = CPLX ? 2 : 1;  // doubles per element
  constexpr int PW = (!CPLX && VEC) ? 2 : 1;
  using PlanA = CopyPlan<AK ? BM : BK, AK ? BK : BM, PW, NTH>;
  using PlanB = CopyPlan<BKM ? BN : BK, BKM ? BK : BN, PW, NTH>;
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
  if constexpr (!GROUPED) {
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

  // ---- per-thread copy geometry (constant over the launch)
  const int a_c = (tid % PlanA::CW) * PW, a_r = tid / PlanA::CW;
  const int b_c = (tid % PlanB::CW) * PW, b_r = tid / PlanB::CW;
  // Rows of the tile that exist in the matrix for the M / N side: fixed per tile.
  const int64_t a_mrem = m - m0, b_nrem = n - n0;

  // ---- load iterator over (segment, k0)
  int64_t seg = seg_begin, seg_end = seg_begin + seg_count;
  int64_t a_off = 0, b_off = 0, kseg = 0, lda = 0, ldb = 0, k0 = 0, s_off = 0;
  auto load_seg = [&](int64_t s) {
    if constexpr (!GROUPED) {
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
      s_off = sd.scale_off;
    }
  };
  int total_steps = 0;
  if constexpr (!GROUPED) {
    total_steps = (int)((args.k + BK - 1) / BK);
  } else {
    for (int64_t s = seg_begin; s < seg_end; s++) total_steps += (int)((args.segs[s].k + BK - 1) / BK);
  }
  if (seg < seg_end) load_seg(seg);

  auto issue_load = [&](int stage) {
    double* As = smem + (size_t)stage * C::stage_elems * RPL;
    double* Bs = As + (size_t)C::PA::elems * RPL;
    const int64_t krem = kseg - k0;  // k rows left in this segment
    // ---- A: rows are M (AK) or K (MN-major); the contiguous index is the other
    {
      const int64_t cont_rem = AK ? krem - a_c : a_mrem - a_c;  // valid contiguous elements from a_c
      const int nv = cont_rem >= PW ? PW : (cont_rem > 0 ? (int)cont_rem : 0);
      const int64_t row_rem = (AK ? a_mrem : krem) - a_r;
      const char* src = Ab + (a_off + (AK ? (k0 + a_c) + (m0 + a_r) * lda : (m0 + a_c) + (k0 + a_r) * lda)) * ES;
      const int64_t rstep = (int64_t)PlanA::RS * lda * ES;
      double* dst = As + ((size_t)a_r * LDA + a_c) * RPL;
#pragma unroll
      for (int it = 0; it < PlanA::IT; it++) {
        const bool rok = it * PlanA::RS < row_rem;
        const int nb = rok ? nv : 0;
        const char* p = nb ? src + it * rstep : Ab;
        double* d = dst + (size_t)it * PlanA::RS * LDA * RPL;
        if constexpr (PW == 2)
          cp_async16n(d, p, nb * 8);
        else if constexpr (CPLX)
          cp_async16n(d, p, nb * 16);
        else
          cp_async8(d, p, nb != 0);
      }
    }
    // ---- B: rows are N (BKM) or K (MN-major)
    {
      const int64_t cont_rem = BKM ? krem - b_c : b_nrem - b_c;
      const int nv = cont_rem >= PW ? PW : (cont_rem > 0 ? (int)cont_rem : 0);
      const int64_t row_rem = (BKM ? b_nrem : krem) - b_r;
      const char* src = Bb + (b_off + (BKM ? (k0 + b_c) + (n0 + b_r) * ldb : (n0 + b_c) + (k0 + b_r) * ldb)) * ES;
      const int64_t rstep = (int64_t)PlanB::RS * ldb * ES;
      double* dst = Bs + ((size_t)b_r * LDB + b_c) * RPL;
#pragma unroll
      for (int it = 0; it < PlanB::IT; it++) {
        const bool rok = it * PlanB::RS < row_rem;
        const int nb = rok ? nv : 0;
        const char* p = nb ? src + it * rstep : Bb;
        double* d = dst + (size_t)it * PlanB::RS * LDB * RPL;
        if constexpr (PW == 2)
          cp_async16n(d, p, nb * 8);
        else if constexpr (CPLX)
          cp_async16n(d, p, nb * 16);
        else
          cp_async8(d, p, nb != 0);
      }
    }
    // ---- the stage's BK scale values (zero past the segment's end)
    if constexpr (SCALE != 0) {
      double* Ss = As + (size_t)(C::PA::elems + C::PB::elems) * RPL;
      if (tid < BK) {
        const bool ok = tid < krem;
        const char* src = (const char*)args.kscale + (s_off + (ok ? k0 + tid : 0)) * ES;
        if constexpr (CPLX)
          cp_async16n(Ss + tid * 2, src, ok ? 16 : 0);
        else
          cp_async8(Ss + tid, src, ok);
      }
    }
  };
  // Loads still to issue: dense runs k0 to kseg; grouped walks the segments.
  auto more = [&]() -> bool {
    if constexpr (!GROUPED)
      return k0 < kseg;
    else
      return seg < seg_end;
  };
  auto advance = [&]() {
    k0 += BK;
    if constexpr (GROUPED) {
      if (k0 >= kseg) {
        seg++;
        k0 = 0;
        if (seg < seg_end) load_seg(seg);
      }
    }
  };

  // f64: one accumulator plane; complex (3M): planes X, Y, Z
  constexpr int PLANES = CPLX ? 3 : 1;
  double acc[MT][NT][4 * PLANES];
#pragma unroll
  for (int i = 0; i < MT; i++)
#pragma unroll
    for (int j = 0; j < NT; j++)
#pragma unroll
      for (int q = 0; q < 4 * PLANES; q++) acc[i][j][q] = 0.0;

  // ---- prologue
#pragma unroll
  for (int s = 0; s < STAGES - 1; s++) {
    if (more()) {
      issue_load(s);
      advance();
    }
    cp_commit();
  }

  int cs = 0, ls = STAGES - 1;  // stage computed / stage loaded
  for (int step = 0; step < total_steps; step++) {
    cp_wait<STAGES - 2>();
    __syncthreads();
    if (more()) {
      issue_load(ls);
      advance();
    }
    cp_commit();
    ls = (ls + 1 == STAGES) ? 0 : ls + 1;
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
      if constexpr (SCALE != 0) {
        // s(k) B(k, j): fragment row t + 4 q of this k8 step.  B rather than A:
        // each B fragment belongs to one warp, while the warps of a CTA row
        // all load the same A fragments, so A would be scaled once per warp.
        const double* Ss = As + (size_t)(C::PA::elems + C::PB::elems) * RPL;
#pragma unroll
        for (int q = 0; q < 2; q++) {
          const int kr = kk + t + 4 * q;
          if constexpr (CPLX && SCALE == 2) {
            const double2 sv = *reinterpret_cast<const double2*>(Ss + (size_t)kr * 2);
#pragma unroll
            for (int j = 0; j < NT; j++) {
              const double re = b[j][q], im = bi[j][q];
              b[j][q] = re * sv.x - im * sv.y;
              bi[j][q] = re * sv.y + im * sv.x;
            }
          } else if constexpr (CPLX) {
            const double sv = Ss[(size_t)kr * 2];
#pragma unroll
            for (int j = 0; j < NT; j++) {
              b[j][q] *= sv;
              bi[j][q] *= sv;
            }
          } else {
            const double sv = Ss[kr];
#pragma unroll
            for (int j = 0; j < NT; j++) b[j][q] *= sv;
          }
        }
      }
      if constexpr (!CPLX) {
#pragma unroll
        for (int i = 0; i < MT; i++)
#pragma unroll
          for (int j = 0; j < NT; j++) dmma(acc[i][j][0], acc[i][j][1], acc[i][j][2], acc[i][j][3], a[i], b[j]);
      } else {
        double as[MT][4], bs[NT][2];
#pragma unroll
        for (int i = 0; i < MT; i++)
#pragma unroll
          for (int q = 0; q < 4; q++) as[i][q] = a[i][q] + ai[i][q];
#pragma unroll
        for (int j = 0; j < NT; j++)
#pragma unroll
          for (int q = 0; q < 2; q++) bs[j][q] = b[j][q] + bi[j][q];
#pragma unroll
        for (int i = 0; i < MT; i++)
#pragma unroll
          for (int j = 0; j < NT; j++) {
            double* cc = acc[i][j];
            dmma(cc[0], cc[1], cc[2], cc[3], a[i], b[j]);      // X += Ar Br
            dmma(cc[4], cc[5], cc[6], cc[7], ai[i], bi[j]);    // Y += Ai Bi
            dmma(cc[8], cc[9], cc[10], cc[11], as[i], bs[j]);  // Z += (Ar + Ai)(Br + Bi)
          }
      }
    }
    cs = (cs + 1 == STAGES) ? 0 : cs + 1;
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
            const double x = acc[i][j][q], y = acc[i][j][4 + q], z = acc[i][j][8 + q];
            double2 v = make_double2(x - y, z - x - y);
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


// Persistent grouped kernel (block-sparse contractions, split-K pieces).
// gridDim.x CTAs, at most as many as fit on the GPU at once, walk the tile
// list (heaviest first).  CTA b starts on tile b; later tiles come from a
// counter in the tile table, so each CTA takes the heaviest tile left when it
// reserves one: greedy list scheduling, as the block scheduler does for a
// grid of one CTA per tile, which matters when tile costs span orders of
// magnitude (U(1) blocks).  Thread 0 reserves tiles into a small shared ring
// up to three ahead of the tile being computed, which covers the tiles whose
// stages are in flight.  The cp.async ring runs across tile boundaries:
// while a tile's last k-steps and its epilogue execute, the next tile's
// first stages are already in flight, so the pipeline fills once per CTA
// rather than once per tile.  Tiles of short, ragged blocks (most of a
// block-sparse contraction) are where that fill would otherwise be paid again
// and again.
// On edge tiles, warp fragments that lie wholly outside the output block
// (rows >= m or columns >= n) and k8 steps past the end of a segment issue no
// MMA: those products are zero.  On ragged blocks that saves the padded part
// of the edge tiles (the c128 MPS chain: 86% useful work at 32 x 64 tile
// granularity, 96% at the 16 x 8 x 8 MMA granularity).  Interior k-steps of
// interior tiles take an unpredicated path.
// A tile whose block has no contracted extent (all its segments empty) runs
// one k-step of zeros and writes a zero tile.
// STR (with AK, BKM and no k-scale): A, B and C are addressed through each
// segment's and problem's index runs, so blocks whose axes are not in GEMM
// order are read and written in place.  A thread's copy rows keep one offset
// each per segment (set when the segment starts); its contraction column
// adds one offset per stage.  With VEC (f64) a copy is a pair of adjacent k
// values: every segment's contraction runs have stride 1 and an even first
// extent, and every offset of a pair's first value is even.
template <bool CPLX, int BM, int BN, int BK, int WM_WARPS, int WN_WARPS, int STAGES, bool AK, bool BKM, bool VEC,
          int SCALE, bool STR = false>
__global__ void __launch_bounds__(WM_WARPS* WN_WARPS * 32, 1)
    dmma_grouped_kernel(const __grid_constant__ KArgs args) {
  static_assert(!STR || (AK && BKM && SCALE == 0), "strided operands: k-major staging, no k-scale");
  pdl_release();
  pdl_wait();  // before the first global access (tile tables, operands)
  using C = Cfg<CPLX, BM, BN, BK, WM_WARPS, WN_WARPS, STAGES, AK, BKM, SCALE>;
  constexpr int NTH = C::kThreads, MT = C::MT, NT = C::NT, ES = C::ES;
  constexpr int LDA = C::PA::value, LDB = C::PB::value;
  constexpr int RPL = CPLX ? 2 : 1;  // doubles per element
  constexpr int PW = (!CPLX && VEC) ? 2 : 1;
  using PlanA = CopyPlan<AK ? BM : BK, AK ? BK : BM, PW, NTH>;
  using PlanB = CopyPlan<BKM ? BN : BK, BKM ? BK : BN, PW, NTH>;
  extern __shared__ __align__(16) double smem[];
  __shared__ int s_kvalid[STAGES];  // k rows of each staged k-step that lie inside its segment
  constexpr int RING = 8;           // reserved tiles: this CTA's j-th tile is s_ring[j % RING]
  __shared__ int s_ring[RING];

  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int wm0 = (warp % WM_WARPS) * C::WM;
  const int wn0 = (warp / WM_WARPS) * C::WN;
  const int G = gridDim.x, cta = blockIdx.x, ntiles = args.ntiles;
  // Tile reservation.  `produced` (the same on every thread) counts the ring
  // entries written; thread 0 writes them.  Every entry is written before a
  // barrier that precedes its first read, and is overwritten only RING
  // entries later, after its tile's compute has started.
  int produced = 3;
  if (tid == 0) {
    s_ring[0] = cta;
    s_ring[1] = G + atomicAdd(args.counter, 1);
    s_ring[2] = G + atomicAdd(args.counter, 1);
  }
  __syncthreads();
  auto tile_of = [&](int j) -> int { return s_ring[j % RING]; };

  const char* Ab = (const char*)args.A;
  const char* Bb = (const char*)args.B;
  // per-thread copy geometry (constant over the launch)
  const int a_c = (tid % PlanA::CW) * PW, a_r = tid / PlanA::CW;
  const int b_c = (tid % PlanB::CW) * PW, b_r = tid / PlanB::CW;

  // ---- load side: the tile whose stages are being issued, and (segment, k0) within it
  int l_i = 0;
  int64_t l_m0 = 0, l_n0 = 0, a_mrem = 0, b_nrem = 0;
  int64_t seg = 0, seg_end = 0, a_off = 0, b_off = 0, kseg = 0, lda = 0, ldb = 0, k0 = 0, s_off = 0;
  int32_t a_row[STR ? PlanA::IT : 1], b_row[STR ? PlanB::IT : 1];  // STR: copy-row offsets in the blocks
  IndexRuns r_ak{}, r_bk{};
  auto load_seg = [&](int64_t sidx) {
    const GroupedSegment sd = args.segs[sidx];
    a_off = sd.a_off;
    b_off = sd.b_off;
    kseg = sd.k;
    lda = sd.lda;
    ldb = sd.ldb;
    s_off = sd.scale_off;
    if constexpr (STR) {
      const StridedSegment ss = args.ssegs[sidx];
      r_ak = ss.ak;
      r_bk = ss.bk;
#pragma unroll
      for (int it = 0; it < PlanA::IT; it++)
        a_row[it] = (int32_t)run_off(ss.am, (uint32_t)(l_m0 + a_r + it * PlanA::RS));
#pragma unroll
      for (int it = 0; it < PlanB::IT; it++)
        b_row[it] = (int32_t)run_off(ss.bn, (uint32_t)(l_n0 + b_r + it * PlanB::RS));
    }
  };
  // Set the load side up on this CTA's l_i-th tile; false when it has no
  // tiles left.  A tile without a non-empty segment gets one null k-step
  // (kseg = 0: the stage is zero-filled and computes nothing).
  auto load_tile = [&]() -> bool {
    const int ti = tile_of(l_i);
    if (ti >= ntiles) return false;
    const int4 td = args.tiles[ti];
    const GroupedProblem pr = args.probs[td.x];
    seg = pr.seg_begin;
    seg_end = pr.seg_begin + pr.seg_count;
    while (seg < seg_end && args.segs[seg].k <= 0) seg++;
    l_m0 = (int64_t)td.y * BM;
    l_n0 = (int64_t)td.z * BN;
    a_mrem = pr.m - l_m0;
    b_nrem = pr.n - l_n0;
    k0 = 0;
    if (seg < seg_end) {
      load_seg(seg);
    } else {
      seg = seg_end - 1;  // the null step: advance() then moves to the next tile
      kseg = 0;
    }
    return true;
  };
  bool loading = load_tile();
  auto advance = [&]() {
    k0 += BK;
    if (k0 >= kseg) {
      k0 = 0;
      seg++;
      while (seg < seg_end && args.segs[seg].k <= 0) seg++;
      if (seg < seg_end) {
        load_seg(seg);
      } else {
        l_i++;
        loading = load_tile();
      }
    }
  };
  auto issue_load = [&](int stage) {
    double* As = smem + (size_t)stage * C::stage_elems * RPL;
    double* Bs = As + (size_t)C::PA::elems * RPL;
    const int64_t krem = kseg - k0;  // k rows left in this segment
    if (tid == 0) s_kvalid[stage] = krem < BK ? (int)krem : BK;
    if constexpr (STR) {
      // A rows m (a_row), column(s) k0 + a_c (+1); B rows n (b_row), k0 + b_c (+1)
      const int64_t ar = krem - a_c, br = krem - b_c;
      const int an = ar >= PW ? PW : (ar > 0 ? (int)ar : 0), bn = br >= PW ? PW : (br > 0 ? (int)br : 0);
      const int64_t ka = an ? a_off + run_off(r_ak, (uint32_t)(k0 + a_c)) : 0;
      const int64_t kb = bn ? b_off + run_off(r_bk, (uint32_t)(k0 + b_c)) : 0;
      double* da = As + ((size_t)a_r * LDA + a_c) * RPL;
      double* db = Bs + ((size_t)b_r * LDB + b_c) * RPL;
#pragma unroll
      for (int it = 0; it < PlanA::IT; it++) {
        const int nb = it * PlanA::RS < a_mrem - a_r ? an : 0;
        const char* p = nb ? Ab + (ka + a_row[it]) * ES : Ab;
        double* d = da + (size_t)it * PlanA::RS * LDA * RPL;
        if constexpr (CPLX)
          cp_async16n(d, p, nb * 16);
        else if constexpr (PW == 2)
          cp_async16n(d, p, nb * 8);
        else
          cp_async8(d, p, nb != 0);
      }
#pragma unroll
      for (int it = 0; it < PlanB::IT; it++) {
        const int nb = it * PlanB::RS < b_nrem - b_r ? bn : 0;
        const char* p = nb ? Bb + (kb + b_row[it]) * ES : Bb;
        double* d = db + (size_t)it * PlanB::RS * LDB * RPL;
        if constexpr (CPLX)
          cp_async16n(d, p, nb * 16);
        else if constexpr (PW == 2)
          cp_async16n(d, p, nb * 8);
        else
          cp_async8(d, p, nb != 0);
      }
      return;
    }
    {
      const int64_t cont_rem = AK ? krem - a_c : a_mrem - a_c;
      const int nv = cont_rem >= PW ? PW : (cont_rem > 0 ? (int)cont_rem : 0);
      const int64_t row_rem = (AK ? a_mrem : krem) - a_r;
      const char* src =
          Ab + (a_off + (AK ? (k0 + a_c) + (l_m0 + a_r) * lda : (l_m0 + a_c) + (k0 + a_r) * lda)) * ES;
      const int64_t rstep = (int64_t)PlanA::RS * lda * ES;
      double* dst = As + ((size_t)a_r * LDA + a_c) * RPL;
#pragma unroll
      for (int it = 0; it < PlanA::IT; it++) {
        const bool rok = it * PlanA::RS < row_rem;
        const int nb = rok ? nv : 0;
        const char* p = nb ? src + it * rstep : Ab;
        double* d = dst + (size_t)it * PlanA::RS * LDA * RPL;
        if constexpr (PW == 2)
          cp_async16n(d, p, nb * 8);
        else if constexpr (CPLX)
          cp_async16n(d, p, nb * 16);
        else
          cp_async8(d, p, nb != 0);
      }
    }
    {
      const int64_t cont_rem = BKM ? krem - b_c : b_nrem - b_c;
      const int nv = cont_rem >= PW ? PW : (cont_rem > 0 ? (int)cont_rem : 0);
      const int64_t row_rem = (BKM ? b_nrem : krem) - b_r;
      const char* src =
          Bb + (b_off + (BKM ? (k0 + b_c) + (l_n0 + b_r) * ldb : (l_n0 + b_c) + (k0 + b_r) * ldb)) * ES;
      const int64_t rstep = (int64_t)PlanB::RS * ldb * ES;
      double* dst = Bs + ((size_t)b_r * LDB + b_c) * RPL;
#pragma unroll
      for (int it = 0; it < PlanB::IT; it++) {
        const bool rok = it * PlanB::RS < row_rem;
        const int nb = rok ? nv : 0;
        const char* p = nb ? src + it * rstep : Bb;
        double* d = dst + (size_t)it * PlanB::RS * LDB * RPL;
        if constexpr (PW == 2)
          cp_async16n(d, p, nb * 8);
        else if constexpr (CPLX)
          cp_async16n(d, p, nb * 16);
        else
          cp_async8(d, p, nb != 0);
      }
    }
    if constexpr (SCALE != 0) {
      double* Ss = As + (size_t)(C::PA::elems + C::PB::elems) * RPL;
      if (tid < BK) {
        const bool ok = tid < krem;
        const char* src = (const char*)args.kscale + (s_off + (ok ? k0 + tid : 0)) * ES;
        if constexpr (CPLX)
          cp_async16n(Ss + tid * 2, src, ok ? 16 : 0);
        else
          cp_async8(Ss + tid, src, ok);
      }
    }
  };

  // ---- compute side: the tile whose k-steps are being computed
  constexpr int PLANES = CPLX ? 3 : 1;
  double acc[MT][NT][4 * PLANES];
#pragma unroll
  for (int i = 0; i < MT; i++)
#pragma unroll
    for (int j = 0; j < NT; j++)
#pragma unroll
      for (int q = 0; q < 4 * PLANES; q++) acc[i][j][q] = 0.0;
  int c_i = 0, csteps = 0, c_prob = 0;
  int64_t cm = 0, cn = 0, c_off = 0, cm0 = 0, cn0 = 0;
  int mrows = 0, ncols = 0;  // rows / columns of this warp's tile that lie in the block
  // C tile (+)= acc for the compute tile (and = acc into every peer copy of
  // C); clears acc.
  auto epilogue = [&]() {
    char* Cb = (char*)args.C + c_off * ES;
    const int np = args.npeers;
    // STR: offsets of this thread's rows and columns in the C block
    int64_t ro[STR ? MT : 1][2], co[STR ? NT : 1][2];
    if constexpr (STR) {
      const StridedProblem sp = args.sprobs[c_prob];
#pragma unroll
      for (int i = 0; i < MT; i++)
#pragma unroll
        for (int h = 0; h < 2; h++) ro[i][h] = run_off(sp.cm, (uint32_t)(cm0 + wm0 + i * 16 + g + 8 * h));
#pragma unroll
      for (int j = 0; j < NT; j++)
#pragma unroll
        for (int b = 0; b < 2; b++) co[j][b] = run_off(sp.cn, (uint32_t)(cn0 + wn0 + j * 8 + 2 * t + b));
    }
    if constexpr (CPLX && !STR) {
      if (np > 0) {
        // The WM_WARPS warps holding the same columns of the CTA tile store
        // them into C and stage 8 of them at a time, all BM rows; bulk copies
        // then send each staged column (the tile's rows of it, contiguous in
        // C: up to BM * 16 bytes per copy) to every peer copy.  The warps go
        // on to the next tile while the copies drain; they wait only before
        // they overwrite the staging, until the copies have read it.  Every
        // warp of a group passes the same group barriers (the epilogue runs
        // on all warps of the CTA together).
        const int grp = warp / WM_WARPS;
        double2* stg = reinterpret_cast<double2*>(smem + C::smem_bytes / sizeof(double)) +
                       (size_t)grp * 8 * C::push_pitch;
        const int nrows = cm - cm0 < BM ? (int)(cm - cm0) : BM;  // rows of the CTA tile in the block
        auto group_sync = [&]() {
          __syncwarp();
          if constexpr (WM_WARPS > 1) {
            static_assert(WN_WARPS <= 4, "one named barrier (1..4) per column group");
            constexpr int n = WM_WARPS * 32;
            if (grp == 0)
              asm volatile("bar.sync 1, %0;\n" ::"n"(n) : "memory");
            else if (grp == 1)
              asm volatile("bar.sync 2, %0;\n" ::"n"(n) : "memory");
            else if (grp == 2)
              asm volatile("bar.sync 3, %0;\n" ::"n"(n) : "memory");
            else
              asm volatile("bar.sync 4, %0;\n" ::"n"(n) : "memory");
          }
        };
#pragma unroll
        for (int j = 0; j < NT; j++) {
          bulk_wait_read();
          group_sync();
#pragma unroll
          for (int i = 0; i < MT; i++)
#pragma unroll
            for (int q = 0; q < 4; q++) {
              const int rl = wm0 + i * 16 + g + 8 * (q >> 1), cl = 2 * t + (q & 1);
              const int64_t row = cm0 + rl, col = cn0 + wn0 + j * 8 + cl;
              const double x = acc[i][j][q], y = acc[i][j][4 + q], z = acc[i][j][8 + q];
              double2 v = make_double2(x - y, z - x - y);
              if (row < cm && col < cn) {
                double2* p = reinterpret_cast<double2*>(Cb) + (row + col * cm);
                if (args.accumulate) {
                  const double2 o = *p;
                  v.x += o.x;
                  v.y += o.y;
                }
                *p = v;
              }
              stg[cl * C::push_pitch + rl] = v;
#pragma unroll
              for (int pl = 0; pl < PLANES; pl++) acc[i][j][4 * pl + q] = 0.0;
            }
          fence_shared_to_bulk();
          group_sync();
          for (int e = (warp % WM_WARPS) * 32 + lane; e < 8 * np; e += 32 * WM_WARPS) {
            const int cl = e & 7;
            const int64_t col = cn0 + wn0 + j * 8 + cl;
            if (col < cn)
              bulk_store(args.peer_c[e >> 3] + (c_off + cm0 + col * cm) * ES, stg + cl * C::push_pitch,
                         (unsigned)nrows * ES);
          }
          bulk_commit();
        }
        return;
      }
    }
#pragma unroll
    for (int i = 0; i < MT; i++)
#pragma unroll
      for (int j = 0; j < NT; j++)
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const int64_t row = cm0 + wm0 + i * 16 + g + 8 * (q >> 1);
          const int64_t col = cn0 + wn0 + j * 8 + 2 * t + (q & 1);
          if (row < cm && col < cn) {
            int64_t e;
            if constexpr (STR)
              e = ro[i][q >> 1] + co[j][q & 1];
            else
              e = row + col * cm;
            if constexpr (CPLX) {
              double2* p = reinterpret_cast<double2*>(Cb) + e;
              const double x = acc[i][j][q], y = acc[i][j][4 + q], z = acc[i][j][8 + q];
              double2 v = make_double2(x - y, z - x - y);
              if (args.accumulate) {
                const double2 o = *p;
                v.x += o.x;
                v.y += o.y;
              }
              *p = v;
              for (int r = 0; r < np; r++) reinterpret_cast<double2*>(args.peer_c[r] + c_off * ES)[e] = v;
            } else {
              double* p = reinterpret_cast<double*>(Cb) + e;
              double v = acc[i][j][q];
              if (args.accumulate) v += *p;
              *p = v;
              for (int r = 0; r < np; r++) reinterpret_cast<double*>(args.peer_c[r] + c_off * ES)[e] = v;
            }
          }
#pragma unroll
          for (int pl = 0; pl < PLANES; pl++) acc[i][j][4 * pl + q] = 0.0;
        }
  };
  // Set the compute side up on this CTA's c_i-th tile; false when its
  // tiles are done.  A tile without k-steps computes the one null step.
  auto compute_tile = [&]() -> bool {
    const int ti = tile_of(c_i);
    if (ti >= ntiles) return false;
    const int4 td = args.tiles[ti];
    const GroupedProblem pr = args.probs[td.x];
    c_prob = td.x;
    cm = pr.m;
    cn = pr.n;
    c_off = pr.c_off;
    cm0 = (int64_t)td.y * BM;
    cn0 = (int64_t)td.z * BN;
    const int64_t mr = cm - cm0 - wm0, nc = cn - cn0 - wn0;
    mrows = mr < 0 ? 0 : (mr > C::WM ? C::WM : (int)mr);
    ncols = nc < 0 ? 0 : (nc > C::WN ? C::WN : (int)nc);
    csteps = td.w;  // the tile's k-steps (at least 1), counted when the table was built
    return true;
  };

  // ---- prologue
#pragma unroll
  for (int s = 0; s < STAGES - 1; s++) {
    if (loading) {
      issue_load(s);
      advance();
    }
    cp_commit();
  }

  bool active = compute_tile();
  int cs = 0, ls = STAGES - 1;  // stage computed / stage loaded
  while (active) {
    // Keep tiles c_i .. c_i + 3 reserved: this iteration computes a step of
    // tile c_i, and after issuing its load the load iterator points at the
    // step STAGES = 3 steps ahead, which (every tile has a step) lies at most
    // three tiles further on.
    if (produced < c_i + 4) {
      if (tid == 0) s_ring[produced % RING] = G + atomicAdd(args.counter, 1);
      produced++;
    }
    cp_wait<STAGES - 2>();
    __syncthreads();
    if (loading) {
      issue_load(ls);
      advance();
    }
    cp_commit();
    ls = (ls + 1 == STAGES) ? 0 : ls + 1;
    const double* As = smem + (size_t)cs * C::stage_elems * RPL;
    const double* Bs = As + (size_t)C::PA::elems * RPL;
    const int kval = s_kvalid[cs];
    // One k-step.  FULL (f64): every MMA of the stage, predicate free, so
    // the fragment loads of consecutive k8 steps overlap the MMAs; the
    // zero-filled rows, columns and k rows of edge tiles add zeros.  The
    // complex kernels skip the MMAs of fragments outside the block and of k8
    // steps past the segment (three MMAs per fragment pair make the skipped
    // work worth its predicates).  Measured on B200 (persistent kernel):
    // one branch per k-step between both paths cost the f64 kernel 11%
    // (DMRG step 4, 1.57 -> 1.74 ms); predicates on every f64 MMA cost 21%;
    // on the c128 MPS chain the predicated path is 3% faster than the
    // unpredicated one.
    auto kstep = [&](auto full_tag) {
      constexpr bool FULL = decltype(full_tag)::value;
#pragma unroll
    for (int kk = 0; kk < BK; kk += 8) {
      if (!FULL && kk >= kval) continue;  // past the segment's end
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
      if constexpr (SCALE != 0) {
        // s(k) B(k, j) as the B fragments leave shared memory (see dmma_gemm_kernel)
        const double* Ss = As + (size_t)(C::PA::elems + C::PB::elems) * RPL;
#pragma unroll
        for (int q = 0; q < 2; q++) {
          const int kr = kk + t + 4 * q;
          if constexpr (CPLX && SCALE == 2) {
            const double2 sv = *reinterpret_cast<const double2*>(Ss + (size_t)kr * 2);
#pragma unroll
            for (int j = 0; j < NT; j++) {
              const double re = b[j][q], im = bi[j][q];
              b[j][q] = re * sv.x - im * sv.y;
              bi[j][q] = re * sv.y + im * sv.x;
            }
          } else if constexpr (CPLX) {
            const double sv = Ss[(size_t)kr * 2];
#pragma unroll
            for (int j = 0; j < NT; j++) {
              b[j][q] *= sv;
              bi[j][q] *= sv;
            }
          } else {
            const double sv = Ss[kr];
#pragma unroll
            for (int j = 0; j < NT; j++) b[j][q] *= sv;
          }
        }
      }
      if constexpr (!CPLX) {
#pragma unroll
        for (int i = 0; i < MT; i++)
#pragma unroll
          for (int j = 0; j < NT; j++)
            if (FULL || (i * 16 < mrows && j * 8 < ncols))
              dmma(acc[i][j][0], acc[i][j][1], acc[i][j][2], acc[i][j][3], a[i], b[j]);
      } else {
        double as[MT][4], bs[NT][2];
#pragma unroll
        for (int i = 0; i < MT; i++)
#pragma unroll
          for (int q = 0; q < 4; q++) as[i][q] = a[i][q] + ai[i][q];
#pragma unroll
        for (int j = 0; j < NT; j++)
#pragma unroll
          for (int q = 0; q < 2; q++) bs[j][q] = b[j][q] + bi[j][q];
#pragma unroll
        for (int i = 0; i < MT; i++)
#pragma unroll
          for (int j = 0; j < NT; j++)
            if (FULL || (i * 16 < mrows && j * 8 < ncols)) {
              double* cc = acc[i][j];
              dmma(cc[0], cc[1], cc[2], cc[3], a[i], b[j]);      // X += Ar Br
              dmma(cc[4], cc[5], cc[6], cc[7], ai[i], bi[j]);    // Y += Ai Bi
              dmma(cc[8], cc[9], cc[10], cc[11], as[i], bs[j]);  // Z += (Ar + Ai)(Br + Bi)
            }
      }
    }
    };
    if constexpr (CPLX)
      kstep(std::false_type{});
    else
      kstep(std::true_type{});
    cs = (cs + 1 == STAGES) ? 0 : cs + 1;
    if (--csteps == 0) {
      epilogue();
      c_i++;
      active = compute_tile();
    }
  }
  cp_wait<0>();
  // Stores into other GPUs' copies of C (the bulk copies complete) are
  // visible system-wide before the kernel completes.
  if (args.npeers) {
    if constexpr (CPLX && !STR) bulk_wait_done();
    __threadfence_system();
  }
  // The last CTA to finish leaves the reservation counters at zero for the
  // next launch over the same table: every other CTA made its last
  // reservation before it counted itself done.
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(args.counter + 1, 1) == G - 1) {
      args.counter[0] = 0;
      args.counter[1] = 0;
      __threadfence();
    }
  }
}

template <bool CPLX, int BM, int BN, int BK, int WMW, int WNW, int ST, bool AK, bool BKM, bool VEC, bool GROUPED,
          int SCALE>
void launch_mode(const KArgs& a, int grid, cudaStream_t s) {
  using C = Cfg<CPLX, BM, BN, BK, WMW, WNW, ST, AK, BKM, SCALE>;
  auto kern = dmma_gemm_kernel<CPLX, BM, BN, BK, WMW, WNW, ST, AK, BKM, VEC, GROUPED, SCALE>;
  ensure_dynamic_smem((const void*)kern, C::smem_bytes);
  launch_pdl(kern, dim3(grid), dim3(C::kThreads), C::smem_bytes, s, a);
  count_launch();
  NDT_CUDA(cudaGetLastError());
}

// CTAs of `kern` resident per SM with `threads` threads and `smem` bytes of
// dynamic shared memory (looked up once per device and kernel).
int resident_per_sm(const void* kern, int threads, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, const void*, size_t>, int> cache;
  const int dev = current_device();
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find({dev, kern, smem});
  if (it != cache.end()) return it->second;
  int nb = 0;
  NDT_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, threads, smem));
  if (nb < 1) nb = 1;
  cache[{dev, kern, smem}] = nb;
  return nb;
}

// Grouped launch: the persistent kernel on min(tiles, resident CTAs) CTAs.
template <bool CPLX, int BM, int BN, int BK, int WMW, int WNW, int ST, bool AK, bool BKM, bool VEC, int SCALE,
          bool STR = false>
void launch_grouped(const KArgs& a, cudaStream_t s) {
  using C = Cfg<CPLX, BM, BN, BK, WMW, WNW, ST, AK, BKM, SCALE>;
  auto kern = dmma_grouped_kernel<CPLX, BM, BN, BK, WMW, WNW, ST, AK, BKM, VEC, SCALE, STR>;
  // complex launches with peer copies of C also stage their epilogue
  const size_t smem = C::smem_bytes + (a.npeers && !STR ? C::push_bytes : 0);
  ensure_dynamic_smem((const void*)kern, smem);
  const int per_sm = resident_per_sm((const void*)kern, C::kThreads, smem);
  const int sms = std::max(1, ctx().sm_count - std::max(0, a.sm_reserve));
  const int grid = (int)std::min<int64_t>(a.ntiles, (int64_t)per_sm * sms);
  launch_pdl(kern, dim3(grid), dim3(C::kThreads), smem, s, a);
  count_launch();
  NDT_CUDA(cudaGetLastError());
}

template <bool CPLX, int BM, int BN, int BK, int WMW, int WNW, int ST, bool AK, bool BKM, bool VEC>
void launch_cfg(const KArgs& a, int grid, cudaStream_t s) {
  if (a.tiles == nullptr)
    launch_mode<CPLX, BM, BN, BK, WMW, WNW, ST, AK, BKM, VEC, false, 0>(a, grid, s);
  else if (a.kscale == nullptr)
    launch_grouped<CPLX, BM, BN, BK, WMW, WNW, ST, AK, BKM, VEC, 0>(a, s);
  else if (!CPLX || a.kscale_real)
    launch_grouped<CPLX, BM, BN, BK, WMW, WNW, ST, AK, BKM, VEC, 1>(a, s);
  else
    launch_grouped<CPLX, BM, BN, BK, WMW, WNW, ST, AK, BKM, VEC, CPLX ? 2 : 1>(a, s);
}

// Tile classes, indexed by `cls`, with their steady-state rate relative to
// the best class (measured on B200 with each class forced: dense 4096^3 and
// 4096 x 4096 x 1024, the DMRG and MPS contractions, both block-sparse
// workloads):
//   f64   0: 64x64x32, 4 warps, two CTAs per SM        1.00
//         1: 128x128x32, 8 warps, one CTA per SM       0.97
//   c128 (3M, 32 x 16 warp tiles: three accumulator planes; 42 TFLOP/s of
//         complex work, 8mnk, on 2048^3, against 33.5 for the 4M kernel and
//         36.3 for cuBLAS zgemm)
//         0: 32x64x16, 4 warps, two CTAs per SM        1.00
//         1: 64x32x16, 4 warps, two CTAs per SM        0.99
//         2: 32x32x16, 2 warps, four CTAs per SM       0.90 (0.985 on dense
//            GEMMs; the lower weight charges its per-tile fill and epilogue,
//            which short-k block-sparse tiles do not amortise)
//         (a 64x64 class of 8 warps fits one CTA per SM by registers and ran
//         10% slower: its barriers stall the whole SM)
// Smaller tiles waste less on the ragged edges of small blocks and fill the
// SMs with fewer tiles; the heuristic weighs that against the rate.
struct TileClass {
  int bm, bn, per_sm;
  double rate;
};
const TileClass kF64Classes[] = {{64, 64, 2, 1.0}, {128, 128, 1, 0.97}};
const TileClass kC128Classes[] = {{32, 64, 2, 1.0}, {64, 32, 2, 0.99}, {32, 32, 4, 0.90}};
int nclasses(bool cplx) { return cplx ? 3 : 2; }
const TileClass& tile_class(bool cplx, int cls) { return cplx ? kC128Classes[cls] : kF64Classes[cls]; }

template <bool CPLX, bool AK, bool BKM, bool VEC>
void launch(const KArgs& a, int grid, int cls, cudaStream_t s) {
  if constexpr (!CPLX) {
    if (cls == 1)
      launch_cfg<false, 128, 128, 32, 2, 4, 3, AK, BKM, VEC>(a, grid, s);
    else
      launch_cfg<false, 64, 64, 32, 2, 2, 3, AK, BKM, VEC>(a, grid, s);
  } else {
    if (cls == 2)
      launch_cfg<true, 32, 32, 16, 1, 2, 3, AK, BKM, false>(a, grid, s);
    else if (cls == 1)
      launch_cfg<true, 64, 32, 16, 2, 2, 3, AK, BKM, false>(a, grid, s);
    else
      launch_cfg<true, 32, 64, 16, 1, 4, 3, AK, BKM, false>(a, grid, s);
  }
}

template <bool CPLX>
void dispatch(const KArgs& a, int grid, int cls, bool ak, bool bk, bool vec, cudaStream_t s) {
  if (!CPLX && vec) {
    if (ak && bk)
      launch<CPLX, true, true, true>(a, grid, cls, s);
    else if (ak && !bk)
      launch<CPLX, true, false, true>(a, grid, cls, s);
    else if (!ak && bk)
      launch<CPLX, false, true, true>(a, grid, cls, s);
    else
      launch<CPLX, false, false, true>(a, grid, cls, s);
    return;
  }
  if (ak && bk)
    launch<CPLX, true, true, false>(a, grid, cls, s);
  else if (ak && !bk)
    launch<CPLX, true, false, false>(a, grid, cls, s);
  else if (!ak && bk)
    launch<CPLX, false, true, false>(a, grid, cls, s);
  else
    launch<CPLX, false, false, false>(a, grid, cls, s);
}

// 16-byte pair copies need 16-byte aligned operand bases and even element
// offsets / leading dimensions.
bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

void gemm(DType dt, int64_t m, int64_t n, int64_t k, GemmOperand A, GemmOperand B, void* Cp, int64_t ldc,
          bool accumulate, cudaStream_t s, bool allow_split_k) {
  if (m <= 0 || n <= 0) return;
  const bool cplx = dt == DType::C128;
  const DeviceCtx& c = ctx();
  // Pick the tile class with the best estimated rate: useful / padded work,
  // times the filled fraction of the last wave, times the class's rate.
  auto waves_eff = [&](int cl) {
    const TileClass& tc = tile_class(cplx, cl);
    const int bm = tc.bm, bn = tc.bn;
    double tiles = (double)((m + bm - 1) / bm) * (double)((n + bn - 1) / bn);
    double slots = (double)c.sm_count * tc.per_sm;
    double waves = std::ceil(tiles / slots);
    double useful = (double)m * n / ((double)((m + bm - 1) / bm) * bm * ((n + bn - 1) / bn) * bn);
    return tiles / (waves * slots) * useful * tc.rate;
  };
  int cls = 0;
  for (int cl = 1; cl < nclasses(cplx); cl++)
    if (waves_eff(cl) > waves_eff(cls)) cls = cl;
  const int bm = tile_class(cplx, cls).bm, bn = tile_class(cplx, cls).bn;
  // Split-K: when the grid leaves much of its last wave idle and k is long,
  // the k-range is cut into S pieces (multiples of 32, at least 16 k-steps of
  // 32 each) computed as S problems of one grouped launch into a workspace,
  // then summed in split order into C (deterministic).  The sum costs about
  // 3% of the GEMM at these sizes.
  {
    const TileClass& tc = tile_class(cplx, cls);
    const double tiles = (double)((m + bm - 1) / bm) * (double)((n + bn - 1) / bn);
    const double slots = (double)c.sm_count * tc.per_sm;
    auto fill = [&](int S) { return tiles * S / (std::ceil(tiles * S / slots) * slots) * (S > 1 ? 0.97 : 1.0); };
    int S = 1;
    for (int cand = 2; cand <= 4 && allow_split_k; cand++)
      if (k / cand >= 16 * 32 && fill(cand) > fill(S) + 0.02) S = cand;
    if (S > 1) {
      std::vector<GroupedProblem> probs(S);
      std::vector<GroupedSegment> segs(S);
      // Pieces of ceil(k / S) rounded up to 32, the last one ending at k: the
      // pieces cover k exactly (k / S >= 512 keeps every piece non-empty).
      const int64_t kc = ((k + S - 1) / S + 31) / 32 * 32;
      for (int sp = 0; sp < S; sp++) {
        const int64_t k0 = sp * kc, k1 = (sp == S - 1) ? k : std::min<int64_t>(k, k0 + kc);
        probs[sp] = GroupedProblem{m, n, (int64_t)sp * m * n, sp, 1};
        segs[sp] = GroupedSegment{A.kmajor ? k0 : k0 * A.ld, B.kmajor ? k0 : k0 * B.ld, k1 - k0, A.ld, B.ld, -1};
      }
      void* w = nullptr;
      w = pool_alloc((size_t)S * m * n * esize(dt), s);
      grouped_gemm(dt, A.ptr, B.ptr, w, A.kmajor, B.kmajor, probs, segs, nullptr, s);
      splitk_reduce(dt, w, S, m, n, Cp, ldc, accumulate, s);
      NDT_CUDA(cudaFreeAsync(w, s));
      return;
    }
  }
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
  const bool vec = aligned16(A.ptr) && aligned16(B.ptr) && A.ld % 2 == 0 && B.ld % 2 == 0;
  if (cplx)
    dispatch<true>(a, grid, cls, A.kmajor, B.kmajor, false, s);
  else
    dispatch<false>(a, grid, cls, A.kmajor, B.kmajor, vec, s);
}

namespace {

struct PlanKey {
  int device = -1;
  int flags = 0;
  std::vector<int64_t> words;  // the problems and segments, verbatim
  bool operator==(const PlanKey& o) const { return device == o.device && flags == o.flags && words == o.words; }
};
struct PlanKeyHash {
  size_t operator()(const PlanKey& k) const {
    uint64_t h = 1469598103934665603ULL ^ (uint64_t)(k.device * 31 + k.flags);
    for (int64_t w : k.words) h = (h ^ (uint64_t)w) * 1099511628211ULL;
    return (size_t)h;
  }
};
struct GroupedPlan {
  char* d = nullptr;  // device table
  size_t off_s = 0, off_t = 0, off_c = 0, off_sp = 0, off_ss = 0;
  int cls = 0, ntiles = 0;
  cudaEvent_t last_use = nullptr;  // the last launch that read the table
  uint64_t tick = 0;
};
constexpr size_t kPlanCacheSize = 64;
std::mutex g_plan_mu;
std::unordered_map<PlanKey, GroupedPlan, PlanKeyHash> g_plans;
uint64_t g_plan_tick = 0;

const GroupedPlan* plan_lookup(const PlanKey& k) {
  std::lock_guard<std::mutex> lk(g_plan_mu);
  auto it = g_plans.find(k);
  if (it == g_plans.end()) return nullptr;
  it->second.tick = ++g_plan_tick;
  return &it->second;
}

// Insert a plan, evicting the least recently used one of a full cache (its
// table is freed once the last launch that read it has completed).
const GroupedPlan* plan_insert(PlanKey&& k, const GroupedPlan& p) {
  std::lock_guard<std::mutex> lk(g_plan_mu);
  if (g_plans.size() >= kPlanCacheSize) {
    auto victim = g_plans.begin();
    for (auto it = g_plans.begin(); it != g_plans.end(); ++it)
      if (it->second.tick < victim->second.tick) victim = it;
    GroupedPlan& v = victim->second;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(victim->first.device);
    cudaEventSynchronize(v.last_use);
    cudaEventDestroy(v.last_use);
    cudaFree(v.d);
    cudaSetDevice(prev);
    g_plans.erase(victim);
  }
  auto r = g_plans.emplace(std::move(k), p);
  r.first->second.tick = ++g_plan_tick;
  return &r.first->second;
}

}  // namespace

void grouped_gemm(DType dt, const void* A, const void* B, void* Cp, bool a_kmajor, bool b_kmajor,
                  const std::vector<GroupedProblem>& probs, const std::vector<GroupedSegment>& segs,
                  const void* kscale, cudaStream_t s, bool kscale_real, int sm_reserve,
                  const std::vector<void*>* peer_copies, const std::vector<StridedProblem>* sprobs,
                  const std::vector<StridedSegment>* ssegs) {
  if (probs.empty()) return;
  const bool cplx = dt == DType::C128;
  const bool strided = sprobs != nullptr;
  if (strided && (!ssegs || sprobs->size() != probs.size() || ssegs->size() != segs.size() || kscale))
    throw Error(ErrKind::InvalidArgument, "strided grouped GEMM: one run set per problem and segment, no k-scale");
  const DeviceCtx& c = ctx();
  // Tile list: every (problem, tile) with its k length, heaviest first so
  // the tail of the launch is made of short tiles.  Each class is scored by
  // its estimated time: the makespan of placing the tiles in that order on
  // the SM slots, each on the slot that frees first (the way the block
  // scheduler hands them out), times the class's cost per k-step.  Grids of
  // more than 64 waves use the mean load (their tail is negligible).
  auto build = [&](int cl, std::vector<int4>& tiles, double* time) {
    const TileClass& tc = tile_class(cplx, cl);
    const int bm = tc.bm, bn = tc.bn;
    const int bk = cplx ? 16 : 32;
    std::vector<std::pair<int64_t, int4>> w;
    for (size_t p = 0; p < probs.size(); p++) {
      const GroupedProblem& pr = probs[p];
      int64_t ktot = 0;
      for (int64_t q = pr.seg_begin; q < pr.seg_begin + pr.seg_count; q++) ktot += (segs[q].k + bk - 1) / bk;
      int64_t mt = (pr.m + bm - 1) / bm, nt = (pr.n + bn - 1) / bn;
      for (int64_t i = 0; i < mt; i++)
        for (int64_t j = 0; j < nt; j++)
          w.push_back({ktot, make_int4((int)p, (int)i, (int)j, (int)std::max<int64_t>(ktot, 1))});
    }
    std::stable_sort(w.begin(), w.end(), [](const auto& x, const auto& y) { return x.first > y.first; });
    tiles.resize(w.size());
    for (size_t i = 0; i < w.size(); i++) tiles[i] = w[i].second;
    const int64_t slots = (int64_t)c.sm_count * tc.per_sm;
    double span = 0;
    if ((int64_t)w.size() <= 64 * slots) {
      std::priority_queue<int64_t, std::vector<int64_t>, std::greater<int64_t>> free_at;
      for (int64_t i = 0; i < slots; i++) free_at.push(0);
      for (const auto& x : w) {
        int64_t t0 = free_at.top();
        free_at.pop();
        free_at.push(t0 + x.first);
        span = std::max(span, (double)(t0 + x.first));
      }
    } else {
      for (const auto& x : w) span += (double)x.first;
      span /= (double)slots;
    }
    // one k-step of a bm x bn tile on a slot that shares its SM with
    // per_sm - 1 others, at the class's relative rate
    *time = span * ((double)bm * bn * bk * tc.per_sm / tc.rate);
  };
  // The plan of a table (tile class, tile order, device copy of the table)
  // depends only on the problems and segments: it is kept per device and
  // reused by later calls with the same table (repeated contractions of one
  // block structure), which then cost one launch and no host planning.
  PlanKey key;
  key.device = c.device;
  // complex launches that push their tiles to peer copies take class 1:
  // its 64-row tiles send 1 KB per column and peer instead of 512 bytes
  const bool push64 = cplx && !strided && peer_copies && !peer_copies->empty();
  key.flags = (cplx ? 1 : 0) | (strided ? 2 : 0) | (push64 ? 4 : 0);
  const size_t bp = probs.size() * sizeof(GroupedProblem), bsg = segs.size() * sizeof(GroupedSegment);
  const size_t bsp = strided ? sprobs->size() * sizeof(StridedProblem) : 0;
  const size_t bss = strided ? ssegs->size() * sizeof(StridedSegment) : 0;
  key.words.resize((bp + bsg + bsp + bss) / 8 + 1);
  key.words[0] = (int64_t)probs.size();
  {
    char* w = (char*)(key.words.data() + 1);
    memcpy(w, probs.data(), bp);
    memcpy(w + bp, segs.data(), bsg);
    if (strided) {
      memcpy(w + bp + bsg, sprobs->data(), bsp);
      memcpy(w + bp + bsg + bsp, ssegs->data(), bss);
    }
  }
  const GroupedPlan* plan = plan_lookup(key);
  if (!plan) {
    std::vector<int4> tiles, cand;
    int cls = 0;
    double best = -1;
    const int cl0 = push64 ? 1 : 0, cl1 = strided ? 1 : (push64 ? 2 : nclasses(cplx));  // strided: class 0 only
    for (int cl = cl0; cl < cl1; cl++) {
      double t;
      build(cl, cand, &t);
      if (best < 0 || t < best) {
        best = t;
        cls = cl;
        tiles.swap(cand);
      }
    }
    // Device-side tables: problems, segments, tiles, and the tile reservation
    // counters (zero; each launch leaves them zero for the next), one allocation.
    const size_t bt = tiles.size() * sizeof(int4);
    GroupedPlan np;
    np.off_s = (bp + 255) / 256 * 256;
    np.off_t = np.off_s + (bsg + 255) / 256 * 256;
    np.off_c = np.off_t + (bt + 255) / 256 * 256;
    np.off_sp = np.off_c + 256;
    np.off_ss = np.off_sp + (bsp + 255) / 256 * 256;
    const size_t total = np.off_ss + bss;
    std::vector<char> host(total, 0);
    memcpy(host.data(), probs.data(), bp);
    memcpy(host.data() + np.off_s, segs.data(), bsg);
    memcpy(host.data() + np.off_t, tiles.data(), bt);
    if (strided) {
      memcpy(host.data() + np.off_sp, sprobs->data(), bsp);
      memcpy(host.data() + np.off_ss, ssegs->data(), bss);
    }
    np.d = (char*)pool_alloc(total, s);
    NDT_CUDA(cudaMemcpyAsync(np.d, host.data(), total, cudaMemcpyHostToDevice, s));
    // the copy reads pageable memory: it has been taken when the call returns
    np.cls = cls;
    np.ntiles = (int)tiles.size();
    NDT_CUDA(cudaEventCreateWithFlags(&np.last_use, cudaEventDisableTiming));
    plan = plan_insert(std::move(key), np);
  }
  char* d = plan->d;
  const int cls = plan->cls;
  KArgs a{};
  a.A = A;
  a.B = B;
  a.C = Cp;
  a.tiles = (const int4*)(d + plan->off_t);
  a.counter = (int*)(d + plan->off_c);
  a.sm_reserve = sm_reserve;
  a.npeers = 0;
  if (peer_copies) {
    if (peer_copies->size() > (size_t)kMaxPeerCopies) throw Error(ErrKind::InvalidArgument, "too many copies of C");
    for (void* p : *peer_copies) a.peer_c[a.npeers++] = (char*)p;
  }
  a.probs = (const GroupedProblem*)d;
  a.segs = (const GroupedSegment*)(d + plan->off_s);
  a.sprobs = strided ? (const StridedProblem*)(d + plan->off_sp) : nullptr;
  a.ssegs = strided ? (const StridedSegment*)(d + plan->off_ss) : nullptr;
  a.kscale = kscale;
  a.kscale_real = kscale_real ? 1 : 0;
  a.accumulate = 0;
  a.ntiles = plan->ntiles;
  int grid = plan->ntiles;
  bool vec = aligned16(A) && aligned16(B);
  for (const GroupedSegment& sg : segs)
    vec = vec && sg.a_off % 2 == 0 && sg.b_off % 2 == 0 && sg.lda % 2 == 0 && sg.ldb % 2 == 0;
  if (strided) {
    // class 0 with k-major staging; f64 pair copies when every pair is
    // adjacent (contraction runs of stride 1, even first extent) and 16-byte
    // aligned (even offsets)
    auto even = [](int64_t x) { return x % 2 == 0; };
    auto pairs = [&](const IndexRuns& rows, const IndexRuns& k, int64_t off) {
      return k.s0 == 1 && (k.e0 == 0x7fffffffu || k.e0 % 2 == 0) && even(k.s1) && even(rows.s0) && even(rows.s1) &&
             even(off);
    };
    bool pv = aligned16(A) && aligned16(B);
    for (size_t q = 0; pv && q < segs.size(); q++)
      pv = pairs((*ssegs)[q].am, (*ssegs)[q].ak, segs[q].a_off) && pairs((*ssegs)[q].bn, (*ssegs)[q].bk, segs[q].b_off);
    if (cplx)
      launch_grouped<true, 32, 64, 16, 1, 4, 3, true, true, false, 0, true>(a, s);
    else if (pv)
      launch_grouped<false, 64, 64, 32, 2, 2, 3, true, true, true, 0, true>(a, s);
    else
      launch_grouped<false, 64, 64, 32, 2, 2, 3, true, true, false, 0, true>(a, s);
  } else if (cplx) {
    dispatch<true>(a, grid, cls, a_kmajor, b_kmajor, false, s);
  } else {
    dispatch<false>(a, grid, cls, a_kmajor, b_kmajor, vec, s);
  }
  NDT_CUDA(cudaEventRecord(plan->last_use, s));
}

}  // namespace ndt
