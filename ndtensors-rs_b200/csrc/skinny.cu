// Skinny contraction: C(i, j) = sum_l X(i, l) Y(l, j) where the row index i
// is long and l (the contracted index) and j are short (<= 32 values each,
// <= 16 for complex).
//
// This is the shape of the two bandwidth-bound steps of a DMRG environment
// update (two-site wavefunction times an MPO tensor: 2^21 rows, k = n = 10)
// and of any contraction where one side is tiny.  The tiled GEMM would pad n
// and k to its tile (64 x 32) and need the permuted operand packed first;
// here X is read through its strides directly (the permutation is folded
// into the addressing), so the contraction is one pass over X and one over C:
//
//   * X arrives in tiles of 256 rows x k values through a 3-stage cp.async
//     ring in shared memory (two tiles in flight per CTA while the third is
//     computed, no registers held by copies in flight), laid out [l][row]
//     with a padded pitch so that the fragment reads below are free of bank
//     conflicts.  The long index i is decomposed into at most kMaxDims
//     merged (extent, stride) axes; the k offsets of l are kernel parameters.
//     In the DMRG steps the fastest axis of i is the fastest of X, so a
//     warp's copies of one l are 256 contiguous bytes;
//   * the arithmetic runs on the FP64 tensor cores (mma.sync m16n8k8 f64):
//     k is padded to KS * 8 (the padding rows of every stage are zeroed once;
//     a last step holding at most 4 values is one m16n8k4 MMA, so k = 10
//     costs 1.5 steps of tensor work, not 2) and n to NT * 8; Y's fragments
//     stay in registers for the whole kernel.
//     Each warp owns 32 rows of a tile (two m16 fragments), so 32 rows cost
//     2 * KS * NT tensor instructions and 8 * KS fragment loads; complex
//     values take four real products (re*re - im*im, re*im + im*re);
//   * C(i, j) lands at i's output offset + j * cj: the M-fastest dense layout
//     the contraction driver expects, with i = M (small n, cj = m) or i = N
//     (small m, cj = 1).
//
// Roofline: HBM.  Algorithmic bytes = (rows * k + rows * n + k * n) * sizeof(T).
#include <algorithm>

#include "ndt_internal.h"

namespace ndt {

namespace {

constexpr int kThreads = 256;  // 8 warps
constexpr int kTileRows = 256;
// Shared-memory row pitch (elements).  A fragment read is served per
// half-warp (f64, 8-byte lanes) or quarter-warp (complex, 16-byte lanes); its
// four t-rows must fall in four different 32-byte bank groups: pitch = 4 mod
// 16 (f64) and 2 mod 8 (complex) give row offsets 0, 32, 64, 96 mod 128 bytes.
template <bool CPLX>
constexpr int pitch() {
  return CPLX ? kTileRows + 2 : kTileRows + 4;
}
constexpr int kMaxDims = 6;
constexpr int kStages = 3;

struct SkArgs {
  const void* X;
  const void* Y;
  void* C;
  int64_t rows, ntiles;
  int nd, k, n;
  int fast;  // tiles never straddle the fastest row axis: row offset = tile base + row * stride
  int pair;   // f64, rows 2p and 2p+1 adjacent in X at a 16-byte boundary: 16-byte copies
  int cpair;  // f64, rows 2p and 2p+1 adjacent in C at a 16-byte boundary: 16-byte stores
  uint32_t ext[kMaxDims];
  int64_t xs[kMaxDims], cs[kMaxDims];  // X / C strides of the merged row axes
  int64_t xk[kSkinnyMax];              // X offset of contracted index l
  int64_t yk[kSkinnyMax], yj[kSkinnyMax];
  int64_t cj;                          // C stride of the small index j
};

__device__ __forceinline__ void row_offsets(const SkArgs& a, int64_t i, int64_t* xo, int64_t* co) {
  uint32_t r = (uint32_t)i;
  int64_t x = 0, c = 0;
#pragma unroll
  for (int d = 0; d < kMaxDims; d++) {
    if (d < a.nd) {
      uint32_t digit = r;
      if (d + 1 < a.nd) {
        const uint32_t q = r / a.ext[d];
        digit = r - q * a.ext[d];
        r = q;
      }
      x += (int64_t)digit * a.xs[d];
      c += (int64_t)digit * a.cs[d];
    }
  }
  *xo = x;
  *co = c;
}

template <int BYTES>
__device__ __forceinline__ void cp_async(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  if constexpr (BYTES == 8)
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(s), "l"(gmem));
  else
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
// 16-byte L1-bypassing copy of which the first `bytes` (8 or 16) are read and
// the rest zero-filled.
__device__ __forceinline__ void cp_async16n(void* smem, const void* gmem, int bytes) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(bytes));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void dmma(double (&c)[4], const double (&a)[4], const double (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
      : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(b[0]), "d"(b[1]));
}
// k = 4 step: A values (row g, col t), (row g + 8, col t) -- the first two of
// the k = 8 fragment -- and B (row t, col g), its first value.
__device__ __forceinline__ void dmma_k4(double (&c)[4], const double (&a)[4], const double (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
      : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
      : "d"(a[0]), "d"(a[1]), "d"(b[0]));
}

template <bool CPLX>
struct Elem;
template <>
struct Elem<false> {
  using T = double;
  __device__ static T zero() { return 0.0; }
};
template <>
struct Elem<true> {
  using T = double2;
  __device__ static T zero() { return make_double2(0.0, 0.0); }
};

// Dynamic shared memory: kStages tiles Xs[k + 1][kPitch] of T; row k of every
// stage stays zero and stands in for the padding rows k..KS*8-1.
// Small real fragment sets (KS, NT <= 2) are held to 85 registers: three
// CTAs per SM, 24 warps to hide the copy and tensor latencies.
template <bool CPLX, int KS, int NT>
__global__ void __launch_bounds__(kThreads, (!CPLX && KS <= 2 && NT <= 2) ? 3 : 1) skinny_kernel(const __grid_constant__ SkArgs a) {
  pdl_release();
  pdl_wait();  // before the first global access
  using T = typename Elem<CPLX>::T;
  constexpr int KP = KS * 8;
  constexpr int ES = sizeof(T);
  constexpr int kPitch = pitch<CPLX>();
  const int STAGE = (a.k + 1) * kPitch;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ int64_t s_cb[kStages];  // C base offset of the tile in each stage (fast mode)
  T* Xs = reinterpret_cast<T*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const T* X = static_cast<const T*>(a.X);
  const T* Y = static_cast<const T*>(a.Y);
  T* C = static_cast<T*>(a.C);
  const int64_t cjt = 2 * t * a.cj;  // this lane's first output column
  // k not a multiple of 8 with at most 4 values in its last k = 8 step: that
  // step is one k = 4 MMA (a quarter of the tensor work at k = 10)
  const bool tail4 = (a.k & 7) != 0 && (a.k & 7) <= 4;
  // per-lane constants: fragment row offsets (rows l >= k read the zero row)
  int foff[KS][2];
#pragma unroll
  for (int ks = 0; ks < KS; ks++)
#pragma unroll
    for (int qh = 0; qh < 2; qh++) foff[ks][qh] = min(ks * 8 + t + 4 * qh, a.k) * kPitch + g;
  // paired stores: this lane's column of each n8 tile and its C offset
  const int odd = g & 1;
  int64_t pcol[NT];
  bool pok[NT];
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    const int j = nt * 8 + 2 * t + odd;
    pok[nt] = j < a.n;
    pcol[nt] = (int64_t)j * a.cj;
  }

  // X / C offsets of row r of a tile: from the tile's base offsets when the
  // tile lies inside one run of the fastest row axis, else by decomposition
  auto offs = [&](int64_t tile, int r, int64_t xb, int64_t cb, int64_t* xo, int64_t* co) {
    if (a.fast) {
      *xo = xb + r * a.xs[0];
      *co = cb + r * a.cs[0];
    } else {
      row_offsets(a, tile * kTileRows + r, xo, co);
    }
  };
  // Fast mode: the X / C base offsets of consecutive tiles follow from one
  // another without a division: the fastest row axis advances by a tile and
  // carries into the slower ones when it wraps.
  struct TileIt {
    uint32_t dig[kMaxDims];
    int64_t xb, cb;
  };
  auto it_init = [&](TileIt& it, int64_t tile) {
    it.xb = it.cb = 0;
    uint32_t r = (uint32_t)(tile * kTileRows);
#pragma unroll
    for (int d = 0; d < kMaxDims; d++) {
      it.dig[d] = 0;
      if (d < a.nd) {
        uint32_t digit = r;
        if (d + 1 < a.nd) {
          const uint32_t q = r / a.ext[d];
          digit = r - q * a.ext[d];
          r = q;
        }
        it.dig[d] = digit;
        it.xb += (int64_t)digit * a.xs[d];
        it.cb += (int64_t)digit * a.cs[d];
      }
    }
  };
  auto it_next = [&](TileIt& it) {
    it.dig[0] += kTileRows;
    it.xb += kTileRows * a.xs[0];
    it.cb += kTileRows * a.cs[0];
#pragma unroll
    for (int d = 0; d + 1 < kMaxDims; d++) {
      if (d + 1 < a.nd && it.dig[d] == a.ext[d]) {
        it.dig[d] = 0;
        it.xb += a.xs[d + 1] - (int64_t)a.ext[d] * a.xs[d];
        it.cb += a.cs[d + 1] - (int64_t)a.ext[d] * a.cs[d];
        it.dig[d + 1] += 1;
      }
    }
  };
  // copy of tile `tile` into `stage`.  Pair mode (f64): thread tid brings
  // rows 2p, 2p+1 (p = tid % 128) for l = h, h + 2, ... (h = tid / 128) in
  // 16-byte L1-bypassing copies; otherwise row tid's k values one by one.
  int64_t xkh[(KP + 1) / 2];  // pair mode: k offsets of l = h, h + 2, ...
#pragma unroll
  for (int u = 0; u < (KP + 1) / 2; u++) {
    const int l = 2 * u + (tid >> 7);
    xkh[u] = l < a.k ? a.xk[l] : 0;
  }
  auto issue = [&](int64_t tile, int stage, int64_t xb, int64_t cb) {
    T* sbase = Xs + stage * STAGE;
    if (tid == 0) s_cb[stage] = cb;  // read when the stage is computed, after a barrier
    if (!CPLX && a.pair) {
      const int p = tid & 127, h = tid >> 7;
      const int64_t i = tile * kTileRows + 2 * p;
      if (i < a.rows) {
        int64_t xo, co;
        offs(tile, 2 * p, xb, cb, &xo, &co);
        const int bytes = i + 1 < a.rows ? 16 : 8;
        const T* src = X + xo;
        T* dst = sbase + 2 * p;
#pragma unroll
        for (int u = 0; u < (KP + 1) / 2; u++)
          if (2 * u + h < a.k) cp_async16n(dst + (2 * u + h) * kPitch, src + xkh[u], bytes);
      }
      return;
    }
    if (tile * kTileRows + tid < a.rows) {
      int64_t xo, co;
      offs(tile, tid, xb, cb, &xo, &co);
      const T* src = X + xo;
      T* dst = sbase + tid;
#pragma unroll
      for (int l = 0; l < KP; l++)
        if (l < a.k) cp_async<ES>(dst + l * kPitch, src + a.xk[l]);
    }
  };
  // Each CTA takes a contiguous run of tiles (consecutive tiles: one
  // offset update each in fast mode).
  const int64_t t0 = blockIdx.x * a.ntiles / gridDim.x, t1 = (blockIdx.x + 1) * a.ntiles / gridDim.x;
  TileIt iti;  // the next tile to issue
  if (a.fast) it_init(iti, t0);
#pragma unroll
  for (int s = 0; s < kStages - 1; s++) {
    const int64_t tile = t0 + s;
    if (tile < t1) {
      issue(tile, s, a.fast ? iti.xb : 0, a.fast ? iti.cb : 0);
      if (a.fast) it_next(iti);
    }
    cp_commit();
  }
  for (int e = tid; e < kStages * kPitch; e += kThreads)
    Xs[(e / kPitch) * STAGE + a.k * kPitch + e % kPitch] = Elem<CPLX>::zero();
  // Y fragments: b_i = Y(ks*8 + t + 4i, nt*8 + g), zero outside k x n
  double br[KS][NT][2], bi[KS][NT][2];
#pragma unroll
  for (int ks = 0; ks < KS; ks++)
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int q = 0; q < 2; q++) {
        const int l = ks * 8 + t + 4 * q, j = nt * 8 + g;
        const T v = (l < a.k && j < a.n) ? Y[a.yk[l] + a.yj[j]] : Elem<CPLX>::zero();
        if constexpr (CPLX) {
          br[ks][nt][q] = v.x;
          bi[ks][nt][q] = v.y;
        } else {
          br[ks][nt][q] = v;
        }
      }

  int stage = 0;
  for (int64_t tile = t0; tile < t1; tile++) {
    cp_wait<kStages - 2>();
    __syncthreads();  // tile landed for all threads; the stage refilled below is free
    {
      const int64_t tn = tile + (kStages - 1);
      if (tn < t1) {
        issue(tn, stage == 0 ? kStages - 1 : stage - 1, a.fast ? iti.xb : 0, a.fast ? iti.cb : 0);
        if (a.fast) it_next(iti);
      }
      cp_commit();
    }
    const T* xs = Xs + stage * STAGE;
    const int64_t xb = 0, cb = a.fast ? s_cb[stage] : 0;  // stores need C's offsets only
#pragma unroll
    for (int mt = 0; mt < 2; mt++) {
      const int row0 = warp * 32 + mt * 16;
      double cr[NT][4], ci[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int q = 0; q < 4; q++) cr[nt][q] = ci[nt][q] = 0.0;
#pragma unroll
      for (int ks = 0; ks < KS; ks++) {
        // the last step holds at most 4 contracted values: one k = 4 MMA
        const bool k4 = ks == KS - 1 && tail4;
        double ar[4], ai[4], nai[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
          if (k4 && q >= 2) {
            ar[q] = ai[q] = nai[q] = 0.0;
            continue;
          }
          const T v = xs[foff[ks][q >> 1] + row0 + 8 * (q & 1)];
          if constexpr (CPLX) {
            ar[q] = v.x;
            ai[q] = v.y;
            nai[q] = -v.y;
          } else {
            ar[q] = v;
          }
        }
        if (k4) {
#pragma unroll
          for (int nt = 0; nt < NT; nt++) {
            dmma_k4(cr[nt], ar, br[ks][nt]);
            if constexpr (CPLX) {
              dmma_k4(cr[nt], nai, bi[ks][nt]);
              dmma_k4(ci[nt], ar, bi[ks][nt]);
              dmma_k4(ci[nt], ai, br[ks][nt]);
            }
          }
        } else {
#pragma unroll
          for (int nt = 0; nt < NT; nt++) {
            dmma(cr[nt], ar, br[ks][nt]);
            if constexpr (CPLX) {
              dmma(cr[nt], nai, bi[ks][nt]);
              dmma(ci[nt], ar, bi[ks][nt]);
              dmma(ci[nt], ai, br[ks][nt]);
            }
          }
        }
      }
      // c0, c1 at (row g, cols 2t, 2t+1); c2, c3 at (row g + 8, same cols)
      if (!CPLX && a.cpair) {
        // 16-byte stores of row pairs: lanes g and g ^ 1 swap one value, so
        // even g holds rows (g, g+1) of column 2t, odd g rows (g-1, g) of 2t+1
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const int rb = row0 + g - odd + 8 * h;  // even row of the pair
          const int64_t ib = tile * kTileRows + rb;
          int64_t xo, co;
          offs(tile, rb, xb, cb, &xo, &co);
#pragma unroll
          for (int nt = 0; nt < NT; nt++) {
            const double v0 = cr[nt][2 * h], v1 = cr[nt][2 * h + 1];
            const double recv = __shfl_xor_sync(0xffffffffu, odd ? v0 : v1, 4);
            const double lo = odd ? recv : v0, hi = odd ? v1 : recv;
            if (pok[nt] && ib < a.rows) {
              double* cp = reinterpret_cast<double*>(C) + co + pcol[nt];
              if (ib + 1 < a.rows)
                *reinterpret_cast<double2*>(cp) = make_double2(lo, hi);
              else
                *cp = lo;
            }
          }
        }
      } else {
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const int r = row0 + g + 8 * h;
          if (tile * kTileRows + r < a.rows) {
            int64_t xo, co;
            offs(tile, r, xb, cb, &xo, &co);
            T* cp = C + co + cjt;
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
              for (int q = 0; q < 2; q++) {
                if (nt * 8 + 2 * t + q < a.n) {
                  if constexpr (CPLX)
                    cp[(nt * 8 + q) * a.cj] = make_double2(cr[nt][2 * h + q], ci[nt][2 * h + q]);
                  else
                    cp[(nt * 8 + q) * a.cj] = cr[nt][2 * h + q];
                }
              }
          }
        }
      }
    }
    stage = stage + 1 == kStages ? 0 : stage + 1;
  }
  asm volatile("cp.async.wait_all;\n" ::);
}

template <bool CPLX, int KS, int NT>
void launch_sk(SkArgs a, cudaStream_t s) {
  auto kern = skinny_kernel<CPLX, KS, NT>;
  const size_t smem = (size_t)kStages * (a.k + 1) * pitch<CPLX>() * (CPLX ? 16 : 8);
  ensure_dynamic_smem((const void*)kern, smem);
  const DeviceCtx& c = ctx();
  int per_sm = 0;
  NDT_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem));
  a.ntiles = (a.rows + kTileRows - 1) / kTileRows;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(a.ntiles, (int64_t)c.sm_count * std::max(per_sm, 1)));
  launch_pdl(kern, dim3(grid), dim3(kThreads), smem, s, a);
  count_launch();
  NDT_CUDA(cudaGetLastError());
}


// k and n rounded up to multiples of 8 (KS, NT in 1..4; 1..2 for complex).
template <bool CPLX>
void dispatch_sk(const SkArgs& a, cudaStream_t s) {
  const int ks = (a.k + 7) / 8, nt = (a.n + 7) / 8;
#define NDT_SK(KS_, NT_) \
  if (ks == KS_ && nt == NT_) return launch_sk<CPLX, KS_, NT_>(a, s);
  NDT_SK(1, 1) NDT_SK(1, 2) NDT_SK(2, 1) NDT_SK(2, 2)
  if constexpr (!CPLX) {
    NDT_SK(1, 3) NDT_SK(1, 4) NDT_SK(2, 3) NDT_SK(2, 4) NDT_SK(3, 1) NDT_SK(3, 2) NDT_SK(3, 3) NDT_SK(3, 4)
    NDT_SK(4, 1) NDT_SK(4, 2) NDT_SK(4, 3) NDT_SK(4, 4)
  }
#undef NDT_SK
  throw Error(ErrKind::InvalidArgument, "skinny contraction outside its range");
}

// Offsets of every value of a short mixed-radix index (fastest axis first).
void offsets(const std::vector<int64_t>& ext, const std::vector<int64_t>& stride, int64_t* out, int64_t count) {
  for (int64_t v = 0; v < count; v++) {
    int64_t r = v, off = 0;
    for (size_t d = 0; d < ext.size(); d++) {
      off += (r % ext[d]) * stride[d];
      r /= ext[d];
    }
    out[v] = off;
  }
}

}  // namespace

bool skinny_contract(DType dt, const void* A, const void* B, void* C, const std::vector<StridedAxis>& M,
                     const std::vector<StridedAxis>& N, const std::vector<ContractedAxis>& K, cudaStream_t s) {
  const bool cplx = dt == DType::C128;
  const int64_t lim = cplx ? 16 : kSkinnyMax;
  constexpr int64_t kMinRows = 2048;
  int64_t m = 1, n = 1, k = 1;
  for (const StridedAxis& x : M) m *= x.n;
  for (const StridedAxis& x : N) n *= x.n;
  for (const ContractedAxis& x : K) k *= x.n;
  if (m <= 0 || n <= 0 || k <= 0 || k > lim) return false;
  const bool small_n = n <= lim && m >= kMinRows;
  const bool small_m = !small_n && m <= lim && n >= kMinRows;
  if (!small_n && !small_m) return false;
  const std::vector<StridedAxis>& big = small_n ? M : N;
  const std::vector<StridedAxis>& sml = small_n ? N : M;
  const int64_t rows = small_n ? m : n;
  if (rows >= ((int64_t)1 << 31)) return false;

  SkArgs a{};
  a.X = small_n ? A : B;
  a.Y = small_n ? B : A;
  a.C = C;
  a.rows = rows;
  a.k = (int)k;
  a.n = (int)(small_n ? n : m);
  // Row axes with their X and C strides; C is dense with M fastest.
  int64_t cstride = small_n ? 1 : m;
  std::vector<int64_t> ext, xs, cs;
  for (const StridedAxis& x : big) {
    if (x.n != 1) {
      const size_t d = ext.size();
      if (d > 0 && xs[d - 1] * ext[d - 1] == x.s && cs[d - 1] * ext[d - 1] == cstride) {
        ext[d - 1] *= x.n;  // contiguous in both X and C: merge
      } else {
        ext.push_back(x.n);
        xs.push_back(x.s);
        cs.push_back(cstride);
      }
    }
    cstride *= x.n;
  }
  if (ext.size() > (size_t)kMaxDims) return false;
  a.nd = (int)ext.size();
  for (int d = 0; d < a.nd; d++) {
    a.ext[d] = (uint32_t)ext[d];
    a.xs[d] = xs[d];
    a.cs[d] = cs[d];
  }
  if (a.nd == 0) {  // a single row
    a.nd = 1;
    a.ext[0] = 1;
  }
  a.fast = (a.nd == 1 || a.ext[0] % kTileRows == 0) ? 1 : 0;
  // Pair mode: every row pair (2p, 2p+1) of a tile is two adjacent elements
  // starting at an even element offset of a 16-byte aligned X.
  bool pair = !cplx && a.fast && a.xs[0] == 1 && ((uintptr_t)(small_n ? A : B) & 15) == 0;
  if (a.nd > 1) pair = pair && a.ext[0] % 2 == 0;
  for (int d = 1; d < a.nd; d++) pair = pair && a.xs[d] % 2 == 0;
  std::vector<int64_t> ke, kx, ky, je, js;
  for (const ContractedAxis& x : K) {
    ke.push_back(x.n);
    kx.push_back(small_n ? x.sa : x.sb);
    ky.push_back(small_n ? x.sb : x.sa);
  }
  for (const StridedAxis& x : sml) {
    je.push_back(x.n);
    js.push_back(x.s);
  }
  offsets(ke, kx, a.xk, k);
  offsets(ke, ky, a.yk, k);
  offsets(je, js, a.yj, a.n);
  for (int l = 0; l < a.k; l++) pair = pair && a.xk[l] % 2 == 0;
  a.pair = pair ? 1 : 0;
  // Store pairs: C rows 2p, 2p+1 adjacent (small n: the row axis is C's
  // fastest) with even column stride and even tile offsets.
  bool cpair = !cplx && small_n && a.fast && a.cs[0] == 1 && m % 2 == 0 && ((uintptr_t)C & 15) == 0;
  if (a.nd > 1) cpair = cpair && a.ext[0] % 2 == 0;
  for (int d = 1; d < a.nd; d++) cpair = cpair && a.cs[d] % 2 == 0;
  a.cpair = cpair ? 1 : 0;
  a.cj = small_n ? m : 1;
  if (cplx)
    dispatch_sk<true>(a, s);
  else
    dispatch_sk<false>(a, s);
  return true;
}

}  // namespace ndt
