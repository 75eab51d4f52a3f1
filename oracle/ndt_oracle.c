/*
 * ndt_oracle.c — CPU oracle for the ndtensors contraction hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the reference answer for tests/, smoke() and bench.py's
 * CPU-baseline leg.  Never part of the product path.
 *
 * Each function restates one reference algorithm (ndtensors-rs,
 * crates/ndtensors/src/...), cited per function.  The restatement keeps the
 * reference's iteration orders, validation order and panic sites so that
 * status codes and (for the naive loop) floating-point results match.  It
 * is compiled with -ffp-contract=off so that a*b+c is never fused, like Rust.
 */
#include "ndt_oracle.h"

#include <stdlib.h>
#include <string.h>

#define MAXR 64 /* maximum rank handled by the oracle */

typedef struct {
  double re, im;
} cplx;

static size_t esize_of(int dtype) { return dtype == 1 ? 16 : 8; }

static size_t prod(const size_t* s, size_t n) {
  size_t p = 1;
  for (size_t i = 0; i < n; i++) p *= s[i];
  return p;
}
static size_t prod_max1(const size_t* s, size_t n) {
  size_t p = prod(s, n);
  return p < 1 ? 1 : p;
}

/* strides.rs:19-33 */
void ndo_compute_strides(const size_t* shape, size_t ndim, size_t* strides) {
  size_t st = 1;
  for (size_t i = 0; i < ndim; i++) {
    strides[i] = st;
    st *= shape[i];
  }
}

/* strides.rs:46-52 */
size_t ndo_cartesian_to_linear(const size_t* idx, const size_t* strides, size_t ndim) {
  size_t l = 0;
  for (size_t i = 0; i < ndim; i++) l += idx[i] * strides[i];
  return l;
}

/* strides.rs:64-73 */
int ndo_linear_to_cartesian(size_t linear, const size_t* shape, size_t ndim, size_t* idx) {
  for (size_t i = 0; i < ndim; i++) {
    if (shape[i] == 0) return NDO_PANIC; /* `linear % 0` panics in Rust */
    idx[i] = linear % shape[i];
    linear /= shape[i];
  }
  return NDO_OK;
}

/* permutedims.rs:198-224 */
int ndo_validate_permutation(const size_t* perm, size_t nperm, size_t ndim) {
  if (nperm != ndim) return NDO_ERR_INVALID_PERMUTATION;
  unsigned char seen[MAXR];
  if (ndim > MAXR) return NDO_PANIC;
  memset(seen, 0, sizeof(seen));
  for (size_t i = 0; i < nperm; i++) {
    if (perm[i] >= ndim) return NDO_ERR_INVALID_PERMUTATION;
    if (seen[perm[i]]) return NDO_ERR_INVALID_PERMUTATION;
    seen[perm[i]] = 1;
  }
  return NDO_OK;
}

/* backend/generic.rs:15-39 over source linear indices [lo, hi). */
int ndo_permutedims_range(int dtype, const void* src, const size_t* shape, size_t ndim,
                          const size_t* perm, void* dst, size_t lo, size_t hi) {
  size_t es = esize_of(dtype);
  size_t new_shape[MAXR], new_strides[MAXR], old_idx[MAXR];
  if (ndim > MAXR) return NDO_PANIC;
  for (size_t i = 0; i < ndim; i++) new_shape[i] = shape[perm[i]];
  ndo_compute_strides(new_shape, ndim, new_strides);
  const unsigned char* s = (const unsigned char*)src;
  unsigned char* d = (unsigned char*)dst;
  for (size_t lin = lo; lin < hi; lin++) {
    if (ndo_linear_to_cartesian(lin, shape, ndim, old_idx) != NDO_OK) return NDO_PANIC;
    size_t lnew = 0;
    for (size_t i = 0; i < ndim; i++) lnew += old_idx[perm[i]] * new_strides[i];
    memcpy(d + lnew * es, s + lin * es, es);
  }
  return NDO_OK;
}

/* permutedims.rs:51-68 */
int ndo_permutedims(int dtype, const void* src, const size_t* shape, size_t ndim,
                    const size_t* perm, size_t nperm, void* dst) {
  int st = ndo_validate_permutation(perm, nperm, ndim);
  if (st != NDO_OK) return st;
  /* DenseTensor::zeros(new_shape): max(1, prod) zero elements */
  size_t total = prod_max1(shape, ndim);
  memset(dst, 0, total * esize_of(dtype));
  /* GenericBackend iterates over src.len() = max(1, prod) elements */
  return ndo_permutedims_range(dtype, src, shape, ndim, perm, dst, 0, total);
}

/* ---------------------------------------------------------------- naive */

static int naive_pairs(const size_t* sa, size_t na, const int32_t* la,
                       const size_t* sb, size_t nb, const int32_t* lb,
                       size_t* npairs, size_t* pa, size_t* pb) {
  /* contract/naive.rs:66-83: first match in B wins, sizes checked */
  size_t np = 0;
  for (size_t i = 0; i < na; i++) {
    if (la[i] < 0) {
      for (size_t j = 0; j < nb; j++) {
        if (la[i] == lb[j]) {
          if (sa[i] != sb[j]) return NDO_ERR_SHAPE_MISMATCH;
          pa[np] = i;
          pb[np] = j;
          np++;
          break;
        }
      }
    }
  }
  *npairs = np;
  return NDO_OK;
}

int ndo_contract_naive_outshape(const size_t* sa, size_t na, const int32_t* la, size_t nla,
                                const size_t* sb, size_t nb, const int32_t* lb, size_t nlb,
                                size_t* out_shape, size_t* out_ndim) {
  if (nla != na) return NDO_ERR_WRONG_NUM_INDICES;
  if (nlb != nb) return NDO_ERR_WRONG_NUM_INDICES;
  if (na > MAXR || nb > MAXR) return NDO_PANIC;
  size_t np, pa[MAXR], pb[MAXR];
  int st = naive_pairs(sa, na, la, sb, nb, lb, &np, pa, pb);
  if (st != NDO_OK) return st;
  size_t k = 0;
  for (size_t i = 0; i < na; i++)
    if (la[i] > 0) out_shape[k++] = sa[i];
  for (size_t j = 0; j < nb; j++)
    if (lb[j] > 0) out_shape[k++] = sb[j];
  if (k == 0) out_shape[k++] = 1; /* naive.rs:112-114 */
  *out_ndim = k;
  return NDO_OK;
}

static void mac(int dtype, void* acc, const void* x, const void* y) {
  if (dtype == 0) {
    double* s = (double*)acc;
    double p = *(const double*)x * *(const double*)y;
    *s = *s + p;
  } else {
    cplx* s = (cplx*)acc;
    const cplx* a = (const cplx*)x;
    const cplx* b = (const cplx*)y;
    double re = a->re * b->re - a->im * b->im;
    double im = a->re * b->im + a->im * b->re;
    s->re = s->re + re;
    s->im = s->im + im;
  }
}

/* contract/naive.rs:45-187 */
int ndo_contract_naive(int dtype,
                       const void* a, size_t len_a, const size_t* sa, size_t na, const int32_t* la, size_t nla,
                       const void* b, size_t len_b, const size_t* sb, size_t nb, const int32_t* lb, size_t nlb,
                       void* out, size_t out_cap) {
  if (nla != na) return NDO_ERR_WRONG_NUM_INDICES;
  if (nlb != nb) return NDO_ERR_WRONG_NUM_INDICES;
  if (na > MAXR || nb > MAXR) return NDO_PANIC;
  size_t np, pa[MAXR], pb[MAXR];
  int st = naive_pairs(sa, na, la, sb, nb, lb, &np, pa, pb);
  if (st != NDO_OK) return st;
  size_t out_shape[2 * MAXR + 1], ond = 0;
  for (size_t i = 0; i < na; i++)
    if (la[i] > 0) out_shape[ond++] = sa[i];
  for (size_t j = 0; j < nb; j++)
    if (lb[j] > 0) out_shape[ond++] = sb[j];
  if (ond == 0) out_shape[ond++] = 1;
  size_t out_total = prod_max1(out_shape, ond); /* result.len() */
  if (out_cap < out_total) return NDO_ERR_CAPACITY;
  size_t es = esize_of(dtype);
  memset(out, 0, out_total * es);

  size_t cdims[MAXR];
  for (size_t p = 0; p < np; p++) cdims[p] = sa[pa[p]];
  size_t ctotal = prod_max1(cdims, np);
  size_t stra[MAXR], strb[MAXR];
  ndo_compute_strides(sa, na, stra);
  ndo_compute_strides(sb, nb, strb);
  /* For each axis, which contracted pair drives it (position of the first
   * pair naming the axis), or -1 when the axis is pinned to index 0. */
  long cpa[MAXR], cpb[MAXR];
  for (size_t i = 0; i < na; i++) {
    cpa[i] = -1;
    for (size_t p = 0; p < np; p++)
      if (pa[p] == i) { cpa[i] = (long)p; break; }
  }
  for (size_t j = 0; j < nb; j++) {
    cpb[j] = -1;
    for (size_t p = 0; p < np; p++)
      if (pb[p] == j) { cpb[j] = (long)p; break; }
  }
  const unsigned char* A = (const unsigned char*)a;
  const unsigned char* B = (const unsigned char*)b;
  unsigned char* C = (unsigned char*)out;
  size_t oidx[2 * MAXR + 1], cidx[MAXR];
  for (size_t ol = 0; ol < out_total; ol++) {
    if (ndo_linear_to_cartesian(ol, out_shape, ond, oidx) != NDO_OK) return NDO_PANIC;
    cplx sum = {0.0, 0.0};
    for (size_t cl = 0; cl < ctotal; cl++) {
      if (ndo_linear_to_cartesian(cl, cdims, np, cidx) != NDO_OK) return NDO_PANIC;
      size_t k = 0, al = 0, bl = 0;
      for (size_t i = 0; i < na; i++) {
        size_t v = 0;
        if (la[i] > 0) v = oidx[k++];
        else if (cpa[i] >= 0) v = cidx[cpa[i]];
        al += v * stra[i];
      }
      for (size_t j = 0; j < nb; j++) {
        size_t v = 0;
        if (lb[j] > 0) v = oidx[k++];
        else if (cpb[j] >= 0) v = cidx[cpb[j]];
        bl += v * strb[j];
      }
      if (al >= len_a || bl >= len_b) return NDO_PANIC; /* get_linear(..).unwrap() */
      mac(dtype, &sum, A + al * es, B + bl * es);
    }
    memcpy(C + ol * es, &sum, es);
  }
  return NDO_OK;
}

/* ------------------------------------------------------------ properties */

typedef struct {
  size_t np, pa[MAXR], pb[MAXR];
  size_t nua, ua[MAXR], nub, ub[MAXR];
  size_t perm_a[MAXR], perm_b[MAXR], perm_c[2 * MAXR];
  int32_t out_labels[2 * MAXR];
  size_t nout;
  size_t dleft, dmid, dright;
  int permute_a, permute_b, permute_c;
} props_t;

static int is_identity(const size_t* p, size_t n) {
  for (size_t i = 0; i < n; i++)
    if (p[i] != i) return 0;
  return 1;
}

/* contract/properties.rs:94-203 */
static void compute_props(const int32_t* la, const size_t* sa, size_t na,
                          const int32_t* lb, const size_t* sb, size_t nb, props_t* P) {
  P->np = 0;
  for (size_t i = 0; i < na; i++) {
    if (la[i] < 0) {
      for (size_t j = 0; j < nb; j++) {
        if (la[i] == lb[j]) {
          P->pa[P->np] = i;
          P->pb[P->np] = j;
          P->np++;
          break;
        }
      }
    }
  }
  P->nua = 0;
  for (size_t i = 0; i < na; i++) {
    int found = 0;
    for (size_t p = 0; p < P->np; p++)
      if (P->pa[p] == i) found = 1;
    if (!found) P->ua[P->nua++] = i;
  }
  P->nub = 0;
  for (size_t j = 0; j < nb; j++) {
    int found = 0;
    for (size_t p = 0; p < P->np; p++)
      if (P->pb[p] == j) found = 1;
    if (!found) P->ub[P->nub++] = j;
  }
  size_t dl = 1, dm = 1, dr = 1;
  for (size_t i = 0; i < P->nua; i++) dl *= sa[P->ua[i]];
  for (size_t p = 0; p < P->np; p++) dm *= sa[P->pa[p]];
  for (size_t j = 0; j < P->nub; j++) dr *= sb[P->ub[j]];
  P->dleft = dl < 1 ? 1 : dl;
  P->dmid = dm < 1 ? 1 : dm;
  P->dright = dr < 1 ? 1 : dr;
  size_t k = 0;
  for (size_t i = 0; i < P->nua; i++) P->perm_a[k++] = P->ua[i];
  for (size_t p = 0; p < P->np; p++) P->perm_a[k++] = P->pa[p];
  P->permute_a = !is_identity(P->perm_a, k);
  k = 0;
  for (size_t p = 0; p < P->np; p++) P->perm_b[k++] = P->pb[p];
  for (size_t j = 0; j < P->nub; j++) P->perm_b[k++] = P->ub[j];
  P->permute_b = !is_identity(P->perm_b, k);
  P->nout = 0;
  for (size_t i = 0; i < P->nua; i++) P->out_labels[P->nout++] = la[P->ua[i]];
  for (size_t j = 0; j < P->nub; j++) P->out_labels[P->nout++] = lb[P->ub[j]];
  /* stable argsort by label (Rust sort_by_key is stable) */
  size_t n = P->nout;
  for (size_t i = 0; i < n; i++) P->perm_c[i] = i;
  for (size_t i = 1; i < n; i++) {
    size_t v = P->perm_c[i];
    size_t j = i;
    while (j > 0 && P->out_labels[P->perm_c[j - 1]] > P->out_labels[v]) {
      P->perm_c[j] = P->perm_c[j - 1];
      j--;
    }
    P->perm_c[j] = v;
  }
  /* permute_c = output_labels != sorted(output_labels) */
  P->permute_c = 0;
  for (size_t i = 0; i < n; i++)
    if (P->out_labels[P->perm_c[i]] != P->out_labels[i]) P->permute_c = 1;
  if (!P->permute_c)
    for (size_t i = 0; i < n; i++) P->perm_c[i] = i;
}

int ndo_contract_properties(const int32_t* la, const size_t* sa, size_t na,
                            const int32_t* lb, const size_t* sb, size_t nb,
                            size_t* npairs, size_t* pairs_a, size_t* pairs_b,
                            size_t* n_unc_a, size_t* unc_a, size_t* n_unc_b, size_t* unc_b,
                            size_t* perm_a, size_t* perm_b, size_t* perm_c,
                            int32_t* output_labels, size_t* dims, int* flags) {
  if (na > MAXR || nb > MAXR) return NDO_PANIC;
  props_t P;
  compute_props(la, sa, na, lb, sb, nb, &P);
  *npairs = P.np;
  for (size_t p = 0; p < P.np; p++) {
    pairs_a[p] = P.pa[p];
    pairs_b[p] = P.pb[p];
  }
  *n_unc_a = P.nua;
  *n_unc_b = P.nub;
  memcpy(unc_a, P.ua, P.nua * sizeof(size_t));
  memcpy(unc_b, P.ub, P.nub * sizeof(size_t));
  memcpy(perm_a, P.perm_a, na * sizeof(size_t));
  memcpy(perm_b, P.perm_b, (P.np + P.nub) * sizeof(size_t));
  memcpy(perm_c, P.perm_c, P.nout * sizeof(size_t));
  memcpy(output_labels, P.out_labels, P.nout * sizeof(int32_t));
  dims[0] = P.dleft;
  dims[1] = P.dmid;
  dims[2] = P.dright;
  flags[0] = P.permute_a;
  flags[1] = P.permute_b;
  flags[2] = P.permute_c;
  return NDO_OK;
}

/* ----------------------------------------------------------- contract_gemm */

/* Permute with the reference's permutedims semantics; a new buffer of
 * max(1, prod) elements is returned in *dst (caller frees). */
static int permute_alloc(int dtype, const void* src, const size_t* shape, size_t ndim,
                         const size_t* perm, size_t nperm, void** dst) {
  size_t es = esize_of(dtype);
  size_t total = prod_max1(shape, ndim);
  *dst = malloc(total * es);
  if (!*dst) return NDO_PANIC;
  int st = ndo_permutedims(dtype, src, shape, ndim, perm, nperm, *dst);
  if (st != NDO_OK) {
    free(*dst);
    *dst = NULL;
  }
  return st;
}

static int gemm_validate(const size_t* sa, size_t na, const int32_t* la, size_t nla,
                         const size_t* sb, size_t nb, const int32_t* lb, size_t nlb) {
  /* contract/gemm.rs:54-79: every matching pair is size-checked */
  if (nla != na) return NDO_ERR_WRONG_NUM_INDICES;
  if (nlb != nb) return NDO_ERR_WRONG_NUM_INDICES;
  if (na > MAXR || nb > MAXR) return NDO_PANIC;
  for (size_t i = 0; i < na; i++)
    if (la[i] < 0)
      for (size_t j = 0; j < nb; j++)
        if (la[i] == lb[j] && sa[i] != sb[j]) return NDO_ERR_SHAPE_MISMATCH;
  return NDO_OK;
}

int ndo_contract_gemm_outshape(const size_t* sa, size_t na, const int32_t* la, size_t nla,
                               const size_t* sb, size_t nb, const int32_t* lb, size_t nlb,
                               size_t* out_shape, size_t* out_ndim) {
  int st = gemm_validate(sa, na, la, nla, sb, nb, lb, nlb);
  if (st != NDO_OK) return st;
  props_t P;
  compute_props(la, sa, na, lb, sb, nb, &P);
  if (P.nua == 0 && P.nub == 0) {
    out_shape[0] = 1;
    *out_ndim = 1;
    return NDO_OK;
  }
  size_t sh[2 * MAXR], k = 0;
  for (size_t i = 0; i < P.nua; i++) sh[k++] = sa[P.ua[i]];
  for (size_t j = 0; j < P.nub; j++) sh[k++] = sb[P.ub[j]];
  for (size_t i = 0; i < k; i++) out_shape[i] = sh[P.perm_c[i]];
  *out_ndim = k;
  return NDO_OK;
}

static void gemm_cm(int dtype, const void* A, const void* B, void* C, size_t m, size_t n, size_t k) {
  /* C[i + j*m] = sum_{l ascending} A[i + l*m] * B[l + j*k] */
  if (dtype == 0) {
    const double* a = (const double*)A;
    const double* b = (const double*)B;
    double* c = (double*)C;
    for (size_t i = 0; i < m; i++)
      for (size_t j = 0; j < n; j++) {
        double s = 0.0;
        for (size_t l = 0; l < k; l++) s = s + a[i + l * m] * b[l + j * k];
        c[i + j * m] = s;
      }
  } else {
    const cplx* a = (const cplx*)A;
    const cplx* b = (const cplx*)B;
    cplx* c = (cplx*)C;
    for (size_t i = 0; i < m; i++)
      for (size_t j = 0; j < n; j++) {
        cplx s = {0.0, 0.0};
        for (size_t l = 0; l < k; l++) mac(1, &s, &a[i + l * m], &b[l + j * k]);
        c[i + j * m] = s;
      }
  }
}

/* contract/gemm.rs:47-236 */
int ndo_contract_gemm(int dtype,
                      const void* a, size_t len_a, const size_t* sa, size_t na, const int32_t* la, size_t nla,
                      const void* b, size_t len_b, const size_t* sb, size_t nb, const int32_t* lb, size_t nlb,
                      void* out, size_t out_cap) {
  int st = gemm_validate(sa, na, la, nla, sb, nb, lb, nlb);
  if (st != NDO_OK) return st;
  props_t P;
  compute_props(la, sa, na, lb, sb, nb, &P);
  size_t es = esize_of(dtype);
  void *aw = NULL, *bw = NULL;
  const void *ap = a, *bp = b;
  size_t alen = len_a, blen = len_b;
  int full = (P.nua == 0 && P.nub == 0);
  int outer = (P.np == 0);
  if (full || !outer) {
    if (P.permute_a) {
      st = permute_alloc(dtype, a, sa, na, P.perm_a, P.nua + P.np, &aw);
      if (st != NDO_OK) return st;
      ap = aw;
    }
    if (P.permute_b) {
      st = permute_alloc(dtype, b, sb, nb, P.perm_b, P.np + P.nub, &bw);
      if (st != NDO_OK) { free(aw); return st; }
      bp = bw;
    }
  }
  if (full) {
    /* contract_full (gemm.rs:98-125): dot over zip(a.data, b.data) */
    if (out_cap < 1) { free(aw); free(bw); return NDO_ERR_CAPACITY; }
    size_t n = alen < blen ? alen : blen;
    cplx s = {0.0, 0.0};
    const unsigned char* A = (const unsigned char*)ap;
    const unsigned char* B = (const unsigned char*)bp;
    for (size_t i = 0; i < n; i++) mac(dtype, &s, A + i * es, B + i * es);
    memcpy(out, &s, es);
    free(aw);
    free(bw);
    return NDO_OK;
  }
  size_t m = P.dleft, kk = P.dmid, n = P.dright;
  /* as_faer_mat asserts rows*cols == len (faer_interop.rs:72-84) */
  if (outer) {
    if (m != alen || n != blen) { free(aw); free(bw); return NDO_PANIC; }
    kk = 1;
  } else {
    if (m * kk != alen || kk * n != blen) { free(aw); free(bw); return NDO_PANIC; }
  }
  size_t sh[2 * MAXR], ond = 0;
  for (size_t i = 0; i < P.nua; i++) sh[ond++] = sa[P.ua[i]];
  for (size_t j = 0; j < P.nub; j++) sh[ond++] = sb[P.ub[j]];
  if (ond == 0) sh[ond++] = 1;
  /* DenseTensor::from_vec(c, output_shape) length check */
  if (m * n != prod_max1(sh, ond)) { free(aw); free(bw); return NDO_ERR_SHAPE_MISMATCH; }
  if (out_cap < m * n) { free(aw); free(bw); return NDO_ERR_CAPACITY; }
  void* c = P.permute_c ? malloc(m * n * es) : out;
  if (!c) { free(aw); free(bw); return NDO_PANIC; }
  gemm_cm(dtype, ap, bp, c, m, n, kk);
  free(aw);
  free(bw);
  if (P.permute_c) {
    st = ndo_permutedims(dtype, c, sh, ond, P.perm_c, ond, out);
    free(c);
    return st;
  }
  return NDO_OK;
}

/* ---------------------------------------------------------- block-sparse */

static const size_t* dim_sizes(const ndo_bs_desc* D, size_t ax) {
  const size_t* p = D->bsz;
  for (size_t i = 0; i < ax; i++) p += D->nblk[i];
  return p;
}
static size_t block_elems(const ndo_bs_desc* D, const size_t* coords) {
  size_t s = 1;
  for (size_t ax = 0; ax < D->ndim; ax++) s *= dim_sizes(D, ax)[coords[ax]];
  return s;
}
static void block_shape(const ndo_bs_desc* D, const size_t* coords, size_t* shape) {
  for (size_t ax = 0; ax < D->ndim; ax++) shape[ax] = dim_sizes(D, ax)[coords[ax]];
}
static size_t dense_extent(const ndo_bs_desc* D, size_t ax) {
  size_t s = 0;
  const size_t* z = dim_sizes(D, ax);
  for (size_t i = 0; i < D->nblk[ax]; i++) s += z[i];
  return s;
}
static size_t block_start(const ndo_bs_desc* D, size_t ax, size_t coord) {
  size_t s = 0;
  const size_t* z = dim_sizes(D, ax);
  for (size_t i = 0; i < coord; i++) s += z[i];
  return s;
}
static int coords_valid(const ndo_bs_desc* D) {
  for (size_t b = 0; b < D->nnzb; b++)
    for (size_t ax = 0; ax < D->ndim; ax++)
      if (D->coords[b * D->ndim + ax] >= D->nblk[ax]) return 0;
  return 1;
}
/* BlockOffsets::from_blocks (block_offsets.rs:76-90): packed in listed order */
static void packed_offsets(const ndo_bs_desc* D, size_t* off) {
  size_t o = 0;
  for (size_t b = 0; b < D->nnzb; b++) {
    off[b] = o;
    o += block_elems(D, D->coords + b * D->ndim);
  }
}

static int lex_cmp(const size_t* x, const size_t* y, size_t n) {
  for (size_t i = 0; i < n; i++) {
    if (x[i] < y[i]) return -1;
    if (x[i] > y[i]) return 1;
  }
  return 0;
}

typedef struct {
  size_t ndim;
  size_t nblk[2 * MAXR + 1];
  size_t* bsz; /* malloc'd */
  size_t nnzb;
  size_t* coords; /* malloc'd, sorted */
  size_t* pair_a; /* per pair: A block index */
  size_t* pair_b;
  size_t* pair_out; /* per pair: output block index */
  size_t npairs;
  props_t P;
} bs_plan_t;

static void bs_plan_free(bs_plan_t* pl) {
  free(pl->bsz);
  free(pl->coords);
  free(pl->pair_a);
  free(pl->pair_b);
  free(pl->pair_out);
}

/* contract/blocksparse.rs:87-141, :186-275 */
static int bs_plan(const ndo_bs_desc* A, const int32_t* la, size_t nla,
                   const ndo_bs_desc* B, const int32_t* lb, size_t nlb, bs_plan_t* pl) {
  memset(pl, 0, sizeof(*pl));
  if (nla != A->ndim) return NDO_ERR_WRONG_NUM_INDICES;
  if (nlb != B->ndim) return NDO_ERR_WRONG_NUM_INDICES;
  if (A->ndim > MAXR || B->ndim > MAXR) return NDO_PANIC;
  if (!coords_valid(A) || !coords_valid(B)) return NDO_PANIC;
  size_t sa[MAXR], sb[MAXR];
  for (size_t i = 0; i < A->ndim; i++) sa[i] = dense_extent(A, i);
  for (size_t j = 0; j < B->ndim; j++) sb[j] = dense_extent(B, j);
  compute_props(la, sa, A->ndim, lb, sb, B->ndim, &pl->P);
  props_t* P = &pl->P;
  for (size_t p = 0; p < P->np; p++) {
    size_t ia = P->pa[p], ib = P->pb[p];
    if (A->nblk[ia] != B->nblk[ib]) return NDO_ERR_SHAPE_MISMATCH;
    const size_t* za = dim_sizes(A, ia);
    const size_t* zb = dim_sizes(B, ib);
    for (size_t q = 0; q < A->nblk[ia]; q++)
      if (za[q] != zb[q]) return NDO_ERR_SHAPE_MISMATCH;
  }
  /* output BlockDims = A free ++ B free, or [BlockDim([1])] */
  size_t nd = 0, nbsz = 0;
  for (size_t i = 0; i < P->nua; i++) nbsz += A->nblk[P->ua[i]];
  for (size_t j = 0; j < P->nub; j++) nbsz += B->nblk[P->ub[j]];
  pl->bsz = (size_t*)malloc((nbsz + 1) * sizeof(size_t));
  nbsz = 0;
  for (size_t i = 0; i < P->nua; i++) {
    size_t ax = P->ua[i];
    pl->nblk[nd++] = A->nblk[ax];
    memcpy(pl->bsz + nbsz, dim_sizes(A, ax), A->nblk[ax] * sizeof(size_t));
    nbsz += A->nblk[ax];
  }
  for (size_t j = 0; j < P->nub; j++) {
    size_t ax = P->ub[j];
    pl->nblk[nd++] = B->nblk[ax];
    memcpy(pl->bsz + nbsz, dim_sizes(B, ax), B->nblk[ax] * sizeof(size_t));
    nbsz += B->nblk[ax];
  }
  if (nd == 0) {
    pl->nblk[nd++] = 1;
    pl->bsz[nbsz++] = 1;
  }
  pl->ndim = nd;
  /* pair scan, A blocks outer, B blocks inner (storage order) */
  size_t cap = 16, np = 0;
  size_t* pcoords = (size_t*)malloc(cap * nd * sizeof(size_t));
  pl->pair_a = (size_t*)malloc(cap * sizeof(size_t));
  pl->pair_b = (size_t*)malloc(cap * sizeof(size_t));
  for (size_t ba = 0; ba < A->nnzb; ba++) {
    const size_t* ca = A->coords + ba * A->ndim;
    for (size_t bb = 0; bb < B->nnzb; bb++) {
      const size_t* cb = B->coords + bb * B->ndim;
      int match = 1;
      for (size_t p = 0; p < P->np; p++)
        if (ca[P->pa[p]] != cb[P->pb[p]]) { match = 0; break; }
      if (!match) continue;
      if (np == cap) {
        cap *= 2;
        pcoords = (size_t*)realloc(pcoords, cap * nd * sizeof(size_t));
        pl->pair_a = (size_t*)realloc(pl->pair_a, cap * sizeof(size_t));
        pl->pair_b = (size_t*)realloc(pl->pair_b, cap * sizeof(size_t));
      }
      size_t k = 0;
      for (size_t i = 0; i < P->nua; i++) pcoords[np * nd + k++] = ca[P->ua[i]];
      for (size_t j = 0; j < P->nub; j++) pcoords[np * nd + k++] = cb[P->ub[j]];
      if (k == 0) pcoords[np * nd + k++] = 0;
      pl->pair_a[np] = ba;
      pl->pair_b[np] = bb;
      np++;
    }
  }
  pl->npairs = np;
  /* distinct output blocks, sorted lexicographically (blocksparse.rs:271-272) */
  size_t* order = (size_t*)malloc((np ? np : 1) * sizeof(size_t));
  for (size_t i = 0; i < np; i++) order[i] = i;
  /* insertion sort by coords, stable (small N in tests; merge below for large) */
  /* use a simple bottom-up merge sort to stay O(N log N) */
  size_t* tmp = (size_t*)malloc((np ? np : 1) * sizeof(size_t));
  for (size_t w = 1; w < np; w *= 2) {
    for (size_t lo = 0; lo < np; lo += 2 * w) {
      size_t mid = lo + w < np ? lo + w : np, hi = lo + 2 * w < np ? lo + 2 * w : np;
      size_t i = lo, j = mid, k = lo;
      while (i < mid && j < hi)
        tmp[k++] = lex_cmp(pcoords + order[j] * nd, pcoords + order[i] * nd, nd) < 0 ? order[j++] : order[i++];
      while (i < mid) tmp[k++] = order[i++];
      while (j < hi) tmp[k++] = order[j++];
    }
    memcpy(order, tmp, np * sizeof(size_t));
  }
  free(tmp);
  pl->coords = (size_t*)malloc((np ? np : 1) * nd * sizeof(size_t));
  pl->pair_out = (size_t*)malloc((np ? np : 1) * sizeof(size_t));
  size_t nout = 0;
  for (size_t r = 0; r < np; r++) {
    size_t p = order[r];
    if (nout == 0 || lex_cmp(pl->coords + (nout - 1) * nd, pcoords + p * nd, nd) != 0) {
      memcpy(pl->coords + nout * nd, pcoords + p * nd, nd * sizeof(size_t));
      nout++;
    }
    pl->pair_out[p] = nout - 1;
  }
  pl->nnzb = nout;
  free(order);
  free(pcoords);
  return NDO_OK;
}

int ndo_bs_contract_plan(const ndo_bs_desc* A, const int32_t* la, size_t nla,
                         const ndo_bs_desc* B, const int32_t* lb, size_t nlb,
                         size_t* out_ndim, size_t* out_nblk, size_t* out_bsz,
                         size_t* out_nnzb, size_t* out_coords, size_t* out_total) {
  bs_plan_t pl;
  int st = bs_plan(A, la, nla, B, lb, nlb, &pl);
  if (st != NDO_OK) { bs_plan_free(&pl); return st; }
  *out_ndim = pl.ndim;
  size_t nbsz = 0;
  for (size_t ax = 0; ax < pl.ndim; ax++) {
    out_nblk[ax] = pl.nblk[ax];
    nbsz += pl.nblk[ax];
  }
  memcpy(out_bsz, pl.bsz, nbsz * sizeof(size_t));
  size_t capb = *out_nnzb;
  *out_nnzb = pl.nnzb;
  ndo_bs_desc O = {pl.ndim, pl.nblk, pl.bsz, pl.nnzb, pl.coords};
  size_t tot = 0;
  for (size_t b = 0; b < pl.nnzb; b++) tot += block_elems(&O, pl.coords + b * pl.ndim);
  *out_total = tot;
  if (out_coords) {
    if (capb < pl.nnzb) { bs_plan_free(&pl); return NDO_ERR_CAPACITY; }
    memcpy(out_coords, pl.coords, pl.nnzb * pl.ndim * sizeof(size_t));
  }
  bs_plan_free(&pl);
  return NDO_OK;
}

int ndo_bs_contract_work(const ndo_bs_desc* A, const int32_t* la, size_t nla,
                         const ndo_bs_desc* B, const int32_t* lb, size_t nlb,
                         size_t* npairs, double* mnk_sum) {
  bs_plan_t pl;
  int st = bs_plan(A, la, nla, B, lb, nlb, &pl);
  if (st != NDO_OK) { bs_plan_free(&pl); return st; }
  double s = 0;
  for (size_t p = 0; p < pl.npairs; p++) {
    double ea = (double)block_elems(A, A->coords + pl.pair_a[p] * A->ndim);
    double eb = (double)block_elems(B, B->coords + pl.pair_b[p] * B->ndim);
    /* m*n*k = (|a| / k) * (|b| / k) * k = |a||b| / k */
    double k = 1;
    const size_t* ca = A->coords + pl.pair_a[p] * A->ndim;
    for (size_t q = 0; q < pl.P.np; q++) k *= (double)dim_sizes(A, pl.P.pa[q])[ca[pl.P.pa[q]]];
    s += k > 0 ? ea * eb / k : 0;
  }
  *npairs = pl.npairs;
  *mnk_sum = s;
  bs_plan_free(&pl);
  return NDO_OK;
}

/* contract/blocksparse.rs:144-180 */
int ndo_bs_contract(int dtype, const ndo_bs_desc* A, const void* a_data, const int32_t* la, size_t nla,
                    const ndo_bs_desc* B, const void* b_data, const int32_t* lb, size_t nlb,
                    void* out, size_t out_cap) {
  bs_plan_t pl;
  int st = bs_plan(A, la, nla, B, lb, nlb, &pl);
  if (st != NDO_OK) { bs_plan_free(&pl); return st; }
  size_t es = esize_of(dtype);
  ndo_bs_desc O = {pl.ndim, pl.nblk, pl.bsz, pl.nnzb, pl.coords};
  size_t* ooff = (size_t*)malloc((pl.nnzb + 1) * sizeof(size_t));
  size_t* aoff = (size_t*)malloc((A->nnzb + 1) * sizeof(size_t));
  size_t* boff = (size_t*)malloc((B->nnzb + 1) * sizeof(size_t));
  packed_offsets(&O, ooff);
  packed_offsets(A, aoff);
  packed_offsets(B, boff);
  size_t total = 0;
  for (size_t b = 0; b < pl.nnzb; b++) total += block_elems(&O, pl.coords + b * pl.ndim);
  if (out_cap < total) { st = NDO_ERR_CAPACITY; goto done; }
  memset(out, 0, total * es);
  {
    unsigned char* firstdone = (unsigned char*)calloc(pl.nnzb + 1, 1);
    const unsigned char* Ad = (const unsigned char*)a_data;
    const unsigned char* Bd = (const unsigned char*)b_data;
    unsigned char* Od = (unsigned char*)out;
    for (size_t ob = 0; ob < pl.nnzb && st == NDO_OK; ob++) {
      size_t oshape[2 * MAXR + 1];
      block_shape(&O, pl.coords + ob * pl.ndim, oshape);
      size_t olen = block_elems(&O, pl.coords + ob * pl.ndim);
      for (size_t p = 0; p < pl.npairs && st == NDO_OK; p++) {
        if (pl.pair_out[p] != ob) continue;
        size_t ba = pl.pair_a[p], bb = pl.pair_b[p];
        size_t ash[MAXR], bsh[MAXR];
        block_shape(A, A->coords + ba * A->ndim, ash);
        block_shape(B, B->coords + bb * B->ndim, bsh);
        size_t alen = prod_max1(ash, A->ndim), blen = prod_max1(bsh, B->ndim);
        size_t csh[2 * MAXR + 1], cnd;
        st = ndo_contract_gemm_outshape(ash, A->ndim, la, nla, bsh, B->ndim, lb, nlb, csh, &cnd);
        if (st != NDO_OK) break;
        size_t clen = prod_max1(csh, cnd);
        void* c = malloc(clen * es);
        st = ndo_contract_gemm(dtype, Ad + aoff[ba] * es, alen, ash, A->ndim, la, nla,
                               Bd + boff[bb] * es, blen, bsh, B->ndim, lb, nlb, c, clen);
        if (st == NDO_OK) {
          if (!firstdone[ob]) {
            /* insertblock: shapes must be equal (blocksparse_tensor.rs:218-223) */
            int same = (cnd == pl.ndim);
            for (size_t i = 0; same && i < cnd; i++)
              if (csh[i] != oshape[i]) same = 0;
            if (!same) st = NDO_ERR_SHAPE_MISMATCH;
            else memcpy(Od + ooff[ob] * es, c, olen * es);
            firstdone[ob] = 1;
          } else {
            size_t n = olen < clen ? olen : clen;
            if (dtype == 0) {
              double* d = (double*)(Od + ooff[ob] * es);
              const double* s = (const double*)c;
              for (size_t i = 0; i < n; i++) d[i] = d[i] + s[i];
            } else {
              cplx* d = (cplx*)(Od + ooff[ob] * es);
              const cplx* s = (const cplx*)c;
              for (size_t i = 0; i < n; i++) {
                d[i].re = d[i].re + s[i].re;
                d[i].im = d[i].im + s[i].im;
              }
            }
          }
        }
        free(c);
      }
    }
    free(firstdone);
  }
done:
  free(ooff);
  free(aoff);
  free(boff);
  bs_plan_free(&pl);
  return st;
}

/* operations/blocksparse.rs:61-129 */
int ndo_bs_permutedims(int dtype, const ndo_bs_desc* A, const void* a_data,
                       const size_t* perm, size_t nperm,
                       size_t* out_nblk, size_t* out_bsz, size_t* out_coords, void* out) {
  size_t nd = A->ndim;
  if (nperm != nd) return NDO_ERR_INVALID_PERMUTATION;
  int st = ndo_validate_permutation(perm, nperm, nd);
  if (st != NDO_OK) return st;
  if (!coords_valid(A)) return NDO_PANIC;
  size_t k = 0;
  for (size_t i = 0; i < nd; i++) {
    out_nblk[i] = A->nblk[perm[i]];
    memcpy(out_bsz + k, dim_sizes(A, perm[i]), A->nblk[perm[i]] * sizeof(size_t));
    k += A->nblk[perm[i]];
  }
  size_t nb = A->nnzb;
  size_t* pc = (size_t*)malloc((nb ? nb : 1) * nd * sizeof(size_t));
  for (size_t b = 0; b < nb; b++)
    for (size_t i = 0; i < nd; i++) pc[b * nd + i] = A->coords[b * nd + perm[i]];
  size_t* order = (size_t*)malloc((nb ? nb : 1) * sizeof(size_t));
  for (size_t i = 0; i < nb; i++) order[i] = i;
  for (size_t i = 1; i < nb; i++) {
    size_t v = order[i], j = i;
    while (j > 0 && lex_cmp(pc + order[j - 1] * nd, pc + v * nd, nd) > 0) {
      order[j] = order[j - 1];
      j--;
    }
    order[j] = v;
  }
  for (size_t r = 0; r < nb; r++) memcpy(out_coords + r * nd, pc + order[r] * nd, nd * sizeof(size_t));
  ndo_bs_desc O = {nd, out_nblk, out_bsz, nb, out_coords};
  size_t* ooff = (size_t*)malloc((nb + 1) * sizeof(size_t));
  size_t* aoff = (size_t*)malloc((nb + 1) * sizeof(size_t));
  packed_offsets(&O, ooff);
  packed_offsets(A, aoff);
  size_t es = esize_of(dtype);
  for (size_t r = 0; r < nb && st == NDO_OK; r++) {
    size_t b = order[r];
    size_t sh[MAXR];
    block_shape(A, A->coords + b * nd, sh);
    st = ndo_permutedims(dtype, (const unsigned char*)a_data + aoff[b] * es, sh, nd, perm, nd,
                         (unsigned char*)out + ooff[r] * es);
  }
  free(pc);
  free(order);
  free(ooff);
  free(aoff);
  return st;
}

/* blocksparse_tensor.rs:290-324 */
int ndo_bs_to_dense(int dtype, const ndo_bs_desc* A, const void* a_data, void* dense) {
  size_t nd = A->ndim, es = esize_of(dtype);
  if (nd > MAXR) return NDO_PANIC;
  if (!coords_valid(A)) return NDO_PANIC;
  size_t shape[MAXR] = {0}, strides[MAXR] = {0};
  for (size_t i = 0; i < nd; i++) shape[i] = dense_extent(A, i);
  ndo_compute_strides(shape, nd, strides);
  memset(dense, 0, prod_max1(shape, nd) * es);
  size_t off = 0;
  for (size_t b = 0; b < A->nnzb; b++) {
    const size_t* c = A->coords + b * nd;
    size_t bs[MAXR], st0[MAXR], idx[MAXR];
    block_shape(A, c, bs);
    for (size_t i = 0; i < nd; i++) st0[i] = block_start(A, i, c[i]);
    size_t n = prod(bs, nd);
    for (size_t e = 0; e < n; e++) {
      ndo_linear_to_cartesian(e, bs, nd, idx);
      size_t l = 0;
      for (size_t i = 0; i < nd; i++) l += (st0[i] + idx[i]) * strides[i];
      memcpy((unsigned char*)dense + l * es, (const unsigned char*)a_data + (off + e) * es, es);
    }
    off += n;
  }
  return NDO_OK;
}

/* blocksparse_tensor.rs:353-391 */
int ndo_bs_from_dense(int dtype, const ndo_bs_desc* A, const void* dense, void* out) {
  size_t nd = A->ndim, es = esize_of(dtype);
  if (nd > MAXR) return NDO_PANIC;
  if (!coords_valid(A)) return NDO_PANIC;
  size_t shape[MAXR] = {0}, strides[MAXR] = {0};
  for (size_t i = 0; i < nd; i++) shape[i] = dense_extent(A, i);
  ndo_compute_strides(shape, nd, strides);
  size_t off = 0;
  for (size_t b = 0; b < A->nnzb; b++) {
    const size_t* c = A->coords + b * nd;
    size_t bs[MAXR], st0[MAXR], idx[MAXR];
    block_shape(A, c, bs);
    for (size_t i = 0; i < nd; i++) st0[i] = block_start(A, i, c[i]);
    size_t n = prod(bs, nd);
    for (size_t e = 0; e < n; e++) {
      ndo_linear_to_cartesian(e, bs, nd, idx);
      size_t l = 0;
      for (size_t i = 0; i < nd; i++) l += (st0[i] + idx[i]) * strides[i];
      memcpy((unsigned char*)out + (off + e) * es, (const unsigned char*)dense + l * es, es);
    }
    off += n;
  }
  return NDO_OK;
}

/* diagblocksparse.rs:86 (diag_size = min(block shape)) */
static size_t diag_size(const ndo_bs_desc* S, const size_t* c) {
  size_t m = (size_t)-1;
  for (size_t ax = 0; ax < S->ndim; ax++) {
    size_t z = dim_sizes(S, ax)[c[ax]];
    if (z < m) m = z;
  }
  return S->ndim ? m : 0;
}

size_t ndo_diag_nnz(const ndo_bs_desc* S) {
  size_t t = 0;
  for (size_t b = 0; b < S->nnzb; b++) t += diag_size(S, S->coords + b * S->ndim);
  return t;
}

/* diagblocksparse_tensor.rs:399-426 */
int ndo_diag_to_dense(int dtype, const ndo_bs_desc* S, const void* s_data, void* dense) {
  size_t nd = S->ndim, es = esize_of(dtype);
  if (nd > MAXR) return NDO_PANIC;
  if (!coords_valid(S)) return NDO_PANIC;
  size_t shape[MAXR] = {0}, strides[MAXR] = {0};
  for (size_t i = 0; i < nd; i++) shape[i] = dense_extent(S, i);
  ndo_compute_strides(shape, nd, strides);
  memset(dense, 0, prod_max1(shape, nd) * es);
  size_t off = 0;
  for (size_t b = 0; b < S->nnzb; b++) {
    const size_t* c = S->coords + b * nd;
    size_t ds = diag_size(S, c);
    for (size_t i = 0; i < ds; i++) {
      size_t l = 0;
      for (size_t ax = 0; ax < nd; ax++) l += (block_start(S, ax, c[ax]) + i) * strides[ax];
      memcpy((unsigned char*)dense + l * es, (const unsigned char*)s_data + (off + i) * es, es);
    }
    off += ds;
  }
  return NDO_OK;
}
