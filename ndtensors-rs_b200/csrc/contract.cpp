// Label planning and the dense contraction driver.
//
// Two label semantics exist in the reference and both are reproduced:
//
//  * Naive (crates/ndtensors/src/contract/naive.rs:45-187) is what the C ABI's
//    ndt_tensor_f64_contract runs.  Output axes are A's positive labels (A
//    order) then B's positive labels (B order), never sorted; contracted pairs
//    are negative labels of A matched to the first equal label of B; every
//    other axis is pinned at index 0; a scalar result has shape [1].
//  * Gemm (contract/gemm.rs:47-236 with properties.rs:94-203) is the TTGT form
//    used per block pair by the block-sparse contraction.  Every non-paired
//    axis is free, and the output is sorted by label (perm_c).
//
// Both lower to one primitive: C[M..., N...] = sum_K A(M, K) B(K, N) with
// arbitrary (extent, stride) lists.  When the M/K (K/N) axes of an operand
// collapse to a strided matrix with a unit stride the DMMA GEMM reads the
// tensor in place (the "permute" is free); otherwise the operand is packed
// once by the gather kernel (permute.cu) into the layout the GEMM reads.
#include <algorithm>
#include <map>

#include "ndt_internal.h"

namespace ndt {

namespace {

using Ax1 = StridedAxis;
using AxK = ContractedAxis;

struct Merged {
  bool ok = true;
  bool empty = true;
  int64_t stride = 1;
  int64_t extent = 1;
};

// Collapse an ordered (fastest first) list of axes into one strided axis.
Merged merge_axes(const std::vector<Ax1>& v) {
  Merged m;
  for (const Ax1& a : v) {
    if (a.n == 1) continue;
    if (m.empty) {
      m.empty = false;
      m.stride = a.s;
      m.extent = a.n;
      continue;
    }
    if (a.s != m.stride * m.extent) m.ok = false;
    m.extent *= a.n;
  }
  return m;
}

struct Operand {
  const void* ptr = nullptr;
  int64_t ld = 1;
  bool kmajor = false;
  void* owned = nullptr;  // packed copy (freed after the GEMM)
};

// Express an operand whose element (r, c) sits at sum(r_digits * rs) +
// sum(c_digits * cs) as a GEMM operand.  For A, rows are M and cols are K
// (MN-major = rows contiguous); for B, rows are K and cols are N (K-major =
// rows contiguous).  `mn_first` tells which of rows/cols is the MN index.
Operand make_operand(DType dt, const void* base, const std::vector<Ax1>& mn, const std::vector<Ax1>& kk,
                     int64_t mn_ext, int64_t k_ext, cudaStream_t s) {
  Operand op;
  Merged M = merge_axes(mn), K = merge_axes(kk);
  const bool m_unit = M.empty || M.stride == 1;
  const bool k_unit = K.empty || K.stride == 1;
  if (M.ok && K.ok && m_unit && (!K.empty ? true : true)) {
    // MN-major: element (i, l) at i + l * ld
    op.ptr = base;
    op.kmajor = false;
    op.ld = K.empty ? std::max<int64_t>(mn_ext, 1) : K.stride;
    if (M.empty || K.empty || K.stride >= 1) return op;
  }
  if (M.ok && K.ok && k_unit) {
    op.ptr = base;
    op.kmajor = true;
    op.ld = M.empty ? std::max<int64_t>(k_ext, 1) : M.stride;
    return op;
  }
  // Pack: choose the layout whose fastest axis is the group holding the
  // operand's smallest stride (a cheaper transpose for the gather kernel).
  int64_t smin_mn = INT64_MAX, smin_k = INT64_MAX;
  for (const Ax1& a : mn)
    if (a.n > 1 && a.s > 0) smin_mn = std::min(smin_mn, a.s);
  for (const Ax1& a : kk)
    if (a.n > 1 && a.s > 0) smin_k = std::min(smin_k, a.s);
  bool kmajor = smin_k < smin_mn;
  GatherDesc g;
  const std::vector<Ax1>& first = kmajor ? kk : mn;
  const std::vector<Ax1>& second = kmajor ? mn : kk;
  for (const Ax1& a : first) {
    g.shape.push_back((size_t)a.n);
    g.src_strides.push_back(a.s);
  }
  for (const Ax1& a : second) {
    g.shape.push_back((size_t)a.n);
    g.src_strides.push_back(a.s);
  }
  size_t elems = (size_t)std::max<int64_t>(1, mn_ext * k_ext);
  int dev = current_device();
  op.owned = dev_alloc(elems * esize(dt), dev);
  if (g.shape.empty()) {
    NDT_CUDA(cudaMemcpyAsync(op.owned, base, esize(dt), cudaMemcpyDeviceToDevice, s));
  } else {
    gather(dt, base, op.owned, g, s);
  }
  op.ptr = op.owned;
  op.kmajor = kmajor;
  op.ld = kmajor ? std::max<int64_t>(k_ext, 1) : std::max<int64_t>(mn_ext, 1);
  return op;
}

// C (dense [M..., N...]) = sum_K A B on the device.
void strided_contract(DType dt, const void* A, const void* B, void* C, const std::vector<Ax1>& M,
                      const std::vector<Ax1>& N, const std::vector<AxK>& K, cudaStream_t s) {
  int64_t m = 1, n = 1, k = 1;
  for (const Ax1& a : M) m *= a.n;
  for (const Ax1& a : N) n *= a.n;
  for (const AxK& a : K) k *= a.n;
  if (skinny_contract(dt, A, B, C, M, N, K, s)) return;
  std::vector<Ax1> ka, kb;
  for (const AxK& a : K) {
    ka.push_back({a.n, a.sa});
    kb.push_back({a.n, a.sb});
  }
  int dev = current_device();
  Operand oa = make_operand(dt, A, M, ka, m, k, s);
  Operand ob = make_operand(dt, B, N, kb, n, k, s);
  // make_operand describes B as (N rows, K cols): "kmajor" there means K is
  // the contiguous index, which is the GEMM's K-major B.
  GemmOperand ga{oa.ptr, oa.ld, oa.kmajor};
  GemmOperand gb{ob.ptr, ob.ld, ob.kmajor};
  gemm(dt, m, n, k, ga, gb, C, std::max<int64_t>(m, 1), false, s);
  if (oa.owned) dev_free(oa.owned, dev);
  if (ob.owned) dev_free(ob.owned, dev);
}

bool has_zero(const std::vector<size_t>& v) {
  for (size_t x : v)
    if (x == 0) return true;
  return false;
}

}  // namespace

// ------------------------------------------------------------------ naive
static Dense contract_naive(const Dense& a, const std::vector<int32_t>& la, const Dense& b,
                            const std::vector<int32_t>& lb) {
  // naive.rs:51-63
  if (la.size() != a.ndim()) throw Error(ErrKind::WrongNumberOfIndices, "labels_a length != ndim(a)");
  if (lb.size() != b.ndim()) throw Error(ErrKind::WrongNumberOfIndices, "labels_b length != ndim(b)");
  const size_t na = a.ndim(), nb = b.ndim();
  // naive.rs:66-83: pairs, first match in B, sizes checked
  std::vector<std::pair<size_t, size_t>> pairs;
  for (size_t i = 0; i < na; i++) {
    if (la[i] >= 0) continue;
    for (size_t j = 0; j < nb; j++) {
      if (la[i] == lb[j]) {
        if (a.shape[i] != b.shape[j]) throw Error(ErrKind::ShapeMismatch, "contracted extents differ");
        pairs.push_back({i, j});
        break;
      }
    }
  }
  std::vector<size_t> out_shape, cdims;
  for (size_t i = 0; i < na; i++)
    if (la[i] > 0) out_shape.push_back(a.shape[i]);
  for (size_t j = 0; j < nb; j++)
    if (lb[j] > 0) out_shape.push_back(b.shape[j]);
  if (out_shape.empty()) out_shape.push_back(1);
  for (auto& p : pairs) cdims.push_back(a.shape[p.first]);
  // The reference divides by every output and contracted extent
  // (strides.rs:64-73 inside its loops), so zero extents panic.
  if (has_zero(out_shape) || has_zero(cdims))
    throw Error(ErrKind::Panic, "zero extent in an output or contracted axis");
  std::vector<size_t> sa = col_major_strides(a.shape), sb = col_major_strides(b.shape);
  // Driving pair of each axis (first pair naming it) or pinned at 0.
  std::vector<long> cpa(na, -1), cpb(nb, -1);
  for (size_t p = 0; p < pairs.size(); p++) {
    if (cpa[pairs[p].first] < 0) cpa[pairs[p].first] = (long)p;
    if (cpb[pairs[p].second] < 0) cpb[pairs[p].second] = (long)p;
  }
  std::vector<Ax1> M, N;
  std::vector<AxK> K(pairs.size());
  int64_t maxa = 0, maxb = 0;
  for (size_t i = 0; i < na; i++) {
    if (la[i] > 0) {
      M.push_back({(int64_t)a.shape[i], (int64_t)sa[i]});
      maxa += (int64_t)(a.shape[i] - 1) * (int64_t)sa[i];
    }
  }
  for (size_t j = 0; j < nb; j++) {
    if (lb[j] > 0) {
      N.push_back({(int64_t)b.shape[j], (int64_t)sb[j]});
      maxb += (int64_t)(b.shape[j] - 1) * (int64_t)sb[j];
    }
  }
  for (size_t p = 0; p < pairs.size(); p++) {
    size_t i = pairs[p].first, j = pairs[p].second;
    K[p].n = (int64_t)a.shape[i];
    K[p].sa = (cpa[i] == (long)p) ? (int64_t)sa[i] : 0;
    K[p].sb = (cpb[j] == (long)p) ? (int64_t)sb[j] : 0;
    maxa += (K[p].n - 1) * K[p].sa;
    maxb += (K[p].n - 1) * K[p].sb;
  }
  // get_linear(..).unwrap() panics when an index leaves the storage
  if (maxa >= (int64_t)a.len() || maxb >= (int64_t)b.len())
    throw Error(ErrKind::Panic, "contraction index outside the tensor's storage");
  Dense out = make_empty_device(a.dt, out_shape);
  const void* pa = a.st->dev_read();
  const void* pb = b.st->dev_read();
  strided_contract(a.dt, pa, pb, out.st->dev, M, N, K, ctx().compute);
  return out;
}

// ------------------------------------------------------------------- gemm
static void validate_perm_like_permutedims(const std::vector<size_t>& perm, size_t ndim) {
  if (perm.size() != ndim) throw Error(ErrKind::InvalidPermutation, "invalid permutation");
  std::vector<char> seen(ndim, 0);
  for (size_t p : perm) {
    if (p >= ndim || seen[p]) throw Error(ErrKind::InvalidPermutation, "invalid permutation");
    seen[p] = 1;
  }
}

// A sub-range [lo, hi) of one free axis of one operand (0: A, 1: B): the
// contraction then produces the matching slab of C.  The operand is read in
// place through its own strides (base moved by lo along the axis).
struct Slab {
  int operand;
  size_t axis, lo, hi;
};

static Dense contract_gemm_sem(const Dense& a, const std::vector<int32_t>& la, const Dense& b,
                               const std::vector<int32_t>& lb, const Slab* slab = nullptr) {
  const size_t na = a.ndim(), nb = b.ndim();
  // gemm.rs:54-79
  if (la.size() != na) throw Error(ErrKind::WrongNumberOfIndices, "labels_a length != ndim(a)");
  if (lb.size() != nb) throw Error(ErrKind::WrongNumberOfIndices, "labels_b length != ndim(b)");
  for (size_t i = 0; i < na; i++)
    if (la[i] < 0)
      for (size_t j = 0; j < nb; j++)
        if (la[i] == lb[j] && a.shape[i] != b.shape[j])
          throw Error(ErrKind::ShapeMismatch, "contracted extents differ");
  // properties.rs:100-122
  std::vector<size_t> pa_, pb_, ua, ub;
  for (size_t i = 0; i < na; i++) {
    if (la[i] >= 0) continue;
    for (size_t j = 0; j < nb; j++)
      if (la[i] == lb[j]) {
        pa_.push_back(i);
        pb_.push_back(j);
        break;
      }
  }
  for (size_t i = 0; i < na; i++)
    if (std::find(pa_.begin(), pa_.end(), i) == pa_.end()) ua.push_back(i);
  for (size_t j = 0; j < nb; j++)
    if (std::find(pb_.begin(), pb_.end(), j) == pb_.end()) ub.push_back(j);
  // perm_a / perm_b (properties.rs:141-158); permutedims validates them
  std::vector<size_t> perm_a(ua), perm_b(pb_);
  perm_a.insert(perm_a.end(), pa_.begin(), pa_.end());
  perm_b.insert(perm_b.end(), ub.begin(), ub.end());
  auto is_id = [](const std::vector<size_t>& p) {
    for (size_t i = 0; i < p.size(); i++)
      if (p[i] != i) return false;
    return true;
  };
  const bool full = ua.empty() && ub.empty();
  const bool outer = pa_.empty();
  if (full || !outer) {
    if (!is_id(perm_a)) {
      validate_perm_like_permutedims(perm_a, na);
      if (has_zero(a.shape)) throw Error(ErrKind::Panic, "permutedims of a zero extent");
    }
    if (!is_id(perm_b)) {
      validate_perm_like_permutedims(perm_b, nb);
      if (has_zero(b.shape)) throw Error(ErrKind::Panic, "permutedims of a zero extent");
    }
  }
  // output labels and perm_c (properties.rs:160-186, stable argsort)
  std::vector<int32_t> olab;
  std::vector<size_t> oshape;
  for (size_t i : ua) {
    olab.push_back(la[i]);
    oshape.push_back(a.shape[i]);
  }
  for (size_t j : ub) {
    olab.push_back(lb[j]);
    oshape.push_back(b.shape[j]);
  }
  std::vector<size_t> perm_c(olab.size());
  for (size_t i = 0; i < perm_c.size(); i++) perm_c[i] = i;
  std::stable_sort(perm_c.begin(), perm_c.end(), [&](size_t x, size_t y) { return olab[x] < olab[y]; });
  bool permute_c = false;
  for (size_t i = 0; i < perm_c.size(); i++)
    if (olab[perm_c[i]] != olab[i]) permute_c = true;

  std::vector<size_t> sa = col_major_strides(a.shape), sb = col_major_strides(b.shape);
  // the operands' extents as read (a slab narrows one free axis) and the
  // element offset of each operand's first element read
  std::vector<size_t> ash(a.shape), bsh(b.shape);
  size_t a0 = 0, b0 = 0, alen = a.len(), blen = b.len();
  if (slab) {
    std::vector<size_t>& sh = slab->operand == 0 ? ash : bsh;
    sh[slab->axis] = slab->hi - slab->lo;
    (slab->operand == 0 ? a0 : b0) = slab->lo * (slab->operand == 0 ? sa : sb)[slab->axis];
    (slab->operand == 0 ? alen : blen) = prod_max1(sh);
    for (size_t i = 0; i < ua.size(); i++) oshape[i] = ash[ua[i]];
    for (size_t j = 0; j < ub.size(); j++) oshape[ua.size() + j] = bsh[ub[j]];
  }
  std::vector<Ax1> M, N;
  std::vector<AxK> K;
  for (size_t i : ua) M.push_back({(int64_t)ash[i], (int64_t)sa[i]});
  for (size_t j : ub) N.push_back({(int64_t)bsh[j], (int64_t)sb[j]});
  for (size_t p = 0; p < pa_.size(); p++)
    K.push_back({(int64_t)a.shape[pa_[p]], (int64_t)sa[pa_[p]], (int64_t)sb[pb_[p]]});
  size_t m = std::max<size_t>(1, prod(std::vector<size_t>(oshape.begin(), oshape.begin() + ua.size())));
  size_t n = std::max<size_t>(1, prod(std::vector<size_t>(oshape.begin() + ua.size(), oshape.end())));
  size_t kk = 1;
  for (size_t p : pa_) kk *= a.shape[p];
  kk = std::max<size_t>(kk, 1);
  const size_t es = esize(a.dt);
  const void* ap = (const char*)a.st->dev_read() + a0 * es;
  const void* bp = (const char*)b.st->dev_read() + b0 * es;
  if (full) {
    // contract_full (gemm.rs:98-125): dot product -> shape [1]
    Dense out = make_empty_device(a.dt, {1});
    strided_contract(a.dt, ap, bp, out.st->dev, {}, {}, K, ctx().compute);
    return out;
  }
  // as_faer_mat asserts rows*cols == len (faer_interop.rs:72-84)
  if (outer) {
    if (m != alen || n != blen) throw Error(ErrKind::Panic, "matrix view size mismatch");
  } else {
    if (m * kk != alen || kk * n != blen) throw Error(ErrKind::Panic, "matrix view size mismatch");
  }
  std::vector<size_t> shape_unsorted = oshape;
  if (shape_unsorted.empty()) shape_unsorted.push_back(1);
  if (m * n != prod_max1(shape_unsorted)) throw Error(ErrKind::ShapeMismatch, "output length mismatch");
  Dense c = make_empty_device(a.dt, shape_unsorted);
  strided_contract(a.dt, ap, bp, c.st->dev, M, N, K, ctx().compute);
  if (!permute_c) return c;
  return permutedims(c, perm_c);
}

// contract_gemm split along a free index (the dense multi-GPU scheme: no
// reduction, each rank owns a slab of C).  The free axis labelled
// `axis_label` (in A or in B, once) is cut into nranks near-equal ranges;
// rank r contracts its range [N r / nranks, N (r + 1) / nranks) and returns
// that slab of C (same label order as contract_gemm's result, the split axis
// narrowed).  A rank whose range is empty gets a zero tensor of the slab's
// shape.
Dense contract_gemm_shard(const Dense& a, const std::vector<int32_t>& la, const Dense& b,
                          const std::vector<int32_t>& lb, int32_t axis_label, int rank, int nranks) {
  if (a.dt != b.dt) throw Error(ErrKind::InvalidArgument, "element types differ");
  if (nranks < 1 || rank < 0 || rank >= nranks) throw Error(ErrKind::InvalidArgument, "need 0 <= rank < nranks");
  if (axis_label <= 0) throw Error(ErrKind::InvalidArgument, "the split label must be a positive (free) label");
  if (la.size() != a.ndim()) throw Error(ErrKind::WrongNumberOfIndices, "labels_a length != ndim(a)");
  if (lb.size() != b.ndim()) throw Error(ErrKind::WrongNumberOfIndices, "labels_b length != ndim(b)");
  Slab sl{-1, 0, 0, 0};
  int hits = 0;
  for (size_t i = 0; i < la.size(); i++)
    if (la[i] == axis_label) sl = Slab{0, i, 0, 0}, hits++;
  for (size_t j = 0; j < lb.size(); j++)
    if (lb[j] == axis_label) sl = Slab{1, j, 0, 0}, hits++;
  if (hits != 1) throw Error(ErrKind::InvalidArgument, "the split label must label exactly one axis of A or B");
  const size_t ext = (sl.operand == 0 ? a.shape : b.shape)[sl.axis];
  sl.lo = ext * (size_t)rank / (size_t)nranks;
  sl.hi = ext * (size_t)(rank + 1) / (size_t)nranks;
  if (sl.hi == sl.lo) {
    // An empty range: a zero tensor of the slab's shape.  Output axes as
    // contract_gemm orders them (properties.rs:100-186): the unpaired axes
    // of A, then of B, stably sorted by label.
    std::vector<char> paired_a(la.size(), 0), paired_b(lb.size(), 0);
    for (size_t i = 0; i < la.size(); i++) {
      if (la[i] >= 0) continue;
      for (size_t j = 0; j < lb.size(); j++)
        if (la[i] == lb[j]) {
          paired_a[i] = 1;
          paired_b[j] = 1;
          break;
        }
    }
    std::vector<std::pair<int32_t, size_t>> out;  // (label, extent)
    for (size_t i = 0; i < la.size(); i++)
      if (!paired_a[i]) out.push_back({la[i], a.shape[i]});
    for (size_t j = 0; j < lb.size(); j++)
      if (!paired_b[j]) out.push_back({lb[j], b.shape[j]});
    std::stable_sort(out.begin(), out.end(), [](const auto& x, const auto& y) { return x.first < y.first; });
    std::vector<size_t> shape;
    for (auto& o : out) shape.push_back(o.first == axis_label ? 0 : o.second);
    if (shape.empty()) shape.push_back(1);
    return make_uniform(a.dt, shape, 0.0, 0.0);
  }
  return contract_gemm_sem(a, la, b, lb, &sl);
}

Dense contract(const Dense& a, const std::vector<int32_t>& la, const Dense& b, const std::vector<int32_t>& lb,
               ContractSemantics sem) {
  if (a.dt != b.dt) throw Error(ErrKind::InvalidArgument, "element types differ");
  return sem == ContractSemantics::Naive ? contract_naive(a, la, b, lb) : contract_gemm_sem(a, la, b, lb);
}

// apply_binary(+) (operations/elementwise.rs:189-210)
Dense add(const Dense& a, const Dense& b) {
  if (a.shape != b.shape) throw Error(ErrKind::ShapeMismatch, "shapes differ");
  Dense out = make_empty_device(a.dt, a.shape);
  size_t n = std::min(a.len(), b.len());
  add_device(a.dt, a.st->dev_read(), b.st->dev_read(), out.st->dev, n, ctx().compute);
  return out;
}

// contract_vjp (contract/naive.rs:222-511), composed from the device
// contraction and permutedims exactly as the reference composes it.
void contract_vjp(const Dense& a, const std::vector<int32_t>& la, const Dense& b, const std::vector<int32_t>& lb,
                  const Dense& grad, Dense* ga, Dense* gb) {
  if (la.size() != a.ndim()) throw Error(ErrKind::WrongNumberOfIndices, "labels_a length != ndim(a)");
  if (lb.size() != b.ndim()) throw Error(ErrKind::WrongNumberOfIndices, "labels_b length != ndim(b)");
  int32_t max_label = 0;
  for (int32_t l : la) max_label = std::max(max_label, l < 0 ? -l : l);
  for (int32_t l : lb) max_label = std::max(max_label, l < 0 ? -l : l);
  bool a_pos = false, b_pos = false;
  for (int32_t l : la) a_pos |= l > 0;
  for (int32_t l : lb) b_pos |= l > 0;
  const bool scalar_out = !a_pos && !b_pos;

  auto scaled = [&](const Dense& src, double re, double im) {
    Dense out = make_empty_device(src.dt, src.shape);
    scale_device(src.dt, src.st->dev_read(), out.st->dev, src.len(), re, im, ctx().compute);
    return out;
  };
  auto grad_scalar = [&](double* re, double* im) {
    if (grad.len() < 1) throw Error(ErrKind::IndexOutOfBounds, "grad_output is empty");
    const double* h = (const double*)grad.st->host_read();
    *re = h[0];
    *im = grad.dt == DType::C128 ? h[1] : 0.0;
  };
  // reshape of a scaled tensor to another shape (Tensor::from_vec length check)
  auto reshaped = [&](Dense t, const std::vector<size_t>& shape) {
    if (prod_max1(shape) != t.len()) throw Error(ErrKind::ShapeMismatch, "reshape length mismatch");
    t.shape = shape;
    return t;
  };

  // ---- grad_a
  if (scalar_out) {
    double re, im;
    grad_scalar(&re, &im);
    Dense r = scaled(b, re, im);
    std::map<int32_t, size_t> b_idx;
    for (size_t i = 0; i < lb.size(); i++) b_idx[lb[i]] = i;  // later entries win
    std::vector<size_t> perm;
    for (int32_t l : la) {
      auto it = b_idx.find(l);
      if (it == b_idx.end()) throw Error(ErrKind::Panic, "label not found in B");
      perm.push_back(it->second);
    }
    bool id = true;
    for (size_t i = 0; i < perm.size(); i++) id &= perm[i] == i;
    *ga = id ? reshaped(r, a.shape) : permutedims(r, perm);
  } else {
    int32_t counter = max_label + 1;
    size_t b_pos_count = 0;
    for (int32_t l : lb) b_pos_count += l > 0;
    std::vector<int32_t> gc_labels, b_pos_contract;
    for (int32_t l : la)
      if (l > 0) gc_labels.push_back(l);
    for (size_t q = 0; q < b_pos_count; q++) {
      gc_labels.push_back(-counter);
      b_pos_contract.push_back(-counter);
      counter++;
    }
    std::map<int32_t, int32_t> b_neg_to_pos;
    std::vector<int32_t> b_new;
    size_t bp = 0;
    for (int32_t l : lb) {
      if (l < 0) {
        b_new.push_back(counter);
        b_neg_to_pos[l] = counter;
        counter++;
      } else {
        b_new.push_back(b_pos_contract.at(bp));
        bp++;
      }
    }
    Dense r = contract(grad, gc_labels, b, b_new, ContractSemantics::Naive);
    std::vector<int32_t> order;
    for (int32_t l : la)
      if (l > 0) order.push_back(l);
    for (int32_t l : lb)
      if (l < 0) order.push_back(b_neg_to_pos.at(l));
    std::vector<size_t> perm;
    for (int32_t l : la) {
      int32_t want;
      if (l > 0) {
        want = l;
      } else {
        auto it = b_neg_to_pos.find(l);
        if (it == b_neg_to_pos.end()) throw Error(ErrKind::Panic, "label has no counterpart in B");
        want = it->second;
      }
      auto pos = std::find(order.begin(), order.end(), want);
      if (pos == order.end()) throw Error(ErrKind::Panic, "label not found");
      perm.push_back((size_t)(pos - order.begin()));
    }
    *ga = permutedims(r, perm);
  }
  // ---- grad_b
  if (scalar_out) {
    double re, im;
    grad_scalar(&re, &im);
    Dense r = scaled(a, re, im);
    std::map<int32_t, size_t> a_idx;
    for (size_t i = 0; i < la.size(); i++) a_idx[la[i]] = i;
    std::vector<size_t> perm;
    for (int32_t l : lb) {
      auto it = a_idx.find(l);
      if (it == a_idx.end()) throw Error(ErrKind::Panic, "label not found in A");
      perm.push_back(it->second);
    }
    bool id = true;
    for (size_t i = 0; i < perm.size(); i++) id &= perm[i] == i;
    *gb = id ? reshaped(r, b.shape) : permutedims(r, perm);
  } else {
    int32_t counter = max_label + 1;
    std::map<int32_t, int32_t> a_neg_to_pos;
    std::vector<int32_t> a_new, a_pos_contract;
    for (int32_t l : la) {
      if (l > 0) {
        a_new.push_back(-counter);
        a_pos_contract.push_back(-counter);
        counter++;
      } else {
        a_new.push_back(counter);
        a_neg_to_pos[l] = counter;
        counter++;
      }
    }
    std::vector<int32_t> gc_labels(a_pos_contract);
    for (int32_t l : lb)
      if (l > 0) gc_labels.push_back(l);
    Dense r = contract(a, a_new, grad, gc_labels, ContractSemantics::Naive);
    std::vector<int32_t> order;
    for (int32_t l : la)
      if (l < 0) order.push_back(a_neg_to_pos.at(l));
    for (int32_t l : lb)
      if (l > 0) order.push_back(l);
    std::vector<size_t> perm;
    for (int32_t l : lb) {
      int32_t want;
      if (l > 0) {
        want = l;
      } else {
        auto it = a_neg_to_pos.find(l);
        if (it == a_neg_to_pos.end()) throw Error(ErrKind::Panic, "label has no counterpart in A");
        want = it->second;
      }
      auto pos = std::find(order.begin(), order.end(), want);
      if (pos == order.end()) throw Error(ErrKind::Panic, "label not found");
      perm.push_back((size_t)(pos - order.begin()));
    }
    *gb = permutedims(r, perm);
  }
}

}  // namespace ndt
