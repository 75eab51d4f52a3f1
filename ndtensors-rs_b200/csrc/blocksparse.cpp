// Block-sparse and diag-block-sparse tensors and their contraction.
//
// Storage model of the reference (storage/blocksparse/*, blocksparse_tensor.rs):
// per-axis block sizes (BlockDim), a list of stored blocks packed in the
// order given (BlockOffsets::from_blocks, block_offsets.rs:76-90), each block
// a column-major dense array.  The data lives in device memory.
//
// contract_blocksparse (contract/blocksparse.rs:87-275) becomes:
//   host   validate (label counts, block counts / sizes on contracted axes),
//          match block pairs with a hash join on the contracted coordinates
//          (same pair set and the same (A, B) storage order as the
//          reference's nnzA x nnzB scan), output blocks sorted
//          lexicographically with packed offsets; per output block its
//          pairs form the device-side table of one grouped GEMM launch;
//   device one grouped DMMA launch (gemm.cu): a CTA owns an output tile and
//          accumulates all matched pairs of its block in registers.
// Operand blocks whose axes are not already [free..., contracted...] (A) /
// [contracted..., free...] (B) are permuted block by block first (TTGT).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <unordered_map>

#include "../../include/ndtensors_capi.h"
#include "ndt_comm.h"
#include "ndt_internal.h"

namespace ndt {

// Which rank holds which output block of a sharded contraction: every rank
// derives the same layout, so the shards can be gathered without exchanging
// their structure.
struct ShardLayout {
  int nranks = 1;
  std::vector<std::vector<size_t>> coords;  // all output blocks, sorted
  std::vector<int> owner;                   // rank holding each of them
};

struct BlockSparseT {
  DType dt = DType::F64;
  std::vector<std::vector<size_t>> bsz;     // per-axis block sizes
  std::vector<std::vector<size_t>> coords;  // stored blocks, storage order
  std::vector<size_t> offs;                 // packed offsets, size nnzb + 1
  std::shared_ptr<Storage> st;
  std::shared_ptr<const ShardLayout> layout;  // set on the shards of a sharded contraction

  size_t ndim() const { return bsz.size(); }
  size_t nnzb() const { return coords.size(); }
  size_t total() const { return offs.empty() ? 0 : offs.back(); }
  std::vector<size_t> block_shape(const std::vector<size_t>& c) const {
    std::vector<size_t> s(c.size());
    for (size_t i = 0; i < c.size(); i++) s[i] = bsz[i][c[i]];
    return s;
  }
  size_t block_elems(const std::vector<size_t>& c) const {
    size_t p = 1;
    for (size_t i = 0; i < c.size(); i++) p *= bsz[i][c[i]];
    return p;
  }
  size_t dense_extent(size_t ax) const {
    size_t s = 0;
    for (size_t x : bsz[ax]) s += x;
    return s;
  }
  size_t block_start(size_t ax, size_t c) const {
    size_t s = 0;
    for (size_t i = 0; i < c; i++) s += bsz[ax][i];
    return s;
  }
  void pack() {
    offs.assign(coords.size() + 1, 0);
    for (size_t b = 0; b < coords.size(); b++) offs[b + 1] = offs[b] + block_elems(coords[b]);
  }
  long find(const std::vector<size_t>& c) const {
    for (size_t b = 0; b < coords.size(); b++)
      if (coords[b] == c) return (long)b;
    return -1;
  }
};

struct DiagBlockSparseT {
  BlockSparseT s;  // coords / block sizes; offs are diagonal offsets
  bool real_valued = true;  // complex values with all imaginary parts zero (set on upload)
  size_t diag_size(const std::vector<size_t>& c) const {
    if (c.empty()) return 0;
    size_t m = SIZE_MAX;
    for (size_t i = 0; i < c.size(); i++) m = std::min(m, s.bsz[i][c[i]]);
    return m;
  }
};

namespace {

void check_structure(const std::vector<std::vector<size_t>>& bsz, const std::vector<std::vector<size_t>>& coords) {
  if (bsz.size() > (size_t)kBsMaxRank) throw Error(ErrKind::InvalidArgument, "block-sparse rank above 16");
  std::map<std::vector<size_t>, int> seen;
  for (const auto& c : coords) {
    if (c.size() != bsz.size()) throw Error(ErrKind::InvalidArgument, "block coordinate rank mismatch");
    for (size_t i = 0; i < c.size(); i++)
      if (c[i] >= bsz[i].size()) throw Error(ErrKind::InvalidArgument, "block coordinate out of range");
    if (seen[c]++) throw Error(ErrKind::InvalidArgument, "duplicate block coordinate");
  }
}

BlockSparseT make_bs(DType dt, const std::vector<std::vector<size_t>>& bsz,
                     const std::vector<std::vector<size_t>>& coords) {
  check_structure(bsz, coords);
  BlockSparseT t;
  t.dt = dt;
  t.bsz = bsz;
  t.coords = coords;
  t.pack();
  t.st = std::make_shared<Storage>(dt, t.total());
  t.st->set_uniform(0.0, 0.0);
  return t;
}

// Per-block permute of a packed tensor: block order[r] (shape sh) goes to
// dst + dst_offs[r] with its axes reordered by perm.  Many small blocks go
// in one launch (the block map kernel: each source element, in its block's
// column-major order, lands at its offset in the permuted block); few or
// large blocks go one tiled permute launch each.
void permute_blocks(DType dt, const void* src, void* dst, const BlockSparseT& t, const std::vector<size_t>& perm,
                    const std::vector<size_t>& dst_offs, const std::vector<size_t>& order, cudaStream_t s) {
  if (t.total() == 0) return;
  if (t.nnzb() <= 16 || t.total() / t.nnzb() >= (size_t)1 << 16) {
    const size_t es = esize(dt);
    for (size_t r = 0; r < order.size(); r++) {
      const size_t b = order[r];
      if (t.block_elems(t.coords[b]) == 0) continue;
      const std::vector<size_t> sh = t.block_shape(t.coords[b]);
      const std::vector<size_t> st = col_major_strides(sh);
      GatherDesc g;
      for (size_t i = 0; i < perm.size(); i++) {
        g.shape.push_back(sh[perm[i]]);
        g.src_strides.push_back((int64_t)st[perm[i]]);
      }
      const char* sp = (const char*)src + t.offs[b] * es;
      char* dp = (char*)dst + dst_offs[r] * es;
      if (g.shape.empty())
        NDT_CUDA(cudaMemcpyAsync(dp, sp, es, cudaMemcpyDeviceToDevice, s));
      else
        gather(dt, sp, dp, g, s);
    }
    return;
  }
  std::vector<int64_t> dst_base(t.nnzb(), 0);
  for (size_t r = 0; r < order.size(); r++) dst_base[order[r]] = (int64_t)dst_offs[r];
  std::vector<int64_t> offs(t.nnzb());
  std::vector<BsBlockDesc> desc(t.nnzb());
  for (size_t b = 0; b < t.nnzb(); b++) {
    offs[b] = (int64_t)t.offs[b];
    const std::vector<size_t> sh = t.block_shape(t.coords[b]);
    std::vector<size_t> psh(perm.size());
    for (size_t i = 0; i < perm.size(); i++) psh[i] = sh[perm[i]];
    const std::vector<size_t> ps = col_major_strides(psh);
    BsBlockDesc& d = desc[b];
    memset(&d, 0, sizeof(d));
    d.ndim = (int32_t)sh.size();
    for (size_t i = 0; i < sh.size(); i++) d.shape[i] = (int64_t)sh[i];
    for (size_t i = 0; i < perm.size(); i++) d.dstride[perm[i]] = (int64_t)ps[i];
    d.dense_base = dst_base[b];
  }
  bs_dense_map(dt, const_cast<void*>(src), dst, offs, desc, (int64_t)t.total(), true, s);
}

bool is_prefix_run(const std::vector<size_t>& v, size_t start) {
  for (size_t i = 0; i < v.size(); i++)
    if (v[i] != start + i) return false;
  return true;
}

// The GEMM index over `axes` (that order, the first fastest) of a block with
// extents `ext` and strides `str`, merged into strided runs (extent-1 axes
// dropped, an axis continuing the previous run joins it).  False when it
// takes more than two runs.
bool index_runs(const std::vector<size_t>& axes, const std::vector<int64_t>& ext, const std::vector<int64_t>& str,
                IndexRuns* out) {
  std::vector<std::pair<int64_t, int64_t>> runs;  // (extent, stride)
  for (size_t a : axes) {
    if (ext[a] == 1) continue;
    if (!runs.empty() && runs.back().first * runs.back().second == str[a])
      runs.back().first *= ext[a];
    else
      runs.push_back({ext[a], str[a]});
  }
  if (runs.size() > 2) return false;
  out->pad = 0;
  out->e0 = 0x7fffffffu;  // one run (or none): every index is below it
  out->s0 = runs.empty() ? 0 : runs[0].second;
  out->s1 = 0;
  if (runs.size() == 2) {
    out->e0 = (uint32_t)runs[0].first;
    out->s1 = runs[1].second;
  }
  return true;
}

// Column-major strides of a block with extents `ext`.
std::vector<int64_t> block_strides(const std::vector<int64_t>& ext) {
  std::vector<int64_t> st(ext.size());
  int64_t s = 1;
  for (size_t i = 0; i < ext.size(); i++) {
    st[i] = s;
    s *= ext[i];
  }
  return st;
}

}  // namespace

// contract_blocksparse (contract/blocksparse.rs:87-183).  With nranks > 1 only
// this rank's output blocks are computed (and stored): output blocks go to
// ranks by longest processing time first on their tensor-core tile cost
// (costliest block to the least loaded rank, ties to the lower rank), so the
// per-rank costs differ by at most one block's.  Every rank derives the same
// assignment from the same operands.
struct ShardPlan {
  std::vector<size_t> blocks;  // output blocks per rank
  std::vector<double> flops;   // real flop per rank
};

// A rank-2 diagonal operand S between A and B, contracted with A's axis
// `a_axis` on one side and with B on the other: S block (q_a, q_b) maps A's
// coordinate q_a on that axis to B's coordinate q_b, and its diagonal starts
// at `off` in S's packed values.  The grouped GEMM applies those values to
// the contracted index as it loads its operands (to B's fragments in shared
// memory), so A . S is never formed.
struct ThroughDiag {
  size_t a_axis = 0;
  std::map<size_t, std::pair<size_t, int64_t>> qmap;  // q_a -> (q_b, off)
  const void* sdata = nullptr;
  bool real = false;  // every diagonal value real (one multiply per component)
};

// Gathered contractions where the ranks cannot write into each other's
// memory (more than kMaxSymRanks ranks, or no CUDA IPC): each rank's output
// blocks (by descending tile cost) are dealt round-robin into this many
// chunks, and chunk c's NCCL all-gather may run while chunk c + 1 computes,
// on SMs that chunk's launch leaves free.  Measured on two B200s (c128 MPS
// chain, bond 8192): one chunk and no reserved SMs is fastest (1.03 ms; two
// chunks 1.07, three chunks with 8 or 16 reserved SMs 1.17 / 1.20): NCCL's
// kernels gain little beside a persistent GEMM that fills every SM.
constexpr int kGatherChunks = 1;
constexpr int kGatherSmReserve = 0;

// Host plan of one block-sparse contraction: everything contract_blocksparse
// derives from the operands' structures and labels (the pair join, the output
// structure and its owners, operand layouts, the grouped launches' tables,
// the transfers of a gathered contraction).  Plans are cached by that
// structure, so repeated contractions of one structure (a sweep over a tensor
// network, a benchmark loop) pay no host planning: one lookup, the launch.
struct PlannedLaunch {
  std::vector<GroupedProblem> probs;
  std::vector<GroupedSegment> segs;
  // strided plans: the index runs of every problem and segment
  std::vector<StridedProblem> sprobs;
  std::vector<StridedSegment> ssegs;
  // gathered mode: this chunk's region of the staging buffer (elements):
  // rank r's blocks of the chunk, packed, at stage_off + r * pad
  size_t stage_off = 0, pad = 0;
};
struct ContractPlan {
  BlockSparseT c;  // output structure (no storage)
  bool zero = false;        // nothing to compute: the output is all zeros
  bool a_kmajor = false, b_kmajor = true;
  bool pack_a = false, pack_b = false;  // operand blocks permuted to [free, contracted] first
  std::vector<size_t> perm_a, perm_b;
  // the GEMM reads A and B and writes C through index runs (no pack, no
  // output permute) instead of packing and permuting
  bool strided = false;
  bool permute_c = false;
  std::vector<size_t> perm_c;
  bool has_td = false;
  std::vector<PlannedLaunch> launches;
  // gathered mode: staging size (elements) and the copy that moves every
  // block from its staging place to its place in the sorted output (bytes)
  size_t stage_total = 0;
  std::vector<int64_t> copy_src, copy_dst, copy_bytes;
  // gathered mode, ranks mapping each other's memory: this rank's blocks at
  // their places in the sorted output, computed once and stored to every rank
  PlannedLaunch direct;
  // ... and the other ranks' blocks (byte ranges, adjacent blocks merged),
  // copied from the mapped buffer into the result once they have arrived
  std::vector<int64_t> peer_off, peer_bytes;
};

namespace {

std::mutex g_bsplan_mu;
std::map<std::vector<int64_t>, std::pair<std::shared_ptr<const ContractPlan>, uint64_t>> g_bsplans;
uint64_t g_bsplan_tick = 0;
constexpr size_t kBsPlanCacheSize = 64;

void key_push(std::vector<int64_t>& k, const std::vector<std::vector<size_t>>& vv) {
  k.push_back((int64_t)vv.size());
  for (const auto& v : vv) {
    k.push_back((int64_t)v.size());
    for (size_t x : v) k.push_back((int64_t)x);
  }
}

}  // namespace

// `select` (nsel output coordinates of rank |ua| + |ub|, natural order):
// compute only those output blocks (the ones the pairs produce), e.g. one
// rank's share when its operands hold only the blocks that share references.
// `gathered`: every output block is kept in the output, this rank computes
// its share into their places, and the plan lists the transfers that bring
// the others' blocks (chunk by chunk, see kGatherChunks).
std::shared_ptr<const ContractPlan> plan_contract(const BlockSparseT& A, const std::vector<int32_t>& la,
                                                  const BlockSparseT& B, const std::vector<int32_t>& lb, int rank,
                                                  int nranks, ShardPlan* plan_only, const size_t* select, size_t nsel,
                                                  const ThroughDiag* td, bool gathered) {
  const size_t na = A.ndim(), nb = B.ndim();
  if (A.dt != B.dt) throw Error(ErrKind::InvalidArgument, "element types differ");
  if (la.size() != na) throw Error(ErrKind::WrongNumberOfIndices, "labels_a length != ndim(a)");
  if (lb.size() != nb) throw Error(ErrKind::WrongNumberOfIndices, "labels_b length != ndim(b)");
  // ---- cache lookup (plan_only queries and selections are not cached)
  std::vector<int64_t> key;
  const bool cached = !plan_only && !select;
  if (cached) {
    key.push_back((int64_t)A.dt);
    key.push_back(rank);
    key.push_back(nranks);
    key.push_back(gathered ? 1 : 0);
    key.push_back((int64_t)la.size());
    for (int32_t l : la) key.push_back(l);
    key.push_back((int64_t)lb.size());
    for (int32_t l : lb) key.push_back(l);
    key_push(key, A.bsz);
    key_push(key, A.coords);
    key_push(key, B.bsz);
    key_push(key, B.coords);
    key.push_back(td ? (int64_t)td->a_axis : -1);
    if (td)
      for (const auto& kv : td->qmap) {
        key.push_back((int64_t)kv.first);
        key.push_back((int64_t)kv.second.first);
        key.push_back(kv.second.second);
      }
    std::lock_guard<std::mutex> lk(g_bsplan_mu);
    auto it = g_bsplans.find(key);
    if (it != g_bsplans.end()) {
      it->second.second = ++g_bsplan_tick;
      return it->second.first;
    }
  }
  auto P = std::make_shared<ContractPlan>();
  // ContractionProperties pairs: first match in B (properties.rs:100-111)
  std::vector<size_t> pa, pb, ua, ub;
  for (size_t i = 0; i < na; i++) {
    if (la[i] >= 0) continue;
    for (size_t j = 0; j < nb; j++)
      if (la[i] == lb[j]) {
        pa.push_back(i);
        pb.push_back(j);
        break;
      }
  }
  for (size_t i = 0; i < na; i++)
    if (std::find(pa.begin(), pa.end(), i) == pa.end()) ua.push_back(i);
  for (size_t j = 0; j < nb; j++)
    if (std::find(pb.begin(), pb.end(), j) == pb.end()) ub.push_back(j);
  // blocksparse.rs:114-132: same block count and sizes on contracted axes
  size_t td_pos = SIZE_MAX;  // position of the diagonal's axis among the contracted pairs
  for (size_t p = 0; p < pa.size(); p++) {
    if (td && pa[p] == td->a_axis) {
      td_pos = p;  // sizes checked against the diagonal operand by the caller
      continue;
    }
    if (A.bsz[pa[p]].size() != B.bsz[pb[p]].size()) throw Error(ErrKind::ShapeMismatch, "block counts differ");
    for (size_t q = 0; q < A.bsz[pa[p]].size(); q++)
      if (A.bsz[pa[p]][q] != B.bsz[pb[p]][q]) throw Error(ErrKind::ShapeMismatch, "block sizes differ");
  }
  P->has_td = td_pos != SIZE_MAX;
  // output BlockDims (blocksparse.rs:186-209)
  BlockSparseT& C = P->c;
  C.dt = A.dt;
  for (size_t i : ua) C.bsz.push_back(A.bsz[i]);
  for (size_t j : ub) C.bsz.push_back(B.bsz[j]);
  const bool scalar_out = C.bsz.empty();
  if (scalar_out) C.bsz.push_back({1});
  // pair scan as a hash join, preserving (A storage order, B storage order)
  auto key_of = [](const std::vector<size_t>& c, const std::vector<size_t>& axes) {
    std::vector<size_t> k;
    for (size_t a : axes) k.push_back(c[a]);
    return k;
  };
  std::map<std::vector<size_t>, std::vector<size_t>> bmap;
  for (size_t b = 0; b < B.nnzb(); b++) bmap[key_of(B.coords[b], pb)].push_back(b);
  std::map<std::vector<size_t>, std::vector<std::pair<size_t, size_t>>> contrib;  // sorted output blocks
  for (size_t a = 0; a < A.nnzb(); a++) {
    std::vector<size_t> k = key_of(A.coords[a], pa);
    if (td_pos != SIZE_MAX) {  // through the diagonal: A's q_a meets B's q_b
      auto q = td->qmap.find(k[td_pos]);
      if (q == td->qmap.end()) continue;
      k[td_pos] = q->second.first;
    }
    auto it = bmap.find(k);
    if (it == bmap.end()) continue;
    for (size_t b : it->second) {
      std::vector<size_t> oc;
      for (size_t i : ua) oc.push_back(A.coords[a][i]);
      for (size_t j : ub) oc.push_back(B.coords[b][j]);
      if (oc.empty()) oc.push_back(0);
      contrib[oc].push_back({a, b});
    }
  }
  if (select) {
    const size_t r = std::max<size_t>(ua.size() + ub.size(), 1);
    std::set<std::vector<size_t>> want;
    for (size_t i = 0; i < nsel; i++) want.insert(std::vector<size_t>(select + i * r, select + (i + 1) * r));
    for (auto it = contrib.begin(); it != contrib.end();) {
      if (want.count(it->first))
        ++it;
      else
        it = contrib.erase(it);
    }
  }
  // TTGT of each pair is contract_gemm on the blocks (gemm.rs:47-236):
  // perm_b with a repeated axis is not a permutation -> InvalidPermutation.
  {
    std::vector<size_t> perm_b(pb);
    perm_b.insert(perm_b.end(), ub.begin(), ub.end());
    bool id = true;
    for (size_t i = 0; i < perm_b.size(); i++) id &= perm_b[i] == i;
    std::vector<char> seen(nb, 0);
    bool valid = perm_b.size() == nb;
    for (size_t p : perm_b) {
      if (p >= nb || seen[p]) valid = false;
      if (p < nb) seen[p] = 1;
    }
    if (!contrib.empty() && !pa.empty() && !id && !valid)
      throw Error(ErrKind::InvalidPermutation, "contracted axes of B repeat");
  }
  // output label order vs contract_gemm's sorted order (properties.rs:169-186)
  std::vector<int32_t> olab;
  for (size_t i : ua) olab.push_back(la[i]);
  for (size_t j : ub) olab.push_back(lb[j]);
  std::vector<size_t>& perm_c = P->perm_c;
  perm_c.resize(olab.size());
  for (size_t i = 0; i < perm_c.size(); i++) perm_c[i] = i;
  std::stable_sort(perm_c.begin(), perm_c.end(), [&](size_t x, size_t y) { return olab[x] < olab[y]; });
  for (size_t i = 0; i < perm_c.size(); i++)
    if (olab[perm_c[i]] != olab[i]) P->permute_c = true;

  // sorted output blocks with their real flops and their cost on the
  // tensor cores: tiles of 64 x 64, k in steps of 16 (a block much smaller
  // than a tile costs a whole tile)
  std::vector<std::vector<size_t>> all_out;
  std::vector<double> work, cost;
  const double cf = A.dt == DType::C128 ? 8.0 : 2.0;
  for (auto& kv : contrib) {
    all_out.push_back(kv.first);
    double w = 0, c = 0;
    for (auto& pr : kv.second) {
      double m = 1, n = 1, k = 1;
      for (size_t i : ua) m *= (double)A.bsz[i][A.coords[pr.first][i]];
      for (size_t j : ub) n *= (double)B.bsz[j][B.coords[pr.second][j]];
      for (size_t i : pa) k *= (double)A.bsz[i][A.coords[pr.first][i]];
      w += cf * m * n * k;
      c += std::ceil(m / 64) * std::ceil(n / 64) * std::ceil(k / 16);
    }
    work.push_back(w);
    cost.push_back(c);
  }
  // Longest processing time first on the tile cost: costliest output block
  // to the least loaded rank (stable order, ties to the lower rank).
  std::vector<int> owner(all_out.size(), 0);
  {
    std::vector<double> load(nranks, 0.0);
    std::vector<size_t> order(all_out.size());
    for (size_t i = 0; i < order.size(); i++) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](size_t x, size_t y) { return cost[x] > cost[y]; });
    for (size_t i : order) {
      int r = 0;
      for (int q = 1; q < nranks; q++)
        if (load[q] < load[r]) r = q;
      owner[i] = r;
      load[r] += cost[i];
    }
  }
  if (plan_only) {
    plan_only->blocks.assign(nranks, 0);
    plan_only->flops.assign(nranks, 0.0);
    for (size_t i = 0; i < owner.size(); i++) {
      plan_only->blocks[owner[i]]++;
      plan_only->flops[owner[i]] += work[i];
    }
    return P;
  }
  if (gathered) {
    C.coords = all_out;
  } else {
    for (size_t i = 0; i < all_out.size(); i++)
      if (owner[i] == rank) C.coords.push_back(all_out[i]);
  }
  if (nranks > 1 && !gathered) {
    auto lay = std::make_shared<ShardLayout>();
    lay->nranks = nranks;
    lay->coords = all_out;
    lay->owner = owner;
    C.layout = lay;
  }
  C.pack();
  if (C.total() == 0 || contrib.empty()) {
    P->zero = true;
  } else {
    // insertblock shape check for the first contribution (blocksparse_tensor.rs:218-223)
    for (size_t ob = 0; ob < C.nnzb(); ob++) {
      std::vector<size_t> sh = C.block_shape(C.coords[ob]);
      if (P->permute_c) {
        std::vector<size_t> sorted(sh.size());
        for (size_t i = 0; i < sh.size(); i++) sorted[i] = sh[perm_c[i]];
        if (sorted != sh) throw Error(ErrKind::ShapeMismatch, "contract_gemm block shape differs from output block");
      }
    }
    for (size_t ob = 0; ob < C.nnzb(); ob++)
      for (auto& pr : contrib[C.coords[ob]]) {
        if (A.block_elems(A.coords[pr.first]) == 0 || B.block_elems(B.coords[pr.second]) == 0)
          throw Error(ErrKind::Panic, "zero-size block in a contracted pair");
      }
    // operand layouts at the tensor level
    if (is_prefix_run(ua, 0) && is_prefix_run(pa, ua.size())) {
      P->a_kmajor = false;
    } else if (is_prefix_run(pa, 0) && is_prefix_run(ua, pa.size())) {
      P->a_kmajor = true;
    } else {
      P->perm_a = ua;
      P->perm_a.insert(P->perm_a.end(), pa.begin(), pa.end());
      P->pack_a = true;
      P->a_kmajor = false;
    }
    if (is_prefix_run(pb, 0) && is_prefix_run(ub, pb.size())) {
      P->b_kmajor = true;
    } else if (is_prefix_run(ub, 0) && is_prefix_run(pb, ub.size())) {
      P->b_kmajor = false;
    } else {
      P->perm_b = pb;
      P->perm_b.insert(P->perm_b.end(), ub.begin(), ub.end());
      P->pack_b = true;
      P->b_kmajor = true;
    }
    // Strided plan: instead of packing an operand or permuting the output,
    // the GEMM addresses every block through its index runs, when each GEMM
    // index of every block takes at most two runs and every block has fewer
    // than 2^31 elements (no k-scale), and when that is not slower: complex
    // tiles lose nothing measurable to the one-element copies (B200, the c128
    // MPS chain with A's axes permuted: 31.4 TFLOP/s either way); f64 tiles
    // copy adjacent k pairs when every contraction run has stride 1 and an
    // even first extent and every row offset is even (the grouped kernel's
    // check; U(1) rank-4 half scale with A's labels (-1, 1, -2, 2): 30.8
    // TFLOP/s in place against 29.6 with A packed first), and otherwise lose
    // about 8% to one-element copies (U(1) rank-4
    // half scale with A's labels (-1, 1, -2, 2): 27.6 TFLOP/s against 29.6
    // with A packed first), so then they take the strided path only while 8%
    // of their GEMM time (at 30 TFLOP/s) stays below the passes it saves
    // (each a read and a write at 6 TB/s, plus 5 us).
    const bool permute_out = P->permute_c;  // the stored C layout, for the runs
    auto seg_runs = [&](size_t a, size_t b, StridedSegment* ss) -> bool {
      std::vector<int64_t> ea(na), eb(nb);
      int64_t ta = 1, tb = 1;
      for (size_t i = 0; i < na; i++) ta *= (ea[i] = (int64_t)A.bsz[i][A.coords[a][i]]);
      for (size_t j = 0; j < nb; j++) tb *= (eb[j] = (int64_t)B.bsz[j][B.coords[b][j]]);
      if (ta >= ((int64_t)1 << 31) || tb >= ((int64_t)1 << 31)) return false;
      const std::vector<int64_t> sa = block_strides(ea), sb = block_strides(eb);
      return index_runs(ua, ea, sa, &ss->am) && index_runs(pa, ea, sa, &ss->ak) && index_runs(pb, eb, sb, &ss->bk) &&
             index_runs(ub, eb, sb, &ss->bn);
    };
    auto prob_runs = [&](size_t ob, StridedProblem* sp) -> bool {
      // C's blocks hold [A free..., B free...] in label-sorted axis order:
      // axis p of the stored block is unsorted axis perm_c[p]
      const std::vector<size_t> sh = C.block_shape(C.coords[ob]);
      std::vector<int64_t> ext(sh.size()), str(sh.size());
      int64_t st = 1;
      for (size_t p = 0; p < sh.size(); p++) {
        const size_t u = permute_out ? perm_c[p] : p;
        ext[u] = (int64_t)sh[u];
        str[u] = st;
        st *= (int64_t)sh[u];
      }
      if (st >= ((int64_t)1 << 31)) return false;
      std::vector<size_t> mi, ni;
      for (size_t i = 0; i < ua.size(); i++) mi.push_back(i);
      for (size_t j = 0; j < ub.size(); j++) ni.push_back(ua.size() + j);
      return index_runs(mi, ext, str, &sp->cm) && index_runs(ni, ext, str, &sp->cn);
    };
    if ((P->pack_a || P->pack_b || P->permute_c) && td_pos == SIZE_MAX) {
      bool ok = true, pairs = true;
      double flops = 0;
      auto even = [](int64_t x) { return x % 2 == 0; };
      auto pair_ok = [&](const IndexRuns& rows, const IndexRuns& k, int64_t off) {
        return k.s0 == 1 && (k.e0 == 0x7fffffffu || k.e0 % 2 == 0) && even(k.s1) && even(rows.s0) &&
               even(rows.s1) && even(off);
      };
      for (size_t ob = 0; ok && ob < C.nnzb(); ob++) {
        StridedProblem sp{};
        ok = prob_runs(ob, &sp);
        for (auto& p2 : contrib[C.coords[ob]]) {
          StridedSegment ss{};
          if (!ok || !(ok = seg_runs(p2.first, p2.second, &ss))) break;
          pairs = pairs && pair_ok(ss.am, ss.ak, (int64_t)A.offs[p2.first]) &&
                  pair_ok(ss.bn, ss.bk, (int64_t)B.offs[p2.second]);
          double m = 1, n = 1, k = 1;
          for (size_t i : ua) m *= (double)A.bsz[i][A.coords[p2.first][i]];
          for (size_t j : ub) n *= (double)B.bsz[j][B.coords[p2.second][j]];
          for (size_t i : pa) k *= (double)A.bsz[i][A.coords[p2.first][i]];
          flops += 2 * m * n * k;
        }
      }
      if (ok && A.dt != DType::C128 && !pairs) {
        const double es = (double)esize(A.dt);
        double saved = 0;
        if (P->pack_a) saved += 2 * (double)A.total() * es / 6e12 + 5e-6;
        if (P->pack_b) saved += 2 * (double)B.total() * es / 6e12 + 5e-6;
        if (P->permute_c) saved += 2 * (double)C.total() * es / 6e12 + 5e-6;
        ok = 0.08 * flops / 30e12 <= saved;
      }
      if (ok) {
        P->strided = true;
        P->pack_a = P->pack_b = P->permute_c = false;
      }
    }
    // device tables: one problem per output block, one segment per pair
    auto make_table = [&](const std::vector<size_t>& obs, PlannedLaunch& L) {
      for (size_t ob : obs) {
        const auto& prs = contrib[C.coords[ob]];
        GroupedProblem pr{};
        int64_t m = 1, n = 1;
        for (size_t i : ua) m *= (int64_t)A.bsz[i][A.coords[prs[0].first][i]];
        for (size_t j : ub) n *= (int64_t)B.bsz[j][B.coords[prs[0].second][j]];
        pr.m = m;
        pr.n = n;
        pr.c_off = (int64_t)C.offs[ob];
        pr.seg_begin = (int64_t)L.segs.size();
        pr.seg_count = (int64_t)prs.size();
        for (auto& p2 : prs) {
          GroupedSegment sg{};
          int64_t k = 1;
          for (size_t i : pa) k *= (int64_t)A.bsz[i][A.coords[p2.first][i]];
          sg.a_off = (int64_t)A.offs[p2.first];
          sg.b_off = (int64_t)B.offs[p2.second];
          sg.k = k;
          sg.lda = P->a_kmajor ? k : m;
          sg.ldb = P->b_kmajor ? k : n;
          sg.scale_off = td_pos != SIZE_MAX ? td->qmap.at(A.coords[p2.first][td->a_axis]).second : -1;
          L.segs.push_back(sg);
          if (P->strided) {
            L.ssegs.emplace_back();
            seg_runs(p2.first, p2.second, &L.ssegs.back());
          }
        }
        L.probs.push_back(pr);
        if (P->strided) {
          L.sprobs.emplace_back();
          prob_runs(ob, &L.sprobs.back());
        }
      }
    };
    if (!gathered) {
      std::vector<size_t> obs(C.nnzb());
      for (size_t i = 0; i < obs.size(); i++) obs[i] = i;
      P->launches.emplace_back();
      make_table(obs, P->launches.back());
    } else {
      // Chunks: every rank's blocks by descending tile cost, dealt round-robin
      // (every rank derives the same chunk of every block, so each transfer's
      // sender and receiver issue it in the same group, in block order).
      std::vector<int> chunk(all_out.size(), 0);
      {
        std::vector<size_t> order(all_out.size());
        for (size_t i = 0; i < order.size(); i++) order[i] = i;
        std::stable_sort(order.begin(), order.end(), [&](size_t x, size_t y) { return cost[x] > cost[y]; });
        std::vector<int> dealt(nranks, 0);
        for (size_t i : order) chunk[i] = dealt[owner[i]]++ % kGatherChunks;
      }
      // Staging layout, chunk-major then rank-major: chunk c's region holds
      // nranks slots of pad_c elements (pad_c: the largest rank's chunk c),
      // rank r's blocks of the chunk packed in sorted order in slot r.  Each
      // rank computes its blocks into its own slot; an in-place all-gather
      // per chunk fills the others; one copy puts every block at its place.
      const size_t es = esize(A.dt);
      std::vector<size_t> stage_of(all_out.size(), 0);
      size_t off = 0;
      for (int c = 0; c < kGatherChunks; c++) {
        P->launches.emplace_back();
        PlannedLaunch& L = P->launches.back();
        std::vector<size_t> fill(nranks, 0);
        for (size_t i = 0; i < all_out.size(); i++)
          if (chunk[i] == c) fill[owner[i]] += C.offs[i + 1] - C.offs[i];
        size_t pad = 0;
        for (size_t f : fill) pad = std::max(pad, f);
        pad = (pad + 1) / 2 * 2;  // slots start 16-byte aligned (f64)
        L.stage_off = off;
        L.pad = pad;
        std::fill(fill.begin(), fill.end(), 0);
        for (size_t i = 0; i < all_out.size(); i++)
          if (chunk[i] == c) {
            stage_of[i] = off + (size_t)owner[i] * pad + fill[owner[i]];
            fill[owner[i]] += C.offs[i + 1] - C.offs[i];
          }
        off += (size_t)nranks * pad;
        std::vector<size_t> mine;
        for (size_t i = 0; i < all_out.size(); i++)
          if (owner[i] == rank && chunk[i] == c) mine.push_back(i);
        make_table(mine, L);
        for (size_t q = 0; q < mine.size(); q++) L.probs[q].c_off = (int64_t)stage_of[mine[q]];
      }
      P->stage_total = off;
      {
        std::vector<size_t> mine;
        for (size_t i = 0; i < all_out.size(); i++)
          if (owner[i] == rank) mine.push_back(i);
        make_table(mine, P->direct);
        for (size_t i = 0; i < all_out.size(); i++) {
          const int64_t o = (int64_t)(C.offs[i] * es), n = (int64_t)((C.offs[i + 1] - C.offs[i]) * es);
          if (owner[i] == rank || n == 0) continue;
          if (!P->peer_off.empty() && P->peer_off.back() + P->peer_bytes.back() == o)
            P->peer_bytes.back() += n;
          else {
            P->peer_off.push_back(o);
            P->peer_bytes.push_back(n);
          }
        }
      }
      for (size_t i = 0; i < all_out.size(); i++) {
        const size_t n = C.offs[i + 1] - C.offs[i];
        if (!n) continue;
        P->copy_src.push_back((int64_t)(stage_of[i] * es));
        P->copy_dst.push_back((int64_t)(C.offs[i] * es));
        P->copy_bytes.push_back((int64_t)(n * es));
      }
    }
  }
  if (cached) {
    std::lock_guard<std::mutex> lk(g_bsplan_mu);
    if (g_bsplans.size() >= kBsPlanCacheSize) {
      auto victim = g_bsplans.begin();
      for (auto it = g_bsplans.begin(); it != g_bsplans.end(); ++it)
        if (it->second.second < victim->second.second) victim = it;
      g_bsplans.erase(victim);
    }
    g_bsplans[key] = {P, ++g_bsplan_tick};
  }
  return P;
}

// contract_blocksparse (contract/blocksparse.rs:87-183), planned by
// plan_contract and run as grouped launches (one, or one per chunk of a
// gathered contraction).  With nranks > 1 only this rank's output blocks are
// computed and stored (longest processing time on the tile cost; every rank
// derives the same assignment).  `gcomm` (gathered mode): rank and nranks are
// the communicator's; when the ranks map each other's output buffers, the
// grouped launch stores every tile of this rank's output blocks into all of
// them as it computes it, then a barrier and a copy into the result;
// otherwise this rank computes into its slot of a staging buffer, chunk by
// chunk, an NCCL all-gather per chunk follows, and one copy kernel puts every
// block at its place in the sorted output.  The result is the unsharded
// tensor on every rank.
BlockSparseT bs_contract(const BlockSparseT& A, const std::vector<int32_t>& la, const BlockSparseT& B,
                         const std::vector<int32_t>& lb, int rank, int nranks, ShardPlan* plan_only = nullptr,
                         const size_t* select = nullptr, size_t nsel = 0, const ThroughDiag* td = nullptr,
                         Comm* gcomm = nullptr) {
  if (gcomm) {
    rank = comm_rank(*gcomm);
    nranks = comm_size(*gcomm);
    if (comm_device(*gcomm) != current_device())
      throw Error(ErrKind::InvalidArgument, "the communicator belongs to another device than the current one");
  }
  std::shared_ptr<const ContractPlan> P =
      plan_contract(A, la, B, lb, rank, nranks, plan_only, select, nsel, td, gcomm != nullptr);
  if (plan_only) return P->c;
  BlockSparseT C = P->c;
  C.st = std::make_shared<Storage>(C.dt, C.total());
  if (P->zero) {
    C.st->set_uniform(0.0, 0.0);
    return C;
  }
  const DeviceCtx& c = ctx();
  cudaStream_t s = c.compute;
  const int dev = current_device();
  const size_t es = esize(A.dt);
  const void* Ad = A.st->dev_read();
  const void* Bd = B.st->dev_read();
  void* Aown = nullptr;
  void* Bown = nullptr;
  if (P->pack_a) {
    std::vector<size_t> order(A.nnzb());
    for (size_t i = 0; i < order.size(); i++) order[i] = i;
    Aown = dev_alloc(A.total() * es, dev);
    permute_blocks(A.dt, Ad, Aown, A, P->perm_a, A.offs, order, s);
    Ad = Aown;
  }
  if (P->pack_b) {
    std::vector<size_t> order(B.nnzb());
    for (size_t i = 0; i < order.size(); i++) order[i] = i;
    Bown = dev_alloc(B.total() * es, dev);
    permute_blocks(B.dt, Bd, Bown, B, P->perm_b, B.offs, order, s);
    Bd = Bown;
  }
  void* Cd = C.st->dev_overwrite();
  void* Cu = P->permute_c ? dev_alloc(C.total() * es, dev) : Cd;
  const void* kscale = P->has_td ? td->sdata : nullptr;
  const bool kreal = P->has_td && td->real;
  // the index runs of a launch's table (strided plans only)
  auto sruns = [&](const PlannedLaunch& L) { return P->strided ? &L.sprobs : nullptr; };
  auto sruns_seg = [&](const PlannedLaunch& L) { return P->strided ? &L.ssegs : nullptr; };
  void* mine = nullptr;
  std::vector<void*> peers(kMaxSymRanks, nullptr);
  const bool direct = gcomm && nranks > 1 && comm_symmetric(*gcomm, C.total() * es, s, &mine, peers.data());
  if (direct) {
    // One launch computes this rank's output blocks and stores every tile
    // into the result and into every other rank's mapped buffer, over
    // NVLink, as it is computed (no separate transfer); a barrier over the
    // ranks, then the other ranks' blocks are copied from this rank's mapped
    // buffer into the result.
    std::vector<void*> others;
    for (int r = 0; r < nranks; r++)
      if (r != rank) others.push_back(peers[r]);
    if (!P->direct.probs.empty())
      grouped_gemm(A.dt, Ad, Bd, Cu, P->a_kmajor, P->b_kmajor, P->direct.probs, P->direct.segs, kscale, s, kreal,
                   0, &others, sruns(P->direct), sruns_seg(P->direct));
    comm_barrier(*gcomm, s, s);
    copy_segments(mine, Cu, P->peer_off, P->peer_off, P->peer_bytes, s);
  } else if (gcomm) {
    // Staged: each chunk into this rank's slots of a staging buffer, an
    // in-place NCCL all-gather per chunk, one copy into the sorted output.
    void* stage = dev_alloc(P->stage_total * es, dev);
    for (const PlannedLaunch& L : P->launches) {
      if (!L.probs.empty())
        grouped_gemm(A.dt, Ad, Bd, stage, P->a_kmajor, P->b_kmajor, L.probs, L.segs, kscale, s, kreal,
                     nranks > 1 ? kGatherSmReserve : 0, nullptr, sruns(L), sruns_seg(L));
      comm_allgather(*gcomm, (char*)stage + L.stage_off * es, L.pad * (es / 8), s);
    }
    comm_join(*gcomm, s);
    copy_segments(stage, Cu, P->copy_src, P->copy_dst, P->copy_bytes, s);
    dev_free(stage, dev);
  } else {
    for (const PlannedLaunch& L : P->launches)
      if (!L.probs.empty())
        grouped_gemm(A.dt, Ad, Bd, Cu, P->a_kmajor, P->b_kmajor, L.probs, L.segs, kscale, s, kreal, 0, nullptr,
                     sruns(L), sruns_seg(L));
  }
  if (P->permute_c) {
    // contract_gemm returns each block in label-sorted order (same shape,
    // checked in the plan); the data is permuted block by block.
    std::vector<size_t> order(C.nnzb());
    for (size_t i = 0; i < order.size(); i++) order[i] = i;
    // blocks of Cu are laid out in the unsorted axis order [A free..., B free...]
    permute_blocks(C.dt, Cu, Cd, C, P->perm_c, C.offs, order, s);
    dev_free(Cu, dev);
  }
  if (Aown) dev_free(Aown, dev);
  if (Bown) dev_free(Bown, dev);
  return C;
}

// permutedims_blocksparse (operations/blocksparse.rs:61-129)
BlockSparseT bs_permutedims(const BlockSparseT& A, const std::vector<size_t>& perm) {
  const size_t nd = A.ndim();
  if (perm.size() != nd) throw Error(ErrKind::InvalidPermutation, "invalid permutation");
  std::vector<char> seen(nd, 0);
  for (size_t p : perm) {
    if (p >= nd || seen[p]) throw Error(ErrKind::InvalidPermutation, "invalid permutation");
    seen[p] = 1;
  }
  BlockSparseT C;
  C.dt = A.dt;
  for (size_t i = 0; i < nd; i++) C.bsz.push_back(A.bsz[perm[i]]);
  std::vector<std::pair<std::vector<size_t>, size_t>> pc;
  for (size_t b = 0; b < A.nnzb(); b++) {
    std::vector<size_t> c(nd);
    for (size_t i = 0; i < nd; i++) c[i] = A.coords[b][perm[i]];
    pc.push_back({c, b});
    if (A.block_elems(A.coords[b]) == 0) throw Error(ErrKind::Panic, "permutedims of a zero-size block");
  }
  std::sort(pc.begin(), pc.end());
  std::vector<size_t> order;
  for (auto& x : pc) {
    C.coords.push_back(x.first);
    order.push_back(x.second);
  }
  C.pack();
  C.st = std::make_shared<Storage>(C.dt, C.total());
  if (C.total() == 0) {
    C.st->set_uniform(0.0, 0.0);
    return C;
  }
  const void* Ad = A.st->dev_read();
  void* Cd = C.st->dev_overwrite();
  std::vector<size_t> dst_offs(C.offs.begin(), C.offs.end() - 1);
  permute_blocks(A.dt, Ad, Cd, A, perm, dst_offs, order, ctx().compute);
  return C;
}

static std::vector<BsBlockDesc> dense_tables(const BlockSparseT& A, std::vector<int64_t>* offs) {
  std::vector<size_t> dshape(A.ndim());
  for (size_t i = 0; i < A.ndim(); i++) dshape[i] = A.dense_extent(i);
  std::vector<size_t> dst = col_major_strides(dshape);
  std::vector<BsBlockDesc> tab;
  offs->clear();
  for (size_t b = 0; b < A.nnzb(); b++) {
    if (A.block_elems(A.coords[b]) == 0) continue;
    BsBlockDesc d{};
    d.ndim = (int32_t)A.ndim();
    d.dense_base = 0;
    for (size_t i = 0; i < A.ndim(); i++) {
      d.shape[i] = (int64_t)A.bsz[i][A.coords[b][i]];
      d.dstride[i] = (int64_t)dst[i];
      d.dense_base += (int64_t)(A.block_start(i, A.coords[b][i]) * dst[i]);
    }
    tab.push_back(d);
    offs->push_back((int64_t)A.offs[b]);
  }
  return tab;
}

// BlockSparseTensor::to_dense (blocksparse_tensor.rs:290-324)
Dense bs_to_dense(const BlockSparseT& A) {
  std::vector<size_t> dshape(A.ndim());
  for (size_t i = 0; i < A.ndim(); i++) dshape[i] = A.dense_extent(i);
  Dense out = make_uniform(A.dt, dshape, 0.0, 0.0);
  if (A.total() == 0) return out;
  void* dd = const_cast<void*>(out.st->dev_read());  // materialise zeros on device
  out.st->dev_overwrite();
  std::vector<int64_t> offs;
  std::vector<BsBlockDesc> tab = dense_tables(A, &offs);
  bs_dense_map(A.dt, const_cast<void*>(A.st->dev_read()), dd, offs, tab, (int64_t)A.total(), true, ctx().compute);
  return out;
}

// BlockSparseTensor::from_dense (blocksparse_tensor.rs:353-391)
BlockSparseT bs_from_dense(const Dense& dense, const std::vector<std::vector<size_t>>& bsz,
                           const std::vector<std::vector<size_t>>& coords) {
  BlockSparseT A = make_bs(dense.dt, bsz, coords);
  std::vector<size_t> dshape(A.ndim());
  for (size_t i = 0; i < A.ndim(); i++) dshape[i] = A.dense_extent(i);
  if (dshape != dense.shape) throw Error(ErrKind::ShapeMismatch, "dense shape does not match block dims");
  if (A.total() == 0) return A;
  void* p = A.st->dev_overwrite();
  std::vector<int64_t> offs;
  std::vector<BsBlockDesc> tab = dense_tables(A, &offs);
  bs_dense_map(A.dt, p, const_cast<void*>(dense.st->dev_read()), offs, tab, (int64_t)A.total(), false,
               ctx().compute);
  return A;
}

static DiagBlockSparseT make_diag(DType dt, const std::vector<std::vector<size_t>>& bsz,
                                  const std::vector<std::vector<size_t>>& coords) {
  check_structure(bsz, coords);
  DiagBlockSparseT S;
  S.s.dt = dt;
  S.s.bsz = bsz;
  S.s.coords = coords;
  // diagblocksparse.rs:218-230: offsets packed by diagonal length
  S.s.offs.assign(coords.size() + 1, 0);
  for (size_t b = 0; b < coords.size(); b++) S.s.offs[b + 1] = S.s.offs[b] + S.diag_size(coords[b]);
  S.s.st = std::make_shared<Storage>(dt, S.s.total());
  S.s.st->set_uniform(0.0, 0.0);
  return S;
}

// DiagBlockSparseTensor::to_dense (diagblocksparse_tensor.rs:399-426)
Dense diag_to_dense(const DiagBlockSparseT& S) {
  const BlockSparseT& t = S.s;
  std::vector<size_t> dshape(t.ndim());
  for (size_t i = 0; i < t.ndim(); i++) dshape[i] = t.dense_extent(i);
  Dense out = make_uniform(t.dt, dshape, 0.0, 0.0);
  if (t.total() == 0) return out;
  void* dd = const_cast<void*>(out.st->dev_read());
  out.st->dev_overwrite();
  std::vector<size_t> dst = col_major_strides(dshape);
  int64_t step = 0;
  for (size_t x : dst) step += (int64_t)x;
  std::vector<BsBlockDesc> tab;
  std::vector<int64_t> offs;
  for (size_t b = 0; b < t.nnzb(); b++) {
    if (S.diag_size(t.coords[b]) == 0) continue;
    BsBlockDesc d{};
    d.ndim = 1;
    for (size_t i = 0; i < t.ndim(); i++) d.dense_base += (int64_t)(t.block_start(i, t.coords[b][i]) * dst[i]);
    d.dstride[0] = step;
    tab.push_back(d);
    offs.push_back((int64_t)t.offs[b]);
  }
  diag_scatter(t.dt, t.st->dev_read(), dd, offs, tab, (int64_t)t.total(), ctx().compute);
  return out;
}

// The diagonal tensor as a block-sparse tensor with dense diagonal blocks
// (the same values as to_dense restricted to the stored blocks).
BlockSparseT diag_to_blocksparse(const DiagBlockSparseT& S) {
  const BlockSparseT& t = S.s;
  BlockSparseT C = make_bs(t.dt, t.bsz, t.coords);
  if (C.total() == 0) return C;
  void* cd = const_cast<void*>(C.st->dev_read());  // zeros on device
  C.st->dev_overwrite();
  std::vector<BsBlockDesc> tab;
  std::vector<int64_t> offs;
  for (size_t b = 0; b < t.nnzb(); b++) {
    size_t ds = S.diag_size(t.coords[b]);
    if (ds == 0) continue;
    std::vector<size_t> st = col_major_strides(C.block_shape(C.coords[b]));
    BsBlockDesc d{};
    d.ndim = 1;
    d.dense_base = (int64_t)C.offs[b];
    for (size_t x : st) d.dstride[0] += (int64_t)x;
    tab.push_back(d);
    offs.push_back((int64_t)t.offs[b]);
  }
  diag_scatter(t.dt, t.st->dev_read(), cd, offs, tab, (int64_t)t.total(), ctx().compute);
  return C;
}

// A (block-sparse) x S (diag-block-sparse): the contraction of A with
// diag_to_blocksparse(S) under contract_blocksparse semantics.  When S is
// rank 2, contracted with A's last axis, its other axis kept, and every A
// block meets at most one S block (and lands in its own output block), the
// product is a diagonal scaling of A's last axis: one elementwise kernel
// instead of a GEMM per block.  Otherwise the general block contraction runs.
BlockSparseT bs_contract_diag(const BlockSparseT& A, const std::vector<int32_t>& la, const DiagBlockSparseT& S,
                              const std::vector<int32_t>& ls) {
  const BlockSparseT& t = S.s;
  const size_t na = A.ndim();
  bool fast = t.ndim() == 2 && na >= 1 && la.size() == na && ls.size() == 2 && A.dt == t.dt;
  size_t js = 0, jo = 1;
  if (fast) {
    // exactly one pair: A's last axis with one S axis; S's other axis positive
    int pairs = 0;
    for (size_t i = 0; i < na; i++)
      if (la[i] < 0 && (la[i] == ls[0] || la[i] == ls[1])) pairs++;
    fast = pairs == 1 && la[na - 1] < 0 && (la[na - 1] == ls[0] || la[na - 1] == ls[1]);
    if (fast) {
      js = la[na - 1] == ls[0] ? 0 : 1;
      jo = 1 - js;
      fast = ls[jo] > 0 && ls[js] != ls[jo];
      // output labels ascending (no contract_gemm re-sort)
      int32_t prev = INT32_MIN;
      for (size_t i = 0; i + 1 < na && fast; i++) {
        if (la[i] <= 0) fast = false;  // all other A axes must be free positive axes
        if (la[i] < prev) fast = false;
        prev = la[i];
      }
      if (fast && ls[jo] < prev) fast = false;
      if (fast && A.bsz[na - 1] != t.bsz[js]) fast = false;
    }
  }
  std::map<size_t, size_t> srow;  // S coordinate on js -> S block
  if (fast) {
    for (size_t b = 0; b < t.nnzb(); b++) {
      size_t key = t.coords[b][js];
      if (srow.count(key)) fast = false;
      srow[key] = b;
    }
  }
  if (!fast) return bs_contract(A, la, diag_to_blocksparse(S), ls, 0, 1);
  BlockSparseT C;
  C.dt = A.dt;
  for (size_t i = 0; i + 1 < na; i++) C.bsz.push_back(A.bsz[i]);
  C.bsz.push_back(t.bsz[jo]);
  std::map<std::vector<size_t>, std::pair<size_t, size_t>> outs;  // sorted: out coords -> (A block, S block)
  for (size_t a = 0; a < A.nnzb(); a++) {
    auto it = srow.find(A.coords[a][na - 1]);
    if (it == srow.end()) continue;
    std::vector<size_t> oc(A.coords[a].begin(), A.coords[a].end() - 1);
    oc.push_back(t.coords[it->second][jo]);
    if (outs.count(oc)) return bs_contract(A, la, diag_to_blocksparse(S), ls, 0, 1);
    outs[oc] = {a, it->second};
  }
  for (auto& kv : outs) C.coords.push_back(kv.first);
  C.pack();
  C.st = std::make_shared<Storage>(C.dt, C.total());
  if (C.total() == 0) {
    C.st->set_uniform(0.0, 0.0);
    return C;
  }
  std::vector<BsBlockDesc> tab;
  std::vector<int64_t> offs;
  size_t ob = 0;
  for (auto& kv : outs) {
    size_t a = kv.second.first, sb = kv.second.second;
    std::vector<size_t> sh = C.block_shape(C.coords[ob]);
    BsBlockDesc d{};
    d.ndim = 3;
    int64_t inner = 1;
    for (size_t i = 0; i + 1 < sh.size(); i++) inner *= (int64_t)sh[i];
    d.shape[0] = inner;
    d.shape[1] = (int64_t)sh.back();
    d.shape[2] = (int64_t)S.diag_size(t.coords[sb]);
    d.dense_base = (int64_t)A.offs[a];
    d.dstride[0] = (int64_t)t.offs[sb];
    if (C.block_elems(C.coords[ob]) > 0) {
      tab.push_back(d);
      offs.push_back((int64_t)C.offs[ob]);
    }
    ob++;
  }
  void* cd = C.st->dev_overwrite();
  bs_diag_scale(A.dt, A.st->dev_read(), t.st->dev_read(), cd, offs, tab, (int64_t)C.total(), ctx().compute);
  return C;
}

// (A . S) . B with S a rank-2 diagonal operand whose two labels are the only
// contracted ones: S's first label is contracted with A (one axis), its second
// with B (one axis); every other label of A and B is positive.  The result is
// contract(contract_diag(A, la, S, (x, P)), sorted(A's labels) ++ (y), B, lb)
// for a fresh positive P, i.e. the A-free ++ B-free axes in label order.
// When S's blocks are square and each of A's
// coordinates on the contracted axis meets at most one S block, this is ONE
// grouped launch that applies S's diagonal to the contracted index as it
// loads the operands (no A . S intermediate); otherwise the two
// contractions run one after the other.  rank / nranks: this rank's share of
// the output blocks, as contract_shard assigns them.
BlockSparseT bs_contract_through_diag(const BlockSparseT& A, const std::vector<int32_t>& la,
                                      const DiagBlockSparseT& S, const std::vector<int32_t>& ls,
                                      const BlockSparseT& B, const std::vector<int32_t>& lb, int rank, int nranks,
                                      Comm* gcomm = nullptr) {
  if (gcomm) {
    rank = comm_rank(*gcomm);
    nranks = comm_size(*gcomm);
  }
  const BlockSparseT& t = S.s;
  if (la.size() != A.ndim()) throw Error(ErrKind::WrongNumberOfIndices, "labels_a length != ndim(a)");
  if (lb.size() != B.ndim()) throw Error(ErrKind::WrongNumberOfIndices, "labels_b length != ndim(b)");
  if (ls.size() != 2 || t.ndim() != 2)
    throw Error(ErrKind::InvalidArgument, "the diagonal operand must be rank 2 with two labels");
  const int32_t x = ls[0], y = ls[1];
  if (x >= 0 || y >= 0 || x == y)
    throw Error(ErrKind::InvalidArgument, "both labels of the diagonal operand must be negative and distinct");
  size_t ax_a = SIZE_MAX, ax_b = SIZE_MAX;
  int32_t pmax = 0;
  for (size_t i = 0; i < la.size(); i++) {
    if (la[i] == x && ax_a == SIZE_MAX)
      ax_a = i;
    else if (la[i] <= 0)
      throw Error(ErrKind::InvalidArgument, "A's labels other than the diagonal's must be positive and single");
    pmax = std::max(pmax, la[i]);
  }
  for (size_t j = 0; j < lb.size(); j++) {
    if (lb[j] == y && ax_b == SIZE_MAX)
      ax_b = j;
    else if (lb[j] <= 0)
      throw Error(ErrKind::InvalidArgument, "B's labels other than the diagonal's must be positive and single");
    pmax = std::max(pmax, lb[j]);
  }
  if (ax_a == SIZE_MAX || ax_b == SIZE_MAX)
    throw Error(ErrKind::InvalidArgument, "A must carry the diagonal's first label and B its second");
  for (int32_t u : la)
    for (int32_t v : lb)
      if (u == v) throw Error(ErrKind::InvalidArgument, "A and B may share no label");
  bool fused = A.dt == B.dt && A.dt == t.dt && A.bsz[ax_a] == t.bsz[0] && t.bsz[1] == B.bsz[ax_b];
  ThroughDiag td;
  td.a_axis = ax_a;
  for (size_t b = 0; b < t.nnzb() && fused; b++) {
    const size_t qa = t.coords[b][0], qb = t.coords[b][1];
    if (t.bsz[0][qa] != t.bsz[1][qb] || td.qmap.count(qa)) fused = false;
    td.qmap[qa] = {qb, (int64_t)t.offs[b]};
  }
  // One launch whenever the structure allows: applying S inside the GEMM
  // (to B's fragments as they leave shared memory, one multiply per
  // component for a real diagonal) costs less than a pass of its own over A,
  // which a sharded rank would pay in full for its 1/nranks of the work.
  if (fused) {
    td.sdata = t.nnzb() ? t.st->dev_read() : nullptr;
    td.real = S.real_valued;
    if (!td.sdata) fused = false;
  }
  if (fused) {
    std::vector<int32_t> lb2(lb);
    lb2[ax_b] = x;  // pair A's axis with B's through the diagonal
    return bs_contract(A, la, B, lb2, rank, nranks, nullptr, nullptr, 0, &td, gcomm);
  }
  const int32_t P = pmax + 1;
  BlockSparseT AS = bs_contract_diag(A, la, S, {x, P});
  std::vector<int32_t> las;
  for (int32_t u : la)
    if (u != x) las.push_back(u);
  std::sort(las.begin(), las.end());
  las.push_back(y);
  return bs_contract(AS, las, B, lb, rank, nranks, nullptr, nullptr, 0, nullptr, gcomm);
}

// The whole output of a sharded contraction on every rank, from this rank's
// shard (which carries the layout: every output block and its owner, so no
// structure is exchanged).
BlockSparseT bs_allgather(const BlockSparseT& shard, Comm& cm) {
  if (!shard.layout) throw Error(ErrKind::InvalidArgument, "allgather needs a shard of a sharded contraction");
  const ShardLayout& L = *shard.layout;
  const int rank = comm_rank(cm), nranks = comm_size(cm);
  if (L.nranks != nranks) throw Error(ErrKind::InvalidArgument, "the shard was cut for another number of ranks");
  if (comm_device(cm) != current_device())
    throw Error(ErrKind::InvalidArgument, "the communicator belongs to another device than the current one");
  std::vector<std::vector<size_t>> mine;
  for (size_t i = 0; i < L.coords.size(); i++)
    if (L.owner[i] == rank) mine.push_back(L.coords[i]);
  if (mine != shard.coords) throw Error(ErrKind::InvalidArgument, "the shard does not belong to this rank");
  BlockSparseT C = make_bs(shard.dt, shard.bsz, L.coords);
  if (C.total() == 0) return C;
  const size_t es = esize(C.dt);
  cudaStream_t s = ctx().compute;
  const int dev = current_device();
  void* d = C.st->dev_overwrite();
  // every rank's shard (its blocks, packed in sorted order) in slot r of a
  // staging buffer of nranks slots of the largest shard's size; one in-place
  // all-gather, then one copy puts every block at its place
  std::vector<size_t> per(nranks, 0), pos(L.coords.size(), 0);
  for (size_t i = 0; i < L.coords.size(); i++) {
    pos[i] = per[L.owner[i]];
    per[L.owner[i]] += C.offs[i + 1] - C.offs[i];
  }
  size_t pad = 0;
  for (size_t x : per) pad = std::max(pad, x);
  pad = (pad + 1) / 2 * 2;
  void* stage = dev_alloc((size_t)nranks * pad * es, dev);
  if (shard.total())
    NDT_CUDA(cudaMemcpyAsync((char*)stage + (size_t)rank * pad * es, shard.st->dev_read(), shard.total() * es,
                             cudaMemcpyDeviceToDevice, s));
  comm_allgather(cm, stage, pad * (es / 8), s);
  comm_join(cm, s);
  std::vector<int64_t> so, dso, nb;
  for (size_t i = 0; i < L.coords.size(); i++) {
    const size_t n = C.offs[i + 1] - C.offs[i];
    if (!n) continue;
    so.push_back((int64_t)(((size_t)L.owner[i] * pad + pos[i]) * es));
    dso.push_back((int64_t)(C.offs[i] * es));
    nb.push_back((int64_t)(n * es));
  }
  copy_segments(stage, d, so, dso, nb, s);
  dev_free(stage, dev);
  return C;
}

// A block-sparse tensor from blocks lying anywhere in device memory: block i
// of `cs` is read at src + src_off[i] elements; the result holds the blocks
// sorted by coordinates, packed (as contract_blocksparse orders its output),
// written by one segmented copy.  Assembles gathered shards.
BlockSparseT bs_from_device_blocks(DType dt, const std::vector<std::vector<size_t>>& bsz,
                                   const std::vector<std::vector<size_t>>& cs, const size_t* src_off,
                                   const void* src, size_t src_len) {
  std::vector<size_t> order(cs.size());
  for (size_t i = 0; i < order.size(); i++) order[i] = i;
  std::sort(order.begin(), order.end(), [&](size_t x, size_t y) { return cs[x] < cs[y]; });
  std::vector<std::vector<size_t>> sorted;
  for (size_t i : order) sorted.push_back(cs[i]);
  BlockSparseT t = make_bs(dt, bsz, sorted);
  if (t.total() == 0) return t;
  const size_t es = esize(dt);
  std::vector<int64_t> so, dso, nb;
  for (size_t r = 0; r < order.size(); r++) {
    const size_t n = t.block_elems(t.coords[r]);
    const size_t o = src_off[order[r]];
    if (o > src_len || n > src_len - o) throw Error(ErrKind::ShapeMismatch, "block outside the source range");
    so.push_back((int64_t)(o * es));
    dso.push_back((int64_t)(t.offs[r] * es));
    nb.push_back((int64_t)(n * es));
  }
  void* d = t.st->dev_overwrite();
  copy_segments(src, d, so, dso, nb, ctx().compute);
  return t;
}

}  // namespace ndt

// =========================================================================
// C ABI (additive: the reference's C ABI has no block-sparse symbols)
// =========================================================================
using namespace ndt;

struct NdtBs {
  BlockSparseT t;
};
struct NdtDiag {
  DiagBlockSparseT t;
};

namespace {

int map_err(const Error& e, int code) {
  set_last_error(e.what());
  switch (e.kind) {
    case ErrKind::Panic:
    case ErrKind::Cuda:
      return NDT_INTERNAL_ERROR;
    case ErrKind::InvalidArgument:
      return NDT_INVALID_ARGUMENT;
    case ErrKind::BlockNotFound:
    case ErrKind::IndexOutOfBounds:
      return NDT_INDEX_OUT_OF_BOUNDS;
    default:
      return code;
  }
}

template <class F>
void* guarded(int* status, int code, F&& f) {
  if (!status) return nullptr;
  try {
    void* r = f();
    *status = NDT_SUCCESS;
    return r;
  } catch (const Error& e) {
    *status = map_err(e, code);
  } catch (const std::exception& e) {
    set_last_error(e.what());
    *status = NDT_INTERNAL_ERROR;
  } catch (...) {
    *status = NDT_INTERNAL_ERROR;
  }
  return nullptr;
}

template <class F>
int guarded_int(int code, F&& f) {
  try {
    return f();
  } catch (const Error& e) {
    return map_err(e, code);
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return NDT_INTERNAL_ERROR;
  } catch (...) {
    return NDT_INTERNAL_ERROR;
  }
}

void read_structure(size_t ndim, const size_t* nblocks, const size_t* block_sizes, size_t nnzb, const size_t* coords,
                    std::vector<std::vector<size_t>>* bsz, std::vector<std::vector<size_t>>* cs) {
  if ((ndim && (!nblocks || !block_sizes)) || (nnzb && ndim && !coords))
    throw Error(ErrKind::InvalidArgument, "NULL structure array");
  size_t k = 0;
  for (size_t i = 0; i < ndim; i++) {
    bsz->push_back(std::vector<size_t>(block_sizes + k, block_sizes + k + nblocks[i]));
    k += nblocks[i];
  }
  for (size_t b = 0; b < nnzb; b++) cs->push_back(std::vector<size_t>(coords + b * ndim, coords + (b + 1) * ndim));
}

std::vector<int32_t> labels(const long* l, size_t n) {
  std::vector<int32_t> v(n);
  for (size_t i = 0; i < n; i++) v[i] = (int32_t)l[i];
  return v;
}

void* bs_new(DType dt, size_t ndim, const size_t* nblocks, const size_t* block_sizes, size_t nnzb,
             const size_t* coords, const double* data, size_t len, int* status) {
  return guarded(status, NDT_SHAPE_MISMATCH, [&]() -> void* {
    std::vector<std::vector<size_t>> bsz, cs;
    read_structure(ndim, nblocks, block_sizes, nnzb, coords, &bsz, &cs);
    BlockSparseT t = make_bs(dt, bsz, cs);
    if (data) {
      if (len != t.total()) throw Error(ErrKind::ShapeMismatch, "data length != total block elements");
      if (t.total()) {
        Dense tmp = make_from_host(dt, data, len, {len});
        t.st = tmp.st;
      }
    }
    return new NdtBs{t};
  });
}

int bs_insert(void* h, const size_t* coords, const double* data, size_t len) {
  if (!h || !coords || !data) return NDT_INVALID_ARGUMENT;
  return guarded_int(NDT_SHAPE_MISMATCH, [&]() {
    BlockSparseT& t = ((NdtBs*)h)->t;
    std::vector<size_t> c(coords, coords + t.ndim());
    long b = t.find(c);
    if (b < 0) return NDT_INDEX_OUT_OF_BOUNDS;  // TensorError::BlockNotFound
    // insertblock: data shape must equal the block shape (blocksparse_tensor.rs:210-235)
    if (len != t.block_elems(c)) return NDT_SHAPE_MISMATCH;
    if (t.st.use_count() > 1) t.st = t.st->clone();
    if (!device_available()) {  // host-only bookkeeping (no computation happens here)
      char* h = (char*)t.st->host_write();
      memcpy(h + t.offs[b] * esize(t.dt), data, len * esize(t.dt));
      return NDT_SUCCESS;
    }
    void* p = const_cast<void*>(t.st->dev_read());
    t.st->dev_overwrite();
    NDT_CUDA(cudaMemcpyAsync((char*)p + t.offs[b] * esize(t.dt), data, len * esize(t.dt), cudaMemcpyHostToDevice,
                             ctx().compute));
    NDT_CUDA(cudaStreamSynchronize(ctx().compute));
    return NDT_SUCCESS;
  });
}

int bs_get(const void* h, const size_t* coords, double* out, size_t len) {
  if (!h || !coords || !out) return NDT_INVALID_ARGUMENT;
  return guarded_int(NDT_SHAPE_MISMATCH, [&]() {
    const BlockSparseT& t = ((const NdtBs*)h)->t;
    std::vector<size_t> c(coords, coords + t.ndim());
    long b = t.find(c);
    if (b < 0) return NDT_INDEX_OUT_OF_BOUNDS;
    if (len < t.block_elems(c)) return NDT_SHAPE_MISMATCH;
    const double* host = (const double*)t.st->host_read();
    memcpy(out, host + t.offs[b] * (esize(t.dt) / 8), t.block_elems(c) * esize(t.dt));
    return NDT_SUCCESS;
  });
}

int bs_structure(const void* h, size_t* nblocks, size_t* block_sizes, size_t* coords, size_t* offsets) {
  if (!h) return NDT_INVALID_ARGUMENT;
  const BlockSparseT& t = ((const NdtBs*)h)->t;
  size_t k = 0;
  for (size_t i = 0; i < t.ndim(); i++) {
    if (nblocks) nblocks[i] = t.bsz[i].size();
    for (size_t x : t.bsz[i]) {
      if (block_sizes) block_sizes[k] = x;
      k++;
    }
  }
  for (size_t b = 0; b < t.nnzb(); b++) {
    for (size_t i = 0; i < t.ndim(); i++)
      if (coords) coords[b * t.ndim() + i] = t.coords[b][i];
    if (offsets) offsets[b] = t.offs[b];
  }
  return NDT_SUCCESS;
}

}  // namespace

extern "C" {

#define NDT_BS_COMMON(T, DT)                                                                                           \
  T* ndt_blocksparse_##DT##_zeros(size_t ndim, const size_t* nblocks, const size_t* block_sizes, size_t nnzb,         \
                                  const size_t* coords, int* status) {                                               \
    return (T*)bs_new(DTYPE_##DT, ndim, nblocks, block_sizes, nnzb, coords, nullptr, 0, status);                     \
  }                                                                                                                  \
  T* ndt_blocksparse_##DT##_from_data(size_t ndim, const size_t* nblocks, const size_t* block_sizes, size_t nnzb,    \
                                      const size_t* coords, const double* data, size_t len, int* status) {           \
    if (!data) {                                                                                                     \
      if (status) *status = NDT_INVALID_ARGUMENT;                                                                    \
      return nullptr;                                                                                                \
    }                                                                                                                \
    return (T*)bs_new(DTYPE_##DT, ndim, nblocks, block_sizes, nnzb, coords, data, len, status);                      \
  }                                                                                                                  \
  T* ndt_blocksparse_##DT##_from_device_ptr(size_t ndim, const size_t* nblocks, const size_t* block_sizes,           \
                                            size_t nnzb, const size_t* coords, const double* dptr, size_t len,       \
                                            int* status) {                                                           \
    return (T*)guarded(status, NDT_SHAPE_MISMATCH, [&]() -> void* {                                                  \
      if (!dptr) throw Error(ErrKind::InvalidArgument, "NULL device pointer");                                       \
      std::vector<std::vector<size_t>> bsz, cs;                                                                      \
      read_structure(ndim, nblocks, block_sizes, nnzb, coords, &bsz, &cs);                                           \
      BlockSparseT t = make_bs(DTYPE_##DT, bsz, cs);                                                                 \
      if (len != t.total()) throw Error(ErrKind::ShapeMismatch, "data length != total block elements");              \
      if (len) t.st = make_from_device(DTYPE_##DT, dptr, len, {len}).st;                                             \
      return new NdtBs{t};                                                                                           \
    });                                                                                                              \
  }                                                                                                                  \
  T* ndt_blocksparse_##DT##_from_device_blocks(size_t ndim, const size_t* nblocks, const size_t* block_sizes,        \
                                               size_t nnzb, const size_t* coords, const size_t* src_offsets,         \
                                               const double* src, size_t src_len, int* status) {                    \
    return (T*)guarded(status, NDT_SHAPE_MISMATCH, [&]() -> void* {                                                  \
      if (nnzb && (!src || !src_offsets)) throw Error(ErrKind::InvalidArgument, "NULL device pointer or offsets");   \
      std::vector<std::vector<size_t>> bsz, cs;                                                                      \
      read_structure(ndim, nblocks, block_sizes, nnzb, coords, &bsz, &cs);                                           \
      return new NdtBs{bs_from_device_blocks(DTYPE_##DT, bsz, cs, src_offsets, src, src_len)};                       \
    });                                                                                                              \
  }                                                                                                                  \
  int ndt_blocksparse_##DT##_shard_layout(const T* t, int* nranks, size_t* nblocks, size_t* coords, int* owners) {   \
    if (!t || !nranks || !nblocks) return NDT_INVALID_ARGUMENT;                                                      \
    const BlockSparseT& b = ((const NdtBs*)t)->t;                                                                    \
    if (!b.layout) return NDT_INVALID_ARGUMENT;                                                                      \
    *nranks = b.layout->nranks;                                                                                      \
    *nblocks = b.layout->coords.size();                                                                              \
    const size_t nd = b.ndim();                                                                                      \
    for (size_t i = 0; i < b.layout->coords.size(); i++) {                                                           \
      if (coords)                                                                                                    \
        for (size_t a = 0; a < nd; a++) coords[i * nd + a] = b.layout->coords[i][a];                                 \
      if (owners) owners[i] = b.layout->owner[i];                                                                    \
    }                                                                                                                \
    return NDT_SUCCESS;                                                                                              \
  }                                                                                                                  \
  void ndt_blocksparse_##DT##_release(T* t) { delete (NdtBs*)t; }                                                    \
  size_t ndt_blocksparse_##DT##_ndim(const T* t) { return t ? ((const NdtBs*)t)->t.ndim() : 0; }                     \
  size_t ndt_blocksparse_##DT##_nnzblocks(const T* t) { return t ? ((const NdtBs*)t)->t.nnzb() : 0; }                \
  size_t ndt_blocksparse_##DT##_nnz(const T* t) { return t ? ((const NdtBs*)t)->t.total() : 0; }                     \
  size_t ndt_blocksparse_##DT##_nblocks_total(const T* t) {                                                          \
    if (!t) return 0;                                                                                                \
    size_t s = 0;                                                                                                    \
    for (auto& v : ((const NdtBs*)t)->t.bsz) s += v.size();                                                          \
    return s;                                                                                                        \
  }                                                                                                                  \
  int ndt_blocksparse_##DT##_structure(const T* t, size_t* nblocks, size_t* block_sizes, size_t* coords,             \
                                       size_t* offsets) {                                                            \
    return bs_structure(t, nblocks, block_sizes, coords, offsets);                                                   \
  }                                                                                                                  \
  int ndt_blocksparse_##DT##_insert_block(T* t, const size_t* coords, const double* data, size_t len) {              \
    return bs_insert(t, coords, data, len);                                                                          \
  }                                                                                                                  \
  int ndt_blocksparse_##DT##_get_block(const T* t, const size_t* coords, double* out, size_t len) {                  \
    return bs_get(t, coords, out, len);                                                                              \
  }                                                                                                                  \
  const double* ndt_blocksparse_##DT##_data(const T* t) {                                                            \
    if (!t) return nullptr;                                                                                          \
    try {                                                                                                            \
      return (const double*)((const NdtBs*)t)->t.st->host_read();                                                    \
    } catch (const std::exception& e) {                                                                              \
      set_last_error(e.what());                                                                                      \
      return nullptr;                                                                                                \
    }                                                                                                                \
  }                                                                                                                  \
  const double* ndt_blocksparse_##DT##_device_ptr(const T* t) {                                                      \
    if (!t) return nullptr;                                                                                          \
    try {                                                                                                            \
      Storage& st = *((const NdtBs*)t)->t.st;                                                                        \
      const double* p = (const double*)st.dev_read();                                                                \
      settle_for_caller(st.device);                                                                                  \
      return p;                                                                                                      \
    } catch (const std::exception& e) {                                                                              \
      set_last_error(e.what());                                                                                      \
      return nullptr;                                                                                                \
    }                                                                                                                \
  }                                                                                                                  \
  double* ndt_blocksparse_##DT##_device_ptr_mut(T* t) {                                                              \
    if (!t) return nullptr;                                                                                          \
    try {                                                                                                            \
      BlockSparseT& b = ((NdtBs*)t)->t;                                                                              \
      if (b.st.use_count() > 1) b.st = b.st->clone(); /* copy on write */                                            \
      double* p = (double*)b.st->dev_write();                                                                        \
      settle_for_caller(b.st->device);                                                                               \
      return p;                                                                                                      \
    } catch (const std::exception& e) {                                                                              \
      set_last_error(e.what());                                                                                      \
      return nullptr;                                                                                                \
    }                                                                                                                \
  }                                                                                                                  \
  T* ndt_blocksparse_##DT##_contract(const T* a, const long* la, size_t na, const T* b, const long* lb, size_t nb,   \
                                     int* status) {                                                                  \
    if (!status) return nullptr;                                                                                     \
    if (!a || !b || (!la && na) || (!lb && nb)) {                                                                    \
      *status = NDT_INVALID_ARGUMENT;                                                                                \
      return nullptr;                                                                                                \
    }                                                                                                                \
    return (T*)guarded(status, NDT_SHAPE_MISMATCH, [&]() -> void* {                                                  \
      return new NdtBs{bs_contract(((const NdtBs*)a)->t, labels(la, na), ((const NdtBs*)b)->t, labels(lb, nb), 0, 1)}; \
    });                                                                                                              \
  }                                                                                                                  \
  T* ndt_blocksparse_##DT##_contract_shard(const T* a, const long* la, size_t na, const T* b, const long* lb,        \
                                           size_t nb, int rank, int nranks, int* status) {                           \
    if (!status) return nullptr;                                                                                     \
    if (!a || !b || (!la && na) || (!lb && nb) || nranks < 1 || rank < 0 || rank >= nranks) {                        \
      *status = NDT_INVALID_ARGUMENT;                                                                                \
      return nullptr;                                                                                                \
    }                                                                                                                \
    return (T*)guarded(status, NDT_SHAPE_MISMATCH, [&]() -> void* {                                                  \
      return new NdtBs{                                                                                              \
          bs_contract(((const NdtBs*)a)->t, labels(la, na), ((const NdtBs*)b)->t, labels(lb, nb), rank, nranks)};    \
    });                                                                                                              \
  }                                                                                                                  \
  T* ndt_blocksparse_##DT##_contract_select(const T* a, const long* la, size_t na, const T* b, const long* lb,       \
                                            size_t nb, const size_t* out_coords, size_t nout, int* status) {        \
    if (!status) return nullptr;                                                                                     \
    if (!a || !b || (!la && na) || (!lb && nb) || (!out_coords && nout)) {                                          \
      *status = NDT_INVALID_ARGUMENT;                                                                                \
      return nullptr;                                                                                                \
    }                                                                                                                \
    return (T*)guarded(status, NDT_SHAPE_MISMATCH, [&]() -> void* {                                                  \
      static const size_t none = 0;                                                                                  \
      return new NdtBs{bs_contract(((const NdtBs*)a)->t, labels(la, na), ((const NdtBs*)b)->t, labels(lb, nb), 0,  \
                                   1, nullptr, nout ? out_coords : &none, nout)};                                    \
    });                                                                                                              \
  }                                                                                                                  \
  T* ndt_blocksparse_##DT##_permutedims(const T* a, const size_t* perm, size_t nperm, int* status) {                 \
    if (!status) return nullptr;                                                                                     \
    if (!a || (!perm && nperm)) {                                                                                    \
      *status = NDT_INVALID_ARGUMENT;                                                                                \
      return nullptr;                                                                                                \
    }                                                                                                                \
    return (T*)guarded(status, NDT_INVALID_PERMUTATION, [&]() -> void* {                                             \
      return new NdtBs{bs_permutedims(((const NdtBs*)a)->t, std::vector<size_t>(perm, perm + nperm))};               \
    });                                                                                                              \
  }

#define DTYPE_f64 DType::F64
#define DTYPE_c64 DType::C128
NDT_BS_COMMON(ndt_blocksparse_f64, f64)
NDT_BS_COMMON(ndt_blocksparse_c64, c64)

// Host-only planning of the sharded contraction: output blocks and real
// flops per rank (no device work).
#define NDT_BS_PLAN(T, DT)                                                                                          \
  int ndt_blocksparse_##DT##_shard_plan(const T* a, const long* la, size_t na, const T* b, const long* lb,         \
                                        size_t nb, int nranks, size_t* blocks_per_rank, double* flops_per_rank) {   \
    if (!a || !b || (!la && na) || (!lb && nb) || nranks < 1) return NDT_INVALID_ARGUMENT;                         \
    return guarded_int(NDT_SHAPE_MISMATCH, [&]() {                                                                 \
      ShardPlan p;                                                                                                 \
      bs_contract(((const NdtBs*)a)->t, labels(la, na), ((const NdtBs*)b)->t, labels(lb, nb), 0, nranks, &p);      \
      for (int r = 0; r < nranks; r++) {                                                                           \
        if (blocks_per_rank) blocks_per_rank[r] = p.blocks[r];                                                     \
        if (flops_per_rank) flops_per_rank[r] = p.flops[r];                                                        \
      }                                                                                                            \
      return NDT_SUCCESS;                                                                                          \
    });                                                                                                            \
  }
NDT_BS_PLAN(ndt_blocksparse_f64, f64)
NDT_BS_PLAN(ndt_blocksparse_c64, c64)

ndt_tensor_f64* ndt_blocksparse_f64_to_dense(const ndt_blocksparse_f64* a, int* status) {
  if (status && !a) {
    *status = NDT_INVALID_ARGUMENT;
    return nullptr;
  }
  return (ndt_tensor_f64*)guarded(status, NDT_SHAPE_MISMATCH,
                                  [&]() -> void* { return new NdtHandle{bs_to_dense(((const NdtBs*)a)->t)}; });
}
ndt_tensor_c64* ndt_blocksparse_c64_to_dense(const ndt_blocksparse_c64* a, int* status) {
  if (status && !a) {
    *status = NDT_INVALID_ARGUMENT;
    return nullptr;
  }
  return (ndt_tensor_c64*)guarded(status, NDT_SHAPE_MISMATCH,
                                  [&]() -> void* { return new NdtHandle{bs_to_dense(((const NdtBs*)a)->t)}; });
}

#define NDT_BS_FROM_DENSE(T, TD, DT)                                                                                  \
  T* ndt_blocksparse_##DT##_from_dense(const TD* dense, size_t ndim, const size_t* nblocks, const size_t* block_sizes, \
                                       size_t nnzb, const size_t* coords, int* status) {                              \
    if (status && !dense) {                                                                                           \
      *status = NDT_INVALID_ARGUMENT;                                                                                 \
      return nullptr;                                                                                                 \
    }                                                                                                                 \
    return (T*)guarded(status, NDT_SHAPE_MISMATCH, [&]() -> void* {                                                   \
      std::vector<std::vector<size_t>> bsz, cs;                                                                       \
      read_structure(ndim, nblocks, block_sizes, nnzb, coords, &bsz, &cs);                                            \
      const Dense& d = ((const NdtHandle*)dense)->t;                                                             \
      if (d.dt != DTYPE_##DT) throw Error(ErrKind::InvalidArgument, "element type mismatch");                         \
      return new NdtBs{bs_from_dense(d, bsz, cs)};                                                                    \
    });                                                                                                               \
  }
NDT_BS_FROM_DENSE(ndt_blocksparse_f64, ndt_tensor_f64, f64)
NDT_BS_FROM_DENSE(ndt_blocksparse_c64, ndt_tensor_c64, c64)

// ---- diag-block-sparse
#define NDT_DIAG(T, TD, TB, DT)                                                                                         \
  T* ndt_diagblocksparse_##DT##_from_data(size_t ndim, const size_t* nblocks, const size_t* block_sizes, size_t nnzb,  \
                                          const size_t* coords, const double* diag, size_t len, int* status) {          \
    return (T*)guarded(status, NDT_SHAPE_MISMATCH, [&]() -> void* {                                                     \
      if (!diag) throw Error(ErrKind::InvalidArgument, "NULL data");                                                    \
      std::vector<std::vector<size_t>> bsz, cs;                                                                         \
      read_structure(ndim, nblocks, block_sizes, nnzb, coords, &bsz, &cs);                                              \
      DiagBlockSparseT S = make_diag(DTYPE_##DT, bsz, cs);                                                              \
      if (len != S.s.total()) throw Error(ErrKind::ShapeMismatch, "diag length != total diagonal elements");            \
      if (len) S.s.st = make_from_host(DTYPE_##DT, diag, len, {len}).st;                                                \
      if (DTYPE_##DT == DType::C128)                                                                                    \
        for (size_t i = 0; i < len && S.real_valued; i++) S.real_valued = diag[2 * i + 1] == 0.0;                       \
      return new NdtDiag{S};                                                                                            \
    });                                                                                                                 \
  }                                                                                                                     \
  void ndt_diagblocksparse_##DT##_release(T* t) { delete (NdtDiag*)t; }                                                 \
  size_t ndt_diagblocksparse_##DT##_nnz(const T* t) { return t ? ((const NdtDiag*)t)->t.s.total() : 0; }                \
  TD* ndt_diagblocksparse_##DT##_to_dense(const T* s, int* status) {                                                    \
    if (status && !s) {                                                                                                 \
      *status = NDT_INVALID_ARGUMENT;                                                                                   \
      return nullptr;                                                                                                   \
    }                                                                                                                   \
    return (TD*)guarded(status, NDT_SHAPE_MISMATCH,                                                                     \
                        [&]() -> void* { return new NdtHandle{diag_to_dense(((const NdtDiag*)s)->t)}; });          \
  }                                                                                                                     \
  TB* ndt_diagblocksparse_##DT##_to_blocksparse(const T* s, int* status) {                                              \
    if (status && !s) {                                                                                                 \
      *status = NDT_INVALID_ARGUMENT;                                                                                   \
      return nullptr;                                                                                                   \
    }                                                                                                                   \
    return (TB*)guarded(status, NDT_SHAPE_MISMATCH,                                                                     \
                        [&]() -> void* { return new NdtBs{diag_to_blocksparse(((const NdtDiag*)s)->t)}; });             \
  }                                                                                                                     \
  TB* ndt_blocksparse_##DT##_contract_diag(const TB* a, const long* la, size_t na, const T* s, const long* ls,          \
                                           size_t ns, int* status) {                                                    \
    if (!status) return nullptr;                                                                                        \
    if (!a || !s || (!la && na) || (!ls && ns)) {                                                                       \
      *status = NDT_INVALID_ARGUMENT;                                                                                   \
      return nullptr;                                                                                                   \
    }                                                                                                                   \
    return (TB*)guarded(status, NDT_SHAPE_MISMATCH, [&]() -> void* {                                                    \
      return new NdtBs{bs_contract_diag(((const NdtBs*)a)->t, labels(la, na), ((const NdtDiag*)s)->t, labels(ls, ns))}; \
    });                                                                                                                 \
  }                                                                                                                     \
  TB* ndt_blocksparse_##DT##_contract_through_diag(const TB* a, const long* la, size_t na, const T* s, const long* ls,  \
                                                   size_t ns, const TB* b, const long* lb, size_t nb, int rank,         \
                                                   int nranks, int* status) {                                          \
    if (!status) return nullptr;                                                                                        \
    if (!a || !s || !b || (!la && na) || (!ls && ns) || (!lb && nb) || nranks < 1 || rank < 0 || rank >= nranks) {     \
      *status = NDT_INVALID_ARGUMENT;                                                                                   \
      return nullptr;                                                                                                   \
    }                                                                                                                   \
    return (TB*)guarded(status, NDT_SHAPE_MISMATCH, [&]() -> void* {                                                    \
      return new NdtBs{bs_contract_through_diag(((const NdtBs*)a)->t, labels(la, na), ((const NdtDiag*)s)->t,           \
                                                labels(ls, ns), ((const NdtBs*)b)->t, labels(lb, nb), rank, nranks)};   \
    });                                                                                                                 \
  }
NDT_DIAG(ndt_diagblocksparse_f64, ndt_tensor_f64, ndt_blocksparse_f64, f64)
NDT_DIAG(ndt_diagblocksparse_c64, ndt_tensor_c64, ndt_blocksparse_c64, c64)

// Gathered multi-GPU contractions over an ndt_comm (comm.cpp).
#define NDT_GATHER(TB, TD, DT)                                                                                          \
  TB* ndt_blocksparse_##DT##_contract_gathered(const TB* a, const long* la, size_t na, const TB* b, const long* lb,   \
                                               size_t nb, ndt_comm* comm, int* status) {                               \
    if (!status) return nullptr;                                                                                        \
    if (!a || !b || !comm || (!la && na) || (!lb && nb)) {                                                              \
      *status = NDT_INVALID_ARGUMENT;                                                                                   \
      return nullptr;                                                                                                   \
    }                                                                                                                   \
    return (TB*)guarded(status, NDT_SHAPE_MISMATCH, [&]() -> void* {                                                    \
      return new NdtBs{bs_contract(((const NdtBs*)a)->t, labels(la, na), ((const NdtBs*)b)->t, labels(lb, nb), 0, 1,   \
                                   nullptr, nullptr, 0, nullptr, &comm_of(comm))};                                      \
    });                                                                                                                 \
  }                                                                                                                     \
  TB* ndt_blocksparse_##DT##_contract_through_diag_gathered(const TB* a, const long* la, size_t na, const TD* s,       \
                                                            const long* ls, size_t ns, const TB* b, const long* lb,     \
                                                            size_t nb, ndt_comm* comm, int* status) {                   \
    if (!status) return nullptr;                                                                                        \
    if (!a || !s || !b || !comm || (!la && na) || (!ls && ns) || (!lb && nb)) {                                         \
      *status = NDT_INVALID_ARGUMENT;                                                                                   \
      return nullptr;                                                                                                   \
    }                                                                                                                   \
    return (TB*)guarded(status, NDT_SHAPE_MISMATCH, [&]() -> void* {                                                    \
      return new NdtBs{bs_contract_through_diag(((const NdtBs*)a)->t, labels(la, na), ((const NdtDiag*)s)->t,           \
                                                labels(ls, ns), ((const NdtBs*)b)->t, labels(lb, nb), 0, 1,             \
                                                &comm_of(comm))};                                                       \
    });                                                                                                                 \
  }                                                                                                                     \
  TB* ndt_blocksparse_##DT##_allgather(const TB* shard, ndt_comm* comm, int* status) {                                \
    if (!status) return nullptr;                                                                                        \
    if (!shard || !comm) {                                                                                              \
      *status = NDT_INVALID_ARGUMENT;                                                                                   \
      return nullptr;                                                                                                   \
    }                                                                                                                   \
    return (TB*)guarded(status, NDT_SHAPE_MISMATCH,                                                                     \
                        [&]() -> void* { return new NdtBs{bs_allgather(((const NdtBs*)shard)->t, comm_of(comm))}; });  \
  }
NDT_GATHER(ndt_blocksparse_f64, ndt_diagblocksparse_f64, f64)
NDT_GATHER(ndt_blocksparse_c64, ndt_diagblocksparse_c64, c64)

}  // extern "C"
