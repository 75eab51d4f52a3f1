// Dense f64 contraction that allocates nothing.
//
// Some callers cannot call cudaMalloc: code running inside a runtime that
// forbids allocation on its hot path, plugins hosted by an application that
// owns the device memory budget, or real-time loops where an allocation (and
// its implicit synchronisation) is not allowed.  For
// them this file provides ndt_b200_contract_f64_noalloc: the same contraction
// as ndt_tensor_f64_contract (the reference's naive-loop label semantics:
// output axes are A's positive labels then B's, unmatched negative labels are
// pinned at index 0, a scalar result has shape [1]), on caller-owned device
// buffers.  Operands that have to be packed before the FP64 tensor-core GEMM
// are packed into the fixed scratch array below instead of pool memory, and
// the GEMM always runs as one launch (never split along k, which would need a
// workspace for the partial sums).
//
// Scratch: g_noalloc_scratch, kNoAllocScratchBytes (16 MiB) per device, held
// by every GPU that loads the library until the process exits.  Requests that
// would need more are rejected with NDT_INVALID_ARGUMENT and a message.  All
// calls share the array and nothing in it survives usefully between calls:
// every byte a call reads was written earlier in the same call, so nothing
// needs clearing; calls that overlap on the GPU (different streams, or
// threads) race on it.
#include <algorithm>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/ndtensors_capi.h"
#include "ndt_internal.h"

using namespace ndt;

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device.  In host code the symbol
// is only a host-side stand-in; the address is looked up once per device,
// with that device current, at the first call on it.
std::mutex g_mu;
void* g_addr[64] = {nullptr};

void* scratch_address(int device) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (device < 0 || device >= 64) throw Error(ErrKind::InvalidArgument, "device index out of range");
  if (!g_addr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) throw_cuda(e, "cudaGetSymbolAddress(g_noalloc_scratch)", __FILE__, __LINE__);
    g_addr[device] = p;
  }
  return g_addr[device];
}

struct Ax1 {
  int64_t n, s;
};

// Collapse an ordered (fastest first) list of axes into one strided axis.
bool merge(const std::vector<Ax1>& v, int64_t* stride, bool* empty) {
  *empty = true;
  int64_t st = 1, ext = 1;
  bool ok = true;
  for (const Ax1& a : v) {
    if (a.n == 1) continue;
    if (*empty) {
      *empty = false;
      st = a.s;
      ext = a.n;
      continue;
    }
    if (a.s != st * ext) ok = false;
    ext *= a.n;
  }
  *stride = st;
  return ok;
}

// How one operand reaches the GEMM: read in place when its axes form a
// unit-stride strided matrix (either orientation), else packed.
struct Layout {
  bool pack;
  bool kmajor;
  int64_t ld;
};
Layout layout(const std::vector<Ax1>& rows, const std::vector<Ax1>& cols, int64_t r_ext, int64_t c_ext) {
  int64_t rs, cs;
  bool re, ce;
  bool rok = merge(rows, &rs, &re), cok = merge(cols, &cs, &ce);
  if (rok && cok && (re || rs == 1)) return Layout{false, false, ce ? std::max<int64_t>(r_ext, 1) : cs};
  if (rok && cok && (ce || cs == 1)) return Layout{false, true, re ? std::max<int64_t>(c_ext, 1) : rs};
  return Layout{true, false, std::max<int64_t>(r_ext, 1)};
}

// Describe one operand for the GEMM, packing it into `scratch` when its
// layout says so.  `rows` are the M (or N) axes.
GemmOperand operand(const double* base, const std::vector<Ax1>& rows, const std::vector<Ax1>& cols,
                    const Layout& L, double* scratch, cudaStream_t s) {
  if (!L.pack) return GemmOperand{base, L.ld, L.kmajor};
  GatherDesc g;
  for (const Ax1& a : rows) {
    g.shape.push_back((size_t)a.n);
    g.src_strides.push_back(a.s);
  }
  for (const Ax1& a : cols) {
    g.shape.push_back((size_t)a.n);
    g.src_strides.push_back(a.s);
  }
  if (g.shape.empty()) {
    NDT_CUDA(cudaMemcpyAsync(scratch, base, sizeof(double), cudaMemcpyDeviceToDevice, s));
  } else {
    gather(DType::F64, base, scratch, g, s);
  }
  return GemmOperand{scratch, L.ld, false};
}

}  // namespace

extern "C" int ndt_b200_contract_f64_noalloc(const double* a, const size_t* shape_a, size_t ndim_a,
                                             const long* labels_a, const double* b, const size_t* shape_b,
                                             size_t ndim_b, const long* labels_b, double* c, size_t c_len,
                                             size_t* out_shape, size_t* out_ndim, void* stream) {
  if (!a || !b || !c || (!shape_a && ndim_a) || (!shape_b && ndim_b) || (!labels_a && ndim_a) ||
      (!labels_b && ndim_b))
    return NDT_INVALID_ARGUMENT;
  try {
    const int dev = current_device();
    ctx(dev);  // per-device context (streams, SM count) on the first call
    double* scratch = (double*)scratch_address(dev);
    cudaStream_t s = (cudaStream_t)stream;
    std::vector<size_t> sa(shape_a, shape_a + ndim_a), sb(shape_b, shape_b + ndim_b);
    // Zero extents: the reference panics (linear_to_cartesian divides by them).
    for (size_t x : sa)
      if (x == 0) {
        set_last_error("ndt_b200_contract_f64_noalloc: A has a zero extent");
        return NDT_INTERNAL_ERROR;
      }
    for (size_t x : sb)
      if (x == 0) {
        set_last_error("ndt_b200_contract_f64_noalloc: B has a zero extent");
        return NDT_INTERNAL_ERROR;
      }
    std::vector<int32_t> la(ndim_a), lb(ndim_b);
    for (size_t i = 0; i < ndim_a; i++) la[i] = (int32_t)labels_a[i];
    for (size_t j = 0; j < ndim_b; j++) lb[j] = (int32_t)labels_b[j];
    // Label pairing as in contract/naive.rs:66-83 (first match in B wins).
    std::vector<std::pair<size_t, size_t>> pairs;
    for (size_t i = 0; i < ndim_a; i++) {
      if (la[i] >= 0) continue;
      for (size_t j = 0; j < ndim_b; j++)
        if (la[i] == lb[j]) {
          if (sa[i] != sb[j]) {
            set_last_error("ndt_b200_contract_f64_noalloc: contracted extents differ for label " +
                           std::to_string(la[i]));
            return NDT_SHAPE_MISMATCH;
          }
          pairs.push_back({i, j});
          break;
        }
    }
    std::vector<size_t> oshape;
    std::vector<Ax1> M, N, KA, KB;
    std::vector<size_t> stra = col_major_strides(sa), strb = col_major_strides(sb);
    for (size_t i = 0; i < ndim_a; i++)
      if (la[i] > 0) {
        oshape.push_back(sa[i]);
        M.push_back({(int64_t)sa[i], (int64_t)stra[i]});
      }
    for (size_t j = 0; j < ndim_b; j++)
      if (lb[j] > 0) {
        oshape.push_back(sb[j]);
        N.push_back({(int64_t)sb[j], (int64_t)strb[j]});
      }
    if (oshape.empty()) oshape.push_back(1);
    std::vector<long> cpa(ndim_a, -1), cpb(ndim_b, -1);
    for (size_t p = 0; p < pairs.size(); p++) {
      if (cpa[pairs[p].first] < 0) cpa[pairs[p].first] = (long)p;
      if (cpb[pairs[p].second] < 0) cpb[pairs[p].second] = (long)p;
    }
    for (size_t p = 0; p < pairs.size(); p++) {
      size_t i = pairs[p].first, j = pairs[p].second;
      KA.push_back({(int64_t)sa[i], cpa[i] == (long)p ? (int64_t)stra[i] : 0});
      KB.push_back({(int64_t)sa[i], cpb[j] == (long)p ? (int64_t)strb[j] : 0});
    }
    int64_t m = 1, n = 1, k = 1;
    for (auto& x : M) m *= x.n;
    for (auto& x : N) n *= x.n;
    for (auto& x : KA) k *= x.n;
    if ((size_t)(m * n) > c_len) {
      set_last_error("output buffer too small for the contraction result");
      return NDT_INVALID_ARGUMENT;
    }
    // Scratch: only the operands that are packed use it, A's part first,
    // then B's at the next 256-byte boundary.
    const Layout lay_a = layout(M, KA, m, k), lay_b = layout(N, KB, n, k);
    const size_t bytes_a = lay_a.pack ? ((size_t)(m * k) * sizeof(double) + 255) / 256 * 256 : 0;
    const size_t need = bytes_a + (lay_b.pack ? (size_t)(k * n) * sizeof(double) : 0);
    if (need > kNoAllocScratchBytes) {
      char msg[256];
      snprintf(msg, sizeof(msg),
               "ndt_b200_contract_f64_noalloc: packing the operands needs %zu bytes of scratch, more than the "
               "fixed %zu bytes this entry point holds; use ndt_tensor_f64_contract",
               need, kNoAllocScratchBytes);
      set_last_error(msg);
      return NDT_INVALID_ARGUMENT;
    }
    if (out_ndim) *out_ndim = oshape.size();
    if (out_shape)
      for (size_t i = 0; i < oshape.size(); i++) out_shape[i] = oshape[i];
    double* scr_a = scratch;
    double* scr_b = (double*)((unsigned char*)scratch + bytes_a);
    GemmOperand ga = operand(a, M, KA, lay_a, scr_a, s);
    GemmOperand gb = operand(b, N, KB, lay_b, scr_b, s);
    // No split-K: its partial sums would need a workspace from the pool.
    gemm(DType::F64, m, n, k, ga, gb, c, std::max<int64_t>(m, 1), false, s, /*allow_split_k=*/false);
    return NDT_SUCCESS;
  } catch (const Error& e) {
    set_last_error(e.what());
    return (e.kind == ErrKind::InvalidArgument) ? NDT_INVALID_ARGUMENT : NDT_INTERNAL_ERROR;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return NDT_INTERNAL_ERROR;
  }
}
