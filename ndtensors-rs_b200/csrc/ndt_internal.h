// Internal declarations of the B200 ndtensors library (libndtensors_capi.so).
//
// Layout of the library:
//   device.cpp       per-device context: compute / upload streams, stream-ordered
//                    device pool, pinned host cache, last-error text
//   tensor.cpp       Storage (device buffer + lazily synced host mirror, copy on
//                    write) and the dense tensor value type
//   capi_dense.cpp   ndt_tensor_f64_* (the reference's C ABI) and ndt_tensor_c64_*
//   permute.cu       strided gather / permutedims kernels and their planner
//   gemm.cu          FP64 tensor-core (DMMA) GEMM: dense (with split-K) and
//                    grouped, f64 and c128
//   skinny.cu        contractions with a short contracted and a short free
//                    extent (strided operand reads, DMMA)
//   contract.cpp     label planning (naive ABI semantics and TTGT semantics),
//                    contraction driver, VJP / JVP compositions
//   contract_noalloc.cu  the allocation-free contraction entry point
//   elementwise.cu   fill, add, scale, split-K sums
//   blocksparse.cpp  block-sparse and diag-block-sparse tensors, block-pair
//                    table, grouped contraction, sharding, ABI exports
//   blocksparse_kernels.cu  block-sparse <-> dense maps, diagonal placement
//                    and scaling
//   fp64_peak.cu     FP64 tensor peak microbenchmark (its own library, for
//                    the bench's roofline)
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace ndt {

// ---------------------------------------------------------------- errors
// Error kinds mirror the reference's TensorError variants plus a "panic"
// kind for the places where the reference panics (its C ABI's catch_unwind
// maps those to NDT_INTERNAL_ERROR).  Each ABI entry point maps kinds onto
// status codes exactly as crates/ndtensors-capi/src/lib.rs does.
enum class ErrKind {
  WrongNumberOfIndices,
  ShapeMismatch,
  InvalidPermutation,
  BlockNotFound,
  IndexOutOfBounds,
  InvalidArgument,
  Panic,  // reference would panic (division by zero extent, failed assert, ...)
  Cuda,   // CUDA runtime failure or no device
};

struct Error : std::runtime_error {
  ErrKind kind;
  Error(ErrKind k, const std::string& m) : std::runtime_error(m), kind(k) {}
};

[[noreturn]] void throw_cuda(cudaError_t e, const char* what, const char* file, int line);
#define NDT_CUDA(x)                                                   \
  do {                                                                \
    cudaError_t _e = (x);                                             \
    if (_e != cudaSuccess) ::ndt::throw_cuda(_e, #x, __FILE__, __LINE__); \
  } while (0)

void set_last_error(const std::string& msg);
const char* last_error();

// ----------------------------------------------------------------- dtypes
enum class DType : int { F64 = 0, C128 = 1 };
inline size_t esize(DType t) { return t == DType::F64 ? 8 : 16; }

// --------------------------------------------------------------- devices
bool device_available();
int current_device();  // throws ErrKind::Cuda when no device is present
struct DeviceCtx {
  int device = -1;
  cudaStream_t compute = nullptr;  // all kernels of the library
  cudaStream_t own_compute = nullptr;  // the library's own compute stream
  cudaStream_t upload = nullptr;   // host->device copies of caller data
  cudaStream_t download = nullptr; // device->host reads of results
  bool external_stream = false;    // compute stream supplied by the caller
  int sm_count = 0;
  size_t smem_optin = 0;
  std::atomic<bool> pool_tuned{false};  // default pool's release threshold raised
};
DeviceCtx& ctx(int device);
DeviceCtx& ctx();  // current device
// A tensor's device buffer is being handed to a caller (device_ptr /
// device_ptr_mut), or a caller's buffer has just been copied in
// (from_device_ptr).  On the library's own stream, wait for it, so that the
// caller's reads and writes, on any stream, see the tensor's values, are not
// overtaken by a fill, upload or kernel still pending for that buffer, and a
// source buffer may be reused at once.  A caller stream installed with
// ndt_b200_set_stream already orders them.
void settle_for_caller(int device);
// Device memory: stream-ordered allocations from the device's default pool
// (release threshold raised so freed blocks are reused, not returned).
void* dev_alloc(size_t bytes, int device);
// A stream-ordered allocation on stream `s` from the current device's pool.
void* pool_alloc(size_t bytes, cudaStream_t s);
void dev_free(void* p, int device);
// Pinned host memory with a size-bucketed cache (host mirrors, staging).
void* pinned_alloc(size_t bytes, bool* pinned);
void pinned_free(void* p, size_t bytes, bool pinned);
void empty_caches();
// Allow `func` (a __global__ function) up to `bytes` of dynamic shared
// memory on the current device.  The attribute is per device and per
// function, so it is set once for each (device, function) and raised when a
// launch needs more.  Thread safe.
void ensure_dynamic_smem(const void* func, size_t bytes);

// ---------------------------------------------------------------- storage
// One buffer of `len` elements.  The device buffer is authoritative once a
// device op has produced it; the host mirror is filled on demand (data(),
// get_linear) and stays valid until the next mutation.  A storage can also be
// "uniform": every element equal to `fill` and nothing materialised yet
// (zeros / ones / fill are lazy).
struct Storage {
  DType dt;
  size_t len = 0;  // elements (max(1, prod(shape)) for dense tensors)
  int device = -1;
  void* dev = nullptr;
  void* host = nullptr;
  bool host_pinned = false;
  bool dev_valid = false;
  bool host_valid = false;
  bool host_external = false;  // a mutable host pointer was handed out
  bool uniform = false;        // all elements == fill, not materialised
  double fill_re = 0.0, fill_im = 0.0;

  Storage(DType t, size_t n) : dt(t), len(n) {}
  ~Storage();
  Storage(const Storage&) = delete;
  Storage& operator=(const Storage&) = delete;

  size_t bytes() const { return len * esize(dt); }
  // Host view: materialises and downloads as needed.
  void* host_read();
  // Host view for mutation: invalidates the device copy.
  void* host_write();
  // Device view for reading by a kernel on the compute stream.
  const void* dev_read();
  // Device view for a kernel that overwrites every element.
  void* dev_overwrite();
  // Device view for writes from outside the library (any subset of the
  // elements): materialised, then the device copy is the only valid one.
  void* dev_write();
  void set_uniform(double re, double im);
  std::shared_ptr<Storage> clone() const;
};

struct Dense {
  DType dt = DType::F64;
  std::vector<size_t> shape;
  std::shared_ptr<Storage> st;
  size_t len() const { return st ? st->len : 0; }
  size_t ndim() const { return shape.size(); }
  void make_unique();  // copy on write (Rc::make_mut)
};

size_t prod(const std::vector<size_t>& v);
size_t prod_max1(const std::vector<size_t>& v);
std::vector<size_t> col_major_strides(const std::vector<size_t>& shape);

Dense make_uniform(DType dt, const std::vector<size_t>& shape, double re, double im);
Dense make_from_host(DType dt, const void* data, size_t len, const std::vector<size_t>& shape);
Dense make_from_device(DType dt, const void* dptr, size_t len, const std::vector<size_t>& shape);
Dense make_empty_device(DType dt, const std::vector<size_t>& shape);  // uninitialised device buffer

// ------------------------------------------------------------- operations
// Strided gather: dst (dense, column-major, shape `shape`) receives
// src[sum_i idx_i * src_strides[i]].  Covers permutedims (strides = permuted
// source strides), TTGT operand packing and axes pinned at index 0.
struct GatherDesc {
  std::vector<size_t> shape;        // destination extents
  std::vector<int64_t> src_strides; // in elements, per destination axis
};
void gather(DType dt, const void* src, void* dst, const GatherDesc& g, cudaStream_t s);
// Programmatic dependent launch (sm_90+).  A kernel launched with
// launch_pdl may be scheduled while the previous kernel on the stream is
// still finishing, so launch latency and its own setup overlap that kernel's
// tail.  Every kernel launched this way executes pdl_wait() before its first
// global memory access (griddepcontrol.wait: the previous grid has completed
// and its writes are visible), and pdl_release() early to let the next
// kernel be scheduled the same way.
__device__ __forceinline__ void pdl_release() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
template <typename... KParams, typename... Args>
void launch_pdl(void (*kern)(KParams...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  NDT_CUDA(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
}
// Number of device kernels launched by this library since load (for benches).
uint64_t launch_count();
void count_launch();

// Dense permutedims with the reference's validation (permutedims.rs:51-68).
Dense permutedims(const Dense& t, const std::vector<size_t>& perm);

// GEMM on device: C[m,n] (+)= sum_k A(i,l) * B(l,j).  A is MN-major
// (A[i + l*lda]) or K-major (A[l + i*lda]); B is K-major (B[l + j*ldb]) or
// MN-major (B[j + l*ldb]); C is column-major with leading dimension ldc.
struct GemmOperand {
  const void* ptr;
  int64_t ld;
  bool kmajor;
};
// allow_split_k = false keeps the launch free of device allocations (split-K
// needs a pool-allocated workspace for its partial sums).
void gemm(DType dt, int64_t m, int64_t n, int64_t k, GemmOperand A, GemmOperand B, void* C,
          int64_t ldc, bool accumulate, cudaStream_t s, bool allow_split_k = true);

// Strided views used by the contraction driver: an axis of one operand
// (extent, element stride) and a contracted axis pair (extent, stride in A,
// stride in B).  Lists are ordered fastest first.
struct StridedAxis {
  int64_t n, s;
};
struct ContractedAxis {
  int64_t n, sa, sb;
};

// Skinny contraction (skinny.cu): C[M..., N...] (dense, M fastest) =
// sum_K A B when K and one of M / N are short (at most kSkinnyMax elements
// each) and the other is long.  It reads both operands through their strides
// in one pass (no packing), so a permuted operand costs nothing extra.
// Returns false, doing nothing, when the shape is outside its range.
constexpr int kSkinnyMax = 32;
bool skinny_contract(DType dt, const void* A, const void* B, void* C, const std::vector<StridedAxis>& M,
                     const std::vector<StridedAxis>& N, const std::vector<ContractedAxis>& K, cudaStream_t s);

// Grouped GEMM over a device-side table.  Each problem is one output block
// C_p (m_p x n_p, column-major, packed) = sum over its segments s of
// A_s (m_p x k_s) * B_s (k_s x n_p).  All operands of one call share the
// majorness flags.  Host arrays are uploaded into `scratch`-owned buffers.
struct GroupedProblem {
  int64_t m, n;
  int64_t c_off;     // element offset of C block
  int64_t seg_begin; // first segment
  int64_t seg_count;
};
struct GroupedSegment {
  int64_t a_off, b_off;  // element offsets into A / B data
  int64_t k;
  int64_t lda, ldb;
  int64_t scale_off;     // offset into the k-scale vector, or -1
};
// Strided operands: one GEMM index (rows, contraction or columns) of a block
// whose axes are not in GEMM order, as at most two strided runs:
// offset(x) = (x % e0) * s0 + (x / e0) * s1.  One run: e0 above every index.
struct IndexRuns {
  uint32_t e0;
  uint32_t pad;
  int64_t s0, s1;
};
struct StridedProblem {
  IndexRuns cm, cn;  // C block: rows and columns (from c_off)
};
struct StridedSegment {
  IndexRuns am, ak;  // A block: rows and contraction (from a_off)
  IndexRuns bk, bn;  // B block: contraction and columns (from b_off)
};
// sm_reserve: SMs left free of the launch's persistent CTAs (room for
// transfer kernels that run beside it, e.g. NCCL's).  peer_copies (at most
// 7): further buffers laid out like C (other GPUs' memory mapped into this
// process) that every output tile is also stored to as it is computed.
// sprobs / ssegs (one per problem / segment, no k-scale): the operands and C
// are addressed through their index runs, so permuted blocks are read and
// written in place (lda, ldb and the majorness flags are then unused).
void grouped_gemm(DType dt, const void* A, const void* B, void* C, bool a_kmajor, bool b_kmajor,
                  const std::vector<GroupedProblem>& probs, const std::vector<GroupedSegment>& segs,
                  const void* kscale, cudaStream_t s, bool kscale_real = false, int sm_reserve = 0,
                  const std::vector<void*>* peer_copies = nullptr,
                  const std::vector<StridedProblem>* sprobs = nullptr,
                  const std::vector<StridedSegment>* ssegs = nullptr);

// Block-sparse device helpers (blocksparse_kernels.cu).  A block table entry
// describes one block: its extents, and for the dense side its start offset
// and the dense strides (meaning of the fields per kernel is documented there).
constexpr int kBsMaxRank = 16;
struct BsBlockDesc {
  int32_t ndim;
  int64_t shape[kBsMaxRank];
  int64_t dstride[kBsMaxRank];
  int64_t dense_base;
};
void bs_dense_map(DType dt, void* packed, void* dense, const std::vector<int64_t>& offs,
                  const std::vector<BsBlockDesc>& blocks, int64_t total, bool to_dense, cudaStream_t s);
void diag_scatter(DType dt, const void* diag, void* out, const std::vector<int64_t>& offs,
                  const std::vector<BsBlockDesc>& blocks, int64_t total, cudaStream_t s);
void bs_diag_scale(DType dt, const void* a, const void* sdiag, void* out, const std::vector<int64_t>& offs,
                   const std::vector<BsBlockDesc>& blocks, int64_t total, cudaStream_t s);
// Byte ranges src + src_off[i] -> dst + dst_off[i] (bytes[i] long, all
// multiples of 8; bases 16-byte aligned) in one launch.
void copy_segments(const void* src, void* dst, const std::vector<int64_t>& src_off, const std::vector<int64_t>& dst_off,
                   const std::vector<int64_t>& bytes, cudaStream_t s);

// Elementwise helpers
void fill_device(DType dt, void* p, size_t n, double re, double im, cudaStream_t s);
void add_device(DType dt, const void* a, const void* b, void* c, size_t n, cudaStream_t s);
void scale_device(DType dt, const void* a, void* c, size_t n, double re, double im, cudaStream_t s);
// C[i + j*ldc] (+)= sum over s < nsplit of W[s][i + j*m] (split-K partials,
// summed in split order).
void splitk_reduce(DType dt, const void* w, int nsplit, int64_t m, int64_t n, void* c, int64_t ldc, bool accumulate,
                   cudaStream_t s);

// Contractions
enum class ContractSemantics { Naive, Gemm };
// contract_gemm on the rank's range of the free axis labelled axis_label
// (near-equal ranges over nranks): that slab of C (contract.cpp).
Dense contract_gemm_shard(const Dense& a, const std::vector<int32_t>& la, const Dense& b,
                          const std::vector<int32_t>& lb, int32_t axis_label, int rank, int nranks);
Dense contract(const Dense& a, const std::vector<int32_t>& la, const Dense& b,
               const std::vector<int32_t>& lb, ContractSemantics sem);
void contract_vjp(const Dense& a, const std::vector<int32_t>& la, const Dense& b,
                  const std::vector<int32_t>& lb, const Dense& grad, Dense* ga, Dense* gb);
Dense add(const Dense& a, const Dense& b);  // apply_binary(+) semantics

}  // namespace ndt

// The object behind an ndt_tensor_f64* / ndt_tensor_c64* handle.
struct NdtHandle {
  ndt::Dense t;
};
