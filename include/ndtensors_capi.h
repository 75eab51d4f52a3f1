/*
 * ndtensors_capi.h — C ABI of the B200 ndtensors library (libndtensors_capi.so).
 *
 * Part 1 is a drop-in for the reference's C ABI
 * (crates/ndtensors-capi/src/lib.rs of ndtensors-rs): same 19 symbols, same
 * signatures, same status codes, same ownership and NULL handling.  Every
 * declaration cites the reference function it replaces.  Computation
 * (permutedims, contract, VJP, JVP) runs on the current CUDA device; the
 * pointers returned by *_data / *_data_mut are host pointers, as in the
 * reference, filled from device memory on demand.
 *
 * Part 2 adds symbols the reference's ABI lacks (its README lists complex
 * and block-sparse tensors as "not yet"): complex128 dense tensors, the TTGT
 * (label-sorted) contraction, block-sparse and diag-block-sparse tensors,
 * device-pointer interop, and stream / diagnostics control.  They follow the
 * same conventions.  Complex values are interleaved (re, im) doubles.
 *
 * Threading: like the reference (Rc-based, not Send), a handle must not be
 * used from two threads at once.  Work is issued on one CUDA stream per
 * device (replaceable with ndt_b200_set_stream).
 */
#ifndef NDTENSORS_CAPI_H
#define NDTENSORS_CAPI_H

#include <stddef.h>

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif
#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: capi/lib.rs:17-25 */
#define NDT_SUCCESS 0
#define NDT_INVALID_ARGUMENT (-1)
#define NDT_SHAPE_MISMATCH (-2)
#define NDT_INDEX_OUT_OF_BOUNDS (-3)
#define NDT_INTERNAL_ERROR (-4)
#define NDT_INVALID_PERMUTATION (-5)

/* Opaque handles (capi/lib.rs:28-65) */
typedef struct ndt_tensor_f64 ndt_tensor_f64;
typedef struct ndt_tensor_c64 ndt_tensor_c64;
typedef struct ndt_blocksparse_f64 ndt_blocksparse_f64;
typedef struct ndt_blocksparse_c64 ndt_blocksparse_c64;
typedef struct ndt_diagblocksparse_f64 ndt_diagblocksparse_f64;
typedef struct ndt_diagblocksparse_c64 ndt_diagblocksparse_c64;

/* ======================= Part 1: the reference's f64 ABI ======================= */

/* capi/lib.rs:81  ndt_tensor_f64_zeros */
ndt_tensor_f64* ndt_tensor_f64_zeros(const size_t* shape, size_t ndim, int* status);
/* capi/lib.rs:138 ndt_tensor_f64_ones */
ndt_tensor_f64* ndt_tensor_f64_ones(const size_t* shape, size_t ndim, int* status);
/* capi/lib.rs:195 ndt_tensor_f64_rand  (uniform [0,1)) */
ndt_tensor_f64* ndt_tensor_f64_rand(const size_t* shape, size_t ndim, int* status);
/* capi/lib.rs:252 ndt_tensor_f64_randn (standard normal) */
ndt_tensor_f64* ndt_tensor_f64_randn(const size_t* shape, size_t ndim, int* status);
/* capi/lib.rs:307 ndt_tensor_f64_from_data (copies; len must be max(1, prod(shape))) */
ndt_tensor_f64* ndt_tensor_f64_from_data(const double* data, size_t len, const size_t* shape, size_t ndim,
                                         int* status);
/* capi/lib.rs:364 ndt_tensor_f64_release (NULL-safe) */
void ndt_tensor_f64_release(ndt_tensor_f64* tensor);
/* capi/lib.rs:374 ndt_tensor_f64_clone (shares storage, copy on write) */
ndt_tensor_f64* ndt_tensor_f64_clone(const ndt_tensor_f64* src);
/* capi/lib.rs:394 ndt_tensor_f64_ndim */
size_t ndt_tensor_f64_ndim(const ndt_tensor_f64* tensor);
/* capi/lib.rs:408 ndt_tensor_f64_len (storage length, max(1, prod(shape))) */
size_t ndt_tensor_f64_len(const ndt_tensor_f64* tensor);
/* capi/lib.rs:429 ndt_tensor_f64_shape */
int ndt_tensor_f64_shape(const ndt_tensor_f64* tensor, size_t* out);
/* capi/lib.rs:454 ndt_tensor_f64_data (host pointer, valid until mutation / release) */
const double* ndt_tensor_f64_data(const ndt_tensor_f64* tensor);
/* capi/lib.rs:471 ndt_tensor_f64_data_mut (copy on write; host pointer) */
double* ndt_tensor_f64_data_mut(ndt_tensor_f64* tensor);
/* capi/lib.rs:489 ndt_tensor_f64_get_linear */
int ndt_tensor_f64_get_linear(const ndt_tensor_f64* tensor, size_t index, double* out);
/* capi/lib.rs:514 ndt_tensor_f64_set_linear */
int ndt_tensor_f64_set_linear(ndt_tensor_f64* tensor, size_t index, double value);
/* capi/lib.rs:539 ndt_tensor_f64_fill */
int ndt_tensor_f64_fill(ndt_tensor_f64* tensor, double value);
/* capi/lib.rs:567 ndt_tensor_f64_permutedims (perm[i] = source axis of output axis i) */
ndt_tensor_f64* ndt_tensor_f64_permutedims(const ndt_tensor_f64* tensor, const size_t* perm, size_t ndim,
                                           int* status);
/* capi/lib.rs:627 ndt_tensor_f64_contract (naive-loop semantics: output axes are
 * A's positive labels then B's, unsorted; scalar result has shape [1]) */
ndt_tensor_f64* ndt_tensor_f64_contract(const ndt_tensor_f64* a, const long* labels_a, size_t ndim_a,
                                        const ndt_tensor_f64* b, const long* labels_b, size_t ndim_b,
                                        int* status);
/* capi/lib.rs:705 ndt_tensor_f64_contract_vjp */
void ndt_tensor_f64_contract_vjp(const ndt_tensor_f64* a, const long* labels_a, size_t ndim_a,
                                 const ndt_tensor_f64* b, const long* labels_b, size_t ndim_b,
                                 const ndt_tensor_f64* grad_output, ndt_tensor_f64** grad_a_out,
                                 ndt_tensor_f64** grad_b_out, int* status);
/* capi/lib.rs:810 ndt_tensor_f64_contract_jvp */
void ndt_tensor_f64_contract_jvp(const ndt_tensor_f64* a, const long* labels_a, size_t ndim_a,
                                 const ndt_tensor_f64* b, const long* labels_b, size_t ndim_b,
                                 const ndt_tensor_f64* tangent_a, const ndt_tensor_f64* tangent_b,
                                 ndt_tensor_f64** primal_out, ndt_tensor_f64** tangent_out, int* status);

/* ============================ Part 2: additive ============================ */

/* TTGT contraction with the reference's contract_gemm semantics
 * (crates/ndtensors/src/contract/gemm.rs:47-95): output axes sorted by label.
 * Status: any TensorError -> NDT_SHAPE_MISMATCH, panic -> NDT_INTERNAL_ERROR. */
ndt_tensor_f64* ndt_tensor_f64_contract_gemm(const ndt_tensor_f64* a, const long* labels_a, size_t ndim_a,
                                             const ndt_tensor_f64* b, const long* labels_b, size_t ndim_b,
                                             int* status);

/* Complex128 dense tensors; element i is (data[2i], data[2i+1]).  Same
 * semantics as the f64 functions of the same name (the reference's generic
 * Tensor<c64>: tensor.rs, permutedims.rs, naive.rs, gemm.rs). */
ndt_tensor_c64* ndt_tensor_c64_zeros(const size_t* shape, size_t ndim, int* status);
ndt_tensor_c64* ndt_tensor_c64_ones(const size_t* shape, size_t ndim, int* status);
ndt_tensor_c64* ndt_tensor_c64_from_data(const double* data_interleaved, size_t len, const size_t* shape,
                                         size_t ndim, int* status);
void ndt_tensor_c64_release(ndt_tensor_c64* tensor);
ndt_tensor_c64* ndt_tensor_c64_clone(const ndt_tensor_c64* src);
size_t ndt_tensor_c64_ndim(const ndt_tensor_c64* tensor);
size_t ndt_tensor_c64_len(const ndt_tensor_c64* tensor);
int ndt_tensor_c64_shape(const ndt_tensor_c64* tensor, size_t* out);
const double* ndt_tensor_c64_data(const ndt_tensor_c64* tensor);
double* ndt_tensor_c64_data_mut(ndt_tensor_c64* tensor);
int ndt_tensor_c64_get_linear(const ndt_tensor_c64* tensor, size_t index, double* re, double* im);
int ndt_tensor_c64_set_linear(ndt_tensor_c64* tensor, size_t index, double re, double im);
int ndt_tensor_c64_fill(ndt_tensor_c64* tensor, double re, double im);
ndt_tensor_c64* ndt_tensor_c64_permutedims(const ndt_tensor_c64* tensor, const size_t* perm, size_t ndim,
                                           int* status);
ndt_tensor_c64* ndt_tensor_c64_contract(const ndt_tensor_c64* a, const long* labels_a, size_t ndim_a,
                                        const ndt_tensor_c64* b, const long* labels_b, size_t ndim_b,
                                        int* status);
ndt_tensor_c64* ndt_tensor_c64_contract_gemm(const ndt_tensor_c64* a, const long* labels_a, size_t ndim_a,
                                             const ndt_tensor_c64* b, const long* labels_b, size_t ndim_b,
                                             int* status);

/* contract_gemm split along one free index for multi-GPU use (no counterpart
 * in the reference; the contraction split is gemm.rs:173-236).  The free axis
 * labelled axis_label (a positive label of exactly one axis of A or B) is cut
 * into nranks near-equal ranges; the call returns this rank's slab of C
 * (range [N*rank/nranks, N*(rank+1)/nranks) of that axis, other axes whole,
 * label-sorted as contract_gemm), reading the operand in place.  No
 * collective: the slabs of all ranks together are contract_gemm's result.
 * An empty range gives a zero tensor of the slab's shape.  Bad rank / nranks
 * or label: NDT_INVALID_ARGUMENT; contraction errors as contract_gemm. */
ndt_tensor_f64* ndt_tensor_f64_contract_gemm_shard(const ndt_tensor_f64* a, const long* labels_a, size_t ndim_a,
                                                   const ndt_tensor_f64* b, const long* labels_b, size_t ndim_b,
                                                   long axis_label, int rank, int nranks, int* status);
ndt_tensor_c64* ndt_tensor_c64_contract_gemm_shard(const ndt_tensor_c64* a, const long* labels_a, size_t ndim_a,
                                                   const ndt_tensor_c64* b, const long* labels_b, size_t ndim_b,
                                                   long axis_label, int rank, int nranks, int* status);

/* Device-pointer interop (the device-pointer ABI proposed in the reference's
 * README, "CUDA support" section).  from_device_ptr copies `len` elements from
 * device memory of the current device (the caller's writes to it must be
 * complete) and returns once they have been read; device_ptr returns the
 * tensor's device buffer for reading (valid until mutation / release);
 * device_ptr_mut returns it for writing from outside the library (copy on
 * write if shared, as data_mut; the device copy then holds the tensor's
 * values, and host views are refreshed from it).  Both return once the
 * library's pending work on the buffer (fills, uploads, kernels) has
 * completed, so reads and writes from any stream are safe.  With a caller
 * stream installed by ndt_b200_set_stream all three return at once, the work
 * being ordered on that stream. */
ndt_tensor_f64* ndt_tensor_f64_from_device_ptr(const double* dptr, size_t len, const size_t* shape, size_t ndim,
                                               int* status);
const double* ndt_tensor_f64_device_ptr(const ndt_tensor_f64* tensor);
double* ndt_tensor_f64_device_ptr_mut(ndt_tensor_f64* tensor);
ndt_tensor_c64* ndt_tensor_c64_from_device_ptr(const double* dptr, size_t len, const size_t* shape, size_t ndim,
                                               int* status);
const double* ndt_tensor_c64_device_ptr(const ndt_tensor_c64* tensor);
double* ndt_tensor_c64_device_ptr_mut(ndt_tensor_c64* tensor);

/* Raw device kernels, no handles, no allocation by the library.
 * dtype: 0 = f64, 1 = complex128.  `stream` is a cudaStream_t; NULL is the
 * legacy default stream, as everywhere in CUDA. */
/* permutedims into a caller buffer: dst has shape perm.map(shape)
 * (operations/permutedims.rs:51-68, backend/generic.rs:15-39). */
int ndt_b200_permutedims_dev(int dtype, const void* src, void* dst, const size_t* shape, size_t ndim,
                             const size_t* perm, size_t nperm, void* stream);
/* C (m x n, column-major, ldc) (+)= A B on FP64 tensor cores.  A is m x k:
 * element (i,l) at A[i + l*lda] (a_kmajor = 0) or A[l + i*lda] (a_kmajor = 1);
 * B is k x n: element (l,j) at B[l + j*ldb] (b_kmajor = 1) or B[j + l*ldb]
 * (b_kmajor = 0).  Stands in for faer's matmul (contract/gemm.rs:209-216). */
int ndt_b200_gemm_dev(int dtype, long m, long n, long k, const void* A, long lda, int a_kmajor, const void* B,
                      long ldb, int b_kmajor, void* C, long ldc, int accumulate, void* stream);

/* Block-sparse tensors (BlockSparseTensor, blocksparse_tensor.rs; storage in
 * storage/blocksparse/).  Structure arguments: ndim axes; nblocks[ax] blocks
 * on axis ax; block_sizes = the sizes of axis 0's blocks, then axis 1's, ...
 * (BlockDim::new, block_dim.rs:45); nnzb stored blocks whose coordinates are
 * coords[b*ndim .. b*ndim+ndim), packed in that order
 * (BlockOffsets::from_blocks, block_offsets.rs:76-90).  Element type as the
 * name says (c64: interleaved re/im; lengths count elements).
 * Errors: invalid / duplicate coordinates -> NDT_INVALID_ARGUMENT, a missing
 * block -> NDT_INDEX_OUT_OF_BOUNDS, a TensorError -> NDT_SHAPE_MISMATCH
 * (NDT_INVALID_PERMUTATION for permutedims), a panic -> NDT_INTERNAL_ERROR. */
/* BlockSparseTensor::zeros (blocksparse_tensor.rs:68) */
ndt_blocksparse_f64* ndt_blocksparse_f64_zeros(size_t ndim, const size_t* nblocks, const size_t* block_sizes,
                                               size_t nnzb, const size_t* coords, int* status);
/* BlockSparse::from_vec with from_blocks offsets (storage.rs:125); len = total stored elements */
ndt_blocksparse_f64* ndt_blocksparse_f64_from_data(size_t ndim, const size_t* nblocks, const size_t* block_sizes,
                                                   size_t nnzb, const size_t* coords, const double* data, size_t len,
                                                   int* status);
/* as from_data, copying from device memory of the current device */
ndt_blocksparse_f64* ndt_blocksparse_f64_from_device_ptr(size_t ndim, const size_t* nblocks,
                                                         const size_t* block_sizes, size_t nnzb,
                                                         const size_t* coords, const double* dptr, size_t len,
                                                         int* status);
void ndt_blocksparse_f64_release(ndt_blocksparse_f64* t);
size_t ndt_blocksparse_f64_ndim(const ndt_blocksparse_f64* t);
size_t ndt_blocksparse_f64_nnzblocks(const ndt_blocksparse_f64* t); /* nnzblocks (blocksparse_tensor.rs:99) */
size_t ndt_blocksparse_f64_nnz(const ndt_blocksparse_f64* t);       /* nnz (blocksparse_tensor.rs:93) */
size_t ndt_blocksparse_f64_nblocks_total(const ndt_blocksparse_f64* t); /* length of block_sizes */
/* block dims, stored block coordinates (storage order) and packed offsets; any pointer may be NULL */
int ndt_blocksparse_f64_structure(const ndt_blocksparse_f64* t, size_t* nblocks, size_t* block_sizes,
                                  size_t* coords, size_t* offsets);
/* insertblock (blocksparse_tensor.rs:210-235): len must equal the block's element count */
int ndt_blocksparse_f64_insert_block(ndt_blocksparse_f64* t, const size_t* coords, const double* data, size_t len);
/* blockview (blocksparse_tensor.rs:158-164): copies the block out (len >= block elements) */
int ndt_blocksparse_f64_get_block(const ndt_blocksparse_f64* t, const size_t* coords, double* out, size_t len);
const double* ndt_blocksparse_f64_data(const ndt_blocksparse_f64* t);       /* host view of packed data */
const double* ndt_blocksparse_f64_device_ptr(const ndt_blocksparse_f64* t); /* device view of packed data */
double* ndt_blocksparse_f64_device_ptr_mut(ndt_blocksparse_f64* t); /* for writing (as the dense device_ptr_mut) */
/* A tensor from blocks lying anywhere in device memory (no counterpart in the reference): block i of
 * the listed structure is read at src + src_offsets[i] elements (each block inside [0, src_len)); the
 * result stores the blocks sorted by coordinates, packed, written by one copy kernel.  Assembles the
 * shards of a sharded contraction gathered into one buffer. */
ndt_blocksparse_f64* ndt_blocksparse_f64_from_device_blocks(size_t ndim, const size_t* nblocks,
                                                            const size_t* block_sizes, size_t nnzb,
                                                            const size_t* coords, const size_t* src_offsets,
                                                            const double* src, size_t src_len, int* status);
/* contract_blocksparse (contract/blocksparse.rs:87-183): one grouped FP64 tensor-core launch */
ndt_blocksparse_f64* ndt_blocksparse_f64_contract(const ndt_blocksparse_f64* a, const long* labels_a,
                                                  size_t ndim_a, const ndt_blocksparse_f64* b, const long* labels_b,
                                                  size_t ndim_b, int* status);
/* `rank`'s FLOP-balanced share of the output blocks (contract_blocksparse split over nranks
 * processes / GPUs; no collective): blocks go to ranks heaviest first, each to the least loaded
 * rank (ties to the lower rank); the returned blocks are sorted. */
ndt_blocksparse_f64* ndt_blocksparse_f64_contract_shard(const ndt_blocksparse_f64* a, const long* labels_a,
                                                        size_t ndim_a, const ndt_blocksparse_f64* b,
                                                        const long* labels_b, size_t ndim_b, int rank, int nranks,
                                                        int* status);
/* The listed output blocks only (coords: nout x output rank, natural order A-free ++ B-free), from
   whatever blocks the operands hold.  A rank of a sharded contraction whose operands carry only the
   blocks its output blocks reference computes its share this way.  No counterpart in the reference. */
ndt_blocksparse_f64* ndt_blocksparse_f64_contract_select(const ndt_blocksparse_f64* a, const long* labels_a,
                                                         size_t ndim_a, const ndt_blocksparse_f64* b,
                                                         const long* labels_b, size_t ndim_b,
                                                         const size_t* out_coords, size_t nout, int* status);
ndt_blocksparse_c64* ndt_blocksparse_c64_contract_select(const ndt_blocksparse_c64* a, const long* labels_a,
                                                         size_t ndim_a, const ndt_blocksparse_c64* b,
                                                         const long* labels_b, size_t ndim_b,
                                                         const size_t* out_coords, size_t nout, int* status);
/* Which rank holds which output block, for a shard returned by contract_shard / contract_through_diag
 * with nranks > 1 (NDT_INVALID_ARGUMENT for any other tensor): *nranks, *nblocks (all output blocks),
 * then, when the arrays are not NULL, the blocks' coordinates (nblocks x ndim, sorted) and owners.
 * Every rank gets the same layout, so shards can be gathered without exchanging their structure. */
int ndt_blocksparse_f64_shard_layout(const ndt_blocksparse_f64* t, int* nranks, size_t* nblocks, size_t* coords,
                                     int* owners);
int ndt_blocksparse_c64_shard_layout(const ndt_blocksparse_c64* t, int* nranks, size_t* nblocks, size_t* coords,
                                     int* owners);
/* Host-only plan of contract_shard: output blocks and real flops per rank (either array may be NULL) */
int ndt_blocksparse_f64_shard_plan(const ndt_blocksparse_f64* a, const long* labels_a, size_t ndim_a,
                                   const ndt_blocksparse_f64* b, const long* labels_b, size_t ndim_b, int nranks,
                                   size_t* blocks_per_rank, double* flops_per_rank);
int ndt_blocksparse_c64_shard_plan(const ndt_blocksparse_c64* a, const long* labels_a, size_t ndim_a,
                                   const ndt_blocksparse_c64* b, const long* labels_b, size_t ndim_b, int nranks,
                                   size_t* blocks_per_rank, double* flops_per_rank);
/* permutedims_blocksparse (operations/blocksparse.rs:61-129) */
ndt_blocksparse_f64* ndt_blocksparse_f64_permutedims(const ndt_blocksparse_f64* t, const size_t* perm, size_t nperm,
                                                     int* status);
/* to_dense / from_dense (blocksparse_tensor.rs:290-391) */
ndt_tensor_f64* ndt_blocksparse_f64_to_dense(const ndt_blocksparse_f64* t, int* status);
ndt_blocksparse_f64* ndt_blocksparse_f64_from_dense(const ndt_tensor_f64* dense, size_t ndim, const size_t* nblocks,
                                                    const size_t* block_sizes, size_t nnzb, const size_t* coords,
                                                    int* status);

/* complex128 block-sparse: same functions */
ndt_blocksparse_c64* ndt_blocksparse_c64_zeros(size_t ndim, const size_t* nblocks, const size_t* block_sizes,
                                               size_t nnzb, const size_t* coords, int* status);
ndt_blocksparse_c64* ndt_blocksparse_c64_from_data(size_t ndim, const size_t* nblocks, const size_t* block_sizes,
                                                   size_t nnzb, const size_t* coords, const double* data, size_t len,
                                                   int* status);
ndt_blocksparse_c64* ndt_blocksparse_c64_from_device_ptr(size_t ndim, const size_t* nblocks,
                                                         const size_t* block_sizes, size_t nnzb,
                                                         const size_t* coords, const double* dptr, size_t len,
                                                         int* status);
void ndt_blocksparse_c64_release(ndt_blocksparse_c64* t);
size_t ndt_blocksparse_c64_ndim(const ndt_blocksparse_c64* t);
size_t ndt_blocksparse_c64_nnzblocks(const ndt_blocksparse_c64* t);
size_t ndt_blocksparse_c64_nnz(const ndt_blocksparse_c64* t);
size_t ndt_blocksparse_c64_nblocks_total(const ndt_blocksparse_c64* t);
int ndt_blocksparse_c64_structure(const ndt_blocksparse_c64* t, size_t* nblocks, size_t* block_sizes,
                                  size_t* coords, size_t* offsets);
int ndt_blocksparse_c64_insert_block(ndt_blocksparse_c64* t, const size_t* coords, const double* data, size_t len);
int ndt_blocksparse_c64_get_block(const ndt_blocksparse_c64* t, const size_t* coords, double* out, size_t len);
const double* ndt_blocksparse_c64_data(const ndt_blocksparse_c64* t);
const double* ndt_blocksparse_c64_device_ptr(const ndt_blocksparse_c64* t);
double* ndt_blocksparse_c64_device_ptr_mut(ndt_blocksparse_c64* t);
ndt_blocksparse_c64* ndt_blocksparse_c64_from_device_blocks(size_t ndim, const size_t* nblocks,
                                                            const size_t* block_sizes, size_t nnzb,
                                                            const size_t* coords, const size_t* src_offsets,
                                                            const double* src, size_t src_len, int* status);
ndt_blocksparse_c64* ndt_blocksparse_c64_contract(const ndt_blocksparse_c64* a, const long* labels_a,
                                                  size_t ndim_a, const ndt_blocksparse_c64* b, const long* labels_b,
                                                  size_t ndim_b, int* status);
ndt_blocksparse_c64* ndt_blocksparse_c64_contract_shard(const ndt_blocksparse_c64* a, const long* labels_a,
                                                        size_t ndim_a, const ndt_blocksparse_c64* b,
                                                        const long* labels_b, size_t ndim_b, int rank, int nranks,
                                                        int* status);
ndt_blocksparse_c64* ndt_blocksparse_c64_permutedims(const ndt_blocksparse_c64* t, const size_t* perm, size_t nperm,
                                                     int* status);
ndt_tensor_c64* ndt_blocksparse_c64_to_dense(const ndt_blocksparse_c64* t, int* status);
ndt_blocksparse_c64* ndt_blocksparse_c64_from_dense(const ndt_tensor_c64* dense, size_t ndim, const size_t* nblocks,
                                                    const size_t* block_sizes, size_t nnzb, const size_t* coords,
                                                    int* status);

/* DiagBlockSparse tensors (diagblocksparse.rs, diagblocksparse_tensor.rs): only
 * the min(block shape) diagonal values of each listed block, packed in the
 * listed order (diagblocksparse.rs:86, :218-230).  The reference has no
 * contraction for them; ndt_blocksparse_*_contract_diag defines one as the
 * block-sparse contraction with the diagonal blocks made dense, and runs it
 * as a fused diagonal scaling when the diagonal tensor is a rank-2 block
 * diagonal contracted with A's last axis. */
ndt_diagblocksparse_f64* ndt_diagblocksparse_f64_from_data(size_t ndim, const size_t* nblocks,
                                                           const size_t* block_sizes, size_t nnzb,
                                                           const size_t* coords, const double* diag, size_t len,
                                                           int* status);
void ndt_diagblocksparse_f64_release(ndt_diagblocksparse_f64* t);
size_t ndt_diagblocksparse_f64_nnz(const ndt_diagblocksparse_f64* t);
ndt_tensor_f64* ndt_diagblocksparse_f64_to_dense(const ndt_diagblocksparse_f64* t, int* status);
ndt_blocksparse_f64* ndt_diagblocksparse_f64_to_blocksparse(const ndt_diagblocksparse_f64* t, int* status);
ndt_blocksparse_f64* ndt_blocksparse_f64_contract_diag(const ndt_blocksparse_f64* a, const long* labels_a,
                                                       size_t ndim_a, const ndt_diagblocksparse_f64* s,
                                                       const long* labels_s, size_t ndim_s, int* status);
ndt_diagblocksparse_c64* ndt_diagblocksparse_c64_from_data(size_t ndim, const size_t* nblocks,
                                                           const size_t* block_sizes, size_t nnzb,
                                                           const size_t* coords, const double* diag, size_t len,
                                                           int* status);
void ndt_diagblocksparse_c64_release(ndt_diagblocksparse_c64* t);
size_t ndt_diagblocksparse_c64_nnz(const ndt_diagblocksparse_c64* t);
ndt_tensor_c64* ndt_diagblocksparse_c64_to_dense(const ndt_diagblocksparse_c64* t, int* status);
ndt_blocksparse_c64* ndt_diagblocksparse_c64_to_blocksparse(const ndt_diagblocksparse_c64* t, int* status);
ndt_blocksparse_c64* ndt_blocksparse_c64_contract_diag(const ndt_blocksparse_c64* a, const long* labels_a,
                                                       size_t ndim_a, const ndt_diagblocksparse_c64* s,
                                                       const long* labels_s, size_t ndim_s, int* status);
/* (A . S) . B with S a rank-2 diagonal between A and B (no counterpart in the reference): labels_s
 * = {x, y}, both negative; x labels one axis of A, y one axis of B, and every other label of A and B
 * is positive.  Equals contract(contract_diag(A, S), B): A's and B's free axes in label order.
 * Sharded (nranks > 1): one grouped launch that applies S's diagonal to the contracted index as it
 * loads the operands (no A . S intermediate) when S's blocks are square and each coordinate of A's
 * contracted axis meets one S block; unsharded, or otherwise, the two contractions in turn (one pass
 * over A costs less than the in-GEMM scaling when a rank does all the work).  rank / nranks as in
 * contract_shard (0, 1: all). */
ndt_blocksparse_f64* ndt_blocksparse_f64_contract_through_diag(
    const ndt_blocksparse_f64* a, const long* labels_a, size_t ndim_a, const ndt_diagblocksparse_f64* s,
    const long* labels_s, size_t ndim_s, const ndt_blocksparse_f64* b, const long* labels_b, size_t ndim_b, int rank,
    int nranks, int* status);
ndt_blocksparse_c64* ndt_blocksparse_c64_contract_through_diag(
    const ndt_blocksparse_c64* a, const long* labels_a, size_t ndim_a, const ndt_diagblocksparse_c64* s,
    const long* labels_s, size_t ndim_s, const ndt_blocksparse_c64* b, const long* labels_b, size_t ndim_b, int rank,
    int nranks, int* status);

/* ---- Multi-GPU: NCCL communicator and gathered block-sparse contractions
 * (no counterpart in the reference, which is single-threaded CPU code; the
 * per-output-block loop these distribute is contract/blocksparse.rs:144-180).
 * One process per GPU.  Rank 0 calls ndt_b200_comm_unique_id and hands the
 * 128 bytes to every rank by its own means (MPI, a TCP store, torch.distributed);
 * each rank, with its GPU current, calls ndt_b200_comm_init.  A caller that
 * already holds an ncclComm_t (for this process's current GPU) wraps it with
 * ndt_b200_comm_from_nccl; it stays the caller's (release does not destroy it).
 * NCCL is loaded at the first of these calls (libnccl.so.2; a copy already
 * loaded in the process, e.g. torch's, is shared).  Release a communicator
 * before its NCCL library's process teardown. */
typedef struct ndt_comm ndt_comm;
int ndt_b200_comm_unique_id(unsigned char* id /* 128 bytes out */);
ndt_comm* ndt_b200_comm_init(const unsigned char* id, int nranks, int rank, int* status);
ndt_comm* ndt_b200_comm_from_nccl(void* nccl_comm /* ncclComm_t */, int* status);
int ndt_b200_comm_rank(const ndt_comm* comm);
int ndt_b200_comm_size(const ndt_comm* comm);
void ndt_b200_comm_release(ndt_comm* comm);

/* contract_blocksparse with the output gathered on every rank (the contract
 * "gather" flag; device list = the communicator's ranks).  Every rank passes
 * the same operands; each computes its share of the output blocks (longest
 * processing time on tile cost, as contract_shard).  On up to 8 ranks that
 * map each other's memory (CUDA IPC), the GEMM stores every output tile into
 * every rank's output buffer as it computes it, a barrier follows, and each
 * rank copies its buffer into the result; otherwise each rank computes into
 * its slot of a staging buffer, an NCCL all-gather follows, and one copy
 * kernel puts every block at its place in the packed, sorted output.  Every
 * rank returns
 * the unsharded result (same structure and values as
 * ndt_blocksparse_*_contract).  Collective: every rank of the communicator
 * must call it, with the same arguments. */
ndt_blocksparse_f64* ndt_blocksparse_f64_contract_gathered(const ndt_blocksparse_f64* a, const long* labels_a,
                                                           size_t ndim_a, const ndt_blocksparse_f64* b,
                                                           const long* labels_b, size_t ndim_b, ndt_comm* comm,
                                                           int* status);
ndt_blocksparse_c64* ndt_blocksparse_c64_contract_gathered(const ndt_blocksparse_c64* a, const long* labels_a,
                                                           size_t ndim_a, const ndt_blocksparse_c64* b,
                                                           const long* labels_b, size_t ndim_b, ndt_comm* comm,
                                                           int* status);
/* (A . S) . B (see contract_through_diag), gathered on every rank as above. */
ndt_blocksparse_f64* ndt_blocksparse_f64_contract_through_diag_gathered(
    const ndt_blocksparse_f64* a, const long* labels_a, size_t ndim_a, const ndt_diagblocksparse_f64* s,
    const long* labels_s, size_t ndim_s, const ndt_blocksparse_f64* b, const long* labels_b, size_t ndim_b,
    ndt_comm* comm, int* status);
ndt_blocksparse_c64* ndt_blocksparse_c64_contract_through_diag_gathered(
    const ndt_blocksparse_c64* a, const long* labels_a, size_t ndim_a, const ndt_diagblocksparse_c64* s,
    const long* labels_s, size_t ndim_s, const ndt_blocksparse_c64* b, const long* labels_b, size_t ndim_b,
    ndt_comm* comm, int* status);
/* The whole output of a sharded contraction on every rank, from each rank's
 * shard (contract_shard / contract_through_diag with rank, nranks = the
 * communicator's).  Collective. */
ndt_blocksparse_f64* ndt_blocksparse_f64_allgather(const ndt_blocksparse_f64* shard, ndt_comm* comm, int* status);
ndt_blocksparse_c64* ndt_blocksparse_c64_allgather(const ndt_blocksparse_c64* shard, ndt_comm* comm, int* status);

/* Dense f64 contraction that allocates no memory (no counterpart in the
 * reference).  For callers that may not call cudaMalloc -- allocation-free
 * hot loops, hosts that own the device memory budget, runtimes that forbid
 * allocation on their hot path.  Same label semantics as
 * ndt_tensor_f64_contract; inputs and the
 * output are caller-owned device buffers (column-major, A and B dense over
 * their shapes, zero extents rejected with NDT_INTERNAL_ERROR); c must hold
 * c_len >= output length elements; out_shape (may be NULL) receives the
 * output shape (up to ndim_a + ndim_b entries, or 1).  An operand whose axes
 * form a unit-stride strided matrix is read in place at any size; one that
 * needs packing is packed into a fixed 16 MiB scratch array in device memory,
 * held by every GPU that loads the library until exit.  Contractions whose
 * packed operands need more are rejected with NDT_INVALID_ARGUMENT (message in
 * ndt_b200_last_error).  The first call on a device creates the library's
 * streams there and looks up that array's device address (make it before any
 * stream capture); it leaves the device's memory pools and their settings
 * untouched.  Calls share the array: calls that overlap on the GPU race. */
int ndt_b200_contract_f64_noalloc(const double* a, const size_t* shape_a, size_t ndim_a, const long* labels_a,
                                  const double* b, const size_t* shape_b, size_t ndim_b, const long* labels_b,
                                  double* c, size_t c_len, size_t* out_shape, size_t* out_ndim, void* stream);

/* Library control and diagnostics */
int ndt_b200_device_available(void);
int ndt_b200_set_stream(void* stream); /* NULL restores the library's own stream */
void* ndt_b200_get_stream(void);
int ndt_b200_synchronize(void);
const char* ndt_b200_last_error(void); /* text of the last failure on this thread */
unsigned long long ndt_b200_launch_count(void); /* kernels launched by this library */
void ndt_b200_empty_cache(void);

#ifdef __cplusplus
}
#endif
#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#endif
