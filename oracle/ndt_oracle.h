/*
 * ndt_oracle.h — CPU oracle for the ndtensors contraction hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference
 * implementation's algorithms (ndtensors-rs, crates/ndtensors/src/...), used as
 * the reference answer in tests/, in __graft_entry__.smoke() and as the timed CPU
 * baseline in bench.py.  The product library (libndtensors_capi.so) never
 * links, loads or calls it.
 *
 * Element types: dtype 0 = f64 (8 bytes), dtype 1 = complex128 stored as an
 * interleaved (re, im) pair of doubles (16 bytes).  All tensors are dense
 * column-major, storage length max(1, prod(shape)) (tensor.rs:45-54).
 *
 * Status values mirror the reference's error kinds so that callers can map
 * them onto the C ABI's NDT_* codes exactly as crates/ndtensors-capi does:
 *   NDO_OK                      success
 *   NDO_ERR_WRONG_NUM_INDICES   TensorError::WrongNumberOfIndices
 *   NDO_ERR_SHAPE_MISMATCH      TensorError::ShapeMismatch
 *   NDO_ERR_INVALID_PERMUTATION TensorError::InvalidPermutation
 *   NDO_ERR_BLOCK_NOT_FOUND     TensorError::BlockNotFound
 *   NDO_PANIC                   a Rust panic inside the reference (division
 *                               by a zero extent, out-of-range get_linear,
 *                               a failed assert_eq!) that catch_unwind turns
 *                               into NDT_INTERNAL_ERROR
 *   NDO_ERR_CAPACITY            caller-provided buffer too small (oracle-only)
 */
#ifndef NDT_ORACLE_H
#define NDT_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NDO_OK 0
#define NDO_ERR_WRONG_NUM_INDICES 1
#define NDO_ERR_SHAPE_MISMATCH 2
#define NDO_ERR_INVALID_PERMUTATION 3
#define NDO_ERR_BLOCK_NOT_FOUND 4
#define NDO_ERR_CAPACITY 8
#define NDO_PANIC 9

/* strides.rs:19-33 */
void ndo_compute_strides(const size_t* shape, size_t ndim, size_t* strides);
/* strides.rs:46-52 */
size_t ndo_cartesian_to_linear(const size_t* idx, const size_t* strides, size_t ndim);
/* strides.rs:64-73; NDO_PANIC on a zero extent (Rust `%` by zero) */
int ndo_linear_to_cartesian(size_t linear, const size_t* shape, size_t ndim, size_t* idx);

/* permutedims.rs:198-224 */
int ndo_validate_permutation(const size_t* perm, size_t nperm, size_t ndim);

/* permutedims.rs:51-68 + backend/generic.rs:15-39.  dst holds max(1, prod)
 * elements in the permuted shape perm.map(shape). */
int ndo_permutedims(int dtype, const void* src, const size_t* shape, size_t ndim,
                    const size_t* perm, size_t nperm, void* dst);
/* Same algorithm restricted to source linear indices [lo, hi): lets a caller
 * spread the reference's per-element loop over host threads. */
int ndo_permutedims_range(int dtype, const void* src, const size_t* shape, size_t ndim,
                          const size_t* perm, void* dst, size_t lo, size_t hi);

/* contract/naive.rs:45-116: validation + output shape of the C ABI contract. */
int ndo_contract_naive_outshape(const size_t* sa, size_t na, const int32_t* la, size_t nla,
                                const size_t* sb, size_t nb, const int32_t* lb, size_t nlb,
                                size_t* out_shape, size_t* out_ndim);
/* contract/naive.rs:45-187: the loop the C ABI's ndt_tensor_f64_contract runs. */
int ndo_contract_naive(int dtype,
                       const void* a, size_t len_a, const size_t* sa, size_t na, const int32_t* la, size_t nla,
                       const void* b, size_t len_b, const size_t* sb, size_t nb, const int32_t* lb, size_t nlb,
                       void* out, size_t out_cap);

/* contract/properties.rs:94-203.  Writes (all arrays caller-sized to
 * na / nb / na+nb): npairs, pairs_a, pairs_b, unc_a (n_unc_a), unc_b
 * (n_unc_b), perm_a (na), perm_b, perm_c, output_labels, dims[3] =
 * {dleft, dmid, dright}, flags[3] = {permute_a, permute_b, permute_c}. */
int ndo_contract_properties(const int32_t* la, const size_t* sa, size_t na,
                            const int32_t* lb, const size_t* sb, size_t nb,
                            size_t* npairs, size_t* pairs_a, size_t* pairs_b,
                            size_t* n_unc_a, size_t* unc_a, size_t* n_unc_b, size_t* unc_b,
                            size_t* perm_a, size_t* perm_b, size_t* perm_c,
                            int32_t* output_labels, size_t* dims, int* flags);

/* contract/gemm.rs:47-95: output shape (after perm_c) of contract_gemm. */
int ndo_contract_gemm_outshape(const size_t* sa, size_t na, const int32_t* la, size_t nla,
                               const size_t* sb, size_t nb, const int32_t* lb, size_t nlb,
                               size_t* out_shape, size_t* out_ndim);
/* contract/gemm.rs:47-236 (TTGT).  The GEMM is a plain column-major i-j-k
 * loop accumulating in increasing k, standing in for faer's matmul. */
int ndo_contract_gemm(int dtype,
                      const void* a, size_t len_a, const size_t* sa, size_t na, const int32_t* la, size_t nla,
                      const void* b, size_t len_b, const size_t* sb, size_t nb, const int32_t* lb, size_t nlb,
                      void* out, size_t out_cap);

/*
 * Block-sparse tensors (storage/blocksparse/ and blocksparse_tensor.rs).
 * A block-sparse tensor is described by
 *   ndim, nblk[ndim]               number of blocks per axis
 *   bsz[sum(nblk)]                 block sizes, axis 0's first (BlockDim::new)
 *   nnzb, coords[nnzb*ndim]        stored blocks, in storage order
 *   data                           blocks packed in that order
 *                                  (BlockOffsets::from_blocks, block_offsets.rs:76-90)
 */
typedef struct {
  size_t ndim;
  const size_t* nblk;
  const size_t* bsz;
  size_t nnzb;
  const size_t* coords;
} ndo_bs_desc;

/* contract/blocksparse.rs:87-141, :186-275: output structure.  On input
 * *out_nnzb is the capacity of out_coords (in blocks); on output it is the
 * number of output blocks (sorted lexicographically).  out_nblk / out_bsz
 * must hold (na + nb) entries / sum of A's and B's block counts (+1). */
int ndo_bs_contract_plan(const ndo_bs_desc* A, const int32_t* la, size_t nla,
                         const ndo_bs_desc* B, const int32_t* lb, size_t nlb,
                         size_t* out_ndim, size_t* out_nblk, size_t* out_bsz,
                         size_t* out_nnzb, size_t* out_coords, size_t* out_total);
/* contract/blocksparse.rs:144-180: per output block, per matched pair,
 * contract_gemm on copied blocks, first insert then add.  out must hold
 * out_total elements laid out per ndo_bs_contract_plan. */
int ndo_bs_contract(int dtype, const ndo_bs_desc* A, const void* a_data, const int32_t* la, size_t nla,
                    const ndo_bs_desc* B, const void* b_data, const int32_t* lb, size_t nlb,
                    void* out, size_t out_cap);
/* Number of matched pairs and sum over pairs of m*n*k (for flop counts). */
int ndo_bs_contract_work(const ndo_bs_desc* A, const int32_t* la, size_t nla,
                         const ndo_bs_desc* B, const int32_t* lb, size_t nlb,
                         size_t* npairs, double* mnk_sum);

/* operations/blocksparse.rs:61-129 (block structure permuted, re-sorted,
 * repacked; each block permuted densely).  out_coords holds nnzb*ndim. */
int ndo_bs_permutedims(int dtype, const ndo_bs_desc* A, const void* a_data,
                       const size_t* perm, size_t nperm,
                       size_t* out_nblk, size_t* out_bsz, size_t* out_coords, void* out);

/* blocksparse_tensor.rs:290-324: dense has max(1, prod(dense_shape)) elements. */
int ndo_bs_to_dense(int dtype, const ndo_bs_desc* A, const void* a_data, void* dense);
/* blocksparse_tensor.rs:353-391 */
int ndo_bs_from_dense(int dtype, const ndo_bs_desc* A, const void* dense, void* out);

/* DiagBlockSparse (storage/blocksparse/diagblocksparse.rs:86-230,
 * diagblocksparse_tensor.rs:399-426): only min(block shape) diagonal values
 * per listed block, packed in the listed order. */
size_t ndo_diag_nnz(const ndo_bs_desc* S);
int ndo_diag_to_dense(int dtype, const ndo_bs_desc* S, const void* s_data, void* dense);

#ifdef __cplusplus
}
#endif
#endif
