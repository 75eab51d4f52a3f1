/*
 * A plain C caller of libndtensors_capi.so: the reference's 19-symbol C ABI
 * (crates/ndtensors-capi/src/lib.rs) used the way a C, Julia or Rust caller
 * binds it -- header, shared library, nothing else.
 *
 *   abi_check host    handle bookkeeping and status codes only (no GPU
 *                     needed); every computation must fail with
 *                     NDT_INTERNAL_ERROR when no device is present
 *   abi_check device  also the computations, against hand-computed answers
 *
 * Exit status 0 when every check passes; each failed check prints a line.
 */
#include <math.h>
#include <stdio.h>
#include <string.h>

#include "ndtensors_capi.h"

static int failures = 0;

#define CHECK(cond, what)                                   \
  do {                                                      \
    if (!(cond)) {                                          \
      fprintf(stderr, "FAIL %s:%d %s\n", __FILE__, __LINE__, what); \
      failures++;                                           \
    }                                                       \
  } while (0)

static int same(const double* x, const double* y, size_t n) {
  for (size_t i = 0; i < n; i++)
    if (fabs(x[i] - y[i]) > 1e-12 * (1.0 + fabs(y[i]))) return 0;
  return 1;
}

int main(int argc, char** argv) {
  const int device = argc > 1 && strcmp(argv[1], "device") == 0;
  int st = 12345;

  /* A = [[1,3,5],[2,4,6]] (2 x 3, column-major data 1..6) */
  const double a_data[6] = {1, 2, 3, 4, 5, 6};
  const size_t a_shape[2] = {2, 3};
  ndt_tensor_f64* A = ndt_tensor_f64_from_data(a_data, 6, a_shape, 2, &st);
  CHECK(A && st == NDT_SUCCESS, "from_data");
  CHECK(ndt_tensor_f64_ndim(A) == 2 && ndt_tensor_f64_len(A) == 6, "ndim / len");
  size_t shp[2] = {0, 0};
  CHECK(ndt_tensor_f64_shape(A, shp) == NDT_SUCCESS && shp[0] == 2 && shp[1] == 3, "shape");
  double v = 0;
  CHECK(ndt_tensor_f64_get_linear(A, 4, &v) == NDT_SUCCESS && v == 5.0, "get_linear");
  CHECK(ndt_tensor_f64_get_linear(A, 6, &v) == NDT_INDEX_OUT_OF_BOUNDS, "get_linear out of range");
  CHECK(ndt_tensor_f64_from_data(a_data, 5, a_shape, 2, &st) == NULL && st == NDT_SHAPE_MISMATCH,
        "from_data length mismatch");
  CHECK(ndt_tensor_f64_zeros(NULL, 2, &st) == NULL && st == NDT_INVALID_ARGUMENT, "zeros(NULL)");

  /* storage length max(1, prod(shape)): a zero extent still holds one element */
  const size_t z_shape[2] = {0, 3};
  ndt_tensor_f64* Z = ndt_tensor_f64_zeros(z_shape, 2, &st);
  CHECK(Z && st == NDT_SUCCESS && ndt_tensor_f64_len(Z) == 1, "zero-extent length");
  ndt_tensor_f64_release(Z);
  ndt_tensor_f64_release(NULL); /* NULL-safe */

  /* clone shares the buffer; mutation copies on write */
  ndt_tensor_f64* A2 = ndt_tensor_f64_clone(A);
  CHECK(A2 != NULL, "clone");
  CHECK(ndt_tensor_f64_set_linear(A2, 0, 100.0) == NDT_SUCCESS, "set_linear");
  CHECK(ndt_tensor_f64_get_linear(A, 0, &v) == NDT_SUCCESS && v == 1.0, "clone is copy on write");
  CHECK(ndt_tensor_f64_fill(A2, 2.5) == NDT_SUCCESS, "fill");
  CHECK(ndt_tensor_f64_data(A2)[5] == 2.5, "data after fill");
  ndt_tensor_f64_release(A2);

  /* permutedims: invalid permutation -> NDT_INVALID_PERMUTATION (checked first) */
  const size_t bad_perm[2] = {0, 0};
  CHECK(ndt_tensor_f64_permutedims(A, bad_perm, 2, &st) == NULL && st == NDT_INVALID_PERMUTATION,
        "invalid permutation");

  const size_t perm[2] = {1, 0};
  ndt_tensor_f64* At = ndt_tensor_f64_permutedims(A, perm, 2, &st);
  if (!device) {
    CHECK(At == NULL && st == NDT_INTERNAL_ERROR, "no device: permutedims fails with NDT_INTERNAL_ERROR");
  } else {
    const double at_ref[6] = {1, 3, 5, 2, 4, 6};
    CHECK(At && st == NDT_SUCCESS && same(ndt_tensor_f64_data(At), at_ref, 6), "transpose");

    /* naive contract: A(1,-1) . At(-1,2) = A A^T = [[35,44],[44,56]] */
    const long la[2] = {1, -1}, lb[2] = {-1, 2};
    ndt_tensor_f64* C = ndt_tensor_f64_contract(A, la, 2, At, lb, 2, &st);
    const double c_ref[4] = {35, 44, 44, 56};
    CHECK(C && st == NDT_SUCCESS && same(ndt_tensor_f64_data(C), c_ref, 4), "contract A A^T");

    /* mismatched contracted extents -> NDT_SHAPE_MISMATCH */
    const long lbad[2] = {-1, 2};
    CHECK(ndt_tensor_f64_contract(A, la, 2, A, lbad, 2, &st) == NULL && st == NDT_SHAPE_MISMATCH,
          "contract shape mismatch");

    /* VJP of C = A At with upstream gradient G = ones(2,2):
       dA = G At^T = [[3,7,11],[3,7,11]], dAt = A^T G = [[3,3],[7,7],[11,11]] */
    const size_t g_shape[2] = {2, 2};
    ndt_tensor_f64* G = ndt_tensor_f64_ones(g_shape, 2, &st);
    ndt_tensor_f64 *gA = NULL, *gB = NULL;
    ndt_tensor_f64_contract_vjp(A, la, 2, At, lb, 2, G, &gA, &gB, &st);
    const double ga_ref[6] = {3, 3, 7, 7, 11, 11}, gb_ref[6] = {3, 7, 11, 3, 7, 11};
    CHECK(st == NDT_SUCCESS && gA && gB, "vjp status");
    if (gA && gB) {
      CHECK(same(ndt_tensor_f64_data(gA), ga_ref, 6), "vjp grad A");
      CHECK(same(ndt_tensor_f64_data(gB), gb_ref, 6), "vjp grad B");
    }
    ndt_tensor_f64_release(gA);
    ndt_tensor_f64_release(gB);
    ndt_tensor_f64_release(G);
    ndt_tensor_f64_release(C);
  }
  ndt_tensor_f64_release(At);
  ndt_tensor_f64_release(A);
  if (failures == 0) printf("abi_check %s: all checks passed\n", device ? "device" : "host");
  return failures ? 1 : 0;
}
