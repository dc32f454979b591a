/*
 * dcf_oracle.h — CPU oracle for the dense-constant folds.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a scalar, plain-C restatement of the
 * reference's per-element fold closures, used by the tests, by the smoke
 * check and as the timed CPU baseline.  The product (libdcfold.so) never
 * links or calls it.
 *
 * The reference (mlirpass, Rust) cannot be built here: no Rust toolchain,
 * and its arithmetic crate mlirformat 0.9.0 (git tag 0.9.0, rev
 * f7aa89884e6d2a38c863b5f82bb5df2f19520cc9) is not vendored.  Each function
 * below cites the reference closure it restates; where the behaviour lives
 * in mlirformat (ApFloat / ApInt arithmetic, the dense text codec), the
 * published IEEE-754 / LLVM APFloat semantics are restated instead, and the
 * result is pinned against the reference's own fixture golden vectors
 * (tests/golden/).
 *
 * The function signatures mirror include/dcfold.h so one test can drive both.
 */
#ifndef DCF_ORACLE_H
#define DCF_ORACLE_H

#include <stdint.h>
#include <stddef.h>
#include "../include/dcfold.h"

#ifdef __cplusplus
extern "C" {
#endif

int dco_binary(int op, int dtype, const void* lhs, int lhs_splat,
               const void* rhs, int rhs_splat, uint64_t n, uint32_t flags,
               void* out, dcf_result* res);
int dco_convert(int op, int from, int to, const void* in, int in_splat,
                uint64_t n, uint32_t flags, void* out, dcf_result* res);
int dco_reciprocal(int dtype, const void* in, int in_splat, uint64_t n,
                   uint32_t flags, void* out, dcf_result* res);
int dco_select(size_t elem_size, const uint8_t* cond, int cond_splat, const void* t, int t_splat,
               const void* f, int f_splat, uint64_t n, void* out, dcf_result* res);
int dco_transpose(size_t elem_size, int rank, const int64_t* in_shape,
                  const int64_t* perms, const void* in, void* out);
int dco_hex_encode(const void* in, uint64_t nbytes, char* out);
int dco_hex_decode(const char* in, uint64_t nchars, void* out);
int dco_splat_check(const void* in, size_t elem_size, uint64_t n);

uint64_t dco_hash(const void* data, uint64_t nbytes);

/* Scalar helpers exposed for the golden-vector tests. */
uint64_t dco_float_convert_bits(int from, int to, uint64_t bits, int* ok);
uint64_t dco_round_from_double(int to, double x);

#ifdef __cplusplus
}
#endif
#endif
