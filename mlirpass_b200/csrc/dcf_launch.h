// dcf_launch.h — internal launch interface between the host runtime and the
// kernel translation units.  Not part of the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/dcfold.h"

namespace dcf {

// One job of a batched step, as the batch kernel reads it from device memory.
struct BatchDesc {
  const void* l;
  const void* r;
  void* o;
  uint64_t n;
  int lsplat;
  int rsplat;
  dcf_status* st;
};

struct EwLaunch {
  int op = 0;
  int dtype = 0;      // operand type
  int out_dtype = 0;  // result type (convert ops); ignored otherwise
  uint32_t flags = 0;
  const void* l = nullptr;
  const void* r = nullptr;
  void* o = nullptr;
  uint64_t n = 0;
  const void* l0 = nullptr;
  const void* r0 = nullptr;
  int lsplat = 0;
  int rsplat = 0;
  uint64_t base = 0;
  dcf_status* st = nullptr;
  cudaStream_t stream = nullptr;
  // batched form (n = the largest job's element count)
  const BatchDesc* batch = nullptr;
  int n_jobs = 0;
};

// Op classes (one place for the runtime, the batch entry points and the
// kernel dispatch).
inline bool op_float_binary(int op) {
  return (op >= DCF_ADDF && op <= DCF_REMF) || op == DCF_CMPF || op == DCF_COPYSIGN;
}
inline bool op_int_binary(int op) {
  return (op >= DCF_ADDI && op <= DCF_MULUI_HI) || op == DCF_CMPI || op == DCF_ADDUI_CARRY || op == DCF_IPOWI;
}
// Unary math folds (element type unchanged), float and integer.
inline bool op_math_float_unary(int op) { return op >= DCF_ABSF && op <= DCF_RSQRT; }
inline bool op_math_int_unary(int op) { return op >= DCF_ABSI && op <= DCF_CTPOP; }
inline bool op_binary(int op) { return op_float_binary(op) || op_int_binary(op); }
// Binary ops whose result elements are i1 bytes.
inline bool op_bool_result(int op) { return op == DCF_CMPI || op == DCF_CMPF || op == DCF_ADDUI_CARRY; }
inline bool op_convert(int op) {
  return (op >= DCF_EXTF && op <= DCF_TRUNCI) || op_math_float_unary(op) || op_math_int_unary(op);
}
// Whether a conversion op accepts the (from, to) element types.
inline bool convert_types_ok(int op, bool from_float, bool from_int, bool to_float, bool to_int, int from, int to) {
  switch (op) {
    case DCF_EXTF: case DCF_TRUNCF: return from_float && to_float;
    case DCF_SITOFP: case DCF_UITOFP: return from_int && to_float;
    case DCF_FPTOSI: case DCF_FPTOUI: return from_float && to_int;
    case DCF_NEGF: case DCF_FLUSH_DENORMALS: return from_float && from == to;
    case DCF_EXTSI: case DCF_EXTUI: case DCF_TRUNCI: return from_int && to_int;
    default:
      if (op_math_float_unary(op)) return from_float && from == to;
      if (op_math_int_unary(op)) return from_int && from == to;
      return false;
  }
}

// Each returns DCF_OK, DCF_EUNSUPPORTED for an (op, type) pair it does not
// handle, or DCF_ECUDA.
int launch_float_binary(const EwLaunch& a);    // addf..minnumf, cmpf
int launch_int_binary(const EwLaunch& a);      // addi..minui, cmpi
int launch_convert(const EwLaunch& a);         // extf, truncf, si/uitofp, fptosi/ui
int launch_reciprocal(const EwLaunch& a);
int launch_math_unary(const EwLaunch& a);     // absf..rsqrt, absi..ctpop

// With a status, 2-byte transposes take the bulk-tensor kernel when the
// shapes and alignment allow (its bounded waits report through st->error).
int launch_transpose2d(size_t elem_size, uint64_t rows, uint64_t cols, const void* in, void* out,
                       cudaStream_t stream, dcf_status* st = nullptr);
int launch_transpose2_tma(const void* in, void* out, uint64_t rows, uint64_t cols, dcf_status* st,
                          cudaStream_t stream);
int launch_permute(size_t elem_size, int rank, const int64_t* in_shape, const int64_t* perms,
                   const void* in, void* out, cudaStream_t stream, dcf_status* st = nullptr);
int launch_hex_encode(const void* in, uint64_t nbytes, char* out, cudaStream_t stream);
int launch_hex_decode(const char* in, uint64_t nchars, void* out, dcf_status* st, cudaStream_t stream);
int launch_hex_decode_pieces(const dcf_hex_piece* pieces, size_t n, uint64_t max_nchars, dcf_status* st,
                             cudaStream_t stream);
int launch_hash_pieces(const dcf_hash_piece* pieces, size_t n, uint64_t max_bytes, uint64_t* out,
                       cudaStream_t stream);
int launch_select(size_t elem_size, const void* cond, int cond_splat, const void* t, int t_splat, const void* f,
                  int f_splat, uint64_t n, void* out, dcf_status* st, cudaStream_t stream);
int launch_splat_check(const void* in, size_t elem_size, uint64_t n, dcf_status* st, cudaStream_t stream);

// Set the per-thread text dcf_last_error() returns; returns `code`.
int record_error(int code, const char* msg);

// Count one kernel launch (dcf_kernel_launches).
void note_launch();
uint64_t launches();

// Dispatch by op (used by the runtime).
int launch_ew(const EwLaunch& a);

size_t dtype_size(int dtype);
bool is_float(int dtype);
bool is_int(int dtype);

}  // namespace dcf
