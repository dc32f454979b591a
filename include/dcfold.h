/*
 * dcfold.h — C ABI of the B200 dense-constant folding library (libdcfold.so).
 *
 * The library folds MLIR ops whose operands are dense constants
 * (DenseElementsAttr) on sm_100a GPUs.  It replaces the per-element loops
 * inside mlirpass's fold hooks; every hook keeps its signature and result:
 *
 *   Folder::binary        src/patterns/arith/canonicalize.rs:203-217
 *   Folder::unary         src/patterns/arith/canonicalize.rs:227-235
 *   Rounded::apply        src/patterns/arith/canonicalize.rs:984-1055
 *   float_convert         src/patterns/arith/canonicalize.rs:727-742
 *   Tf::transpose         src/patterns/tosa/canonicalize.rs:497-511
 *   Tf::reciprocal        src/patterns/tosa/canonicalize.rs:596-605
 *
 * Conventions
 *   - Element data is raw little-endian element storage: i1 and i8 one byte
 *     per element (i1 holds 0 or 1), i16/f16/bf16 two bytes, i32/f32 four,
 *     i64/f64 eight, f8 kinds one byte.  This is the storage of
 *     `Const.values` in the reference and the byte order of the
 *     `dense<"0x…">` hex form.
 *   - "Splat" operands hold exactly one element and broadcast over `n`
 *     (Const::at on a splat, src/patterns/arith/canonicalize.rs:214-215).
 *   - A fold is all-or-nothing, like `collect::<Option<Vec<_>>>()` in the
 *     reference: when any element refuses (divide by zero, INT_MIN / -1,
 *     shift >= width, inexact truncf, NaN -> int, ...) the call still returns
 *     0 but sets `folded = 0` and `first_fail_index` to the lowest refusing
 *     element.  The output buffer then holds no meaningful data.
 *   - Return value: 0 on success (folded or refused), a negative DCF_E* code
 *     on a runtime error; dcf_last_error() then names it.  There is no CPU
 *     fallback: without a usable GPU every compute entry point returns
 *     DCF_ENODEV.
 *
 * Host entry points (dcf_binary, dcf_convert, ...) take HOST pointers,
 * which may be pageable (staged through the library's pinned buffers) or
 * pinned (copied directly); the work is split into row blocks over the
 * GPUs chosen by dcf_init.  *_async entry points take DEVICE pointers
 * (the kernel runs on the device that owns the output pointer) and a
 * cudaStream_t, and report through a device-side dcf_status that the caller
 * fills with 0xFF bytes first (dcf_status_reset_async).
 */
#ifndef DCFOLD_H
#define DCFOLD_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types.  Integer kinds are signless two's complement, as MLIR's
 * iN; float kinds are the IEEE-like layouts of `float_layout`
 * (src/patterns/arith/canonicalize.rs:36-48). */
typedef enum dcf_dtype {
  DCF_I1 = 1,
  DCF_I8 = 2,
  DCF_I16 = 3,
  DCF_I32 = 4,
  DCF_I64 = 5,
  DCF_F16 = 16,
  DCF_BF16 = 17,
  DCF_F32 = 18,
  DCF_F64 = 19,
  DCF_F8E5M2 = 20,
  DCF_F8E4M3 = 21,
  DCF_F8E3M4 = 22
} dcf_dtype;

/* Fold operations.  The names are the arith / tosa op names. */
typedef enum dcf_op {
  /* float binary: Rounded::apply and minmax
   * (src/patterns/arith/canonicalize.rs:336-375, 132-150, 984-1055) */
  DCF_ADDF = 1,
  DCF_SUBF = 2,
  DCF_MULF = 3,
  DCF_DIVF = 4,
  DCF_MAXIMUMF = 5,
  DCF_MINIMUMF = 6,
  DCF_MAXNUMF = 7,
  DCF_MINNUMF = 8,
  /* remf: the exact IEEE remainder of truncating division (fmod), the
   * closure `x % y` of src/patterns/arith/canonicalize.rs:387 */
  DCF_REMF = 9,
  /* integer binary (src/patterns/arith/canonicalize.rs:277-325, 469-683) */
  DCF_ADDI = 16,
  DCF_SUBI = 17,
  DCF_MULI = 18,
  DCF_ANDI = 19,
  DCF_ORI = 20,
  DCF_XORI = 21,
  DCF_SHLI = 22,
  DCF_SHRUI = 23,
  DCF_SHRSI = 24,
  DCF_DIVSI = 25,
  DCF_DIVUI = 26,
  DCF_REMSI = 27,
  DCF_REMUI = 28,
  DCF_MAXSI = 29,
  DCF_MAXUI = 30,
  DCF_MINSI = 31,
  DCF_MINUI = 32,
  /* rounding divisions (src/patterns/arith/canonicalize.rs:287-317,
   * 557-595): refuse on a zero divisor and on signed overflow */
  DCF_CEILDIVUI = 33,
  DCF_CEILDIVSI = 34,
  DCF_FLOORDIVSI = 35,
  /* high half of the double-width product: the second result of
   * mulsi_extended / mului_extended (canonicalize.rs:928-949); the low half
   * is DCF_MULI */
  DCF_MULSI_HI = 36,
  DCF_MULUI_HI = 37,
  /* compares producing i1 bytes (src/patterns/arith/canonicalize.rs:94-130,
   * 791-839); the predicate goes in the flags (DCF_FLAG_PRED) */
  DCF_CMPI = 48,
  DCF_CMPF = 49,
  /* carry bit of addui_extended (canonicalize.rs:878-893): i1 bytes,
   * (a + b mod 2^w) <u a.  The borrow of subui_extended is DCF_CMPI ult. */
  DCF_ADDUI_CARRY = 50,
  /* unary conversions (src/patterns/arith/canonicalize.rs:400-434, 717-762) */
  DCF_EXTF = 64,
  DCF_TRUNCF = 65,
  DCF_SITOFP = 66,
  DCF_UITOFP = 67,
  DCF_FPTOSI = 68,
  DCF_FPTOUI = 69,
  /* more unary element maps through dcf_convert: negf (sign flip,
   * canonicalize.rs:327-333), flush_denormals (:69-77, :376-385), and the
   * integer width changes extsi / extui / trunci (:388-398, :685-706; also
   * index_cast / index_castui, :435-454, with index as i64) */
  DCF_NEGF = 70,
  DCF_FLUSH_DENORMALS = 71,
  DCF_EXTSI = 72,
  DCF_EXTUI = 73,
  DCF_TRUNCI = 74,
  /* tosa.reciprocal, 1/x round-to-nearest-even
   * (src/patterns/tosa/canonicalize.rs:596-605; layerwise pass) */
  DCF_RECIPROCAL = 80,
  /* math dialect folds that are exact (ArithFolder::math,
   * src/patterns/math/canonicalize.rs:145-234), unary through dcf_convert
   * with from == to:
   *   absf        sign cleared (every float type)
   *   ceil, floor, roundeven
   *               to an integral value; a NaN comes back quieted (every
   *               float type, FloatFolds::integral :87-92)
   *   round, trunc, sqrt
   *               f32 / f64 only (any other type refuses); sqrt refuses a
   *               negative operand (sign bit set, -0 and -NaN included);
   *               a NaN comes back quieted
   *   rsqrt       1 / sqrt(x) rounded twice, f32 / f64 only; refuses a
   *               negative operand; a NaN comes back quieted
   *   absi (wrapping), ctlz, cttz, ctpop (of zero: the width)
   * and binary through dcf_binary:
   *   copysign    lhs with rhs's sign bit (every float type)
   *   ipowi       wrapping power by squaring; a negative exponent gives
   *               1 for base 1, +-1 for base -1 by parity, 0 otherwise,
   *               and refuses base 0; i1 refuses (IntFolds::ipowi :95-124)
   * The inexact ones (sin, exp, log, pow, ...) are the host C library's
   * results in the reference and are not offered. */
  DCF_ABSF = 96,
  DCF_CEIL = 97,
  DCF_FLOOR = 98,
  DCF_ROUNDEVEN = 99,
  DCF_ROUND = 100,
  DCF_TRUNC = 101,
  DCF_SQRT = 102,
  DCF_RSQRT = 103,
  DCF_ABSI = 104,
  DCF_CTLZ = 105,
  DCF_CTTZ = 106,
  DCF_CTPOP = 107,
  DCF_COPYSIGN = 112,
  DCF_IPOWI = 113
} dcf_op;

/* Flags word.
 * bits 0-2  : rounding mode of addf/subf/mulf/divf, the `roundingmode`
 *             property: 0 nearest-even, 1 downward, 2 upward, 3 toward
 *             zero, 4 nearest-away (RoundingMode, canonicalize.rs:952-974)
 * bits 8-11 : cmpi / cmpf predicate number (canonicalize.rs:9-18, 109-130)
 * bit 16    : NaN produced by an invalid operation (inf-inf, 0*inf, 0/0)
 *             is the negative quiet NaN instead of the positive one.  The
 *             reference's float arithmetic lives in an un-vendored crate;
 *             the default follows LLVM APFloat (positive quiet NaN). */
#define DCF_FLAG_ROUND_MASK 0x7u
#define DCF_FLAG_PRED_SHIFT 8
#define DCF_FLAG_PRED_MASK (0xFu << DCF_FLAG_PRED_SHIFT)
#define DCF_FLAG_PRED(p) (((uint32_t)(p) & 0xFu) << DCF_FLAG_PRED_SHIFT)
#define DCF_FLAG_NEG_DEFAULT_NAN (1u << 16)

/* Error codes (negative return values). */
#define DCF_OK 0
#define DCF_EINVAL (-1)
#define DCF_ENODEV (-2)
#define DCF_ENOMEM (-3)
#define DCF_ECUDA (-4)
#define DCF_EUNSUPPORTED (-5)
#define DCF_ETIMEOUT (-6)
#define DCF_EPARSE (-7)

/* Outcome of one fold (host entry points). */
typedef struct dcf_result {
  uint8_t folded;   /* 1: every element folded and `out` holds n elements */
  uint8_t is_splat; /* 1: all n output elements are bitwise equal */
  uint8_t reserved[6];
  uint64_t first_fail_index; /* lowest refusing element, UINT64_MAX if none */
} dcf_result;

/* Device-side status written by the *_async entry points.  Reset it to all
 * 0xFF bytes before a fold; afterwards `first_fail == UINT64_MAX` means
 * folded, `splat_word != 0` means all output elements are equal, and
 * `error != 0xFFFFFFFF` means a kernel gave up a bounded wait on its own
 * copies (the fold's output is then not valid; dcf_status_read reports
 * DCF_ETIMEOUT). */
typedef struct dcf_status {
  unsigned long long first_fail;
  unsigned int splat_word;
  unsigned int error;
} dcf_status;

/* One job of a batched fold (dcf_batch): one elementwise fold of one
 * isolated function.  Splat operands are given by pointer with their
 * *_splat flag set. */
typedef struct dcf_job {
  uint32_t op;      /* dcf_op */
  uint32_t dtype;   /* element type of the operands */
  uint32_t out_dtype; /* element type of the result (convert ops) */
  uint32_t flags;
  const void* lhs;  /* host pointer */
  const void* rhs;  /* host pointer, NULL for unary ops */
  void* out;        /* host pointer, n elements of out_dtype */
  uint64_t n;
  uint8_t lhs_splat;
  uint8_t rhs_splat;
  uint8_t reserved[6];
  dcf_result result; /* filled by dcf_batch */
} dcf_job;

/* ---- context -------------------------------------------------------- */

/* Choose the GPUs the host entry points shard over: devices 0..n_gpus-1,
 * or the list in DCF_DEVICES (comma separated) when set.  n_gpus <= 0
 * means every visible device.  Called implicitly with 1 by the first host
 * entry point.  Replaces the host thread pool that runs one task per
 * isolated function (src/pass.rs:280-341).  Returns the number of GPUs
 * in use, or a negative DCF_E* code. */
int dcf_init(int n_gpus);

/* Release all device and pinned memory and streams. */
int dcf_shutdown(void);

/* Number of GPUs the host entry points shard over (after dcf_init). */
int dcf_device_count(void);

/* Text of the last error on this thread ("" if none). */
const char* dcf_last_error(void);

/* Library version string. */
const char* dcf_version(void);

/* Size in bytes of one element of `dtype`, 0 if unknown. */
size_t dcf_dtype_size(dcf_dtype dtype);

/* Number of kernels this library has launched in this process (all
 * devices).  No counterpart in the reference; used by benchmarks to report
 * how much of the timed work ran in the library's own kernels. */
uint64_t dcf_kernel_launches(void);

/* ---- host entry points ---------------------------------------------- */

/* Elementwise binary fold over n result elements: out[i] = op(lhs[i],
 * rhs[i]).  Replaces the loop at src/patterns/arith/canonicalize.rs:214-216
 * for int_binary / float_binary / rounded_binary / cmpi.  Compare ops write
 * i1 bytes. */
int dcf_binary(dcf_op op, dcf_dtype dtype, const void* lhs, int lhs_splat,
               const void* rhs, int rhs_splat, uint64_t n, uint32_t flags,
               void* out, dcf_result* res);

/* Elementwise conversion fold (extf, truncf, sitofp, uitofp, fptosi,
 * fptoui, negf, flush_denormals, extsi, extui, trunci, and the unary math
 * folds with from == to) from `from` to `to`.  Replaces the Const::map
 * closures at src/patterns/arith/canonicalize.rs:327-333, 376-434, 685-762
 * and src/patterns/math/canonicalize.rs:127-234. */
int dcf_convert(dcf_op op, dcf_dtype from, dcf_dtype to, const void* in,
                int in_splat, uint64_t n, uint32_t flags, void* out,
                dcf_result* res);

/* 1/x per element, round-to-nearest-even, for float types.  Replaces
 * Tf::reciprocal (src/patterns/tosa/canonicalize.rs:596-605) and is the
 * element step of the layerwise reciprocal fold. */
int dcf_reciprocal(dcf_dtype dtype, const void* in, int in_splat, uint64_t n,
                   uint32_t flags, void* out, dcf_result* res);

/* Elementwise select over dense constants: out[i] = cond[i] != 0 ? t[i] :
 * f[i], with i1 condition bytes and values of elem_size bytes (1, 2, 4 or
 * 8); a splat operand holds one element.  Never refuses.  Replaces the
 * value loop of Folder::select (src/patterns/arith/canonicalize.rs:869-875);
 * the shortcuts before it (:842-868) stay in the caller. */
int dcf_select(size_t elem_size, const void* cond, int cond_splat,
               const void* t, int t_splat, const void* f, int f_splat,
               uint64_t n, void* out, dcf_result* res);

/* Permute a dense row-major tensor of `rank` dims: out has shape
 * in_shape[perms[i]].  elem_size is 1, 2, 4 or 8 bytes.  Rank 2 with
 * perms {1,0} takes the tiled transpose kernel.  The element step of the
 * layerwise transpose fold; the reference folds only splat or identity
 * transposes (src/patterns/tosa/canonicalize.rs:497-511). */
int dcf_transpose(size_t elem_size, int rank, const int64_t* in_shape,
                  const int64_t* perms, const void* in, void* out,
                  dcf_result* res);

/* Hex codec of the dense<"0x…"> literal body (without the quotes and the
 * 0x prefix): nbytes raw bytes <-> 2*nbytes uppercase hex characters.
 * Stands in for the dense text codec of the un-vendored mlirformat
 * (Const::try_from / Attribute::from(Const), re-exported at src/lib.rs:48).
 * dcf_hex_decode accepts upper and lower case and returns DCF_EPARSE on
 * any other character. */
int dcf_hex_encode(const void* in, uint64_t nbytes, char* out);
int dcf_hex_decode(const char* in, uint64_t nchars, void* out);

/* Whether all n elements of size elem_size are bitwise equal (the splat
 * test that decides `dense<v>` versus the full literal).  *is_splat gets 1
 * or 0. */
int dcf_splat_check(const void* in, size_t elem_size, uint64_t n,
                    int* is_splat);

/* Run many independent folds (one per isolated function) with one launch
 * per step per GPU; jobs are assigned to GPUs by balanced byte count.
 * Each job's `result` is filled.  Jobs whose `op` is DCF_RECIPROCAL or a
 * convert ignore rhs.  Replaces the per-function task fan-out of
 * src/pass.rs:280-341 for the fold-only work of each function. */
int dcf_batch(dcf_job* jobs, size_t n_jobs);

/* As dcf_batch, but the jobs' lhs / rhs / out are DEVICE pointers (all on
 * one device) and the call allocates no memory at all: no cudaMalloc, no
 * cudaFree, no pinned or host heap.  No counterpart in the reference.  It
 * is for callers that cannot allocate device memory when they fold: an
 * embedding runtime whose caching allocator already holds all of HBM (a
 * cudaMalloc would fail or fragment it), or latency-sensitive code that
 * cannot take the device-wide synchronisation cudaMalloc / cudaFree may
 * cause.  Its scratch (one descriptor and one status per job) is a fixed
 * file-scope device array of 64 KiB, so a call takes at most 1024 jobs and
 * a larger list is rejected with DCF_EINVAL.  The first call on a device
 * looks up that array's device address (cudaGetSymbolAddress).  All calls
 * share the array and each re-initialises what it uses; calls whose work
 * overlaps on the GPU (from two threads or streams at once) race on it and
 * must be serialised by the caller.  Work runs on `stream`; the call
 * returns when its results are in each job's `result`. */
int dcf_batch_noalloc(dcf_job* jobs, size_t n_jobs, void* stream);

/* ---- device entry points (caller-owned device memory, async) -------- */

/* Fill a device dcf_status with 0xFF bytes on `stream`. */
int dcf_status_reset_async(dcf_status* status, void* stream);

/* As dcf_binary, on device pointers of the current device (a splat
 * operand is a device pointer to its one element).  Nothing is
 * synchronised: read the outcome with dcf_status_read. */
int dcf_binary_async(dcf_op op, dcf_dtype dtype, const void* lhs,
                     int lhs_splat, const void* rhs, int rhs_splat, uint64_t n,
                     uint32_t flags, void* out, dcf_status* status,
                     void* stream);

int dcf_convert_async(dcf_op op, dcf_dtype from, dcf_dtype to, const void* in,
                      int in_splat, uint64_t n, uint32_t flags, void* out,
                      dcf_status* status, void* stream);

int dcf_reciprocal_async(dcf_dtype dtype, const void* in, int in_splat,
                         uint64_t n, uint32_t flags, void* out,
                         dcf_status* status, void* stream);

int dcf_select_async(size_t elem_size, const void* cond, int cond_splat,
                     const void* t, int t_splat, const void* f, int f_splat,
                     uint64_t n, void* out, dcf_status* status,
                     void* stream);

/* 2-D transpose of a rows x cols row-major matrix on device pointers. */
int dcf_transpose2d_async(size_t elem_size, uint64_t rows, uint64_t cols,
                          const void* in, void* out, void* stream);

/* N-D permutation (as dcf_transpose) on device pointers; rank <= 8. */
int dcf_permute_async(size_t elem_size, int rank, const int64_t* in_shape,
                      const int64_t* perms, const void* in, void* out,
                      void* stream);

/* As dcf_permute_async, with a device status (reset it first).  Transposes
 * of 2-byte elements (a swap of two groups of dims, both extents of the
 * 2-D view multiples of 8, 16-byte aligned buffers) run as a bulk-tensor
 * (TMA) pipeline whose bounded waits report through status->error. */
int dcf_permute_status_async(size_t elem_size, int rank,
                             const int64_t* in_shape, const int64_t* perms,
                             const void* in, void* out, dcf_status* status,
                             void* stream);

/* Splat test on device memory: afterwards status->splat_word != 0 when all
 * n elements equal element 0 (the all-values test of Tf::splat,
 * src/patterns/tosa/canonicalize.rs:97-100).  Reset the status first. */
int dcf_splat_check_async(const void* in, size_t elem_size, uint64_t n,
                          dcf_status* status, void* stream);

int dcf_hex_encode_async(const void* in, uint64_t nbytes, char* out,
                         void* stream);
int dcf_hex_decode_async(const char* in, uint64_t nchars, void* out,
                         dcf_status* status, void* stream);

/* One literal of a batched hex decode: nchars characters at `in` become
 * nchars / 2 bytes at `out` (both device pointers). */
typedef struct dcf_hex_piece {
  const char* in;
  void* out;
  uint64_t nchars;
} dcf_hex_piece;

/* Decode n literals with one launch (per 65535 pieces).  `pieces` is a
 * DEVICE array of n descriptors that the caller has written; max_nchars
 * bounds every piece's nchars (it sizes the grid, so split very long
 * literals into pieces of similar length).  A piece whose output is 8-byte
 * aligned is decoded 16 characters per thread step at any text alignment;
 * when its text is not 16-byte aligned the kernel reads the whole aligned
 * 16-byte blocks around it, so up to 15 bytes before the text and 16 bytes
 * after it must be readable device memory.  An invalid character or an odd
 * length sets status->first_fail.  The literal-by-literal decode of many
 * constants that a module parse needs, without one launch per constant.
 * Reset the status first. */
int dcf_hex_decode_many_async(const dcf_hex_piece* pieces, size_t n,
                              uint64_t max_nchars, dcf_status* status,
                              void* stream);

/* One byte range of a batched hash (device pointer). */
typedef struct dcf_hash_piece {
  const void* data;
  uint64_t nbytes;
} dcf_hash_piece;

/* 64-bit hashes of n device byte ranges with one launch (per 65535):
 * out[i] (device) gets the hash of pieces[i] (a DEVICE array); max_bytes
 * bounds every piece's length.  Equal bytes give equal hashes; a caller
 * that deduplicates constants confirms equal hashes byte for byte.  The
 * hash is the sum over 8-byte words w_i (the last zero-padded) of
 * mix(w_i ^ i * 0x9E3779B97F4A7C15) plus mix(nbytes), mix being the
 * SplitMix64 finaliser.  Stands in for the O(bytes) Attribute equality of
 * the greedy driver's constant folder (src/rewrite.rs:689-728). */
int dcf_hash_many_async(const dcf_hash_piece* pieces, size_t n,
                        uint64_t max_bytes, uint64_t* out, void* stream);

/* Read a device dcf_status back into a dcf_result (synchronises stream). */
int dcf_status_read(const dcf_status* status, void* stream, dcf_result* res);

#ifdef __cplusplus
}
#endif

#endif /* DCFOLD_H */
