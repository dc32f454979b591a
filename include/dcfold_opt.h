/*
 * dcfold_opt.h — C ABI of libdcfold_opt.so, the pass driver that runs the
 * dense-constant folds of mlirpass's pipelines on MLIR text with libdcfold.
 *
 * It stands in for the parts of mlirpass around the fold hooks that a
 * fold-only run needs: reading and printing the generic form, the greedy
 * rewrite driver (src/rewrite.rs:785-906), `canonicalize` as a bare flag
 * (src/pass.rs:693-695) and nested `func.func(...)` pipelines whose
 * functions the reference runs as parallel tasks (src/pass.rs:280-341), plus
 * the `tosa-layerwise-constant-fold` pass that the reference lacks.  Only
 * folds run: the reference's canonicalization rewrite patterns are not
 * restated.
 */
#ifndef DCFOLD_OPT_H
#define DCFOLD_OPT_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Phase timings and counters of one run (milliseconds / counts). */
typedef struct dcf_opt_stats {
  double parse_ms;   /* text -> IR */
  double run_ms;     /* the pipeline, including host<->device transfers and
                        bringing every folded constant back to host memory */
  double print_ms;   /* IR -> text */
  unsigned long long folds, refused, h2d_bytes, d2h_bytes, batches;
  /* parts of run_ms, summed over the GPUs: packing constants into the
   * pinned staging slots and copying them in (with their decode), the fold
   * launches and their statuses, and bringing results back to the host */
  double upload_ms, fold_ms, download_ms;
} dcf_opt_stats;

/* Run `pipeline` ("canonicalize", or "builtin.module(func.func(P,...))" with
 * P in canonicalize, tosa-layerwise-constant-fold) over the module `text`
 * on GPUs 0..n_gpus-1 (n_gpus < 0: every GPU).  n_gpus == 0 runs host-only:
 * parsing, printing and the folds decided without element work (shortcuts)
 * succeed, and any fold that needs element work fails with an error; there
 * is no CPU fallback.  `flags` is a mask of DCF_OPT_* bits: with
 * DCF_OPT_SPLIT_INPUT_FILE chunks separated by "// -----" lines are run
 * separately; with DCF_OPT_LOCAL_SCOPE (mlir-opt's --mlir-print-local-scope)
 * a module is not followed by a blank line; with DCF_OPT_DEBUGINFO
 * (--mlir-print-debuginfo) locations are printed, without it op and block
 * argument locations and `#loc` aliases are dropped.  Alias definitions
 * that the printed module does not use are dropped.  On success *out is a
 * buffer holding the
 * printed module (give it back with dcf_opt_free) and the return value is 0;
 * otherwise a negative code and dcf_opt_last_error() says why. */
#define DCF_OPT_SPLIT_INPUT_FILE 1
#define DCF_OPT_LOCAL_SCOPE 2
#define DCF_OPT_DEBUGINFO 4
/* By default every float and integer constant the module holds is printed
 * from its values (dcf_opt_print_element for each element; large non-splat
 * values as uppercase hex), as the reference re-reads every such dense
 * attribute at import (canonical_floats, src/ir.rs:2149-2164) and prints it
 * back.  With DCF_OPT_VERBATIM parsed constants keep their input text
 * instead, which is the same text when mlir-opt printed the input. */
#define DCF_OPT_VERBATIM 8

int dcf_opt_run(const char* text, size_t len, const char* pipeline, int n_gpus, int flags,
                char** out, size_t* out_len, dcf_opt_stats* stats);

/* Give back an output buffer.  The library keeps the last buffer given
 * back, with its pages mapped, for a later run whose output fits it. */
void dcf_opt_free(char* p);

const char* dcf_opt_last_error(void);

/* The text of one element of a dense attribute whose element type is
 * `dtype` (a dcf_dtype of dcfold.h), as the printer writes it and as
 * mlir-opt does: a float in six-digit scientific form ("1.000000e+00") when
 * that text parses back to the same bits, else in the shortest form that
 * round-trips ("2.00000024", "3.0757404601899907E-5") when it has a decimal
 * point, else as its hex bit pattern ("0x7FC00000"); an integer in decimal,
 * i1 as true / false.  This decides the printed text of every folded
 * constant of up to 100 elements, which mlirpass must print byte for byte
 * as mlir-opt does (its printing goes through mlirformat's Const ->
 * Attribute, src/ir.rs:2149-2164).  Writes the text and a NUL into out
 * (cap bytes); returns its length, or a negative value if dtype is not an
 * element type or cap is too small. */
int dcf_opt_print_element(int dtype, unsigned long long bits, char* out, size_t cap);

#ifdef __cplusplus
}
#endif

#endif
