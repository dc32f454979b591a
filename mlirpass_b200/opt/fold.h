// fold.h — the fold hooks and the greedy rewrite driver of dcfold-opt.
//
// Host-side restatement of the mlirpass code that sits around the element
// loops libdcfold replaces:
//   ArithFolder::fold   src/patterns/arith/canonicalize.rs:270-491 (shortcuts,
//                       then the loop -> a FoldRequest for the GPU)
//   Tf::fold            src/patterns/tosa/canonicalize.rs:189-232, 497-511, 596-605
//   Body::fold_with     src/patterns/canonicalize.rs:328-378
//   materialize         src/patterns/arith/canonicalize.rs:1845-1859,
//                       src/patterns/tosa/canonicalize.rs:1237-1241
//   apply_greedily      src/rewrite.rs:679-906 (worklist, constant hoisting
//                       and dedup, fold-then-patterns, replace_folded)
// plus the two constant-fold patterns of the new tosa-layerwise-constant-fold
// pass (upstream MLIR semantics: reciprocal and transpose of a constant with
// a single use, or a splat).  The canonicalization *patterns* of the
// reference are not restated: only folds run here.
//
// The driver is resumable.  When a fold needs element work it hands back a
// FoldRequest and stops; the scheduler runs the requests of many isolated
// functions as one batch on the GPU, then resumes every driver.
#pragma once

#include <memory>
#include <string>
#include <vector>

#include "engine.h"
#include "ir.h"

namespace dco {

struct GreedyConfig {
  bool top_down = false;
  bool fold = true;
  bool cse_constants = true;
  int max_iterations = 10;
  bool layerwise = false;  // add the tosa-layerwise-constant-fold patterns
};

class Greedy {
 public:
  Greedy(Module& m, Region* region, GreedyConfig cfg, Engine& eng);
  ~Greedy();
  // Run until the driver needs element work (returns the request, to be
  // executed before the next call) or has finished (returns nullptr).
  FoldRequest* step();
  bool done() const;
  bool converged() const;
  Engine& engine();

 private:
  struct Impl;
  std::unique_ptr<Impl> impl_;
};

struct PassStats {
  uint64_t folds = 0, refused = 0, shortcuts = 0;
};

// Run a pass pipeline on the module.  Accepted forms:
//   "canonicalize"                      (module-level, like --canonicalize)
//   "builtin.module(func.func(P1,P2,...))" with P in
//     {canonicalize, tosa-layerwise-constant-fold}
// Functions of a nested pipeline are spread over `engines` (one per GPU) and
// their element folds are batched per round.
void run_pipeline(Module& m, const std::string& pipeline, std::vector<Engine*>& engines, PassStats* stats);

// Bring every device-resident constant of the module to the host.
void fetch_results(Module& m, std::vector<Engine*>& engines);

}  // namespace dco
