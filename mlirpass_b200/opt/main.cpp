// main.cpp — the C ABI (include/dcfold_opt.h) and the `dcfold-opt` command
// line of the pass driver.
#include <cctype>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iostream>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/dcfold_opt.h"
#include "engine.h"
#include "fold.h"
#include "ir.h"

namespace {

thread_local std::string g_opt_err;

using Clock = std::chrono::steady_clock;
double ms_since(Clock::time_point t) { return std::chrono::duration<double, std::milli>(Clock::now() - t).count(); }

struct Engines {
  std::vector<std::unique_ptr<dco::Engine>> own;
  std::vector<dco::Engine*> list;
  explicit Engines(int n) {
    if (n == 0) {  // host-only
      own.push_back(std::make_unique<dco::Engine>(-1));
      list.push_back(own.back().get());
      return;
    }
    int visible = 0;
    if (cudaGetDeviceCount(&visible) != cudaSuccess || visible <= 0)
      throw std::runtime_error("no CUDA device available; dcfold-opt has no CPU fallback");
    if (n <= 0 || n > visible) n = visible;
    for (int i = 0; i < n; i++) {
      own.push_back(std::make_unique<dco::Engine>(i));
      list.push_back(own.back().get());
    }
    // DCF_OPT_RANGES_PER_GPU (default 1): element ranges per GPU for bare
    // canonicalize, each run by an engine (stream) of its own.
    const char* e = getenv("DCF_OPT_RANGES_PER_GPU");
    const int k = e && atoi(e) > 0 ? atoi(e) : 1;
    std::vector<dco::Engine*> subs(list);
    for (int r = 1; r < k; r++)
      for (int i = 0; i < n; i++) {
        own.push_back(std::make_unique<dco::Engine>(i));
        subs.push_back(own.back().get());
      }
    if (subs.size() > 1) sharded = std::make_unique<dco::ShardedEngine>(subs);
  }
  // Bare `canonicalize` runs the whole module as one unit (the reference
  // runs it on one thread); over several GPUs its large constants are split
  // into element ranges, one per GPU.  Nested pipelines place whole
  // functions on the GPUs instead.
  std::vector<dco::Engine*> for_pipeline(const std::string& pipeline) {
    size_t a = pipeline.find_first_not_of(" \t-");
    if (sharded && a != std::string::npos && pipeline.compare(a, 12, "canonicalize") == 0) return {sharded.get()};
    return list;
  }
  std::unique_ptr<dco::ShardedEngine> sharded;
  dco::Engine* of(const dco::DenseValue& v) {
    if (sharded && !v.parts.empty()) return sharded.get();
    if (v.dev)
      for (auto* e : list)
        if (e->device() == v.dev->device) return e;
    return list[0];
  }
};

std::string hex_hook(dco::DenseValue& v, void* ctx) { return ((Engines*)ctx)->of(v)->hex_of(v); }
uint64_t bits_hook(dco::DenseValue& v, void* ctx) { return ((Engines*)ctx)->of(v)->bits0_of(v); }

// Whether the copy engine can read `text` in place (page-locked memory).
bool is_pinned(std::string_view text) {
  if (text.empty()) return false;
  for (const char* p : {text.data(), text.data() + text.size() - 1}) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    if (a.type != cudaMemoryTypeHost) return false;
  }
  return true;
}

// Chunks of --split-input-file: the text between lines that read exactly
// "// -----" (trailing blanks allowed), as Invocation::chunks splits
// (src/pass.rs:704-716).
std::vector<std::string_view> split_chunks(std::string_view text, bool split) {
  std::vector<std::string_view> out;
  if (!split) {
    out.push_back(text);
    return out;
  }
  static constexpr std::string_view kMarker = "// -----";
  size_t start = 0;
  for (size_t at = 0; at < text.size();) {
    size_t nl = text.find('\n', at);
    const size_t end = nl == std::string_view::npos ? text.size() : nl + 1;
    std::string_view line = text.substr(at, end - at);
    while (!line.empty() && isspace((unsigned char)line.back())) line.remove_suffix(1);
    if (line == kMarker) {
      out.push_back(text.substr(start, at - start));
      start = end;
    }
    at = end;
  }
  out.push_back(text.substr(start));
  return out;
}

// Output buffers.  Printing a large module into fresh memory spends much
// of its time in page faults, so the last buffer given back with
// dcf_opt_free is kept (its pages stay mapped) and serves the next run
// whose output fits in it without wasting more than half of it.  Each
// buffer carries its capacity in a 64-byte header.
constexpr size_t kOutHeader = 64;
std::mutex g_out_mu;
char* g_out_keep = nullptr;  // a header address, or null

size_t out_cap(char* hdr) { return *(size_t*)hdr; }

char* out_alloc(size_t n) {
  {
    std::lock_guard<std::mutex> g(g_out_mu);
    if (g_out_keep && out_cap(g_out_keep) >= n && out_cap(g_out_keep) / 2 <= n) {
      char* h = g_out_keep;
      g_out_keep = nullptr;
      return h + kOutHeader;
    }
  }
  char* h = (char*)malloc(n + kOutHeader);
  if (!h) return nullptr;
  *(size_t*)h = n;
  return h + kOutHeader;
}

void out_free(char* p) {
  if (!p) return;
  char* h = p - kOutHeader;
  std::lock_guard<std::mutex> g(g_out_mu);
  if (g_out_keep && out_cap(g_out_keep) >= out_cap(h)) {
    free(h);
    return;
  }
  free(g_out_keep);
  g_out_keep = h;
}

// The printed result (handed to the C API's caller as is; dcf_opt_free).
struct Output {
  char* p = nullptr;
  size_t n = 0;
};

Output run_all(std::string_view text, const std::string& pipeline, int n_gpus, int flags, dcf_opt_stats* st) {
  Engines eng(n_gpus);
  dcf_opt_stats total{};
  const auto chunks = split_chunks(text, (flags & DCF_OPT_SPLIT_INPUT_FILE) != 0);
  const size_t tail = (flags & DCF_OPT_LOCAL_SCOPE) ? 0 : 1;
  // Modules stay alive until the text is assembled: the printed parts
  // point into their constants.
  std::vector<std::unique_ptr<dco::Module>> mods;
  std::vector<dco::PrintedModule> parts;
  for (size_t i = 0; i < chunks.size(); i++) {
    auto t0 = Clock::now();
    mods.push_back(dco::parse_module(chunks[i], (flags & DCF_OPT_VERBATIM) == 0));
    dco::Module& m = *mods.back();
    total.parse_ms += ms_since(t0);
    if (i == 0 && is_pinned(text))
      for (auto& e : eng.own) e->set_pinned_source(text.data(), text.size(), eng.list.size() == 1);
    t0 = Clock::now();
    dco::PassStats ps;
    std::vector<dco::Engine*> engines = eng.for_pipeline(pipeline);
    dco::run_pipeline(m, pipeline, engines, &ps);
    dco::fetch_results(m, engines);
    total.run_ms += ms_since(t0);
    total.folds += ps.folds;
    total.refused += ps.refused;
    t0 = Clock::now();
    dco::PrintHooks hooks;
    hooks.hex_of = hex_hook;
    hooks.bits0_of = bits_hook;
    hooks.ctx = &eng;
    hooks.debuginfo = (flags & DCF_OPT_DEBUGINFO) != 0;
    parts.push_back(dco::print_module_parts(m, hooks));
    total.print_ms += ms_since(t0);
  }
  auto t0 = Clock::now();
  // Each chunk's module and, unless printing in local scope, one more
  // newline; the chunks joined by the marker line (Invocation::print and
  // Invocation::run, src/pass.rs:761-767 and :817-820).
  static const char sep[] = "// -----\n";
  Output out;
  for (size_t i = 0; i < parts.size(); i++) out.n += parts[i].size() + tail + (i ? sizeof sep - 1 : 0);
  out.p = out_alloc(out.n + 1);
  if (!out.p) throw std::runtime_error("out of memory for the printed module");
  size_t at = 0;
  for (size_t i = 0; i < parts.size(); i++) {
    if (i) {
      memcpy(out.p + at, sep, sizeof sep - 1);
      at += sizeof sep - 1;
    }
    parts[i].write_to(out.p + at);
    at += parts[i].size();
    if (tail) out.p[at++] = '\n';
  }
  out.p[out.n] = 0;
  total.print_ms += ms_since(t0);
  for (auto& e : eng.own) {
    total.h2d_bytes += e->stats.h2d_bytes;
    total.d2h_bytes += e->stats.d2h_bytes;
    total.batches += e->stats.batches;
    total.upload_ms += e->stats.upload_ms;
    total.download_ms += e->stats.download_ms;
    total.fold_ms += e->stats.device_ms;
  }
  if (st) *st = total;
  return out;
}

}  // namespace

extern "C" int dcf_opt_run(const char* text, size_t len, const char* pipeline, int n_gpus, int flags,
                           char** out, size_t* out_len, dcf_opt_stats* stats) {
  if (!text || !pipeline || !out) {
    g_opt_err = "null argument";
    return -1;
  }
  try {
    const Output r = run_all(std::string_view(text, len), pipeline, n_gpus, flags, stats);
    *out = r.p;
    if (out_len) *out_len = r.n;
    return 0;
  } catch (const std::exception& e) {
    g_opt_err = e.what();
    return -1;
  }
}

extern "C" void dcf_opt_free(char* p) { out_free(p); }

extern "C" const char* dcf_opt_last_error(void) { return g_opt_err.c_str(); }

extern "C" int dcf_opt_print_element(int dtype, unsigned long long bits, char* out, size_t cap) {
  std::string s;
  switch (dtype) {
    case DCF_F16: case DCF_BF16: case DCF_F32: case DCF_F64: case DCF_F8E5M2: case DCF_F8E4M3: case DCF_F8E3M4:
      s = dco::print_float_literal(bits, dtype);
      break;
    case DCF_I1: case DCF_I8: case DCF_I16: case DCF_I32: case DCF_I64:
      s = dco::print_int_literal(bits, dtype);
      break;
    default:
      g_opt_err = "not an element type";
      return -1;
  }
  if (!out || s.size() + 1 > cap) {
    g_opt_err = "output buffer too small";
    return -1;
  }
  memcpy(out, s.c_str(), s.size() + 1);
  return (int)s.size();
}

#ifdef DCFOLD_OPT_MAIN
int main(int argc, char** argv) {
  std::string input = "-", output = "-", pipeline;
  int gpus = 1;
  int flags = 0;
  bool timing = false;
  for (int i = 1; i < argc; i++) {
    std::string a = argv[i];
    if (a == "--canonicalize" || a == "-canonicalize" || a.rfind("--canonicalize=", 0) == 0 ||
        a.rfind("-canonicalize=", 0) == 0)
      pipeline = "canonicalize";
    else if (a.rfind("--pass-pipeline=", 0) == 0 || a.rfind("-pass-pipeline=", 0) == 0)
      pipeline = a.substr(a.find('=') + 1);
    else if (a == "--split-input-file" || a == "-split-input-file")
      flags |= DCF_OPT_SPLIT_INPUT_FILE;
    else if (a == "--mlir-print-local-scope" || a == "-mlir-print-local-scope")
      flags |= DCF_OPT_LOCAL_SCOPE;
    else if (a == "--mlir-print-debuginfo" || a == "-mlir-print-debuginfo")
      flags |= DCF_OPT_DEBUGINFO;
    else if (a.rfind("--gpus=", 0) == 0)
      gpus = atoi(a.c_str() + 7);
    else if (a == "--timing")
      timing = true;
    else if (a == "-o" && i + 1 < argc)
      output = argv[++i];
    else if (a.rfind("--mlir-", 0) == 0 || a.rfind("-mlir-", 0) == 0 || a == "--allow-unregistered-dialect")
      continue;  // printing flags: the output is always generic form
    else if (a[0] != '-' || a == "-")
      input = a;
    else {
      fprintf(stderr, "dcfold-opt: unknown option %s\n", a.c_str());
      return 2;
    }
  }
  if (pipeline.empty()) {
    fprintf(stderr, "usage: dcfold-opt [--canonicalize | --pass-pipeline=...] [--gpus=N] [--split-input-file] "
                    "[--timing] [-o out] [in.mlir]\n");
    return 2;
  }
  std::stringstream buf;
  if (input == "-") buf << std::cin.rdbuf();
  else {
    std::ifstream f(input, std::ios::binary);
    if (!f) {
      fprintf(stderr, "dcfold-opt: cannot read %s\n", input.c_str());
      return 1;
    }
    buf << f.rdbuf();
  }
  const std::string text = buf.str();
  dcf_opt_stats st{};
  try {
    const Output r = run_all(text, pipeline, gpus, flags, &st);
    if (output == "-") fwrite(r.p, 1, r.n, stdout);
    else {
      std::ofstream f(output, std::ios::binary);
      f.write(r.p, (std::streamsize)r.n);
    }
    out_free(r.p);
  } catch (const std::exception& e) {
    fprintf(stderr, "dcfold-opt: %s\n", e.what());
    return 1;
  }
  if (timing)
    fprintf(stderr,
            "{\"parse_ms\": %.3f, \"run_ms\": %.3f, \"print_ms\": %.3f, \"folds\": %llu, \"refused\": %llu, "
            "\"h2d_bytes\": %llu, \"d2h_bytes\": %llu, \"batches\": %llu}\n",
            st.parse_ms, st.run_ms, st.print_ms, st.folds, st.refused, st.h2d_bytes, st.d2h_bytes, st.batches);
  return 0;
}
#endif
