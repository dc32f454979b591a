"""Build libdcfold.so (sm_100a) in-tree, and the CPU oracle beside the tests.

    python -m mlirpass_b200.build          # library + oracle
    python -m mlirpass_b200.build --lib    # library only

The library is compiled with nvcc for sm_100a only, with IEEE-exact
float settings (-fmad=false -ftz=false -prec-div=true -prec-sqrt=true),
and links the CUDA runtime statically so it needs no torch at run time.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libdcfold.so")
ORACLE_SRC = os.path.join(ROOT, "oracle", "dcf_oracle.c")
ORACLE_LIB = os.path.join(ROOT, "oracle", "_build", "libdcforacle.so")
GEN_SRC = os.path.join(PKG, "gen", "dcf_gen.c")
GEN_LIB = os.path.join(PKG, "libdcfgen.so")

# The float and conversion kernel families are split by layout so that the
# (template-heavy) translation units compile in parallel.
SOURCES = ["dcf_ew_float.cu", "dcf_ew_float_f32.cu", "dcf_ew_float_f64.cu", "dcf_ew_float_h.cu",
           "dcf_ew_float_f8.cu", "dcf_ew_int.cu", "dcf_ew_convert.cu", "dcf_ew_convert_ff.cu",
           "dcf_ew_convert_if.cu", "dcf_ew_convert_fi.cu", "dcf_ew_math.cu", "dcf_misc.cu", "dcf_transpose_tma.cu", "dcf_runtime.cu",
           "dcf_noalloc.cu", "dcf_rt.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2",
    "-fmad=false", "-ftz=false", "-prec-div=true", "-prec-sqrt=true",
    "--expt-relaxed-constexpr",
    "-I", os.path.join(ROOT, "include"),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hs + [os.path.join(ROOT, "include", "dcfold.h")]


def build_lib(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    cc = nvcc()
    hdrs = _headers()
    objs = []
    jobs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale(o, [s] + hdrs):
            jobs.append([cc, *NVCC_FLAGS, "-c", s, "-o", o])
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for cmd, res in zip(jobs, ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), jobs)):
                if verbose or res.returncode:
                    sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
                if res.returncode:
                    raise RuntimeError(f"nvcc failed on {cmd[-3]}")
    if force or jobs or _stale(LIB, objs):
        cmd = [cc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", LIB, *objs,
               "-cudart", "static", "-lpthread", "-ldl", "-lrt"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode:
            sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
            raise RuntimeError("link of libdcfold.so failed")
    return LIB


OPT_SOURCES = ["ir.cpp", "float_text.cpp", "hex_host.cpp", "engine.cpp", "sharded.cpp", "fold.cpp", "main.cpp"]
OPT_LIB = os.path.join(PKG, "libdcfold_opt.so")
OPT_BIN = os.path.join(PKG, "dcfold-opt")


def _cuda_home() -> str:
    return os.path.dirname(os.path.dirname(os.path.realpath(nvcc())))


def build_opt(force: bool = False) -> list[str]:
    """The pass driver: libdcfold_opt.so and the dcfold-opt executable."""
    srcs = [os.path.join(PKG, "opt", f) for f in OPT_SOURCES]
    deps = srcs + [os.path.join(PKG, "opt", f) for f in ("ir.h", "engine.h", "fold.h", "cuda_rt.h")] + \
        [os.path.join(ROOT, "include", "dcfold.h"), os.path.join(ROOT, "include", "dcfold_opt.h"), LIB]
    cuda = _cuda_home()
    cxx = os.environ.get("CXX", "g++")
    common = ["-std=c++17", "-O2", "-fPIC", "-Wall", "-I", os.path.join(cuda, "include")]
    # No CUDA runtime of its own: the driver's runtime calls go through
    # libdcfold.so's (opt/cuda_rt.h), one runtime per process.
    link = ["-L", PKG, "-ldcfold", "-Wl,-rpath,$ORIGIN", "-lpthread", "-ldl", "-lrt"]
    out = []
    for target, extra in ((OPT_LIB, ["-shared"]), (OPT_BIN, ["-DDCFOLD_OPT_MAIN"])):
        if force or _stale(target, deps):
            cmd = [cxx, *common, *extra, "-o", target, *srcs, *link]
            res = subprocess.run(cmd, capture_output=True, text=True)
            if res.returncode:
                sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
                raise RuntimeError(f"build of {os.path.basename(target)} failed")
        out.append(target)
    return out


def build_oracle(force: bool = False) -> str:
    os.makedirs(os.path.dirname(ORACLE_LIB), exist_ok=True)
    deps = [ORACLE_SRC, os.path.join(ROOT, "oracle", "dcf_oracle.h"), os.path.join(ROOT, "include", "dcfold.h")]
    if force or _stale(ORACLE_LIB, deps):
        cc = os.environ.get("CC", "gcc")
        cmd = [cc, "-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
               "-Wall", "-o", ORACLE_LIB, ORACLE_SRC, "-lm"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode:
            sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
            raise RuntimeError("oracle build failed")
    return ORACLE_LIB


def build_gen(force: bool = False) -> str:
    """The host generator of the synthetic workloads (libdcfgen.so)."""
    if force or _stale(GEN_LIB, [GEN_SRC]):
        cc = os.environ.get("CC", "gcc")
        cmd = [cc, "-O3", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math", "-Wall",
               "-o", GEN_LIB, GEN_SRC, "-lpthread"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode:
            sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
            raise RuntimeError("build of libdcfgen.so failed")
    return GEN_LIB


def main(argv: list[str]) -> None:
    force = "--force" in argv
    if "--oracle" not in argv:
        print(build_lib(verbose="-v" in argv, force=force))
        for t in build_opt(force=force):
            print(t)
        print(build_gen(force=force))
    if "--lib" not in argv:
        print(build_oracle(force=force))


if __name__ == "__main__":
    main(sys.argv[1:])
