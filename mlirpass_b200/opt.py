"""Binding of libdcfold_opt.so: run mlirpass pipelines' dense-constant folds
on MLIR text (include/dcfold_opt.h).

    out, stats = run(text, "canonicalize")
    out, stats = run(text, "builtin.module(func.func(tosa-layerwise-constant-fold,canonicalize))", n_gpus=8)

n_gpus=0 runs host-only: parsing, printing and the folds decided without
element work succeed; a fold that needs element work raises (no CPU
fallback).
"""
from __future__ import annotations

import ctypes
import os
import time

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdcfold_opt.so")
BIN_PATH = os.path.join(_HERE, "dcfold-opt")


class Stats(ctypes.Structure):
    _fields_ = [("parse_ms", ctypes.c_double), ("run_ms", ctypes.c_double), ("print_ms", ctypes.c_double),
                ("folds", ctypes.c_ulonglong), ("refused", ctypes.c_ulonglong), ("h2d_bytes", ctypes.c_ulonglong),
                ("d2h_bytes", ctypes.c_ulonglong), ("batches", ctypes.c_ulonglong), ("upload_ms", ctypes.c_double),
                ("fold_ms", ctypes.c_double), ("download_ms", ctypes.c_double)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


class OptError(RuntimeError):
    pass


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python -m mlirpass_b200.build` first")
        L = ctypes.CDLL(LIB_PATH)
        L.dcf_opt_run.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_int, ctypes.c_int,
                                  ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_size_t),
                                  ctypes.POINTER(Stats)]
        L.dcf_opt_run.restype = ctypes.c_int
        L.dcf_opt_free.argtypes = [ctypes.c_void_p]
        L.dcf_opt_last_error.restype = ctypes.c_char_p
        _lib = L
    return _lib


def _buffer(text):
    """(address, size, keep-alive) of the text argument."""
    if isinstance(text, str):
        text = text.encode()
    if isinstance(text, (bytes, bytearray)):
        buf = ctypes.create_string_buffer(0) if not text else None
        if buf is not None:
            return ctypes.addressof(buf), 0, buf
        if isinstance(text, bytes):
            return ctypes.cast(ctypes.c_char_p(text), ctypes.c_void_p).value, len(text), text
        arr = (ctypes.c_char * len(text)).from_buffer(text)
        return ctypes.addressof(arr), len(text), arr
    if hasattr(text, "data_ptr"):            # a torch uint8 tensor (for example in pinned memory)
        return text.data_ptr(), text.numel() * text.element_size(), text
    if hasattr(text, "ctypes"):              # a numpy array
        return text.ctypes.data, text.nbytes, text
    raise TypeError("text must be str, bytes, bytearray, a numpy array or a torch tensor")


def pinned_text(text):
    """Copy text into page-locked host memory (a torch uint8 tensor).  The
    driver copies constants straight from pinned text to the GPU instead of
    staging them through its own pinned slots."""
    import numpy as np
    import torch
    data = text.encode() if isinstance(text, str) else text
    t = torch.empty(len(data), dtype=torch.uint8, pin_memory=True)
    t.numpy()[:] = np.frombuffer(data, dtype=np.uint8)
    return t


def run(text, pipeline: str, n_gpus: int = 1, split_input_file: bool = False, as_bytes: bool = False,
        as_array: bool = False, local_scope: bool = False, debuginfo: bool = False, verbatim: bool = False):
    """Run `pipeline` over `text` (str, bytes, or a uint8 buffer such as
    pinned_text's); returns (printed module, stats dict).  The module is
    str, bytes with as_bytes=True, or with as_array=True a numpy uint8 view
    of the driver's own output buffer (no copy; freed with the array).
    local_scope prints as mlir-opt's --mlir-print-local-scope ends a module
    (no blank line after it); debuginfo prints locations, as
    --mlir-print-debuginfo does; verbatim keeps parsed constants' input text
    instead of printing them from their values (DCF_OPT_VERBATIM)."""
    addr, size, keep = _buffer(text)
    out = ctypes.c_void_p()
    n = ctypes.c_size_t()
    st = Stats()
    t0 = time.perf_counter()
    rc = lib().dcf_opt_run(addr, size, pipeline.encode(), n_gpus, int(split_input_file) | (2 if local_scope else 0) | (4 if debuginfo else 0) | (8 if verbatim else 0),
                           ctypes.byref(out),
                           ctypes.byref(n), ctypes.byref(st))
    call_ms = (time.perf_counter() - t0) * 1e3
    del keep
    if rc != 0:
        raise OptError(lib().dcf_opt_last_error().decode())
    if as_array:
        import weakref
        import numpy as np
        # The finaliser hangs on the base array: every view of it (this
        # slice included) keeps the buffer alive.
        base = np.ctypeslib.as_array((ctypes.c_uint8 * max(1, n.value)).from_address(out.value))
        weakref.finalize(base, lib().dcf_opt_free, out.value)
        arr = base[:n.value]
        d = st.as_dict()
        d["call_ms"] = call_ms
        return arr, d
    try:
        # ctypes.string_at takes a C int size: copy through a sized array so
        # outputs above 2 GiB work.
        b = bytes((ctypes.c_char * n.value).from_address(out.value)) if n.value else b""
    finally:
        lib().dcf_opt_free(out)
    d = st.as_dict()
    d["call_ms"] = call_ms
    return (b if as_bytes else b.decode()), d
