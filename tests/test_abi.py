"""The C-ABI library (CPU-side checks): it loads, exports every entry point
include/dcfold.h declares with the signature the binding uses, and with no
GPU a compute call fails loudly (ENODEV) instead of computing on the CPU.
"""
import ctypes
import os
import re

import numpy as np
import pytest

import mlirpass_b200 as m
from conftest import ROOT, have_gpu

HEADER = os.path.join(ROOT, "include", "dcfold.h")


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dcf_[a-z0-9_]+)\s*\(", text)))


def test_header_declarations_match_binding():
    names = declared()
    assert len(names) >= 20
    assert set(names) == set(m.SIGNATURES), set(names) ^ set(m.SIGNATURES)


def test_library_exports_every_symbol():
    assert os.path.exists(m.LIB_PATH), "run python -m mlirpass_b200.build"
    L = ctypes.CDLL(m.LIB_PATH)
    for name in declared():
        assert hasattr(L, name), name
    assert m.lib().dcf_version().startswith(b"dcfold")
    assert m.lib().dcf_dtype_size(m.DTYPES["bf16"]) == 2
    assert m.lib().dcf_dtype_size(m.DTYPES["i64"]) == 8


def test_enums_match_header():
    text = open(HEADER).read()
    for name, val in m.DTYPES.items():
        tag = "DCF_" + name.upper()
        assert re.search(rf"\b{tag}\s*=\s*{val}\b", text), tag
    for name, val in m.OPS.items():
        tag = "DCF_" + name.upper()
        assert re.search(rf"\b{tag}\s*=\s*{val}\b", text), tag


def test_struct_layouts():
    assert ctypes.sizeof(m.Result) == 16
    assert ctypes.sizeof(m.Status) == 16
    assert ctypes.sizeof(m.Job) == 4 * 4 + 3 * 8 + 8 + 8 + 16


@pytest.mark.skipif(have_gpu(), reason="checks the no-GPU failure path")
def test_no_cpu_fallback_without_gpu():
    a = np.ones(16, np.float32)
    with pytest.raises(m.DcfError) as e:
        m.binary("addf", "f32", a, a)
    assert e.value.code == -2
    assert "no CPU fallback" in str(e.value)
