"""The synthetic workload generators: the C generator (libdcfgen.so) gives
exactly the values of the numpy definitions in mlirpass_b200/workloads.py,
and the MLIR text of every configuration is the same whichever way it is
assembled (one str, or one bytearray built in place)."""
import numpy as np
import pytest

from mlirpass_b200 import mlir_gen as G
from mlirpass_b200 import workloads as W


@pytest.mark.parametrize("seed,n,start", [(1, 1000, 0), (2**63 + 5, 777, 3), (5010, 3_000_001, 0), (7, 1, 12)])
def test_splitmix64_c_equals_numpy(seed, n, start):
    assert np.array_equal(W.splitmix64(seed, n, start), W.splitmix64_np(seed, n, start))


@pytest.mark.parametrize("seed,n,lo,hi", [(2000, 3_000_001, -4.0, 4.0), (5011, 65536, -1.0, 1.0),
                                          (5000, 1 << 21, -0.1, 0.1), (1000, 3, -1.0, 1.0)])
def test_uniform_c_equals_numpy(seed, n, lo, hi):
    assert np.array_equal(W.uniform_f32(seed, n, lo, hi).view(np.uint32),
                          W.uniform_f32_np(seed, n, lo, hi).view(np.uint32))
    assert np.array_equal(W.uniform_bf16_bits(seed, n, lo, hi), W.uniform_bf16_bits_np(seed, n, lo, hi))


def test_hex_upper():
    a = np.random.default_rng(1).integers(0, 256, (5 << 20) + 3, dtype=np.uint8)
    assert W.hex_upper(a) == a.tobytes().hex().upper()
    assert W.hex_upper(np.zeros(0, np.uint8)) == ""


def test_module_text_and_bytes_agree():
    for text, mod in [(G.config1_text(), G.config1_module()), (G.config2_text(64), G.config2_module(64)),
                      (G.config3_text("i64", 16, 8), G.config3_module("i64", 16, 8)),
                      (G.config4_text(4096, True), G.config4_module(4096, True)),
                      (G.config5_text(3, 8, 16), G.config5_module(3, 8, 16))]:
        assert bytes(mod.tobytes()) == text.encode()
