"""Row-block sharding of one fold over several GPUs in one process
(dcf_init(n)), against the oracle.  Runs only where at least two GPUs are
visible."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ngpus():
    import torch
    return torch.cuda.device_count()


@pytest.fixture
def multi(dcf):
    n = _ngpus()
    if n < 2:
        pytest.skip("needs two or more GPUs")
    import os
    os.environ.pop("DCF_DEVICES", None)
    got = dcf.init(n)
    assert got == n and dcf.device_count() == n
    yield dcf
    dcf.init(1)


def test_row_blocks_match_oracle(multi, oracle):
    rng = np.random.default_rng(4)
    n = 50_000_017                      # not a multiple of the row-block granularity
    a = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    for op in ("addf", "maximumf", "divf"):
        g, c = multi.binary(op, "f32", a, b), oracle.binary(op, "f32", a, b)
        assert g.folded == c.folded and g.is_splat == c.is_splat
        assert np.array_equal(g.out, c.out), op


def test_refusal_index_across_blocks(multi, oracle):
    n = 40_000_000
    x = np.arange(n, dtype=np.int32)
    y = np.ones(n, dtype=np.int32)
    y[n - 3] = 0                        # in the last GPU's block
    y[n // 2 + 7] = 0                   # in a middle block
    g, c = multi.binary("divsi", "i32", x, y), oracle.binary("divsi", "i32", x, y)
    assert not g.folded and g.first_fail_index == c.first_fail_index == n // 2 + 7


def test_splat_across_blocks(multi):
    n = 30_000_000
    a = np.full(n, 1.5, np.float32)
    b = np.full(n, 2.0, np.float32)
    g = multi.binary("mulf", "f32", a, b)
    assert g.folded and g.is_splat and np.all(g.out.view(np.float32) == 3.0)
    b[-1] = 3.0                          # differs only in the last block
    g = multi.binary("mulf", "f32", a, b)
    assert g.folded and not g.is_splat


def test_batch_balanced_over_gpus(multi, oracle):
    jobs = [{"op": "mulf", "dtype": "f32", "lhs": np.full(65536, i, np.float32),
             "rhs": np.arange(65536, dtype=np.float32)} for i in range(64)]
    res = multi.batch(jobs)
    for j, r in zip(jobs, res):
        c = oracle.binary("mulf", "f32", j["lhs"], j["rhs"])
        assert r.folded and np.array_equal(r.out, c.out)
