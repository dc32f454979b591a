"""dcf_batch_noalloc: the fold entry point that allocates nothing.

It exists for callers that cannot allocate device memory while folding:
an embedding runtime whose caching allocator already holds all of HBM, or
latency-sensitive code that cannot take the synchronisation cudaMalloc may
cause.  Its scratch is a fixed file-scope device array inside the library.

The test folds through the new entry point (via the C ABI) twice in a row
with different data, so the second call runs on scratch that the first one
left behind, and checks every job against the existing device entry points
(dcf_binary_async / dcf_convert_async / dcf_reciprocal_async): same fold
decision, same lowest refusing index, same splat flag, and bit-identical
results.  This file sorts last so that a run stopping at the first failure
has already run every other test.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _jobs(seed):
    import torch
    g = torch.Generator().manual_seed(seed)
    dev = "cuda"
    n = 300_001
    a = torch.randn(n, generator=g).to(dev)
    b = torch.randn(n, generator=g).to(dev)
    x = torch.randint(-2**31, 2**31 - 1, (n,), dtype=torch.int32, generator=g).to(dev)
    y = torch.randint(1, 1000, (n,), dtype=torch.int32, generator=g).to(dev)
    y[1234 + seed] = 0                                           # refuses at this index
    t = (torch.randn(n, generator=g).view(torch.int32) & 0x7FFF0000 | 0x00000000).view(torch.float32).to(dev)
    r = (torch.randn(n, generator=g) * 8).to(torch.bfloat16).to(dev)
    s = torch.tensor([0.25 * (seed + 1)], dtype=torch.float32, device=dev)
    p = torch.randint(-2**62, 2**62, (n,), dtype=torch.int64, generator=g).to(dev)
    q = torch.randint(-2**62, 2**62, (n,), dtype=torch.int64, generator=g).to(dev)
    return [
        {"op": "addf", "dtype": "f32", "lhs": a, "rhs": b, "out": torch.empty_like(a)},
        {"op": "divsi", "dtype": "i32", "lhs": x, "rhs": y, "out": torch.empty_like(x)},
        {"op": "truncf", "dtype": "f32", "out_dtype": "bf16", "lhs": t,
         "out": torch.empty(n, dtype=torch.int16, device=dev)},
        {"op": "reciprocal", "dtype": "bf16", "lhs": r, "out": torch.empty_like(r)},
        {"op": "maximumf", "dtype": "f32", "lhs": a, "rhs": s, "rhs_splat": True, "out": torch.empty_like(a)},
        {"op": "cmpi", "dtype": "i64", "lhs": p, "rhs": q, "flags": 2 << 8,
         "out": torch.empty(n, dtype=torch.uint8, device=dev)},
        {"op": "addf", "dtype": "f32", "lhs": a[1:], "rhs": b[1:], "out": torch.empty(n - 1, device=dev)},
        {"op": "rsqrt", "dtype": "f32", "out_dtype": "f32", "lhs": a.abs(), "out": torch.empty_like(a)},
        {"op": "ipowi", "dtype": "i32", "lhs": x, "rhs": y, "out": torch.empty_like(x)},
    ]


def _existing(dcf, j):
    """The same fold through the existing (allocating) device entry points."""
    import torch
    out = torch.empty_like(j["out"])
    st = torch.empty(2, dtype=torch.int64, device="cuda")
    dcf.status_reset(st)
    n = j["out"].numel()
    if j["op"] == "reciprocal":
        dcf.reciprocal_async(j["dtype"], j["lhs"], out, st, n=n)
    elif j["op"] in dcf.CONVERT_OPS:
        dcf.convert_async(j["op"], j["dtype"], j["out_dtype"], j["lhs"], out, st, n=n)
    else:
        dcf.binary_async(j["op"], j["dtype"], j["lhs"], j["rhs"], out, st, n=n,
                         rhs_splat=j.get("rhs_splat", False), flags=j.get("flags", 0))
    return dcf.status_read(st), out


def _bits(t):
    import torch
    return t.contiguous().view(torch.uint8).cpu().numpy()


def test_noalloc_matches_existing_entry_points_twice(dcf):
    import torch
    for call in range(2):
        jobs = _jobs(call)
        got = dcf.batch_noalloc(jobs)
        torch.cuda.synchronize()
        for j, r in zip(jobs, got):
            want, out = _existing(dcf, j)
            assert r.folded == want.folded, (call, j["op"])
            assert r.first_fail_index == want.first_fail_index, (call, j["op"])
            if want.folded:
                assert r.is_splat == want.is_splat, (call, j["op"])
                assert np.array_equal(_bits(j["out"]), _bits(out)), (call, j["op"])
        assert not got[1].folded and got[1].first_fail_index == 1234 + call


def test_noalloc_rejects_more_jobs_than_its_scratch_holds(dcf):
    import torch
    a = torch.ones(8, device="cuda")
    jobs = [{"op": "addf", "dtype": "f32", "lhs": a, "rhs": a, "out": torch.empty_like(a)}] * (dcf.NOALLOC_MAX_JOBS + 1)
    with pytest.raises(dcf.DcfError) as e:
        dcf.batch_noalloc(jobs)
    assert e.value.code == -1 and "at most 1024 jobs" in str(e.value)
