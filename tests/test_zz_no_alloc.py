"""dcf_batch_noalloc: the fold entry point that allocates nothing.

It exists for callers that cannot allocate device memory while folding:
an embedding runtime whose caching allocator already holds all of HBM, or
latency-sensitive code that cannot take the synchronisation cudaMalloc may
cause.  Its scratch is a fixed file-scope device array inside the library.

The tests fold through the new entry point (via the C ABI) twice in a row
with different data, so the second call runs on scratch that the first one
left behind, and check every job bit for bit against the oracle (the CPU
restatement of the reference's fold closures) and against the existing
device entry points (dcf_binary_async / dcf_convert_async /
dcf_reciprocal_async): same fold decision, same lowest refusing index,
same splat flag, identical result bits.  They also check that a call
leaves the device's free memory unchanged, that calls from several host
threads at once on one GPU give the same results as calls one after the
other, that buffers which are not device memory (or too small for the job)
are rejected before anything runs, and that the caller's current device is
kept.  This file sorts last so that a run stopping at the first failure has
already run every other test.
"""
import threading

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


def _host(t):
    import torch
    return t.contiguous().view(torch.uint8).cpu().numpy()


def _bits(t, dtype):
    """A device tensor's bytes as the oracle's storage array of `dtype`."""
    import mlirpass_b200 as m
    return _host(t).view(m.storage(dtype))


def _oracle(oracle, j):
    n = j["out"].numel()
    dt = j["dtype"]
    if j["op"] == "reciprocal":
        return oracle.reciprocal(dt, _bits(j["lhs"], dt), n=n)
    import mlirpass_b200 as m
    if j["op"] in m.CONVERT_OPS:
        return oracle.convert(j["op"], dt, j["out_dtype"], _bits(j["lhs"], dt), n=n)
    return oracle.binary(j["op"], dt, _bits(j["lhs"], dt), _bits(j["rhs"], dt), n=n,
                         rhs_splat=j.get("rhs_splat", False), flags=j.get("flags", 0))


def _check(jobs, got, oracle, dcf, tag):
    for j, r in zip(jobs, got):
        want = _oracle(oracle, j)
        assert r.folded == want.folded, (tag, j["op"])
        assert r.first_fail_index == want.first_fail_index, (tag, j["op"])
        if want.folded:
            assert r.is_splat == want.is_splat, (tag, j["op"])
            assert _host(j["out"]).tobytes() == want.out.tobytes(), (tag, j["op"])
        ex, out = _existing(dcf, j)
        assert (ex.folded, ex.first_fail_index) == (r.folded, r.first_fail_index), (tag, j["op"])
        if ex.folded:
            assert ex.is_splat == r.is_splat and np.array_equal(_host(out), _host(j["out"])), (tag, j["op"])


def test_noalloc_matches_oracle_twice_and_allocates_nothing(dcf, oracle):
    import torch
    for call in range(2):
        jobs = _jobs(call)
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        got = dcf.batch_noalloc(jobs)
        torch.cuda.synchronize()
        free1 = torch.cuda.mem_get_info()[0]
        if call == 1:
            # The first call looked up the scratch array's address; from then
            # on a call changes nothing in the device's memory use.
            assert free1 == free0, (free0, free1)
        _check(jobs, got, oracle, dcf, call)
        assert not got[1].folded and got[1].first_fail_index == 1234 + call


def test_noalloc_calls_from_several_threads_take_turns(dcf, oracle):
    # Four host threads fold different job lists on one GPU at once (each on
    # its own stream); every result must equal the oracle's, as when the
    # calls run one after the other.
    import torch
    lists = [_jobs(10 + k) for k in range(4)]
    streams = [torch.cuda.Stream() for _ in lists]
    torch.cuda.synchronize()
    results, errors = [None] * len(lists), []

    def work(k):
        try:
            for _ in range(3):
                results[k] = dcf.batch_noalloc(lists[k], stream=streams[k])
        except Exception as e:  # noqa: BLE001 - reported below
            errors.append(e)

    threads = [threading.Thread(target=work, args=(k,)) for k in range(len(lists))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    torch.cuda.synchronize()
    for k, jobs in enumerate(lists):
        _check(jobs, results[k], oracle, dcf, f"thread {k}")


def test_noalloc_rejects_more_jobs_than_its_scratch_holds(dcf):
    import torch
    a = torch.ones(8, device="cuda")
    jobs = [{"op": "addf", "dtype": "f32", "lhs": a, "rhs": a, "out": torch.empty_like(a)}] * (dcf.NOALLOC_MAX_JOBS + 1)
    with pytest.raises(dcf.DcfError) as e:
        dcf.batch_noalloc(jobs)
    assert e.value.code == -1 and "at most 1024 jobs" in str(e.value)


def test_noalloc_rejects_host_and_short_buffers_and_keeps_the_device(dcf):
    import torch
    a = torch.ones(1024, device="cuda")
    out = torch.empty_like(a)
    host = np.ones(1024, dtype=np.float32)
    before = torch.cuda.current_device()
    # an operand in host memory
    arr = dcf.device_jobs([{"op": "addf", "dtype": "f32", "lhs": a, "rhs": a, "out": out}])
    arr[0].rhs = host.ctypes.data
    with pytest.raises(dcf.DcfError) as e:
        dcf.run_device_jobs(arr)
    assert e.value.code == -1 and "device buffers" in str(e.value)
    # an element count far beyond any allocation on the device
    arr = dcf.device_jobs([{"op": "addf", "dtype": "f32", "lhs": a, "rhs": a, "out": out, "n": 1 << 40}])
    with pytest.raises(dcf.DcfError) as e:
        dcf.run_device_jobs(arr)
    assert e.value.code == -1
    assert torch.cuda.current_device() == before
    # a valid call afterwards still folds
    got = dcf.batch_noalloc([{"op": "addf", "dtype": "f32", "lhs": a, "rhs": a, "out": out}])
    torch.cuda.synchronize()
    assert got[0].folded and bool((out == 2).all())
