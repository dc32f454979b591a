"""The device-pointer entry points (*_async) on torch CUDA tensors,
including unaligned views that take the scalar kernel path, against the
oracle."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _t(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.parametrize("offset", [0, 1, 3])
def test_binary_async(offset, dcf, oracle):
    import torch
    rng = np.random.default_rng(offset)
    n = 100_003
    a = rng.standard_normal(n + offset).astype(np.float32)
    b = rng.standard_normal(n + offset).astype(np.float32)
    ta, tb = _t(a), _t(b)
    out = torch.empty(n + offset, dtype=torch.float32, device="cuda")
    st = torch.empty(2, dtype=torch.int64, device="cuda")
    for op in ("addf", "divf", "maximumf"):
        dcf.status_reset(st)
        dcf.binary_async(op, "f32", ta[offset:], tb[offset:], out[offset:], st, n=n)
        r = dcf.status_read(st)
        c = oracle.binary(op, "f32", a[offset:], b[offset:])
        assert r.folded == c.folded and r.is_splat == c.is_splat
        assert np.array_equal(out[offset:].cpu().numpy().view(np.uint32), c.out)


def test_convert_and_reciprocal_async(dcf, oracle):
    import torch
    rng = np.random.default_rng(5)
    n = 65_536
    x = (rng.standard_normal(n).astype(np.float32).view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)
    tx = _t(x)
    out = torch.empty(n, dtype=torch.int16, device="cuda")
    st = torch.empty(2, dtype=torch.int64, device="cuda")
    dcf.status_reset(st)
    dcf.convert_async("truncf", "f32", "bf16", tx, out, st)
    r = dcf.status_read(st)
    c = oracle.convert("truncf", "f32", "bf16", x)
    assert r.folded and c.folded
    assert np.array_equal(out.cpu().numpy().view(np.uint16), c.out)
    rec = torch.empty(n, dtype=torch.float32, device="cuda")
    dcf.status_reset(st)
    dcf.reciprocal_async("f32", tx, rec, st)
    assert dcf.status_read(st).folded
    assert np.array_equal(rec.cpu().numpy().view(np.uint32), oracle.reciprocal("f32", x).out)


def test_refusal_reports_first_index_async(dcf):
    import torch
    n = 1 << 20
    a = torch.arange(n, dtype=torch.int32, device="cuda")
    b = torch.ones(n, dtype=torch.int32, device="cuda")
    b[777_777] = 0
    b[900_000] = 0
    out = torch.empty_like(a)
    st = torch.empty(2, dtype=torch.int64, device="cuda")
    dcf.status_reset(st)
    dcf.binary_async("divsi", "i32", a, b, out, st)
    r = dcf.status_read(st)
    assert not r.folded and r.first_fail_index == 777_777


def test_hex_and_transpose_async(dcf, oracle):
    import torch
    rng = np.random.default_rng(9)
    data = rng.integers(0, 256, 1 << 16, dtype=np.uint8)
    td = _t(data)
    enc = torch.empty(2 << 16, dtype=torch.uint8, device="cuda")
    dcf.hex_encode_async(td, 1 << 16, enc)
    back = torch.empty(1 << 16, dtype=torch.uint8, device="cuda")
    st = torch.empty(2, dtype=torch.int64, device="cuda")
    dcf.status_reset(st)
    dcf.hex_decode_async(enc, 2 << 16, back, st)
    torch.cuda.synchronize()
    assert enc.cpu().numpy().tobytes() == oracle.hex_encode(data.tobytes())
    assert np.array_equal(back.cpu().numpy(), data)
    x = rng.integers(0, 1 << 16, size=(256, 384), dtype=np.uint16)
    tx = _t(x.view(np.int16))
    out = torch.empty(384 * 256, dtype=torch.int16, device="cuda")
    dcf.transpose2d_async(2, 256, 384, tx, out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint16).reshape(384, 256), x.T)
