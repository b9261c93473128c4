"""vadd / sum / fused vadd+sum / demo block reduce on the GPU, through the C
ABI, against the CPU oracle. Bars: vadd and block partials bit-exact; the
fp64-combined sum within 1e-6 relative of the oracle's fp64 sum."""
from __future__ import annotations

import ctypes
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
SUM_RTOL = 1e-6


# (1 << 25) + 12345: the bulk-copy kernel, with a tail past its last whole
# 2048-element chunk
@pytest.mark.parametrize("n", [0, 1, 3, 64, 1000, 1 << 20, (1 << 22) + 7, (1 << 25) + 12345])
def test_vadd_bit_exact(gpu, dev, orc, n):
    rng = np.random.default_rng(n)
    a = rng.random(n, dtype=np.float32)
    b = rng.random(n, dtype=np.float32)
    da, db, dc = dev.put(a), dev.put(b), dev.alloc(max(4 * n, 4))
    assert gpu.vadd_f32(da.ptr, db.ptr, dc.ptr, n) == 0
    assert gpu.vcDeviceSynchronize() == 0
    assert np.array_equal(dc.to_host(np.float32, n), orc.vadd(a, b))


@pytest.mark.parametrize("offset", [1, 2, 3])
def test_vadd_unaligned(gpu, dev, orc, offset):
    n = 100_003
    rng = np.random.default_rng(offset)
    a = rng.standard_normal(n + offset).astype(np.float32)
    b = rng.standard_normal(n + offset).astype(np.float32)
    da, db, dc = dev.put(a), dev.put(b), dev.alloc(4 * (n + offset))
    assert gpu.vadd_f32(da.ptr + 4 * offset, db.ptr + 4 * offset, dc.ptr + 4 * offset, n) == 0
    assert gpu.vcDeviceSynchronize() == 0
    got = dc.to_host(np.float32, n + offset)[offset:]
    assert np.array_equal(got, orc.vadd(a[offset:], b[offset:]))


def _read_f64(d):
    return float(d.to_host(np.float64, 1)[0])


@pytest.mark.parametrize("n", [0, 1, 5, 4096, 1_000_003, 1 << 24])
def test_sum_within_1e6(gpu, dev, orc, n):
    x = np.random.default_rng(n + 11).random(n, dtype=np.float32)
    dx, dout = dev.put(x), dev.alloc(8)
    assert gpu.sum_f32(dx.ptr, n, dout.ptr) == 0
    assert gpu.vcDeviceSynchronize() == 0
    got, ref = _read_f64(dout), orc.sum_f64(x)
    assert got == pytest.approx(ref, rel=SUM_RTOL, abs=1e-12)


@pytest.mark.parametrize("n", [7, 1 << 20, 3_000_001, 1 << 25, (1 << 25) + 12345])
def test_vadd_sum_fused(gpu, dev, orc, n):
    rng = np.random.default_rng(n)
    a = rng.random(n, dtype=np.float32)
    b = rng.random(n, dtype=np.float32)
    da, db, dc, dout = dev.put(a), dev.put(b), dev.alloc(4 * n), dev.alloc(8)
    for _ in range(2):  # twice: the scratch ticket must be reset by the kernel
        assert gpu.vadd_sum_f32(da.ptr, db.ptr, dc.ptr, n, dout.ptr) == 0
        assert gpu.vcDeviceSynchronize() == 0
        c_ref = orc.vadd(a, b)
        assert np.array_equal(dc.to_host(np.float32, n), c_ref)
        assert _read_f64(dout) == pytest.approx(orc.sum_f64(c_ref), rel=SUM_RTOL)


def test_sum_deterministic(gpu, dev):
    x = np.random.default_rng(9).standard_normal(5_000_000).astype(np.float32)
    dx, dout = dev.put(x), dev.alloc(8)
    vals = set()
    for _ in range(3):
        assert gpu.sum_f32(dx.ptr, x.size, dout.ptr) == 0
        gpu.vcDeviceSynchronize()
        vals.add(_read_f64(dout))
    assert len(vals) == 1


@pytest.mark.parametrize("n,block", [(128, 32), (1000, 48), (777, 7), (4096, 256), (5000, 1024),
                                     (64, 1)])
def test_block_reduce_bit_exact(gpu, dev, orc, n, block):
    x = np.random.default_rng(n * block).standard_normal(n).astype(np.float32)
    groups = (n + block - 1) // block
    dx, dout = dev.put(x), dev.alloc(4 * groups)
    assert gpu.block_reduce_f32(dx.ptr, dout.ptr, n, block, groups) == 0
    gpu.vcDeviceSynchronize()
    assert np.array_equal(dout.to_host(np.float32, groups), orc.block_reduce(x, block, groups))


def test_legacy_vadd_and_reduce_demos(gpu, dev):
    """The demos' own launches through vcLoadKernel / vcLaunchKernel
    (test/vadd.vc:30-43, test/reduce.vc:47-75) with their known answers."""
    kat = json.load(open(os.path.join(GOLDEN, "kat.json")))
    a = np.array(kat["vadd"]["a"], np.float32)
    b = np.array(kat["vadd"]["b"], np.float32)
    da, db, dc = dev.put(a), dev.put(b), dev.alloc(64 * 4)
    err, k = gpu.vcGetKernel("vadd")
    assert err == 0
    assert gpu.vcLaunchKernel(k, 64, 32, [gpu.ptr(da.ptr), gpu.ptr(db.ptr), gpu.ptr(dc.ptr),
                                          gpu.i32(64)]) == 0
    assert gpu.vcDeviceSynchronize() == 0
    assert dc.to_host(np.float32, 64).tolist() == kat["vadd"]["c"]
    gpu.vcReleaseKernel(k)

    x = np.arange(128, dtype=np.float32)
    dx, dout = dev.put(x), dev.alloc(4 * 4)
    err, k = gpu.vcGetKernel("blockReduce")
    assert gpu.vcLaunchKernel(k, 128, 32, [gpu.ptr(dx.ptr), gpu.ptr(dout.ptr), gpu.i32(128)]) == 0
    assert gpu.vcDeviceSynchronize() == 0
    assert dout.to_host(np.float32, 4).tolist() == kat["reduce"]["partials"]
    # A launch that would overrun the output buffer is refused on the host.
    assert gpu.vcLaunchKernel(k, 256, 32, [gpu.ptr(dx.ptr), gpu.ptr(dout.ptr), gpu.i32(256)]) \
        == gpu.VCError.InvalidValue
    gpu.vcReleaseKernel(k)


def test_native_sum_through_registry(gpu, dev, orc):
    n = 123_457
    x = np.random.default_rng(1).random(n, dtype=np.float32)
    dx, dout = dev.put(x), dev.alloc(8)
    err, k = gpu.vcGetKernel("vc.sum")
    assert err == 0
    assert gpu.vcLaunchKernel(k, 1, 1, [gpu.ptr(dx.ptr), gpu.i64(n), gpu.ptr(dout.ptr)]) == 0
    assert gpu.vcDeviceSynchronize() == 0
    assert _read_f64(dout) == pytest.approx(orc.sum_f64(x), rel=SUM_RTOL)
    gpu.vcReleaseKernel(k)


# ---- cross-GPU sum through mailboxes (vc_vadd_sum_f32_allreduce)
def test_allreduce_one_rank_equals_fused_sum(gpu, dev, orc):
    """world = 1: the exchange runs against this GPU's own mailbox and gives
    the fused sum; consecutive epochs alternate the two slots."""
    n = (1 << 20) + 5
    rng = np.random.default_rng(11)
    a = rng.random(n, dtype=np.float32)
    b = rng.random(n, dtype=np.float32)
    da, db, dc, dout = dev.put(a), dev.put(b), dev.alloc(4 * n), dev.alloc(8)
    err, mb = gpu.peer_mailbox_alloc()
    assert err == 0 and mb
    try:
        ref = orc.sum_f64(orc.vadd(a, b))
        for epoch in (1, 2, 3):
            assert gpu.vadd_sum_f32_allreduce(da.ptr, db.ptr, dc.ptr, n, dout.ptr, [mb], 0,
                                              epoch) == 0
            assert gpu.vcDeviceSynchronize() == 0
            got = float(dout.to_host(np.float64, 1)[0])
            assert abs(got - ref) <= SUM_RTOL * abs(ref)
        assert np.array_equal(dc.to_host(np.float32, n), orc.vadd(a, b))
        assert gpu.kernel_error(True) == 0
    finally:
        gpu.peer_mailbox_free(mb)


def test_allreduce_silent_peer_times_out(gpu, dev):
    """A rank whose peer never arrives: the kernel's bounded wait ends (about
    2 s), the result is NaN and the timeout is recorded; the context stays
    usable. The "peer" is a second mailbox on this GPU that nothing writes."""
    n = 4096
    da, db, dc, dout = dev.put(np.ones(n, np.float32)), dev.put(np.ones(n, np.float32)), \
        dev.alloc(4 * n), dev.alloc(8)
    err, own = gpu.peer_mailbox_alloc()
    err2, silent = gpu.peer_mailbox_alloc()
    assert err == 0 and err2 == 0
    try:
        gpu.kernel_error(True)
        assert gpu.vadd_sum_f32_allreduce(da.ptr, db.ptr, dc.ptr, n, dout.ptr, [own, silent], 0,
                                          1) == 0
        assert gpu.vcDeviceSynchronize() == 0
        assert np.isnan(dout.to_host(np.float64, 1)[0])
        assert gpu.kernel_error(True) != 0
        # Still usable: a one-rank call right after succeeds.
        assert gpu.vadd_sum_f32_allreduce(da.ptr, db.ptr, dc.ptr, n, dout.ptr, [own], 0, 2) == 0
        assert gpu.vcDeviceSynchronize() == 0
        assert float(dout.to_host(np.float64, 1)[0]) == 2.0 * n
    finally:
        gpu.peer_mailbox_free(own)
        gpu.peer_mailbox_free(silent)


def test_allreduce_rejects_bad_arguments(gpu, dev):
    d = dev.alloc(1024)
    err, mb = gpu.peer_mailbox_alloc()
    assert err == 0
    try:
        bad = gpu.VCError.InvalidValue
        assert gpu.vadd_sum_f32_allreduce(d.ptr, d.ptr, d.ptr, 16, d.ptr, [mb], 0, 0) == bad
        assert gpu.vadd_sum_f32_allreduce(d.ptr, d.ptr, d.ptr, 16, d.ptr, [mb], 1, 1) == bad
        assert gpu.vadd_sum_f32_allreduce(d.ptr, d.ptr, d.ptr, 16, d.ptr, [mb] * 9, 0, 1) == bad
        assert gpu.vadd_sum_f32_allreduce(d.ptr, d.ptr, d.ptr, 16, d.ptr, [mb, 0], 0, 1) == bad
        assert gpu.peer_ipc_open(b"\0" * 10)[0] == bad
    finally:
        gpu.peer_mailbox_free(mb)


def test_vadd_sum_full_size_2p30(gpu):
    """The benchmark size, 2^30 fp32 elements (12 GiB of operands): c = a + b
    bit-identical to torch's IEEE add, the sum within 1e-6 of an fp64
    reduction, also through the one-rank exchange path."""
    import torch
    n = 1 << 30
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.rand(n, device="cuda", generator=g)
    b = torch.rand(n, device="cuda", generator=g)
    c = torch.empty_like(a)
    out = torch.zeros(1, dtype=torch.float64, device="cuda")
    assert gpu.vadd_sum_f32(a.data_ptr(), b.data_ptr(), c.data_ptr(), n, out.data_ptr()) == 0
    torch.cuda.synchronize()
    assert torch.equal(c, a + b)
    ref = c.double().sum().item()
    assert abs(out.item() - ref) <= SUM_RTOL * abs(ref)
    err, mb = gpu.peer_mailbox_alloc()
    assert err == 0
    try:
        out.zero_()
        assert gpu.vadd_sum_f32_allreduce(a.data_ptr(), b.data_ptr(), c.data_ptr(), n,
                                          out.data_ptr(), [mb], 0, 1) == 0
        torch.cuda.synchronize()
        assert abs(out.item() - ref) <= SUM_RTOL * abs(ref)
    finally:
        gpu.peer_mailbox_free(mb)
    assert gpu.kernel_error(True) == 0
    del a, b, c
    torch.cuda.empty_cache()
