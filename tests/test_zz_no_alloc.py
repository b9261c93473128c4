"""vc_sum_f32_noalloc: the sum for callers that cannot allocate device memory
while they run (a process whose device budget is reserved up front, a
latency-critical loop that must not enter the driver allocator, a library
callback that must not allocate as a side effect). It keeps its block
partials in a fixed array compiled into the library instead of a buffer the
runtime allocates on first use.

Checked through the C ABI against the existing entry point vc_sum_f32 on two
calls in a row (the second call finds the first call's partials and ticket
state in the shared array). Both entries launch the same kernel on the same
grid and add the same partials in the same order, so the results must be
bit-identical; both are also held to the sum bar of the other tests (1e-6
relative to the oracle's fp64 sum). The file sorts last so that a run stopping
at the first failure has already run every other test; it also passes on its
own in a fresh process."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
SUM_RTOL = 1e-6  # the bar of tests/test_gpu_stream.py


def _sum_both(gpu, dev, x, offset_floats=0, stream=None):
    """Both entries over x, placed `offset_floats` floats past a 256-byte
    aligned allocation (offset 1: not 16-byte aligned, the scalar kernel)."""
    buf = np.zeros(x.size + offset_floats, np.float32)
    buf[offset_floats:] = x
    dx = dev.put(buf)
    xp = dx.ptr + 4 * offset_floats
    out_ref, out_na = dev.alloc(8), dev.alloc(8)
    assert gpu.sum_f32(xp, x.size, out_ref.ptr, stream) == gpu.VCError.Success
    assert gpu.sum_f32_noalloc(xp, x.size, out_na.ptr, stream) == gpu.VCError.Success
    assert gpu.vcDeviceSynchronize() == gpu.VCError.Success
    return float(out_ref.to_host(np.float64, 1)[0]), float(out_na.to_host(np.float64, 1)[0])


def _check(orc, x, ref, got):
    assert got == ref  # same kernel, grid and order: bit-identical
    exact = orc.sum_f64(x)
    assert abs(got - exact) <= SUM_RTOL * abs(exact) + 1e-9


def test_noalloc_sum_matches_existing_entry_on_two_calls(gpu, dev, orc):
    rng = np.random.default_rng(2024)
    inputs = [rng.random(3_000_001, dtype=np.float32),                 # ragged tail
              rng.standard_normal((1 << 22) + 3).astype(np.float32)]   # signed, larger
    for x in inputs:  # two calls in a row through the same static scratch
        ref, got = _sum_both(gpu, dev, x)
        _check(orc, x, ref, got)
    assert gpu.kernel_error(True) == 0


def test_noalloc_sum_unaligned_empty_and_stream(gpu, dev, orc):
    rng = np.random.default_rng(7)
    x = rng.random(1_000_003, dtype=np.float32)
    for _ in range(2):                       # unaligned input: the scalar kernel
        ref, got = _sum_both(gpu, dev, x, offset_floats=1)
        _check(orc, x, ref, got)
    ref, got = _sum_both(gpu, dev, np.zeros(0, np.float32))   # n = 0 gives 0.0
    assert ref == 0.0 and got == 0.0
    err, s = gpu.vcStreamCreate()
    assert err == gpu.VCError.Success
    try:
        for _ in range(2):                   # on a created stream
            ref, got = _sum_both(gpu, dev, x, stream=s)
            _check(orc, x, ref, got)
    finally:
        assert gpu.vcStreamDestroy(s) == gpu.VCError.Success
    assert gpu.kernel_error(True) == 0


def test_noalloc_sum_rejects_bad_arguments(gpu, dev):
    out = dev.alloc(8)
    assert gpu.sum_f32_noalloc(None, 16, out.ptr) == gpu.VCError.InvalidValue
    assert gpu.sum_f32_noalloc(out.ptr, 16, None) == gpu.VCError.InvalidValue
    assert gpu.sum_f32_noalloc(out.ptr, -1, out.ptr) == gpu.VCError.InvalidValue
