"""vc_sum_f32_noalloc: the sum for callers that cannot allocate device memory
while they run (a process whose device budget is reserved up front, a
latency-critical loop that must not enter the driver allocator, a library
callback that must not allocate as a side effect). It keeps its block
partials in a fixed array compiled into the library instead of a buffer the
runtime allocates on first use.

Checked through the C ABI against the existing entry point vc_sum_f32, with
the tolerance the other sum tests use, on two calls in a row (the second call
finds the first call's partials and ticket state in the shared array). The
file sorts last so that a run stopping at the first failure has already run
every other test; it also passes on its own in a fresh process."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
SUM_RTOL = 1e-6  # the bar of tests/test_gpu_stream.py


def _sum_both(gpu, dev, x):
    dx = dev.put(x)
    out_ref, out_na = dev.alloc(8), dev.alloc(8)
    assert gpu.sum_f32(dx.ptr, x.size, out_ref.ptr) == gpu.VCError.Success
    assert gpu.sum_f32_noalloc(dx.ptr, x.size, out_na.ptr) == gpu.VCError.Success
    assert gpu.vcDeviceSynchronize() == gpu.VCError.Success
    return float(out_ref.to_host(np.float64, 1)[0]), float(out_na.to_host(np.float64, 1)[0])


def test_noalloc_sum_matches_existing_entry_on_two_calls(gpu, dev):
    rng = np.random.default_rng(2024)
    inputs = [rng.random(3_000_001, dtype=np.float32),                 # ragged tail
              rng.standard_normal((1 << 22) + 3).astype(np.float32)]   # signed, larger
    for x in inputs:  # two calls in a row through the same static scratch
        ref, got = _sum_both(gpu, dev, x)
        assert got == pytest.approx(ref, rel=SUM_RTOL, abs=1e-9)
    assert gpu.kernel_error(True) == 0


def test_noalloc_sum_rejects_bad_arguments(gpu, dev):
    out = dev.alloc(8)
    assert gpu.sum_f32_noalloc(None, 16, out.ptr) == gpu.VCError.InvalidValue
    assert gpu.sum_f32_noalloc(out.ptr, -1, out.ptr) == gpu.VCError.InvalidValue
