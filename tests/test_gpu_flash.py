"""Flash-attention forward on the GPU through the C ABI against the fp64
oracle (the reference's referenceAttn restated).
Bars: fp32 path <= 1e-4 absolute (the demo's own check, flash_attn.vc:230-236);
fp16 path <= 2e-3 and bf16 path <= 1e-2 absolute (fp64 softmax over the
rounded inputs)."""
from __future__ import annotations

import math
import os
import struct

import numpy as np
import pytest

from conftest import half_bits_to_f32, to_half_bits

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOL = {"f32": 1e-4, "f16": 2e-3, "bf16": 1e-2}
LOG2E = 1.4426950408889634


def load_vcfa(path):
    raw = open(path, "rb").read()
    nh, seq, hd, causal = (int(v) for v in struct.unpack("<4f", raw[4:20]))
    body = np.frombuffer(raw[20:], "<f4")
    e = nh * seq * hd
    return (nh, seq, hd, causal), [body[i * e:(i + 1) * e].copy() for i in range(5)]


@pytest.mark.parametrize("causal", [0, 1])
def test_flash_attn_demo_legacy_launch(gpu, dev, causal):
    """examples/flash_attn.vc end to end: its inputs, its launch
    (grid NHEAD*SEQ elements, block BR), its scale and its 1e-4 check against
    the reference's host output stored in the golden fixture."""
    (nh, seq, hd, c), (Q, K, V, _, O_host) = load_vcfa(
        os.path.join(GOLDEN, f"fa_demo_causal{causal}.bin"))
    dq, dk, dv, do = dev.put(Q), dev.put(K), dev.put(V), dev.alloc(Q.nbytes)
    err, k = gpu.vcGetKernel("flashAttn")
    scale = np.float32(LOG2E / math.sqrt(hd))
    assert gpu.vcLaunchKernel(k, nh * seq, 16, [gpu.ptr(dq.ptr), gpu.ptr(dk.ptr), gpu.ptr(dv.ptr),
                                                gpu.ptr(do.ptr), gpu.f32(scale),
                                                gpu.i32(causal)]) == 0
    assert gpu.vcDeviceSynchronize() == 0
    assert np.abs(do.to_host(np.float32, Q.size) - O_host).max() <= TOL["f32"]
    gpu.vcReleaseKernel(k)


def test_flash_attn_legacy_constants(gpu, dev, orc):
    """NHEAD/SEQ/HDIM are compile-time in the demo; vcKernelSetConstant sets them."""
    nh, seq, hd = 3, 96, 32
    Q, K, V = orc.fa_inputs(99, nh * seq * hd)
    scale = np.float32(LOG2E / math.sqrt(hd))
    dq, dk, dv, do = dev.put(Q), dev.put(K), dev.put(V), dev.alloc(Q.nbytes)
    err, k = gpu.vcGetKernel("flashAttn")
    for name, v in (("NHEAD", nh), ("SEQ", seq), ("HDIM", hd)):
        assert gpu.vcKernelSetConstant(k, name, v) == 0
    args = [gpu.ptr(dq.ptr), gpu.ptr(dk.ptr), gpu.ptr(dv.ptr), gpu.ptr(do.ptr), gpu.f32(scale),
            gpu.i32(1)]
    assert gpu.vcLaunchKernel(k, nh * seq, 16, args) == 0
    assert gpu.vcDeviceSynchronize() == 0
    ref = orc.attention(Q, K, V, nh, seq, hd, scale, True)
    assert np.abs(do.to_host(np.float32, Q.size) - ref).max() <= TOL["f32"]
    # A grid that does not match NHEAD*SEQ is refused.
    assert gpu.vcLaunchKernel(k, 64, 16, args) == gpu.VCError.InvalidValue
    gpu.vcReleaseKernel(k)


@pytest.mark.parametrize("BH,N,d,causal", [(1, 256, 64, False), (2, 100, 16, True),
                                           (3, 333, 128, False), (2, 64, 32, True),
                                           (2, 97, 24, True), (1, 130, 48, False),
                                           (1, 64, 100, True), (3, 40, 8, False),
                                           (2, 77, 17, True), (1, 50, 3, False)])
def test_flash_f32_vs_oracle(gpu, dev, orc, BH, N, d, causal):
    """d % 4 != 0 (17, 3) stages K / V with 4-byte copies, the rest with
    16-byte copies."""
    rng = np.random.default_rng(BH * N + d)
    Q, K, V = (rng.standard_normal(BH * N * d).astype(np.float32) for _ in range(3))
    s = np.float32(LOG2E / math.sqrt(d))
    dq, dk, dv, do = dev.put(Q), dev.put(K), dev.put(V), dev.alloc(Q.nbytes)
    assert gpu.flash_fwd(dq.ptr, dk.ptr, dv.ptr, do.ptr, BH, N, d, s, causal, gpu.Dtype.F32) == 0
    assert gpu.vcDeviceSynchronize() == 0
    ref = orc.attention(Q, K, V, BH, N, d, s, causal)
    assert np.abs(do.to_host(np.float32, Q.size) - ref).max() <= TOL["f32"]


def test_flash_f32_unaligned_kv_pointers(gpu, dev, orc):
    """K and V starting 4 bytes past a 16-byte boundary take the 4-byte
    staging path with the same result."""
    BH, N, d = 2, 90, 32
    rng = np.random.default_rng(5)
    Q, K, V = (rng.standard_normal(BH * N * d).astype(np.float32) for _ in range(3))
    s = np.float32(LOG2E / math.sqrt(d))
    pad = np.zeros(1, np.float32)
    dq = dev.put(Q)
    dk, dv = dev.put(np.concatenate([pad, K])), dev.put(np.concatenate([pad, V]))
    do = dev.alloc(Q.nbytes)
    assert gpu.flash_fwd(dq.ptr, dk.ptr + 4, dv.ptr + 4, do.ptr, BH, N, d, s, True,
                         gpu.Dtype.F32) == 0
    assert gpu.vcDeviceSynchronize() == 0
    ref = orc.attention(Q, K, V, BH, N, d, s, True)
    assert np.abs(do.to_host(np.float32, Q.size) - ref).max() <= TOL["f32"]


@pytest.mark.parametrize("BH,N,d,causal", [(8, 1024, 64, True), (4, 2048, 128, False),
                                           (16, 520, 24, False)])
def test_flash_f32_large_grid_vs_oracle(gpu, dev, orc, BH, N, d, causal):
    """Grids that fill the GPU take the 8-rows-per-block variant; checked on
    the first and last slices, first and last 40 rows."""
    rng = np.random.default_rng(BH * N + d + 1)
    Q, K, V = (rng.standard_normal(BH * N * d).astype(np.float32) for _ in range(3))
    s = np.float32(LOG2E / math.sqrt(d))
    dq, dk, dv, do = dev.put(Q), dev.put(K), dev.put(V), dev.alloc(Q.nbytes)
    assert gpu.flash_fwd(dq.ptr, dk.ptr, dv.ptr, do.ptr, BH, N, d, s, causal, gpu.Dtype.F32) == 0
    assert gpu.vcDeviceSynchronize() == 0
    got = do.to_host(np.float32, Q.size).reshape(BH, N, d)
    for bh in ((0, 1), (BH - 1, BH)):
        for rows in ((0, 40), (N - 40, N)):
            ref = orc.attention(Q, K, V, BH, N, d, s, causal, bh_range=bh,
                                row_range=rows).reshape(BH, N, d)
            err = np.abs(got[bh[0]:bh[1], rows[0]:rows[1]] - ref[bh[0]:bh[1], rows[0]:rows[1]]).max()
            assert err <= TOL["f32"], (bh, rows, err)


def _run_tc(gpu, dev, orc, BH, N, d, causal, bf16, seed=0, scale_in=1.0, bh_check=None,
            row_check=None, qk_scale=1.0):
    rng = np.random.default_rng(seed)
    raw = [(rng.standard_normal(BH * N * d) * scale_in * (qk_scale if i < 2 else 1.0))
           .astype(np.float32) for i in range(3)]
    bits, vals = zip(*(to_half_bits(x, bf16) for x in raw))
    s = np.float32(LOG2E / math.sqrt(d))
    dq, dk, dv = (dev.put(b) for b in bits)
    do = dev.alloc(BH * N * d * 2)
    dt = gpu.Dtype.BF16 if bf16 else gpu.Dtype.F16
    err = gpu.flash_fwd(dq.ptr, dk.ptr, dv.ptr, do.ptr, BH, N, d, s, causal, dt)
    assert err == 0, err
    assert gpu.vcDeviceSynchronize() == 0
    assert gpu.kernel_error(True) == 0
    got = half_bits_to_f32(do.to_host(np.uint16, BH * N * d), bf16).reshape(BH, N, d)
    ref = orc.attention(*vals, BH, N, d, s, causal, bh_range=bh_check,
                        row_range=row_check).reshape(BH, N, d)
    b0, b1 = bh_check or (0, BH)
    r0, r1 = row_check or (0, N)
    err = np.abs(got[b0:b1, r0:r1] - ref[b0:b1, r0:r1]).max()
    assert np.isfinite(got).all()
    assert err <= TOL["bf16" if bf16 else "f16"], err
    return got


@pytest.mark.parametrize("BH,N,d,causal", [(2, 128, 128, False), (2, 128, 128, True),
                                           (3, 512, 128, True), (2, 200, 128, False),
                                           (2, 333, 64, True), (1, 1024, 64, False),
                                           (4, 1, 128, True), (1, 640, 128, False)])
@pytest.mark.parametrize("bf16", [False, True])
def test_flash_tcgen05_vs_oracle(gpu, dev, orc, BH, N, d, causal, bf16):
    _run_tc(gpu, dev, orc, BH, N, d, causal, bf16, seed=BH + N + d + causal,
            scale_in=0.5 if bf16 else 1.0)


def test_flash_tcgen05_large_scores_rescale(gpu, dev, orc):
    # Q and K scaled x4 give scores spanning hundreds of log2 units: exercises
    # the conditional rescale of O (max growing by more than 2^8 mid-row).
    # V keeps unit variance, so the absolute bar keeps its meaning.
    _run_tc(gpu, dev, orc, 2, 512, 128, False, False, seed=3, qk_scale=4.0)
    _run_tc(gpu, dev, orc, 2, 512, 128, True, True, seed=4, qk_scale=4.0)


def test_flash_tcgen05_causal_fp16_8x16x4096_sampled(gpu, dev, orc):
    """The causal fp16 benchmark workload: B=8, H=16, N=4096, d=128; rows checked
    on a sample (4 slices x 64 rows, including the last rows of the sequence)."""
    _run_tc(gpu, dev, orc, 128, 4096, 128, True, False, seed=3, bh_check=(60, 64),
            row_check=(4032, 4096))


def test_flash_tcgen05_bf16_32x32x8192_full_shape_sampled(gpu, orc):
    """The bf16 attention benchmark workload at its own shape: B=32, H=32 (1024 slices),
    N=8192, d=128, non-causal, Q/K/V ~ 0.5 N(0,1) rounded to bf16 (2 GiB per
    tensor, generated on the device). The whole launch runs; the fp64 oracle
    checks 4 slices (the first, the last, and both sides of an 8-GPU shard
    boundary) x the first and last 64 query rows, within the bf16 bar."""
    import torch
    BH, N, d = 1024, 8192, 128
    g = torch.Generator(device="cuda").manual_seed(4)

    def gen():
        return (torch.randn(BH, N, d, device="cuda", generator=g) * 0.5).to(torch.bfloat16)

    q, k, v = gen(), gen(), gen()
    o = torch.empty_like(q)
    s = np.float32(LOG2E / math.sqrt(d))
    torch.cuda.synchronize()
    assert gpu.flash_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), BH, N, d, s,
                         False, gpu.Dtype.BF16) == 0
    assert gpu.vcDeviceSynchronize() == 0
    assert gpu.kernel_error(True) == 0
    slices = [0, 127, 128, 1023]
    idx = torch.tensor(slices, device="cuda")
    qs, ks, vs, os_ = (t.index_select(0, idx).float().cpu().numpy() for t in (q, k, v, o))
    del q, k, v, o
    torch.cuda.empty_cache()
    assert np.isfinite(os_).all()
    for rows in ((0, 64), (N - 64, N)):
        ref = orc.attention(qs, ks, vs, len(slices), N, d, s, False,
                            row_range=rows).reshape(len(slices), N, d)
        err = np.abs(os_[:, rows[0]:rows[1]] - ref[:, rows[0]:rows[1]]).max()
        assert err <= TOL["bf16"], (rows, err)


def test_flash_rejects_bad_shapes(gpu, dev):
    d = dev.alloc(1 << 16)
    # head dim 96 has no tensor-core path
    assert gpu.flash_fwd(d.ptr, d.ptr, d.ptr, d.ptr, 1, 64, 96, 0.1, False, gpu.Dtype.F16) \
        == gpu.VCError.InvalidValue
    # buffers smaller than BH*N*d are refused before launch
    assert gpu.flash_fwd(d.ptr, d.ptr, d.ptr, d.ptr, 8, 4096, 128, 0.1, False, gpu.Dtype.F16) \
        == gpu.VCError.InvalidValue
