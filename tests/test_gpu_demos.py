"""The reference demos' remaining checks and independent large-shape checks:

* matmulTiled (examples/matmul_bench.vc:22-54) through its own launch, with
  its own inputs (0.1 i + 0.01 j / 0.1 j + 0.01 i) and its own bar: 1e-4
  relative against an fp64 loop (matmul_bench.vc:109-125).
* The flash-attention demo's cross-check workflow applied to our kernel: our
  fp32 output goes into a VCFA dump, which is read back and judged with the
  criteria of the reference's examples/compare_flash_attn.py (1e-5 between
  the kernel, PyTorch's FlashAttention and the host reference).
* Full-size attention configs against an independent implementation (PyTorch
  SDPA, fp32 math on the GPU): every row of the causal fp16 config, 128
  slices of the bf16 config.
"""
from __future__ import annotations

import math
import os

import numpy as np
import pytest

from conftest import half_bits_to_f32, to_half_bits

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
LOG2E = 1.4426950408889634


@pytest.mark.parametrize("N", [64, 100, 256, 512])
def test_matmul_tiled_demo(gpu, dev, orc, N):
    i = np.arange(N, dtype=np.float32)[:, None]
    j = np.arange(N, dtype=np.float32)[None, :]
    A = (np.float32(0.1) * i + np.float32(0.01) * j).astype(np.float32)
    B = (np.float32(0.1) * j + np.float32(0.01) * i).astype(np.float32)
    dA, dB, dC = dev.put(A), dev.put(B), dev.alloc(N * N * 4)
    err, k = gpu.vcGetKernel("matmulTiled")
    assert err == 0
    # The demo's launch: grid (N, N) elements, block 16 x 16.
    assert gpu.vcLaunchKernel2D(k, N, N, 16, 16, [gpu.ptr(dA.ptr), gpu.ptr(dB.ptr),
                                                  gpu.ptr(dC.ptr), gpu.i32(N)]) == 0
    assert gpu.vcDeviceSynchronize() == 0
    got = dC.to_host(np.float32, N * N).reshape(N, N).astype(np.float64)
    ref = orc.gemm(A, B, N, N, N, N, N, True)
    rel = np.abs(got - ref) / np.where(ref != 0, np.abs(ref), 1.0)
    assert rel.max() <= 1e-4
    gpu.vcReleaseKernel(k)


@pytest.mark.parametrize("causal", [0, 1])
def test_vcfa_dump_of_our_kernel_passes_reference_criteria(gpu, dev, tmp_path, causal):
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    from vkcuda_b200 import vcfa
    meta, blobs = vcfa.read(os.path.join(GOLDEN, f"fa_demo_causal{causal}.bin"))
    nh, seq, hd = meta["nhead"], meta["seq"], meta["hdim"]
    Q, K, V, O_host = blobs["q"], blobs["k"], blobs["v"], blobs["o_hostref"]
    dq, dk, dv, do = dev.put(Q), dev.put(K), dev.put(V), dev.alloc(Q.nbytes)
    err, k = gpu.vcGetKernel("flashAttn")
    scale = np.float32(LOG2E / math.sqrt(hd))
    assert gpu.vcLaunchKernel(k, nh * seq, 16, [gpu.ptr(dq.ptr), gpu.ptr(dk.ptr), gpu.ptr(dv.ptr),
                                                gpu.ptr(do.ptr), gpu.f32(scale),
                                                gpu.i32(causal)]) == 0
    assert gpu.vcDeviceSynchronize() == 0
    O_ours = do.to_host(np.float32, Q.size)
    gpu.vcReleaseKernel(k)
    path = str(tmp_path / f"causal{causal}.bin")
    vcfa.write(path, nh, seq, hd, causal, Q, K, V, O_ours, O_host)
    meta2, b2 = vcfa.read(path)
    assert meta2 == meta and np.array_equal(b2["o_kernel"], O_ours)
    # The reference script's comparisons (compare_flash_attn.py:123-151).
    shape = (1, nh, seq, hd)
    q, kk, v = (torch.from_numpy(b2[n].copy()).reshape(shape) for n in ("q", "k", "v"))
    mask = torch.tril(torch.ones(seq, seq, dtype=torch.bool)) if causal else None
    with sdpa_kernel(SDPBackend.FLASH_ATTENTION):
        o_torch = F.scaled_dot_product_attention(q, kk, v, attn_mask=mask)
    o_kernel = torch.from_numpy(b2["o_kernel"]).reshape(shape)
    o_hostref = torch.from_numpy(b2["o_hostref"]).reshape(shape)
    worst = lambda a, b: (a.double() - b.double()).abs().max().item()  # noqa: E731
    assert worst(o_torch, o_kernel) <= 1e-5
    assert worst(o_kernel, o_hostref) <= 1e-5


def _torch_ref_fp32(q, k, v, causal):
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel
    with sdpa_kernel(SDPBackend.MATH):
        return F.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=causal)


def test_flash_causal_fp16_8x16x4096_all_rows_vs_torch(gpu):
    """B=8, H=16, N=4096, d=128, fp16, causal: every row against torch fp32."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(33)
    BH, N, d = 128, 4096, 128
    q, k, v = (torch.randn(BH, N, d, device="cuda", generator=g).half() for _ in range(3))
    o = torch.empty_like(q)
    assert gpu.flash_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), BH, N, d,
                         LOG2E / math.sqrt(d), True, gpu.Dtype.F16) == 0
    torch.cuda.synchronize()
    worst = 0.0
    for c in range(0, BH, 32):
        ref = _torch_ref_fp32(q[c:c + 32], k[c:c + 32], v[c:c + 32], True)
        worst = max(worst, (o[c:c + 32].float() - ref).abs().max().item())
        del ref
    assert worst <= 2e-3, worst


def test_flash_bf16_32x32x8192_slices_vs_torch(gpu):
    """B=32, H=32, N=8192, d=128, bf16 (inputs 0.5 N(0,1)): 128 of the 1024
    slices (the first and last 64) against torch fp32."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(44)
    BH, N, d = 1024, 8192, 128
    q, k, v = ((torch.randn(BH, N, d, device="cuda", generator=g) * 0.5).bfloat16()
               for _ in range(3))
    o = torch.empty_like(q)
    assert gpu.flash_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), BH, N, d,
                         LOG2E / math.sqrt(d), False, gpu.Dtype.BF16) == 0
    torch.cuda.synchronize()
    worst = 0.0
    for c in list(range(0, 64, 8)) + list(range(BH - 64, BH, 8)):
        ref = _torch_ref_fp32(q[c:c + 8], k[c:c + 8], v[c:c + 8], False)
        worst = max(worst, (o[c:c + 8].float() - ref).abs().max().item())
        del ref
    assert worst <= 1e-2, worst
    del q, k, v, o
    torch.cuda.empty_cache()
