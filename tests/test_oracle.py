"""The CPU oracle pinned against the reference: its own compiled host code
(oracle/_ref), the golden fixtures and known answers, and an independent
implementation (torch SDPA in fp64). CPU only."""
from __future__ import annotations

import json
import math
import os
import struct

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load_vcfa(path):
    """Reader for the demo's VCFA dump (examples/flash_attn.vc:240-267)."""
    raw = open(path, "rb").read()
    assert raw[:4] == b"VCFA"
    nhead, seq, hdim, causal = (int(v) for v in struct.unpack("<4f", raw[4:20]))
    body = np.frombuffer(raw[20:], "<f4")
    e = nhead * seq * hdim
    assert body.size == 5 * e
    blobs = [body[i * e:(i + 1) * e].copy() for i in range(5)]
    return (nhead, seq, hdim, causal), blobs


@pytest.fixture(scope="module")
def kat():
    with open(os.path.join(GOLDEN, "kat.json")) as f:
        return json.load(f)


@pytest.mark.parametrize("causal", [0, 1])
def test_generator_matches_reference_build(orc, causal):
    ref = orc.ref_fa_inputs(12345 + causal)
    if ref is None:
        pytest.skip("oracle/_ref not built (reference tree absent when building)")
    mine = orc.fa_inputs(12345 + causal, 2 * 64 * 16)
    for a, b in zip(ref, mine):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("causal", [0, 1])
def test_attention_matches_reference_build(orc, causal):
    q, k, v = orc.fa_inputs(12345 + causal, 2 * 64 * 16)
    s = orc.demo_scale(16)
    ref = orc.ref_fa_attention(q, k, v, s, bool(causal))
    if ref is None:
        pytest.skip("oracle/_ref not built")
    assert np.array_equal(orc.attention(q, k, v, 2, 64, 16, s, bool(causal)), ref)


@pytest.mark.parametrize("causal", [0, 1])
def test_attention_matches_golden_vcfa(orc, causal):
    (nh, seq, hd, c), (Q, K, V, O_torch, O_host) = load_vcfa(
        os.path.join(GOLDEN, f"fa_demo_causal{causal}.bin"))
    assert (nh, seq, hd, c) == (2, 64, 16, causal)
    q, k, v = orc.fa_inputs(12345 + causal, nh * seq * hd)
    assert np.array_equal(q, Q) and np.array_equal(k, K) and np.array_equal(v, V)
    o = orc.attention(Q, K, V, nh, seq, hd, orc.demo_scale(hd), bool(causal))
    assert np.array_equal(o, O_host)
    # The fixture's second output is PyTorch FlashAttention; the reference's
    # own cross-check allows 1e-5 (examples/compare_flash_attn.py:64).
    assert np.abs(o - O_torch).max() <= 1e-5


@pytest.mark.parametrize("BH,N,d,causal", [(3, 77, 32, False), (2, 130, 64, True), (1, 5, 8, True)])
def test_attention_matches_torch_math_fp64(orc, BH, N, d, causal):
    import torch
    import torch.nn.functional as F
    rng = np.random.default_rng(7)
    Q, K, V = (rng.standard_normal((BH, N, d)).astype(np.float32) for _ in range(3))
    scale_log2 = math.log2(math.e) / math.sqrt(d)
    o = orc.attention(Q, K, V, BH, N, d, np.float32(scale_log2), causal).reshape(BH, N, d)
    mask = torch.tril(torch.ones(N, N, dtype=torch.bool)) if causal else None
    ref = F.scaled_dot_product_attention(
        *(torch.from_numpy(x).double() for x in (Q, K, V)), attn_mask=mask,
        scale=float(np.float32(scale_log2)) / math.log2(math.e)).numpy()
    assert np.abs(o - ref).max() <= 1e-6


def test_attention_row_sampling(orc):
    rng = np.random.default_rng(3)
    BH, N, d = 4, 64, 16
    Q, K, V = (rng.standard_normal(BH * N * d).astype(np.float32) for _ in range(3))
    full = orc.attention(Q, K, V, BH, N, d, 0.3, True).reshape(BH, N, d)
    part = orc.attention(Q, K, V, BH, N, d, 0.3, True, bh_range=(1, 3),
                         row_range=(10, 20)).reshape(BH, N, d)
    assert np.array_equal(part[1:3, 10:20], full[1:3, 10:20])
    assert not part[0].any() and not part[3].any()


def test_gemm_wmma_kat(orc, kat):
    A = np.array(kat["wmma_gemm"]["A"], np.float32)
    B = np.array(kat["wmma_gemm"]["B"], np.float32)
    D = orc.gemm(A, B, 8, 8, 16, 16, 8, True, Cin=np.ones((8, 8), np.float32), ldc=8)
    assert np.array_equal(D, np.array(kat["wmma_gemm"]["D"], np.float64))


@pytest.mark.parametrize("N", [128, 256])
def test_gemm_coopmat_kat(orc, kat, N):
    L = 1024
    n = np.arange(N)[:, None]
    m = np.arange(L)[None, :]
    A = ((n * 3 + m * 5) % 7).astype(np.float32)
    B = ((n * 2 + m * 3) % 7).astype(np.float32)
    D = orc.gemm(A, B, N, N, N, L, L, True)
    ent = kat["matmul_coopmat"][str(N)]
    Di = D.astype(np.int64)
    assert int(Di.sum()) == ent["sum"] and int((Di * Di).sum()) == ent["sumsq"]
    if "full" in ent:
        assert np.array_equal(Di, np.array(ent["full"], np.int64))


def test_gemm_layouts_agree(orc):
    rng = np.random.default_rng(1)
    M, N, K = 33, 17, 40
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    d1 = orc.gemm(A, B, M, N, K, K, N, True)
    d2 = orc.gemm(A, np.ascontiguousarray(B.T), M, N, K, K, K, False)
    ref = A.astype(np.float64) @ B.astype(np.float64)
    assert np.abs(d1 - ref).max() < 1e-12 and np.abs(d2 - ref).max() < 1e-12


def test_vadd_and_sum(orc, kat):
    a = np.array(kat["vadd"]["a"], np.float32)
    b = np.array(kat["vadd"]["b"], np.float32)
    assert np.array_equal(orc.vadd(a, b), np.array(kat["vadd"]["c"], np.float32))
    rng = np.random.default_rng(5)
    x = rng.random(3_000_001, dtype=np.float32)
    assert orc.sum_f64(x) == pytest.approx(math.fsum(x.astype(np.float64)), rel=1e-12)
    assert orc.sum_f64(x, threads=1) == orc.sum_f64(x, threads=4)
    assert orc.sum_f64(np.zeros(0, np.float32)) == 0.0


def _tree_py(x, block, groups):
    out = []
    for g in range(groups):
        s = [np.float32(x[g * block + t]) if g * block + t < len(x) else np.float32(0)
             for t in range(block)]
        h = block // 2
        while h > 0:
            for t in range(h):
                s[t] = np.float32(s[t] + s[t + h])
            h //= 2
        out.append(s[0])
    return np.array(out, np.float32)


def test_block_reduce_kat(orc, kat):
    x = np.arange(kat["reduce"]["n"], dtype=np.float32)
    out = orc.block_reduce(x, kat["reduce"]["block"])
    assert out.tolist() == kat["reduce"]["partials"]


@pytest.mark.parametrize("n,block", [(100, 32), (200, 48), (77, 7), (1, 1), (1000, 256)])
def test_block_reduce_tree_order(orc, n, block):
    x = np.random.default_rng(n).standard_normal(n).astype(np.float32)
    groups = (n + block - 1) // block
    assert np.array_equal(orc.block_reduce(x, block), _tree_py(x, block, groups))
