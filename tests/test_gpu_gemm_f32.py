"""fp32 GEMM (vc_gemm with VC_DTYPE_F32, and matmulTiled) on the GPU against
the fp64 oracle.

The tensor-core path splits each fp32 operand into hi (tf32) and lo parts
and accumulates hi*hi in tf32 and lo*hi + hi*lo in bf16. Bars:
* the reference's own: 1e-4 relative error against an fp64 loop on its
  inputs 0.1 i + 0.01 j / 0.1 j + 0.01 i (examples/matmul_bench.vc:109-125),
  at its sizes 128..1024 and beyond;
* random inputs of both signs: |D - D_ref| <= 2e-5 * (|A| |B|)_ij, the sum
  of absolute products (the split's worst case is ~2^-17 = 7.6e-6 of it; a
  single tf32 product per term would exceed the bar by ~25x).
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
BOUND = 2e-5


def _demo_inputs(N):
    i = np.arange(N, dtype=np.float32)[:, None]
    j = np.arange(N, dtype=np.float32)[None, :]
    A = (np.float32(0.1) * i + np.float32(0.01) * j).astype(np.float32)
    B = (np.float32(0.1) * j + np.float32(0.01) * i).astype(np.float32)
    return A, B


def _run(gpu, dev, orc, M, N, K, b_kn, lda=None, ldb=None, ldd=None, with_c=False, seed=0,
         rows=None, scale=1.0):
    rng = np.random.default_rng(seed)
    lda = lda or K
    ldb = ldb or (N if b_kn else K)
    ldd = ldd or N
    A = (rng.uniform(-1, 1, (M, lda)) * scale).astype(np.float32)
    B = rng.uniform(-1, 1, (K, ldb) if b_kn else (N, ldb)).astype(np.float32)
    cin = rng.standard_normal((M, N)).astype(np.float32) if with_c else None
    dA, dB, dD = dev.put(A), dev.put(B), dev.alloc(M * ldd * 4)
    dC = dev.put(cin) if with_c else None
    err = gpu.gemm(dA.ptr, dB.ptr, dD.ptr, dC.ptr if dC else None, M, N, K, lda, ldb, ldd,
                   N if with_c else 0, gpu.Dtype.F32, b_kn)
    assert err == 0, err
    assert gpu.vcDeviceSynchronize() == 0
    got = dD.to_host(np.float32, M * ldd).reshape(M, ldd)[:, :N].astype(np.float64)
    ref = orc.gemm(A, B, M, N, K, lda, ldb, b_kn, Cin=cin, ldc=N, rows=rows)
    mag = orc.gemm(np.abs(A), np.abs(B), M, N, K, lda, ldb, b_kn, rows=rows)
    r0, r1 = rows or (0, M)
    excess = np.abs(got[r0:r1] - ref[r0:r1]) - BOUND * mag[r0:r1] - 1e-30
    assert excess.max() <= 0, (np.abs(got[r0:r1] - ref[r0:r1]) / (mag[r0:r1] + 1e-30)).max()
    return got


@pytest.mark.parametrize("N", [128, 256, 512, 1024, 1000, 2048])
def test_matmul_tiled_demo_sizes_relative_1e4(gpu, dev, orc, N):
    """matmulTiled's launch (grid (N, N) elements, block 16 x 16) at the demo's
    sizes; N % 4 == 0 runs on the tensor cores."""
    A, B = _demo_inputs(N)
    dA, dB, dC = dev.put(A), dev.put(B), dev.alloc(N * N * 4)
    err, k = gpu.vcGetKernel("matmulTiled")
    assert err == 0
    assert gpu.vcLaunchKernel2D(k, N, N, 16, 16, [gpu.ptr(dA.ptr), gpu.ptr(dB.ptr),
                                                  gpu.ptr(dC.ptr), gpu.i32(N)]) == 0
    assert gpu.vcDeviceSynchronize() == 0
    got = dC.to_host(np.float32, N * N).reshape(N, N).astype(np.float64)
    ref = orc.gemm(A, B, N, N, N, N, N, True)
    rel = np.abs(got - ref) / np.where(ref != 0, np.abs(ref), 1.0)
    assert rel.max() <= 1e-4, rel.max()
    # inside the demo's bar with room: the tensor cores' truncating fp32
    # accumulation is bounded to one 512-deep K chunk (same-sign data shows
    # its bias in full), the chunks are added with round-to-nearest
    assert rel.max() <= 3e-5, rel.max()
    gpu.vcReleaseKernel(k)


@pytest.mark.parametrize("M,N,K", [(128, 256, 32), (256, 512, 512), (300, 500, 200),
                                   (4, 4, 4), (129, 260, 1000), (1024, 1024, 1024),
                                   (40, 8, 72), (512, 768, 33 * 4)])
@pytest.mark.parametrize("b_kn", [True, False])
def test_gemm_f32_random_vs_oracle(gpu, dev, orc, M, N, K, b_kn):
    _run(gpu, dev, orc, M, N, K, b_kn, seed=M * 7 + N * 3 + K + int(b_kn))


@pytest.mark.parametrize("b_kn", [True, False])
def test_gemm_f32_split_k_small_grid_deterministic(gpu, dev, orc, b_kn):
    """1024 x 1024 x 1024 fills 16 of the GPU's SM pairs, so K is split in
    two halves that both add onto a zeroed C: results within the bar, with
    the addend, and identical on a second call."""
    M = N = K = 1024
    rng = np.random.default_rng(21 + int(b_kn))
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N) if b_kn else (N, K)).astype(np.float32)
    cin = rng.standard_normal((M, N)).astype(np.float32)
    dA, dB, dC, dD = dev.put(A), dev.put(B), dev.put(cin), dev.alloc(M * N * 4)
    outs = []
    for _ in range(2):
        assert gpu.gemm(dA.ptr, dB.ptr, dD.ptr, dC.ptr, M, N, K, K, N if b_kn else K, N, N,
                        gpu.Dtype.F32, b_kn) == 0
        assert gpu.vcDeviceSynchronize() == 0
        outs.append(dD.to_host(np.float32, M * N).reshape(M, N))
    assert np.array_equal(outs[0], outs[1])
    ldb = N if b_kn else K
    ref = orc.gemm(A, B, M, N, K, K, ldb, b_kn, Cin=cin, ldc=N)
    mag = orc.gemm(np.abs(A), np.abs(B), M, N, K, K, ldb, b_kn)
    assert (np.abs(outs[0].astype(np.float64) - ref) <= BOUND * mag + 1e-6).all()
    # In place (D is Cin): the same shape must not zero D before reading the
    # addend, so it runs unsplit; same bar.
    assert gpu.gemm(dA.ptr, dB.ptr, dC.ptr, dC.ptr, M, N, K, K, ldb, N, N,
                    gpu.Dtype.F32, b_kn) == 0
    assert gpu.vcDeviceSynchronize() == 0
    inplace = dC.to_host(np.float32, M * N).reshape(M, N).astype(np.float64)
    assert (np.abs(inplace - ref) <= BOUND * mag + 1e-6).all()


def test_gemm_f32_with_addend_and_strides(gpu, dev, orc):
    _run(gpu, dev, orc, 200, 300, 256, True, lda=260, ldb=304, ldd=308, with_c=True, seed=5)
    _run(gpu, dev, orc, 200, 300, 256, False, lda=260, ldb=264, ldd=300, with_c=True, seed=6)


def test_gemm_f32_unaligned_strides_use_simt_path(gpu, dev, orc):
    # lda = 37 floats (148 bytes) breaks TMA's 16-byte stride rule: the
    # CUDA-core path serves it with the same contract and bar.
    _run(gpu, dev, orc, 65, 33, 37, True, lda=37, ldb=33, ldd=33, seed=9)
    # matmulTiled at N = 131 (524-byte rows) likewise.
    N = 131
    A, B = _demo_inputs(N)
    dA, dB, dC = dev.put(A), dev.put(B), dev.alloc(N * N * 4)
    err, k = gpu.vcGetKernel("matmulTiled")
    assert gpu.vcLaunchKernel2D(k, N, N, 16, 16, [gpu.ptr(dA.ptr), gpu.ptr(dB.ptr),
                                                  gpu.ptr(dC.ptr), gpu.i32(N)]) == 0
    assert gpu.vcDeviceSynchronize() == 0
    got = dC.to_host(np.float32, N * N).reshape(N, N).astype(np.float64)
    ref = orc.gemm(A, B, N, N, N, N, N, True)
    assert (np.abs(got - ref) / np.abs(ref)).max() <= 1e-4
    gpu.vcReleaseKernel(k)


def test_gemm_f32_wide_exponent_range(gpu, dev, orc):
    """Rows scaled over 2^-60 .. 2^60: the split is relative, so the bound
    holds row by row."""
    rng = np.random.default_rng(11)
    M, N, K = 256, 256, 256
    A = (rng.uniform(-1, 1, (M, K)) * np.exp2(rng.integers(-60, 61, (M, 1)))).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    dA, dB, dD = dev.put(A), dev.put(B), dev.alloc(M * N * 4)
    assert gpu.gemm(dA.ptr, dB.ptr, dD.ptr, None, M, N, K, K, N, N, 0, gpu.Dtype.F32, True) == 0
    assert gpu.vcDeviceSynchronize() == 0
    got = dD.to_host(np.float32, M * N).reshape(M, N).astype(np.float64)
    ref = orc.gemm(A, B, M, N, K, K, N, True)
    mag = orc.gemm(np.abs(A), np.abs(B), M, N, K, K, N, True)
    assert (np.abs(got - ref) <= BOUND * mag).all()


def test_gemm_f32_nonfinite_inputs_propagate(gpu, dev):
    """An infinity or NaN in A makes its row of D NaN (an infinity meets a
    zero low part, where an fp32 FMA loop would give inf); other rows stay
    exact."""
    M = N = K = 128
    A = np.ones((M, K), np.float32)
    B = np.ones((K, N), np.float32)
    A[3, 5] = np.inf
    A[7, 9] = np.nan
    dA, dB, dD = dev.put(A), dev.put(B), dev.alloc(M * N * 4)
    assert gpu.gemm(dA.ptr, dB.ptr, dD.ptr, None, M, N, K, K, N, N, 0, gpu.Dtype.F32, True) == 0
    assert gpu.vcDeviceSynchronize() == 0
    got = dD.to_host(np.float32, M * N).reshape(M, N)
    assert np.isnan(got[3]).all()
    assert np.isnan(got[7]).all()
    rest = np.delete(got, [3, 7], axis=0)
    assert (rest == K).all()


def test_gemm_f32_4096_sampled_rows_and_column_sums(gpu, dev, orc):
    M = N = K = 4096
    got = _run(gpu, dev, orc, M, N, K, True, seed=42, rows=(4000, 4096))
    rng = np.random.default_rng(42)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    expect = A.astype(np.float64).sum(0) @ B.astype(np.float64)
    mag = np.abs(A).astype(np.float64).sum(0) @ np.abs(B).astype(np.float64)
    assert (np.abs(got.sum(0) - expect) <= BOUND * mag).all()


def test_gemm_f32_grouped_tile_order_large_b(gpu, dev, orc):
    """B of 4608 x 4096 fp32 (72 MiB) exceeds the size above which tiles run
    in groups of 8 pair rows; M = 2304 is 9 pair rows (a partial last group)."""
    _run(gpu, dev, orc, 2304, 4096, 4608, True, seed=77, rows=(2240, 2304))
    _run(gpu, dev, orc, 2304, 4096, 4608, False, seed=78, rows=(0, 48))


def test_gemm_f32_rejects_bad_shapes(gpu, dev):
    d = dev.alloc(4096)
    F32 = gpu.Dtype.F32
    assert gpu.gemm(d.ptr, d.ptr, d.ptr, None, 0, 8, 8, 8, 8, 8, 0, F32) == gpu.VCError.InvalidValue
    # lda < K
    assert gpu.gemm(d.ptr, d.ptr, d.ptr, None, 8, 8, 8, 4, 8, 8, 0, F32) == gpu.VCError.InvalidValue
    # 64 x 64 fp32 operands need 16 KiB each: refused before launch, while
    # 32 x 32 (4 KiB each) fits.
    assert gpu.gemm(d.ptr, d.ptr, d.ptr, None, 64, 64, 64, 64, 64, 64, 0, F32) == gpu.VCError.InvalidValue
    a, b, c = dev.alloc(4096), dev.alloc(4096), dev.alloc(4096)
    assert gpu.gemm(a.ptr, b.ptr, c.ptr, None, 32, 32, 32, 32, 32, 32, 0, F32) == 0
    assert gpu.vcDeviceSynchronize() == 0
