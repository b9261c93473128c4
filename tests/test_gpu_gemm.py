"""GEMM on the GPU through the C ABI against the fp64 oracle.
Bars: the reference's integer known answers bit-exact; random fp16/bf16 inputs
within 1e-3 * sqrt(K) absolute of the fp64 product of the rounded inputs."""
from __future__ import annotations

import hashlib
import json
import math
import os

import numpy as np
import pytest

from conftest import to_half_bits

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def kat():
    return json.load(open(os.path.join(GOLDEN, "kat.json")))


def test_wmma_gemm_demo_exact(gpu, dev, kat):
    """test/wmma_gemm.vc through the legacy launch: D = A*B + C, exact."""
    A = np.array(kat["wmma_gemm"]["A"], np.float16)
    B = np.array(kat["wmma_gemm"]["B"], np.float16)
    C = np.ones((8, 8), np.float32)
    dA, dB, dC, dD = dev.put(A), dev.put(B), dev.put(C), dev.alloc(256)
    err, k = gpu.vcGetKernel("wmma_gemm")
    assert gpu.vcLaunchKernel(k, 1, 32, [gpu.ptr(dA.ptr), gpu.ptr(dB.ptr), gpu.ptr(dC.ptr),
                                         gpu.ptr(dD.ptr)]) == 0
    assert gpu.vcDeviceSynchronize() == 0
    assert np.array_equal(dD.to_host(np.float32, 64).reshape(8, 8),
                          np.array(kat["wmma_gemm"]["D"], np.float32))
    gpu.vcReleaseKernel(k)


@pytest.mark.parametrize("N", [128, 256, 512, 1024])
def test_matmul_coopmat_demo_exact(gpu, dev, kat, N):
    """examples/matmul_coopmat_bench.vc's launch (grid (N/16*32, N/16), block
    32, row stride L = 1024) with its integer inputs: exact."""
    L = 1024
    n = np.arange(N)[:, None]
    m = np.arange(L)[None, :]
    A = ((n * 3 + m * 5) % 7).astype(np.float16)
    B = ((n * 2 + m * 3) % 7).astype(np.float16)
    dA, dB, dC = dev.put(A), dev.put(B), dev.alloc(N * L * 4)
    err, k = gpu.vcGetKernel("matmulCoopmat")
    assert gpu.vcLaunchKernel2D(k, (N // 16) * 32, N // 16, 32, 1,
                                [gpu.ptr(dA.ptr), gpu.ptr(dB.ptr), gpu.ptr(dC.ptr), gpu.i32(N)]) == 0
    assert gpu.vcDeviceSynchronize() == 0
    C = dC.to_host(np.float32, N * L).reshape(N, L)[:, :N].astype(np.int64)
    ent = kat["matmul_coopmat"][str(N)]
    assert int(C.sum()) == ent["sum"] and int((C * C).sum()) == ent["sumsq"]
    assert C[0, :16].tolist() == ent["row0"]
    if "full" in ent:
        assert np.array_equal(C, np.array(ent["full"], np.int64))
    gpu.vcReleaseKernel(k)


def test_integer_kat_4096_exact(gpu, dev, kat):
    """The coopmat formulas scaled to 4096^3 (partial sums < 2^24): exact."""
    N = 4096
    n = np.arange(N)[:, None]
    m = np.arange(N)[None, :]
    A = ((n * 3 + m * 5) % 7).astype(np.float16)
    B = ((n * 2 + m * 3) % 7).astype(np.float16)
    dA, dB, dD = dev.put(A), dev.put(B), dev.alloc(N * N * 4)
    assert gpu.gemm(dA.ptr, dB.ptr, dD.ptr, None, N, N, N, N, N, N, 0, gpu.Dtype.F16, True) == 0
    assert gpu.vcDeviceSynchronize() == 0
    C = dD.to_host(np.float32, N * N).reshape(N, N).astype(np.int64)
    ent = kat["matmul_coopmat"]["4096"]
    assert int(C.sum()) == ent["sum"]
    assert hashlib.sha256(np.ascontiguousarray(C).tobytes()).hexdigest() == ent["sha256"]


def _run_gemm(gpu, dev, orc, M, N, K, bf16, b_kn, with_c=False, lda=None, ldb=None, ldd=None,
              seed=0, rows=None):
    rng = np.random.default_rng(seed)
    lda = lda or K
    ldb = ldb or (N if b_kn else K)
    ldd = ldd or N
    a32 = rng.uniform(-1, 1, (M, lda)).astype(np.float32)
    b32 = rng.uniform(-1, 1, (K, ldb) if b_kn else (N, ldb)).astype(np.float32)
    abits, aval = to_half_bits(a32, bf16)
    bbits, bval = to_half_bits(b32, bf16)
    cin = rng.standard_normal((M, N)).astype(np.float32) if with_c else None
    dA, dB, dD = dev.put(abits), dev.put(bbits), dev.alloc(M * ldd * 4)
    dC = dev.put(cin) if with_c else None
    dt = gpu.Dtype.BF16 if bf16 else gpu.Dtype.F16
    err = gpu.gemm(dA.ptr, dB.ptr, dD.ptr, dC.ptr if dC else None, M, N, K, lda, ldb, ldd,
                   N if with_c else 0, dt, b_kn)
    assert err == 0, err
    assert gpu.vcDeviceSynchronize() == 0
    got = dD.to_host(np.float32, M * ldd).reshape(M, ldd)[:, :N]
    ref = orc.gemm(aval, bval, M, N, K, lda, ldb, b_kn, Cin=cin, ldc=N, rows=rows)
    r0, r1 = rows or (0, M)
    err = np.abs(got[r0:r1].astype(np.float64) - ref[r0:r1]).max()
    assert err <= 1e-3 * math.sqrt(K), err
    return got


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 512), (300, 500, 200),
                                   (1, 1, 1), (129, 257, 1000), (1024, 1024, 1024), (37, 8, 72),
                                   # CTA-pair kernel with an odd number of 64-deep K
                                   # blocks: the last barrier stage's second block
                                   # lies past K (zero-filled)
                                   (256, 256, 192), (384, 768, 320)])
@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("b_kn", [True, False])
def test_gemm_random_vs_oracle(gpu, dev, orc, M, N, K, bf16, b_kn):
    if K % 8 and K > 1:
        pytest.skip("row strides are padded below")
    lda = ((K + 7) // 8) * 8
    ldb = ((N + 7) // 8) * 8 if b_kn else lda
    _run_gemm(gpu, dev, orc, M, N, K, bf16, b_kn, lda=lda, ldb=ldb, ldd=((N + 3) // 4) * 4,
              seed=M * 7 + N * 3 + K)


def test_gemm_with_addend(gpu, dev, orc):
    _run_gemm(gpu, dev, orc, 200, 300, 256, False, True, with_c=True, seed=5)


def test_gemm_unaligned_strides_use_simt_path(gpu, dev, orc):
    # lda = 37 elements breaks TMA's 16-byte stride rule: the CUDA-core path
    # serves it with the same contract.
    _run_gemm(gpu, dev, orc, 65, 33, 37, False, True, lda=37, ldb=33, ldd=33, seed=9)


def test_gemm_grouped_tile_order_large_b(gpu, dev, orc):
    """B of 4608 x 8192 fp16 (72 MiB) exceeds the size above which the pair
    kernel orders its tiles in groups of 8 pair rows; M = 2304 is 9 pair
    rows, so the last group is partial. Rows of the partial group and the
    first group are checked against the oracle."""
    M, N, K = 2304, 8192, 4608
    _run_gemm(gpu, dev, orc, M, N, K, False, True, seed=77, rows=(2240, 2304))
    _run_gemm(gpu, dev, orc, M, N, K, True, True, seed=78, rows=(0, 48))


def test_gemm_4096_sampled_rows_and_column_sums(gpu, dev, orc):
    M = N = K = 4096
    got = _run_gemm(gpu, dev, orc, M, N, K, False, True, seed=42, rows=(4000, 4096))
    # Size-independent property over the full product: column sums of D equal
    # (column sums of A) * B, in fp64.
    rng = np.random.default_rng(42)
    a32 = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b32 = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    _, aval = to_half_bits(a32, False)
    _, bval = to_half_bits(b32, False)
    expect = aval.astype(np.float64).sum(0) @ bval.astype(np.float64)
    assert np.abs(got.astype(np.float64).sum(0) - expect).max() <= 1e-3 * math.sqrt(K) * math.sqrt(M)


def test_gemm_rejects_bad_shapes(gpu, dev):
    d = dev.alloc(1024)
    assert gpu.gemm(d.ptr, d.ptr, d.ptr, None, 0, 8, 8, 8, 8, 8, 0) == gpu.VCError.InvalidValue
    assert gpu.gemm(d.ptr, d.ptr, d.ptr, None, 8, 8, 8, 4, 8, 8, 0) == gpu.VCError.InvalidValue
    # Buffers too small for the shape are refused before launch.
    assert gpu.gemm(d.ptr, d.ptr, d.ptr, None, 64, 64, 64, 64, 64, 64, 0) == gpu.VCError.InvalidValue
