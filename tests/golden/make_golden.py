"""Generate the golden fixtures in tests/golden/ (run here, where the reference
tree is mounted; the fixtures are committed and travel without it).

    python tests/golden/make_golden.py [--reference DIR]   (default: oracle.build_ref.reference_dir())

Writes:
  fa_demo_causal0.bin, fa_demo_causal1.bin
      The flash-attention demo case (examples/flash_attn.vc: 2 heads x 64 x 16,
      seed 12345 + causal) in the demo's own VCFA dump format
      (flash_attn.vc:240-267): magic, {NHEAD, SEQ, HDIM, causal} as float32,
      then Q, K, V, O_kernel, O_hostref. Q/K/V and O_hostref come from the
      reference's own host code compiled by oracle/build_ref.py; the O_kernel
      slot holds PyTorch's FlashAttention (CPU) output, since the reference's
      Vulkan kernel cannot run here. Each file is then checked with the
      reference's own examples/compare_flash_attn.py `check()` (tolerance
      1e-5 against torch FLASH and MATH backends).
  kat.json
      Known answers of the integer demos, computed with numpy int64 (not with
      the oracle): wmma_gemm's 8x8x16 D = A*B + C (test/wmma_gemm.vc:45-53),
      matmulCoopmat's N x N products for N = 128..1024 and 4096 as
      checksums plus the full 128 case (matmul_coopmat_bench.vc:138-143),
      vadd's demo output (test/vadd.vc:30) and reduce's per-block partials
      (test/reduce.vc:47-75).
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)


def write_vcfa(path, nhead, seq, hdim, causal, blobs):
    with open(path, "wb") as f:
        f.write(b"VCFA")
        f.write(struct.pack("<4f", nhead, seq, hdim, causal))
        for b in blobs:
            f.write(np.ascontiguousarray(b, np.float32).astype("<f4").tobytes())


def coopmat_inputs(N: int, L: int):
    n = np.arange(N, dtype=np.int64)[:, None]
    m = np.arange(L, dtype=np.int64)[None, :]
    A = (n * 3 + m * 5) % 7
    B = (n * 2 + m * 3) % 7
    return A, B


def int_checksum(C: np.ndarray) -> dict:
    C = C.astype(np.int64)
    return {
        "sum": int(C.sum()),
        "sumsq": int((C * C).sum()),
        "row0": [int(v) for v in C[0, :16]],
        "sha256": hashlib.sha256(np.ascontiguousarray(C).tobytes()).hexdigest(),
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", default="")
    args = ap.parse_args()

    from oracle import build_ref, oracle

    args.reference = args.reference or build_ref.reference_dir()
    build_ref.build(args.reference, quiet=True)
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    spec = importlib.util.spec_from_file_location(
        "compare_flash_attn", os.path.join(args.reference, "examples", "compare_flash_attn.py"))
    cmp = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(cmp)

    nhead, seq, hdim = oracle.DEMO_SHAPE
    for causal in (0, 1):
        Q, K, V = oracle.ref_fa_inputs(12345 + causal)
        scale = oracle.demo_scale(hdim)
        o_host = oracle.ref_fa_attention(Q, K, V, scale, bool(causal))
        q, k, v = (torch.from_numpy(x.copy()).reshape(1, nhead, seq, hdim) for x in (Q, K, V))
        mask = torch.tril(torch.ones(seq, seq, dtype=torch.bool)) if causal else None
        with sdpa_kernel(SDPBackend.FLASH_ATTENTION):
            o_flash = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
        path = os.path.join(HERE, f"fa_demo_causal{causal}.bin")
        write_vcfa(path, nhead, seq, hdim, causal,
                   [Q, K, V, o_flash.reshape(-1).numpy(), o_host])
        if not cmp.check(path, True, cmp.TOL):
            raise SystemExit(f"{path}: reference check failed")

    kat = {}
    # wmma_gemm: A[i][k] = (i+k)%5 (8x16), B[k][j] = (k-j+7)%5 (16x8), C = 1.
    i = np.arange(8)[:, None]
    kk = np.arange(16)[None, :]
    A = (i + kk) % 5
    kc = np.arange(16)[:, None]
    j = np.arange(8)[None, :]
    B = (kc - j + 7) % 5
    D = A.astype(np.int64) @ B.astype(np.int64) + 1
    kat["wmma_gemm"] = {"A": A.tolist(), "B": B.tolist(), "D": D.tolist()}
    # matmulCoopmat: N x N corner with row stride L = 1024, K = N.
    kat["matmul_coopmat"] = {}
    for N in (128, 256, 512, 1024):
        A, B = coopmat_inputs(N, 1024)
        C = np.rint(A[:, :N].astype(np.float64) @ B[:N, :N].astype(np.float64)).astype(np.int64)
        entry = int_checksum(C)
        if N == 128:
            entry["full"] = C.tolist()
        kat["matmul_coopmat"][str(N)] = entry
    # Same formulas at 4096 (row stride 4096): the scaled-up integer KAT.
    A, B = coopmat_inputs(4096, 4096)
    # float64 BLAS product: every partial sum is an integer below 2^53, so it
    # is exact (an int64 matmul has no BLAS path and takes tens of minutes).
    C = np.rint(A.astype(np.float64) @ B.astype(np.float64)).astype(np.int64)
    kat["matmul_coopmat"]["4096"] = int_checksum(C)
    # vadd demo: a[i] = i, b[i] = 2, N = 64.
    kat["vadd"] = {"a": list(range(64)), "b": [2] * 64, "c": [i + 2 for i in range(64)]}
    # reduce demo: in[i] = i, N = 128, block 32 -> 4 partials.
    x = np.arange(128)
    kat["reduce"] = {"n": 128, "block": 32,
                     "partials": [int(x[b * 32:(b + 1) * 32].sum()) for b in range(4)]}
    with open(os.path.join(HERE, "kat.json"), "w") as f:
        json.dump(kat, f, indent=1)
    print("golden fixtures written")


if __name__ == "__main__":
    main()
