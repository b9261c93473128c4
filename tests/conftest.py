"""Shared fixtures. Tests marked `gpu` need a CUDA device (B200); the rest run
on CPU. GPU tests talk to the kernels only through the C ABI of
libVCRuntime.so (vkcuda_b200.vc) and check them against the CPU oracle."""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs on the B200 box)")


def _ensure_built():
    from vkcuda_b200 import vc
    if not os.path.exists(vc.LIB_PATH):
        from vkcuda_b200 import build
        build.build()
    from oracle import oracle
    if not os.path.exists(oracle.LIB_PATH):
        oracle.build()


@pytest.fixture(scope="session")
def vc():
    _ensure_built()
    from vkcuda_b200 import vc as _vc
    _vc.library()
    return _vc


@pytest.fixture(scope="session")
def orc():
    _ensure_built()
    from oracle import oracle
    return oracle


@pytest.fixture(scope="session")
def gpu(vc):
    """Initialised runtime on a real GPU; fails (does not skip) without one."""
    err = vc.vcInit()
    assert err == vc.VCError.Success, f"vcInit failed: {err!r} (no CUDA device?)"
    assert vc.vcSetDevice(0) == vc.VCError.Success
    yield vc
    assert vc.kernel_error(True) == 0, "a kernel left a device error code"


class Dev:
    """A device buffer owned by the test (vcMalloc / vcFree)."""

    def __init__(self, vc, nbytes: int):
        self.vc = vc
        err, self.ptr = vc.vcMalloc(nbytes)
        assert err == vc.VCError.Success, err
        self.nbytes = nbytes

    @classmethod
    def from_host(cls, vc, arr: np.ndarray) -> "Dev":
        arr = np.ascontiguousarray(arr)
        d = cls(vc, max(arr.nbytes, 1))
        if arr.nbytes:
            assert vc.vcMemcpy(d.ptr, arr, arr.nbytes, vc.VCMemcpyKind.HostToDevice) == 0
        return d

    def to_host(self, dtype, count: int) -> np.ndarray:
        out = np.empty(count, dtype)
        if out.nbytes:
            assert self.vc.vcMemcpy(out, self.ptr, out.nbytes, self.vc.VCMemcpyKind.DeviceToHost) == 0
        return out

    def free(self):
        if self.ptr:
            assert self.vc.vcFree(self.ptr) == 0
            self.ptr = 0

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


@pytest.fixture
def dev(gpu):
    made = []

    class _F:
        @staticmethod
        def alloc(nbytes):
            d = Dev(gpu, nbytes)
            made.append(d)
            return d

        @staticmethod
        def put(arr):
            d = Dev.from_host(gpu, arr)
            made.append(d)
            return d

    yield _F
    for d in made:
        d.free()


def to_half_bits(x: np.ndarray, bf16: bool):
    """Round fp32 values to fp16/bf16 (RNE). Returns (raw uint16 bits, values
    widened back to fp32)."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x, np.float32))
    h = t.to(torch.bfloat16 if bf16 else torch.float16)
    return h.view(torch.int16).numpy().view(np.uint16).copy(), h.float().numpy()


def half_bits_to_f32(bits: np.ndarray, bf16: bool) -> np.ndarray:
    import torch
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
    return t.view(torch.bfloat16 if bf16 else torch.float16).float().numpy()


def spirv_module(entry: str) -> list:
    """The words of a minimal SPIR-V module (header, Shader capability,
    logical/GLSL450 memory model, one GLCompute OpEntryPoint named `entry`):
    what vcLoadKernel is given by generated host code, reduced to the parts a
    loader reads (SPIR-V 1.0 spec, section 2.3 physical layout)."""
    name = entry.encode() + b"\0"
    name += b"\0" * (-len(name) % 4)
    name_words = [int.from_bytes(name[i:i + 4], "little") for i in range(0, len(name), 4)]
    words = [0x07230203, 0x00010000, 0, 2, 0]          # magic, version 1.0, generator, bound, schema
    words += [(2 << 16) | 17, 1]                         # OpCapability Shader
    words += [(3 << 16) | 14, 0, 1]                      # OpMemoryModel Logical GLSL450
    words += [((3 + len(name_words)) << 16) | 15, 5, 1] + name_words  # OpEntryPoint GLCompute %1
    return words


def spirv_glsl_module(buffers, push) -> list:
    """Words of a SPIR-V module shaped like the VC compiler's GLSL backend
    output for one kernel (lib/Codegen/ASTToGLSL.cpp:955-1008 in the
    reference): entry "main"; one storage-buffer block per pointer parameter,
    `buffer Bi { T name[]; }` at binding i; one push-constant block with the
    scalar parameters in order. `buffers` and `push` are lists of (name,
    "f32" | "i32"). Only the instructions a loader reads are emitted."""
    def lit(text):
        b = text.encode() + b"\0"
        b += b"\0" * (-len(b) % 4)
        return [int.from_bytes(b[i:i + 4], "little") for i in range(0, len(b), 4)]

    def ins(op, *operands):
        return [((1 + len(operands)) << 16) | op, *operands]

    ids = iter(range(1, 1000))
    main, f32, i32 = next(ids), next(ids), next(ids)
    words = ins(17, 1) + ins(14, 0, 1) + ins(15, 5, main, *lit("main"))
    words += ins(22, f32, 32) + ins(21, i32, 32, 1)
    tid = {"f32": f32, "i32": i32}
    for b, (name, ty) in enumerate(buffers):
        rt, st, ptr, var = next(ids), next(ids), next(ids), next(ids)
        words += ins(29, rt, tid[ty]) + ins(30, st, rt)
        words += ins(5, st, *lit(f"B{b}")) + ins(6, st, 0, *lit(name)) + ins(71, st, 2)
        words += ins(32, ptr, 12, st) + ins(59, ptr, var, 12)
        words += ins(71, var, 34, 0) + ins(71, var, 33, b)
    if push:
        st, ptr, var = next(ids), next(ids), next(ids)
        words += ins(30, st, *[tid[ty] for _, ty in push]) + ins(5, st, *lit("PC"))
        for m, (name, _) in enumerate(push):
            words += ins(6, st, m, *lit(name))
        words += ins(32, ptr, 9, st) + ins(59, ptr, var, 9)
    return [0x07230203, 0x00010000, 0, 1000, 0] + words


GLSL_DEMO_INTERFACES = {
    "vadd": ([("a", "f32"), ("b", "f32"), ("c", "f32")], [("n", "i32")]),
    "blockReduce": ([("inBuf", "f32"), ("outBuf", "f32")], [("N", "i32")]),
    "flashAttn": ([("Q", "f32"), ("K", "f32"), ("V", "f32"), ("O", "f32")],
                  [("scale", "f32"), ("causal", "i32")]),
    "matmulTiled": ([("A", "f32"), ("B", "f32"), ("C", "f32")], [("N", "i32")]),
    "fillPattern": ([("a", "i32")], [("base", "i32"), ("n", "i32")]),
}
