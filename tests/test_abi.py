"""libVCRuntime.so on CPU: it loads without a GPU, exports every symbol the
headers declare, and the host-side logic (error codes, kernel registry,
argument checks, fault injection) behaves as the reference API specifies."""
from __future__ import annotations

import os
import re
import subprocess
import sys

import pytest

from conftest import GLSL_DEMO_INTERFACES, spirv_glsl_module, spirv_module

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_c_symbols():
    text = open(os.path.join(ROOT, "include", "vc_b200.h")).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char \*)\s*(vc_\w+)\(", text, re.M)))


def _declared_cpp_functions():
    text = open(os.path.join(ROOT, "include", "vc", "Runtime", "VCRuntime.h")).read()
    return sorted(set(re.findall(r"^(?:VCError|const char \*)\s*(vc\w+)\(", text, re.M)))


def _exported(lib_path, demangle):
    cmd = ["nm", "-D", "--defined-only"] + (["-C"] if demangle else []) + [lib_path]
    return subprocess.run(cmd, capture_output=True, text=True, check=True).stdout


def test_library_loads_and_exports_c_abi(vc):
    syms = _declared_c_symbols()
    assert len(syms) >= 59
    out = _exported(vc.LIB_PATH, False)
    exported = set(re.findall(r" T (vc_\w+)$", out, re.M))
    missing = [s for s in syms if s not in exported]
    assert not missing, missing
    # ...and the Python mirror binds exactly those.
    assert set(vc.SIGNATURES) == set(syms)


def test_library_exports_cpp_api(vc):
    out = _exported(vc.LIB_PATH, True)
    missing = [f for f in _declared_cpp_functions() if f"vc::{f}(" not in out]
    assert not missing, missing


def test_error_strings(vc):
    assert vc.vcErrorString(vc.VCError.Success) == "success"
    assert vc.vcErrorString(vc.VCError.InvalidKernel) == "invalid kernel"
    assert vc.vcErrorString(vc.VCError.NotReady) == "not ready"
    assert vc.vcErrorString(99) == "unknown error"


def _no_gpu():
    import torch
    return not torch.cuda.is_available()


@pytest.mark.skipif(not _no_gpu(), reason="checks the no-device behaviour")
def test_no_device_behaviour(vc):
    # vcGetDeviceCount initialises lazily and reports 0 devices with Success
    # when initialisation fails (reference VCRuntime.cpp:5037-5047).
    assert vc.vcGetDeviceCount() == (vc.VCError.Success, 0)
    assert vc.vcInit() == vc.VCError.InitializationError
    assert vc.vcSetDevice(0) == vc.VCError.InitializationError
    assert vc.vcGetDevice()[0] == vc.VCError.InitializationError
    err, p = vc.vcMalloc(64)
    assert err == vc.VCError.InitializationError and p == 0


def test_kernel_registry_host_logic(vc):
    for name in ["flashAttn", "wmma_gemm", "matmulCoopmat", "matmulTiled", "vadd", "blockReduce",
                 "fillPattern", "matmul",
                 "vc.gemm", "vc.flash_fwd", "vc.vadd", "vc.sum", "vc.vadd_sum",
                 "vc.block_reduce"]:
        err, k = vc.vcGetKernel(name)
        assert err == vc.VCError.Success and k, name
        assert vc.vcReleaseKernel(k) == vc.VCError.Success
        # The reference-style load: a SPIR-V module whose entry names the kernel.
        err, k = vc.vcLoadKernel(spirv_module(name), name)
        assert err == vc.VCError.Success and k, name
        assert vc.vcReleaseKernel(k) == vc.VCError.Success
    # A missing module, one shorter than the 5-word header, or one without the
    # SPIR-V magic is InvalidValue before the entry is looked at
    # (reference lib/Runtime/VCRuntime.cpp:4261-4268).
    assert vc.vcLoadKernel(None, "vadd")[0] == vc.VCError.InvalidValue
    assert vc.vcLoadKernel([], "vadd")[0] == vc.VCError.InvalidValue
    assert vc.vcLoadKernel([0x07230203, 0x00010000, 0, 1], "vadd")[0] == vc.VCError.InvalidValue
    assert vc.vcLoadKernel([0xdeadbeef, 0x00010000, 0, 1, 0], "vadd")[0] == vc.VCError.InvalidValue
    assert vc.vcLoadKernel([0x07230203, 0x00010000, 0, 1, 0], "vadd")[0] == vc.VCError.Success
    # A well-formed module whose entry names no kernel here: InvalidKernel.
    assert vc.vcLoadKernel(spirv_module("noSuchKernel"), "noSuchKernel")[0] == vc.VCError.InvalidKernel
    assert vc.vcLoadKernel(spirv_module("main"), "main")[0] == vc.VCError.InvalidKernel
    assert vc.vcGetKernel("noSuchKernel")[0] == vc.VCError.InvalidKernel
    err, k = vc.vcGetKernel("flashAttn")
    assert vc.vcKernelSetConstant(k, "SEQ", 128) == vc.VCError.Success
    assert vc.vcKernelSetConstant(k, "NOPE", 1) == vc.VCError.InvalidValue
    assert vc.vcKernelSetConstant(k, "SEQ", 0) == vc.VCError.InvalidValue
    vc.vcReleaseKernel(k)


def test_glsl_backend_modules_resolve_by_interface(vc):
    """A GLSL-backend module names its entry "main"; its storage-buffer and
    push-constant member names and types identify the demo kernel."""
    for name, (bufs, push) in GLSL_DEMO_INTERFACES.items():
        err, k = vc.vcLoadKernel(spirv_glsl_module(bufs, push), "main")
        assert err == vc.VCError.Success and k, name
        vc.vcReleaseKernel(k)
    # Another kernel's interface (a renamed parameter, a wrong element type,
    # a missing scalar) is not taken for a demo kernel.
    assert vc.vcLoadKernel(spirv_glsl_module([("x", "f32"), ("b", "f32"), ("c", "f32")],
                                             [("n", "i32")]), "main")[0] == vc.VCError.InvalidKernel
    assert vc.vcLoadKernel(spirv_glsl_module([("a", "i32"), ("b", "f32"), ("c", "f32")],
                                             [("n", "i32")]), "main")[0] == vc.VCError.InvalidKernel
    assert vc.vcLoadKernel(spirv_glsl_module([("a", "f32"), ("b", "f32"), ("c", "f32")], []),
                           "main")[0] == vc.VCError.InvalidKernel
    # A malformed module (a runtime array whose element type is itself, bound
    # as an eighth buffer) is refused, not followed.
    w = spirv_glsl_module(*GLSL_DEMO_INTERFACES["vadd"])
    w += [(3 << 16) | 29, 900, 900, (3 << 16) | 30, 901, 900,
          (4 << 16) | 6, 901, 0, int.from_bytes(b"x\0\0\0", "little"),
          (4 << 16) | 32, 902, 12, 901, (4 << 16) | 59, 902, 903, 12,
          (4 << 16) | 71, 903, 33, 7]
    assert vc.vcLoadKernel(w, "main")[0] == vc.VCError.InvalidKernel
    # Truncated instruction streams end the read, without reading past the end.
    w = spirv_glsl_module(*GLSL_DEMO_INTERFACES["vadd"])
    for cut in range(5, len(w), 7):
        assert vc.vcLoadKernel(w[:cut], "main")[0] in (vc.VCError.InvalidKernel,
                                                      vc.VCError.Success)


def test_glsl_backend_module_identity_is_reported():
    out = subprocess.run(
        [sys.executable, "-c",
         "import sys; sys.path.insert(0, 'tests')\n"
         "from conftest import GLSL_DEMO_INTERFACES, spirv_glsl_module\n"
         "from vkcuda_b200 import vc\n"
         "b, p = GLSL_DEMO_INTERFACES['blockReduce']\n"
         "print(int(vc.vcLoadKernel(spirv_glsl_module(b, p), 'main')[0]))\n"],
        capture_output=True, text=True, cwd=ROOT, env=dict(os.environ, VC_DEBUG="1"), timeout=120)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == "0"
    assert "interface inBuf:f32,outBuf:f32;N:i32 is blockReduce" in out.stderr


def test_load_kernel_from_file(vc, tmp_path):
    # Whole words with the last one zero-padded, as the reference reads a file
    # (VCRuntime.cpp:4378-4387): a 3-byte file is one word, too short.
    import struct
    short = tmp_path / "short.spv"
    short.write_bytes(b"\x03\x02\x23")
    assert vc.vcLoadKernelFromFile(str(short), "vadd")[0] == vc.VCError.InvalidValue
    assert vc.vcLoadKernelFromFile(str(tmp_path / "absent.spv"), "vadd")[0] == vc.VCError.InvalidValue
    good = tmp_path / "vadd.spv"
    good.write_bytes(struct.pack(f"<{len(spirv_module('vadd'))}I", *spirv_module("vadd")))
    err, k = vc.vcLoadKernelFromFile(str(good), "vadd")
    assert err == vc.VCError.Success and k
    vc.vcReleaseKernel(k)


def test_launch_argument_checks(vc):
    # Null kernel -> InvalidKernel; zero block -> InvalidValue (both before
    # any device work, as in the reference wrappers VCRuntime.cpp:5584-5609).
    assert vc.vcLaunchKernel(None, 64, 32, []) == vc.VCError.InvalidKernel
    err, k = vc.vcGetKernel("vadd")
    assert vc.vcLaunchKernel(k, 64, 0, []) == vc.VCError.InvalidValue
    vc.vcReleaseKernel(k)
    assert vc.vcMemcpy(None, None, 4, vc.VCMemcpyKind.HostToDevice) == vc.VCError.InvalidValue
    assert vc.vcMemset(None, 0, 4) == vc.VCError.InvalidValue
    assert vc.vcFree(None) == vc.VCError.Success
    assert vc.vcMemcpy2DAsync(1, 4, 1, 4, 4, 1, vc.VCMemcpyKind.HostToDevice) == vc.VCError.InvalidValue


def _run_child(code: str, env_extra: dict) -> str:
    env = dict(os.environ, **env_extra)
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env,
                         cwd=ROOT, timeout=120)
    assert res.returncode == 0, res.stderr
    return res.stdout.strip()


def test_fault_injection_malloc_and_launch():
    # The 2nd vcMalloc and the 1st launch fail with the injected codes, before
    # any device is touched (host-side failure injection, no GPU needed).
    out = _run_child(
        "from vkcuda_b200 import vc\n"
        "a = int(vc.vcMalloc(16)[0]); b = int(vc.vcMalloc(16)[0]); c = int(vc.vcMalloc(16)[0])\n"
        "k = vc.vcGetKernel('vadd')[1]\n"
        "l1 = int(vc.vcLaunchKernel(k, 64, 32, [])); l2 = int(vc.vcLaunchKernel(k, 64, 32, []))\n"
        "print(a, b, c, l1, l2)\n",
        {"VC_FAULT_INJECT": "malloc:2,launch:1"})
    a, b, c, l1, l2 = (int(x) for x in out.split())
    assert b == 2                      # OutOfMemory injected on call 2
    assert a == c and a in (0, 5)      # real result: Success on a GPU, InitializationError on CPU
    assert l1 == 8                     # Unknown injected on launch 1
    assert l2 != 8


def test_python_mirror_covers_the_api(vc):
    """Every vc:: function of the header has a Python mirror of the same name,
    except the storage-image and printf-layer calls (graphics API, out of
    scope on this runtime)."""
    text = open(os.path.join(ROOT, "include", "vc", "Runtime", "VCRuntime.h")).read()
    names = sorted(set(re.findall(r"^(?:VCError|const char \*)\s*(vc\w+)\(", text, re.M)))
    out_of_scope = {"vcCreateImage1D", "vcCreateImage2D", "vcCreateImage2DArray",
                    "vcCreateImage3D", "vcDestroyImage", "vcMemcpyToImage",
                    "vcMemcpyFromImage", "vcEnableKernelPrintf"}
    missing = [n for n in names if n not in out_of_scope and not hasattr(vc, n)]
    assert not missing, missing
