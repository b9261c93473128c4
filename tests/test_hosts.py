"""Compiled C++ host programs link against libVCRuntime unchanged.

tests/hosts/*.cpp are host programs in the form the VC compiler's host
emitter writes (lib/Codegen/ASTToHost.cpp:238-248, 406-428, 1261-1318 in the
reference): the vc:: runtime header, `using namespace vc`, an embedded SPIR-V
module per kernel, `vcLoadKernel(words, len, "<entry>", &handle)` and a
`VCKernelArg[]` launch. They bind the C++ API by its mangled names and struct
layouts, as generated code does. On CPU each is compiled and linked (every
vc:: symbol it names must resolve); on a GPU each runs and must print the
demo's own PASS line (test/vadd.vc, test/reduce.vc, examples/flash_attn.vc,
test/multigpu.vc, examples/matmul_coopmat_bench.vc)."""
from __future__ import annotations

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOSTS = os.path.join(ROOT, "tests", "hosts")
PROGRAMS = {
    "vadd_host": "vector_add: PASS",
    "block_reduce_host": "block_reduce: PASS",
    "flash_attn_host": "flash_attn: PASS",
    "multigpu_host": "multigpu: PASS",
    "matmul_coopmat_host": "matmul_coopmat_bench: PASS",
}


def _gxx():
    for cand in ("/usr/bin/g++", shutil.which("g++")):
        if cand and os.path.exists(cand):
            return cand
    pytest.skip("no g++")


def _build(vc, orc, name: str, outdir: str) -> str:
    libdir = os.path.dirname(vc.LIB_PATH)
    oracle_dir = os.path.dirname(orc.LIB_PATH)
    exe = os.path.join(outdir, name)
    cmd = [_gxx(), "-std=c++20", "-O2", "-fno-rtti", "-I", os.path.join(ROOT, "include"),
           os.path.join(HOSTS, name + ".cpp"), "-o", exe,
           "-L", libdir, "-lVCRuntime", f"-Wl,-rpath,{libdir}",
           "-L", oracle_dir, "-l:" + os.path.basename(orc.LIB_PATH), f"-Wl,-rpath,{oracle_dir}",
           "-Wl,--no-undefined"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    return exe


@pytest.mark.parametrize("name", sorted(PROGRAMS))
def test_host_program_compiles_and_links(vc, orc, name, tmp_path):
    _build(vc, orc, name, str(tmp_path))


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(PROGRAMS))
def test_host_program_runs_on_gpu(gpu, orc, name, tmp_path):
    exe = _build(gpu, orc, name, str(tmp_path))
    res = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    assert PROGRAMS[name] in res.stdout, res.stdout
