"""Runtime API semantics on the GPU, mirroring the reference's runtime demos
(test/event.vc, test/profiling.vc, test/stream_query.vc, test/graph.vc,
test/multigpu.vc): allocation registry, blocking vs async copies, memset
rules, streams, events and elapsed time, graph record/replay, host callbacks,
peer copies, and the bounded-wait failure path."""
from __future__ import annotations

import ctypes
import subprocess
import threading

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_device_properties(gpu):
    err, n = gpu.vcGetDeviceCount()
    assert err == 0 and n >= 1
    err, p = gpu.vcGetDeviceProperties(0)
    assert err == 0
    assert p.multiProcessorCount >= 100 and p.warpSize == 32 and p.major >= 10
    assert gpu.vcGetDeviceProperties(n)[0] == gpu.VCError.InvalidDevice
    assert gpu.vcSetDevice(n) == gpu.VCError.InvalidDevice
    assert gpu.vcGetDevice() == (gpu.VCError.Success, 0)


def test_pointer_attributes_and_free(gpu):
    err, d = gpu.vcMalloc(4096)
    err2, h = gpu.vcMallocHost(1024)
    assert err == 0 and err2 == 0
    e, a = gpu.vcPointerGetAttributes(d)
    assert e == 0 and a.memoryType == gpu.VCMemoryType.Device and a.size == 4096
    e, a = gpu.vcPointerGetAttributes(d + 100)  # interior pointer
    assert a.memoryType == gpu.VCMemoryType.Device and a.devicePointer == d
    e, a = gpu.vcPointerGetAttributes(h)
    assert a.memoryType == gpu.VCMemoryType.Host and a.hostPointer == h
    stack = ctypes.c_int(0)
    e, a = gpu.vcPointerGetAttributes(ctypes.addressof(stack))
    assert a.memoryType == gpu.VCMemoryType.Unregistered and a.size == 0
    assert gpu.vcFree(d) == 0 and gpu.vcFree(h) == 0
    e, a = gpu.vcPointerGetAttributes(d)
    assert a.memoryType == gpu.VCMemoryType.Unregistered
    assert gpu.vcFree(d) == gpu.VCError.InvalidValue  # no longer a VC allocation


def test_copies_and_memset(gpu, dev):
    x = np.arange(1024, dtype=np.int32)
    d1, d2 = dev.put(x), dev.alloc(4096)
    assert gpu.vcMemcpy(d2.ptr, d1.ptr, 4096, gpu.VCMemcpyKind.DeviceToDevice) == 0
    assert np.array_equal(d2.to_host(np.int32, 1024), x)
    assert gpu.vcMemset(d2.ptr, 0x01, 4096) == 0
    assert (d2.to_host(np.int32, 1024) == 0x01010101).all()
    assert gpu.vcMemset(d2.ptr, 0, 6) == gpu.VCError.InvalidValue       # count % 4
    assert gpu.vcMemset(d2.ptr, 0, 8192) == gpu.VCError.InvalidValue    # past the allocation
    # 2D pitched copy: 4 rows of 16 bytes from pitch 64 to pitch 32.
    assert gpu.vcMemcpy2DAsync(d2.ptr, 32, d1.ptr, 64, 16, 4, gpu.VCMemcpyKind.DeviceToDevice) == 0
    gpu.vcStreamSynchronize(None)
    got = d2.to_host(np.int32, 32).reshape(4, 8)[:, :4]
    assert np.array_equal(got, x.reshape(-1, 16)[:4, :4])
    assert gpu.vcMemset2DAsync(d2.ptr, 32, 0, 16, 4) == 0
    gpu.vcStreamSynchronize(None)
    assert (d2.to_host(np.int32, 32).reshape(4, 8)[:, :4] == 0).all()


def test_async_copy_stream_and_events(gpu, dev):
    n = 1 << 22
    x = np.random.default_rng(0).random(n, dtype=np.float32)
    err, hbuf = gpu.vcMallocHost(x.nbytes)
    ctypes.memmove(hbuf, x.ctypes.data, x.nbytes)
    d = dev.alloc(x.nbytes)
    err, s = gpu.vcStreamCreate()
    err, e0 = gpu.vcEventCreate()
    err, e1 = gpu.vcEventCreate()
    # Elapsed time of never-recorded events is InvalidValue (reference contract).
    assert gpu.vcEventElapsedTime(e0, e1)[0] == gpu.VCError.InvalidValue
    assert gpu.vcEventRecord(e0, s) == 0
    assert gpu.vcMemcpyAsyncS(d.ptr, hbuf, x.nbytes, gpu.VCMemcpyKind.HostToDevice, s) == 0
    assert gpu.vcEventRecord(e1, s) == 0
    assert gpu.vcEventSynchronize(e1) == 0
    err, done = gpu.vcEventQuery(e1)
    assert err == 0 and done == 1
    err, ms = gpu.vcEventElapsedTime(e0, e1)
    assert err == 0 and ms > 0.0
    err, done = gpu.vcStreamQuery(s)
    assert done == 1
    # Cross-stream dependency: default stream waits on e1 before reading.
    assert gpu.vcStreamWaitEvent(None, e1) == 0
    assert np.array_equal(d.to_host(np.float32, n), x)
    for e in (e0, e1):
        gpu.vcEventDestroy(e)
    gpu.vcStreamDestroy(s)
    gpu.vcFree(hbuf)


def test_graph_record_replay(gpu, dev, orc):
    n = 100_000
    rng = np.random.default_rng(4)
    a = rng.random(n, dtype=np.float32)
    b = rng.random(n, dtype=np.float32)
    da, db, dc = dev.put(a), dev.put(b), dev.alloc(4 * n)
    err, k = gpu.vcGetKernel("vadd")
    err, g = gpu.vcGraphCreate()
    assert gpu.vcGraphBeginRecord(g) == 0
    assert gpu.vcLaunchKernel(k, n, 256, [gpu.ptr(da.ptr), gpu.ptr(db.ptr), gpu.ptr(dc.ptr),
                                          gpu.i32(n)]) == 0
    # The recorded launch reads c back into a: a <- a + b on every replay.
    assert gpu.vcMemcpyAsync(da.ptr, dc.ptr, 4 * n, gpu.VCMemcpyKind.DeviceToDevice) == 0
    assert gpu.vcGraphEndRecord(g) == 0
    ref = a.copy()
    for _ in range(3):
        assert gpu.vcGraphLaunch(g, None) == 0
        ref = orc.vadd(ref, b)
    assert gpu.vcStreamSynchronize(None) == 0
    assert np.array_equal(da.to_host(np.float32, n), ref)
    assert gpu.vcGraphReset(g) == 0
    assert gpu.vcGraphLaunch(g, None) == gpu.VCError.InvalidValue  # reset graphs are empty
    gpu.vcGraphDestroy(g)
    gpu.vcReleaseKernel(k)


def test_host_func_runs_after_stream_work(gpu, dev):
    fired = threading.Event()
    seen = []

    def cb(_user):
        seen.append(1)
        fired.set()

    d = dev.alloc(1 << 20)
    assert gpu.vcMemsetAsyncS(d.ptr, 0, 1 << 20, None) == 0
    assert gpu.vcLaunchHostFunc(None, cb) == 0
    assert fired.wait(10.0) and seen == [1]


def test_peer_copy_same_device(gpu, dev):
    """test/multigpu.vc degrades to a 0 -> 0 peer copy on one device."""
    x = 1000 + np.arange(1024, dtype=np.int32)
    src, dst = dev.put(x), dev.alloc(4096)
    assert gpu.vcMemcpyPeer(dst.ptr, 0, src.ptr, 0, 4096) == 0
    assert np.array_equal(dst.to_host(np.int32, 1024), x)
    err, n = gpu.vcGetDeviceCount()
    assert gpu.vcMemcpyPeer(dst.ptr, n, src.ptr, 0, 4096) == gpu.VCError.InvalidDevice
    assert gpu.vcMemcpyPeer(dst.ptr, 0, src.ptr, 0, 8192) == gpu.VCError.InvalidValue


def test_bounded_wait_reports_timeout_and_context_survives(gpu, dev, orc):
    # A device wait on a barrier nothing arrives on gives up after ~2 ms and
    # reports its code (3); the context stays usable afterwards.
    assert gpu.selftest_bounded_wait(2000) == 3
    a = np.ones(1000, np.float32)
    da, dc = dev.put(a), dev.alloc(4000)
    assert gpu.vadd_f32(da.ptr, da.ptr, dc.ptr, 1000) == 0
    assert gpu.vcDeviceSynchronize() == 0
    assert (dc.to_host(np.float32, 1000) == 2.0).all()
    assert gpu.kernel_error(True) == 0


def test_indirect_launch_reads_workgroups_from_device(gpu, dev, orc):
    """vcLaunchKernelIndirect: the workgroup counts {x, y, z} come from a device
    buffer at a byte offset (reference VCRuntime.h:722-740)."""
    n = 4096
    rng = np.random.default_rng(8)
    a = rng.random(n, dtype=np.float32)
    b = rng.random(n, dtype=np.float32)
    da, db, dc = dev.put(a), dev.put(b), dev.alloc(4 * n)
    # {x, y, z} = {n/256 - 4, 1, 1} at byte offset 8: the last 4 workgroups
    # (1024 elements) are not launched and keep their zeros.
    ind = dev.put(np.array([7, 7, n // 256 - 4, 1, 1], np.uint32))
    assert gpu.vcMemset(dc.ptr, 0, 4 * n) == 0
    err, k = gpu.vcGetKernel("vadd")
    args = [gpu.ptr(da.ptr), gpu.ptr(db.ptr), gpu.ptr(dc.ptr), gpu.i32(n)]
    assert gpu.vcLaunchKernelIndirect(k, ind.ptr, 8, (256, 1, 1), args) == 0
    assert gpu.vcDeviceSynchronize() == 0
    got = dc.to_host(np.float32, n)
    assert np.array_equal(got[:n - 1024], orc.vadd(a, b)[:n - 1024])
    assert not got[n - 1024:].any()
    # Counts past the end of the buffer are refused.
    assert gpu.vcLaunchKernelIndirect(k, ind.ptr, 16, (256, 1, 1), args) == gpu.VCError.InvalidValue
    gpu.vcReleaseKernel(k)


def _child(code: str, env: dict) -> subprocess.CompletedProcess:
    import os
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    return subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                          env=dict(os.environ, **env), cwd=root, timeout=300)


def test_profile_table_at_shutdown(gpu):
    """VC_PROFILE=1: per-op GPU spans summarised at vcShutdown (reference
    VCRuntime.cpp:1976-2078)."""
    r = _child("from vkcuda_b200 import vc\n"
               "import numpy as np\n"
               "assert vc.vcInit() == 0\n"
               "e, d = vc.vcMalloc(1 << 20)\n"
               "x = np.ones(1 << 18, np.float32)\n"
               "assert vc.vcMemcpy(d, x, x.nbytes, vc.VCMemcpyKind.HostToDevice) == 0\n"
               "e, k = vc.vcGetKernel('vadd')\n"
               "assert vc.vcLaunchKernel(k, 1 << 18, 256, [vc.ptr(d), vc.ptr(d), vc.ptr(d), vc.i32(1 << 18)]) == 0\n"
               "assert vc.vcDeviceSynchronize() == 0\n"
               "assert vc.vcShutdown() == 0\n", {"VC_PROFILE": "1"})
    assert r.returncode == 0, r.stderr
    assert "vc profile:" in r.stderr and "vadd" in r.stderr and "memcpy H2D" in r.stderr


def test_sync_timeout_returns_not_ready(gpu):
    """VC_SYNC_TIMEOUT_MS bounds host waits: a deadline shorter than the queued
    work returns NotReady (the work completes afterwards)."""
    r = _child("from vkcuda_b200 import vc\n"
               "assert vc.vcInit() == 0\n"
               "n = 1 << 28\n"
               "e, a = vc.vcMalloc(4 * n); e, c = vc.vcMalloc(4 * n)\n"
               "assert vc.vcMemsetAsync(a, 0, 4 * n) == 0\n"
               "for _ in range(40):\n"
               "    assert vc.vadd_f32(a, a, c, n) == 0\n"
               "r1 = int(vc.vcStreamSynchronize(None))\n"
               "import time\n"
               "for _ in range(2000):\n"
               "    if int(vc.vcStreamSynchronize(None)) == 0: break\n"
               "    time.sleep(0.005)\n"
               "r2 = int(vc.vcStreamSynchronize(None))\n"
               "print(r1, r2)\n", {"VC_SYNC_TIMEOUT_MS": "1"})
    assert r.returncode == 0, r.stderr
    r1, r2 = (int(x) for x in r.stdout.split())
    assert r1 == int(gpu.VCError.NotReady) and r2 == 0


def test_multigpu_demo_semantics(gpu, dev):
    """test/multigpu.vc on two devices: pattern 1000+i on device 0, peer copy
    0 -> 1, a launch on device 1 writes 2000+i, and a device-1 buffer is freed
    while device 0 is current. Skipped with one device (the reference then
    degrades to a 0 -> 0 copy, covered above)."""
    err, n = gpu.vcGetDeviceCount()
    if n < 2:
        pytest.skip("needs two devices")
    count = 1024
    pat = (1000 + np.arange(count)).astype(np.float32)
    src = dev.put(pat)                                       # on device 0
    assert gpu.vcSetDevice(1) == 0
    err, dst = gpu.vcMalloc(4 * count)
    err, two = gpu.vcMalloc(4 * count)
    assert gpu.vcMemcpyPeer(dst, 1, src.ptr, 0, 4 * count) == 0
    back = np.empty(count, np.float32)
    assert gpu.vcMemcpy(back, dst, 4 * count, gpu.VCMemcpyKind.DeviceToHost) == 0
    assert np.array_equal(back, pat)
    ones = np.full(count, 1000.0, np.float32)
    assert gpu.vcMemcpy(two, ones, 4 * count, gpu.VCMemcpyKind.HostToDevice) == 0
    assert gpu.vadd_f32(dst, two, dst, count) == 0             # launch on device 1
    assert gpu.vcDeviceSynchronize() == 0
    assert gpu.vcMemcpy(back, dst, 4 * count, gpu.VCMemcpyKind.DeviceToHost) == 0
    assert np.array_equal(back, (2000 + np.arange(count)).astype(np.float32))
    assert gpu.vcSetDevice(0) == 0
    assert gpu.vcFree(dst) == 0 and gpu.vcFree(two) == 0      # device-1 buffers, device 0 current


def test_poison_fill_outputs(gpu):
    """VC_POISON=1 (the NaN-canary debug aid that stands in for an
    initialisation checker): every launch first fills the region its kernel's
    contract says it writes with 0xFF bytes, so a skipped element would read
    back NaN. Kernels that write their whole output give unchanged results;
    an in-place call (output sharing memory with an input) is not poisoned."""
    r = _child("from vkcuda_b200 import vc\n"
               "import numpy as np\n"
               "assert vc.vcInit() == 0\n"
               "n = 1000\n"
               "a = np.arange(n, dtype=np.float32); b = np.full(n, 2.0, np.float32)\n"
               "e, da = vc.vcMalloc(4 * n); e, db = vc.vcMalloc(4 * n); e, dc = vc.vcMalloc(4 * n)\n"
               "assert vc.vcMemcpy(da, a, 4 * n, vc.VCMemcpyKind.HostToDevice) == 0\n"
               "assert vc.vcMemcpy(db, b, 4 * n, vc.VCMemcpyKind.HostToDevice) == 0\n"
               "e, k = vc.vcGetKernel('vadd')\n"
               "assert vc.vcLaunchKernel(k, n, 32, [vc.ptr(da), vc.ptr(db), vc.ptr(dc), vc.i32(n)]) == 0\n"
               "c = np.empty(n, np.float32)\n"
               "assert vc.vcMemcpy(c, dc, 4 * n, vc.VCMemcpyKind.DeviceToHost) == 0\n"
               "assert np.array_equal(c, a + b)\n"
               "import sys; print('INPLACE', file=sys.stderr, flush=True)\n"
               "assert vc.vcLaunchKernel(k, n, 32, [vc.ptr(da), vc.ptr(db), vc.ptr(da), vc.i32(n)]) == 0\n"
               "assert vc.vcMemcpy(c, da, 4 * n, vc.VCMemcpyKind.DeviceToHost) == 0\n"
               "assert np.array_equal(c, a + b)\n"
               "print('GEMM', file=sys.stderr, flush=True)\n"
               "M = N = K = 256\n"
               "A = (np.arange(M * K) % 7).astype(np.float16); B = (np.arange(K * N) % 5).astype(np.float16)\n"
               "e, dA = vc.vcMalloc(2 * M * K); e, dB = vc.vcMalloc(2 * K * N); e, dD = vc.vcMalloc(4 * M * N)\n"
               "assert vc.vcMemcpy(dA, A, A.nbytes, vc.VCMemcpyKind.HostToDevice) == 0\n"
               "assert vc.vcMemcpy(dB, B, B.nbytes, vc.VCMemcpyKind.HostToDevice) == 0\n"
               "assert vc.gemm(dA, dB, dD, None, M, N, K, K, N, N, 0, vc.Dtype.F16, True) == 0\n"
               "D = np.empty(M * N, np.float32)\n"
               "assert vc.vcMemcpy(D, dD, D.nbytes, vc.VCMemcpyKind.DeviceToHost) == 0\n"
               "ref = A.astype(np.float64).reshape(M, K) @ B.astype(np.float64).reshape(K, N)\n"
               "assert np.array_equal(D.reshape(M, N), ref)\n"
               "assert vc.vcShutdown() == 0\n",
               {"VC_POISON": "1", "VC_DEBUG": "1"})
    assert r.returncode == 0, r.stderr
    before, _, rest = r.stderr.partition("INPLACE")
    inplace, _, gemm = rest.partition("GEMM")
    assert "vc: poison vadd output" in before
    assert "vc: poison vadd output" not in inplace      # c shares memory with a
    assert "vc: poison vc.gemm output" in gemm and "256 x 1024 bytes" in gemm


def test_bounds_check_selftest(gpu):
    """The bounds-checked vadd (what VC_CHECK_BOUNDS=1 selects), told its
    output holds 1000 of the 1024 elements it is given (all of them real
    memory), refuses indices 1000..1023 on the device: error word 4, the
    first 1000 written, the rest untouched; the context stays usable."""
    assert gpu.selftest_bounds_check() == 4
    assert gpu.kernel_error(True) == 0


def test_check_bounds_env_runs_checked_forms(gpu):
    """VC_CHECK_BOUNDS=1: vadd, fillPattern and blockReduce (registry launches)
    and the native vadd / block-reduce entries run their bounds-checked forms
    with in-range launches: exact results, a clean error word, and each launch
    named in the VC_DEBUG log."""
    r = _child("from vkcuda_b200 import vc\n"
               "import numpy as np\n"
               "assert vc.vcInit() == 0\n"
               "n = 1000\n"
               "a = np.arange(n, dtype=np.float32); b = np.full(n, 2.0, np.float32)\n"
               "e, da = vc.vcMalloc(4 * n); e, db = vc.vcMalloc(4 * n); e, dc = vc.vcMalloc(4 * n)\n"
               "assert vc.vcMemcpy(da, a, 4 * n, vc.VCMemcpyKind.HostToDevice) == 0\n"
               "assert vc.vcMemcpy(db, b, 4 * n, vc.VCMemcpyKind.HostToDevice) == 0\n"
               "e, k = vc.vcGetKernel('vadd')\n"
               "assert vc.vcLaunchKernel(k, n, 32, [vc.ptr(da), vc.ptr(db), vc.ptr(dc), vc.i32(n)]) == 0\n"
               "c = np.empty(n, np.float32)\n"
               "assert vc.vcMemcpy(c, dc, 4 * n, vc.VCMemcpyKind.DeviceToHost) == 0\n"
               "assert np.array_equal(c, a + b)\n"
               "assert vc.vadd_f32(da, db, dc, n) == 0 and vc.vcDeviceSynchronize() == 0\n"
               "assert vc.vcMemcpy(c, dc, 4 * n, vc.VCMemcpyKind.DeviceToHost) == 0\n"
               "assert np.array_equal(c, a + b)\n"
               "e, k = vc.vcGetKernel('fillPattern')\n"
               "assert vc.vcLaunchKernel(k, n, 32, [vc.ptr(dc), vc.i32(7), vc.i32(n)]) == 0\n"
               "ci = np.empty(n, np.int32)\n"
               "assert vc.vcMemcpy(ci, dc, 4 * n, vc.VCMemcpyKind.DeviceToHost) == 0\n"
               "assert np.array_equal(ci, 7 + np.arange(n, dtype=np.int32))\n"
               "e, k = vc.vcGetKernel('blockReduce')\n"
               "N, block = 1024, 32\n"
               "x = np.arange(N, dtype=np.float32)\n"
               "e, dx = vc.vcMalloc(4 * N); e, do = vc.vcMalloc(4 * (N // block))\n"
               "assert vc.vcMemcpy(dx, x, 4 * N, vc.VCMemcpyKind.HostToDevice) == 0\n"
               "assert vc.vcLaunchKernel(k, N, block, [vc.ptr(dx), vc.ptr(do), vc.i32(N)]) == 0\n"
               "out = np.empty(N // block, np.float32)\n"
               "assert vc.vcMemcpy(out, do, out.nbytes, vc.VCMemcpyKind.DeviceToHost) == 0\n"
               "assert np.array_equal(out, x.reshape(-1, block).sum(axis=1))\n"
               "assert vc.block_reduce_f32(dx, do, N, block, N // block) == 0\n"
               "assert vc.vcDeviceSynchronize() == 0\n"
               "assert vc.vcMemcpy(out, do, out.nbytes, vc.VCMemcpyKind.DeviceToHost) == 0\n"
               "assert np.array_equal(out, x.reshape(-1, block).sum(axis=1))\n"
               "assert vc.kernel_error(True) == 0\n"
               "assert vc.vcShutdown() == 0\n",
               {"VC_CHECK_BOUNDS": "1", "VC_DEBUG": "1"})
    assert r.returncode == 0, r.stderr
    for name in ("vadd", "vc_vadd_f32", "fillPattern", "blockReduce", "vc_block_reduce_f32"):
        assert f"vc: bounds-checked {name} launch" in r.stderr, name


def test_glsl_backend_modules_launch(gpu, dev):
    """Modules shaped like the GLSL backend's (entry "main") resolve by their
    interface and run the demo kernels: vadd (test/vadd.vc) and blockReduce
    (test/reduce.vc) with the demos' own launches and exact checks."""
    from conftest import GLSL_DEMO_INTERFACES, spirv_glsl_module
    n = 64
    a = np.arange(n, dtype=np.float32)
    b = np.full(n, 2.0, np.float32)
    da, db, dc = dev.put(a), dev.put(b), dev.alloc(4 * n)
    err, k = gpu.vcLoadKernel(spirv_glsl_module(*GLSL_DEMO_INTERFACES["vadd"]), "main")
    assert err == gpu.VCError.Success
    assert gpu.vcLaunchKernel(k, n, 32, [gpu.ptr(da.ptr), gpu.ptr(db.ptr), gpu.ptr(dc.ptr),
                                         gpu.i32(n)]) == 0
    assert gpu.vcDeviceSynchronize() == 0
    assert np.array_equal(dc.to_host(np.float32, n), a + b)
    gpu.vcReleaseKernel(k)
    N, block = 128, 32
    x = np.arange(N, dtype=np.float32)
    dx, dout = dev.put(x), dev.alloc(4 * (N // block))
    err, k = gpu.vcLoadKernel(spirv_glsl_module(*GLSL_DEMO_INTERFACES["blockReduce"]), "main")
    assert err == gpu.VCError.Success
    assert gpu.vcLaunchKernel(k, N, block, [gpu.ptr(dx.ptr), gpu.ptr(dout.ptr), gpu.i32(N)]) == 0
    assert gpu.vcDeviceSynchronize() == 0
    expect = x.reshape(-1, block).sum(axis=1)
    assert np.array_equal(dout.to_host(np.float32, N // block), expect)
    gpu.vcReleaseKernel(k)

