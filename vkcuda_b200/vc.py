"""Python mirror of the VC runtime API (include/vc/Runtime/VCRuntime.h in
junka/vkcuda), bound with ctypes to the flat C ABI of libVCRuntime.so
(include/vc_b200.h).

Names, argument meaning and error behaviour follow the reference header:
every call returns a ``VCError`` (allocation-style calls return
``(VCError, value)``); nothing raises except a missing library. Device
pointers are plain integers (device addresses). Host buffers may be numpy
arrays, ``bytes``/``bytearray``, ctypes objects or integer addresses.

    from vkcuda_b200 import vc
    vc.vcInit()
    err, d_a = vc.vcMalloc(n * 4)
    vc.vcMemcpy(d_a, host_a, n * 4, vc.VCMemcpyKind.HostToDevice)
    err, k = vc.vcGetKernel("vadd")
    vc.vcLaunchKernel(k, n, 256, [vc.ptr(d_a), vc.ptr(d_b), vc.ptr(d_c), vc.i32(n)])
"""
from __future__ import annotations

import ctypes
import enum
import os
from typing import Iterable, Optional, Sequence, Tuple, Union

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libVCRuntime.so")


class VCError(enum.IntEnum):
    """Reference VCRuntime.h:64-74."""
    Success = 0
    InvalidValue = 1
    OutOfMemory = 2
    InvalidKernel = 3
    InvalidDevice = 4
    InitializationError = 5
    MapFailed = 6
    NotReady = 7
    Unknown = 8


class VCMemcpyKind(enum.IntEnum):
    """Reference VCRuntime.h:77-81."""
    HostToDevice = 0
    DeviceToHost = 1
    DeviceToDevice = 2


class VCMemoryType(enum.IntEnum):
    """Reference VCRuntime.h:308-314."""
    Unregistered = 0
    Device = 1
    Host = 2
    Managed = 3


class Dtype(enum.IntEnum):
    """Element types of the native entries (include/vc_b200.h)."""
    F32 = 0
    F16 = 1
    BF16 = 2


class VCKernelArg(ctypes.Structure):
    """Byte-compatible with vc::VCKernelArg (reference VCRuntime.h:690-694)."""
    POINTER, SCALAR, IMAGE = 0, 1, 2
    _fields_ = [("kind", ctypes.c_int), ("data", ctypes.c_void_p), ("size", ctypes.c_size_t)]


class VCDeviceProperties(ctypes.Structure):
    """Byte-compatible with vc::VCDeviceProperties (reference VCRuntime.h:255-268)."""
    _fields_ = [("name", ctypes.c_char * 256), ("totalGlobalMem", ctypes.c_size_t),
                ("sharedMemPerBlock", ctypes.c_size_t),
                ("sharedMemPerMultiprocessor", ctypes.c_size_t), ("warpSize", ctypes.c_int),
                ("maxThreadsPerBlock", ctypes.c_int), ("maxThreadsDim", ctypes.c_int * 3),
                ("maxGridSize", ctypes.c_int * 3), ("clockRate", ctypes.c_int),
                ("multiProcessorCount", ctypes.c_int), ("major", ctypes.c_int),
                ("minor", ctypes.c_int)]


class VCPointerAttributes(ctypes.Structure):
    """Byte-compatible with vc::VCPointerAttributes (reference VCRuntime.h:321-326)."""
    _fields_ = [("memoryType", ctypes.c_int), ("devicePointer", ctypes.c_void_p),
                ("hostPointer", ctypes.c_void_p), ("size", ctypes.c_size_t)]


class VCRuntimeError(RuntimeError):
    def __init__(self, err: int, what: str = ""):
        self.err = VCError(err) if 0 <= err <= 8 else err
        super().__init__(f"{what}: {vcErrorString(err)} ({err})" if what else vcErrorString(err))


_lib: Optional[ctypes.CDLL] = None

_VP, _SZ, _I, _U, _LL, _I64, _F = (ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_uint,
                                   ctypes.c_longlong, ctypes.c_int64, ctypes.c_float)
_PVP, _PI = ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_int)
HOSTFN = ctypes.CFUNCTYPE(None, ctypes.c_void_p)

# name -> (restype, argtypes); every symbol of include/vc_b200.h.
SIGNATURES = {
    "vc_init": (_I, []), "vc_shutdown": (_I, []),
    "vc_get_device_count": (_I, [_PI]), "vc_get_device": (_I, [_PI]),
    "vc_set_device": (_I, [_I]),
    "vc_get_device_properties": (_I, [ctypes.POINTER(VCDeviceProperties), _I]),
    "vc_occupancy_max_potential_block_size": (_I, [_PI, _PI, _VP, _SZ, _I]),
    "vc_pointer_get_attributes": (_I, [ctypes.POINTER(VCPointerAttributes), _VP]),
    "vc_malloc": (_I, [_PVP, _SZ]), "vc_malloc_host": (_I, [_PVP, _SZ]),
    "vc_malloc_managed": (_I, [_PVP, _SZ]), "vc_free": (_I, [_VP]),
    "vc_malloc_async": (_I, [_PVP, _SZ, _VP]), "vc_free_async": (_I, [_VP, _VP]),
    "vc_memcpy": (_I, [_VP, _VP, _SZ, _I]), "vc_memcpy_s": (_I, [_VP, _VP, _SZ, _I, _VP]),
    "vc_memcpy_async_s": (_I, [_VP, _VP, _SZ, _I, _VP]),
    "vc_memcpy_async": (_I, [_VP, _VP, _SZ, _I]),
    "vc_memcpy_peer": (_I, [_VP, _I, _VP, _I, _SZ]),
    "vc_memcpy_peer_async": (_I, [_VP, _I, _VP, _I, _SZ, _VP]),
    "vc_memset": (_I, [_VP, _I, _SZ]), "vc_memset_async_s": (_I, [_VP, _I, _SZ, _VP]),
    "vc_memcpy_2d_async": (_I, [_VP, _SZ, _VP, _SZ, _SZ, _SZ, _I, _VP]),
    "vc_memset_2d_async": (_I, [_VP, _SZ, _I, _SZ, _SZ, _VP]),
    "vc_device_synchronize": (_I, []), "vc_stream_create": (_I, [_PVP]),
    "vc_stream_destroy": (_I, [_VP]), "vc_stream_synchronize": (_I, [_VP]),
    "vc_stream_query": (_I, [_VP, _PI]), "vc_launch_host_func": (_I, [_VP, HOSTFN, _VP]),
    "vc_event_create": (_I, [_PVP]), "vc_event_destroy": (_I, [_VP]),
    "vc_event_record": (_I, [_VP, _VP]), "vc_stream_wait_event": (_I, [_VP, _VP]),
    "vc_event_query": (_I, [_VP, _PI]), "vc_event_synchronize": (_I, [_VP]),
    "vc_event_elapsed_time": (_I, [ctypes.POINTER(ctypes.c_float), _VP, _VP]),
    "vc_graph_create": (_I, [_PVP]), "vc_graph_destroy": (_I, [_VP]),
    "vc_graph_begin_record": (_I, [_VP]), "vc_graph_end_record": (_I, [_VP]),
    "vc_graph_launch": (_I, [_VP, _VP]), "vc_graph_reset": (_I, [_VP]),
    "vc_load_kernel": (_I, [ctypes.POINTER(ctypes.c_uint32), _SZ, ctypes.c_char_p, _PVP]),
    "vc_load_kernel_from_file": (_I, [ctypes.c_char_p, ctypes.c_char_p, _PVP]),
    "vc_release_kernel": (_I, [_VP]),
    "vc_launch_kernel": (_I, [_VP, _U, _U, ctypes.POINTER(VCKernelArg), _I]),
    "vc_launch_kernel_s": (_I, [_VP, _U, _U, ctypes.POINTER(VCKernelArg), _I, _VP]),
    "vc_launch_kernel_2d_s": (_I, [_VP, _U, _U, _U, _U, ctypes.POINTER(VCKernelArg), _I, _VP]),
    "vc_launch_kernel_indirect_s": (_I, [_VP, _VP, _SZ, _U, _U, _U, ctypes.POINTER(VCKernelArg),
                                         _I, _VP]),
    "vc_error_string": (ctypes.c_char_p, [_I]),
    "vc_get_kernel": (_I, [ctypes.c_char_p, _PVP]),
    "vc_kernel_set_constant": (_I, [_VP, ctypes.c_char_p, _LL]),
    "vc_kernel_error": (_I, [_I]), "vc_selftest_bounded_wait": (_I, [_U]),
    "vc_selftest_bounds_check": (_I, []),
    "vc_vadd_f32": (_I, [_VP, _VP, _VP, _I64, _VP]),
    "vc_sum_f32": (_I, [_VP, _I64, _VP, _VP]),
    "vc_sum_f32_noalloc": (_I, [_VP, _I64, _VP, _VP]),
    "vc_vadd_sum_f32": (_I, [_VP, _VP, _VP, _I64, _VP, _VP]),
    "vc_peer_mailbox_alloc": (_I, [ctypes.POINTER(ctypes.c_void_p)]),
    "vc_peer_mailbox_free": (_I, [_VP]),
    "vc_peer_ipc_get_handle": (_I, [_VP, _VP]),
    "vc_peer_ipc_open": (_I, [_VP, ctypes.POINTER(ctypes.c_void_p)]),
    "vc_peer_ipc_close": (_I, [_VP]),
    "vc_vadd_sum_f32_allreduce": (_I, [_VP, _VP, _VP, _I64, _VP, ctypes.POINTER(ctypes.c_void_p),
                                       _I, _I, ctypes.c_ulonglong, _VP]),
    "vc_block_reduce_f32": (_I, [_VP, _VP, _I, _I, _I, _VP]),
    "vc_gemm": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I, _I64, _I64, _I64, _I64, _I, _I, _VP]),
    "vc_flash_fwd": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I, _F, _I, _I, _VP]),
}


def library() -> ctypes.CDLL:
    """Load libVCRuntime.so (built by ``python -m vkcuda_b200.build``).

    Raises when the library is missing: there is no fallback path."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing; build it with `python -m vkcuda_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def _addr(x) -> Optional[int]:
    """Address of a host or device buffer (int, numpy array, ctypes object, torch tensor)."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "__array_interface__"):
        return x.__array_interface__["data"][0]
    if isinstance(x, (bytearray, memoryview)):
        return ctypes.addressof(ctypes.c_char.from_buffer(x))
    if isinstance(x, bytes):
        return ctypes.cast(ctypes.c_char_p(x), ctypes.c_void_p).value
    return ctypes.addressof(x)


def _stream(s) -> Optional[int]:
    if s is None:
        return None
    if hasattr(s, "cuda_stream"):
        return s.cuda_stream
    return int(s)


def check(err, what: str = "") -> None:
    """Raise VCRuntimeError for a non-Success code (helper, not in the reference)."""
    if int(err) != 0:
        raise VCRuntimeError(int(err), what)


# ------------------------------------------------------------ runtime calls
def vcInit() -> VCError: return VCError(library().vc_init())
def vcShutdown() -> VCError: return VCError(library().vc_shutdown())


def vcGetDeviceCount() -> Tuple[VCError, int]:
    n = ctypes.c_int(0)
    return VCError(library().vc_get_device_count(ctypes.byref(n))), n.value


def vcGetDevice() -> Tuple[VCError, int]:
    n = ctypes.c_int(-1)
    return VCError(library().vc_get_device(ctypes.byref(n))), n.value


def vcSetDevice(device: int) -> VCError: return VCError(library().vc_set_device(device))


def vcGetDeviceProperties(device: int) -> Tuple[VCError, VCDeviceProperties]:
    p = VCDeviceProperties()
    return VCError(library().vc_get_device_properties(ctypes.byref(p), device)), p


def vcOccupancyMaxPotentialBlockSize(kernel, dyn_smem: int = 0, limit: int = 0):
    mg, bs = ctypes.c_int(0), ctypes.c_int(0)
    e = library().vc_occupancy_max_potential_block_size(ctypes.byref(mg), ctypes.byref(bs),
                                                       kernel, dyn_smem, limit)
    return VCError(e), mg.value, bs.value


def vcPointerGetAttributes(ptr) -> Tuple[VCError, VCPointerAttributes]:
    a = VCPointerAttributes()
    return VCError(library().vc_pointer_get_attributes(ctypes.byref(a), _addr(ptr))), a


def _alloc(fn, nbytes: int, *extra) -> Tuple[VCError, int]:
    p = ctypes.c_void_p(0)
    e = fn(ctypes.byref(p), nbytes, *extra)
    return VCError(e), (p.value or 0)


def vcMalloc(nbytes: int): return _alloc(library().vc_malloc, nbytes)
def vcMallocHost(nbytes: int): return _alloc(library().vc_malloc_host, nbytes)
def vcMallocManaged(nbytes: int): return _alloc(library().vc_malloc_managed, nbytes)
def vcMallocAsync(nbytes: int, stream=None): return _alloc(library().vc_malloc_async, nbytes, _stream(stream))
def vcFree(ptr) -> VCError: return VCError(library().vc_free(_addr(ptr)))
def vcFreeAsync(ptr, stream=None) -> VCError: return VCError(library().vc_free_async(_addr(ptr), _stream(stream)))


def vcMemcpy(dst, src, count: int, kind) -> VCError:
    return VCError(library().vc_memcpy(_addr(dst), _addr(src), count, int(kind)))


def vcMemcpyS(dst, src, count: int, kind, stream=None) -> VCError:
    return VCError(library().vc_memcpy_s(_addr(dst), _addr(src), count, int(kind), _stream(stream)))


def vcMemcpyAsyncS(dst, src, count: int, kind, stream=None) -> VCError:
    return VCError(library().vc_memcpy_async_s(_addr(dst), _addr(src), count, int(kind), _stream(stream)))


def vcMemcpyAsync(dst, src, count: int, kind) -> VCError:
    return VCError(library().vc_memcpy_async(_addr(dst), _addr(src), count, int(kind)))


def vcMemcpyPeer(dst, dst_dev: int, src, src_dev: int, count: int) -> VCError:
    return VCError(library().vc_memcpy_peer(_addr(dst), dst_dev, _addr(src), src_dev, count))


def vcMemcpyPeerAsync(dst, dst_dev: int, src, src_dev: int, count: int, stream=None) -> VCError:
    return VCError(library().vc_memcpy_peer_async(_addr(dst), dst_dev, _addr(src), src_dev, count,
                                                  _stream(stream)))


def vcMemset(ptr, value: int, count: int) -> VCError:
    return VCError(library().vc_memset(_addr(ptr), value, count))


def vcMemsetAsyncS(ptr, value: int, count: int, stream=None) -> VCError:
    return VCError(library().vc_memset_async_s(_addr(ptr), value, count, _stream(stream)))


def vcMemsetAsync(ptr, value: int, count: int) -> VCError:
    """Asynchronous fill on the default stream (reference VCRuntime.h:486)."""
    return vcMemsetAsyncS(ptr, value, count, None)


def vcMemsetS(ptr, value: int, count: int, stream=None) -> VCError:
    """Fill on `stream`, then wait for it (reference VCRuntime.h:477)."""
    e = vcMemsetAsyncS(ptr, value, count, stream)
    return e if e != VCError.Success else vcStreamSynchronize(stream)


def vcMemcpy2DAsync(dst, dpitch, src, spitch, width, height, kind, stream=None) -> VCError:
    return VCError(library().vc_memcpy_2d_async(_addr(dst), dpitch, _addr(src), spitch, width,
                                                height, int(kind), _stream(stream)))


def vcMemcpy2DS(dst, dpitch, src, spitch, width, height, kind, stream=None) -> VCError:
    """2D copy on `stream`, then wait for it (reference VCRuntime.h:496)."""
    e = vcMemcpy2DAsync(dst, dpitch, src, spitch, width, height, kind, stream)
    return e if e != VCError.Success else vcStreamSynchronize(stream)


def vcMemcpy2D(dst, dpitch, src, spitch, width, height, kind) -> VCError:
    return vcMemcpy2DS(dst, dpitch, src, spitch, width, height, kind, None)


def vcMemset2DAsync(dst, pitch, value, width, height, stream=None) -> VCError:
    return VCError(library().vc_memset_2d_async(_addr(dst), pitch, value, width, height,
                                                _stream(stream)))


def vcMemset2D(dst, pitch, value, width, height) -> VCError:
    e = vcMemset2DAsync(dst, pitch, value, width, height, None)
    return e if e != VCError.Success else vcStreamSynchronize(None)


def vcMallocHostAsync(nbytes: int, stream=None): return vcMallocHost(nbytes)
def vcMallocManagedS(nbytes: int, stream=None): return vcMallocManaged(nbytes)


def vcDeviceSynchronize() -> VCError: return VCError(library().vc_device_synchronize())


def vcStreamCreate() -> Tuple[VCError, int]:
    return _alloc(lambda p, _n: library().vc_stream_create(p), 0)


def vcStreamDestroy(stream) -> VCError: return VCError(library().vc_stream_destroy(_stream(stream)))
def vcStreamSynchronize(stream=None) -> VCError: return VCError(library().vc_stream_synchronize(_stream(stream)))


def vcStreamQuery(stream=None) -> Tuple[VCError, int]:
    d = ctypes.c_int(0)
    return VCError(library().vc_stream_query(_stream(stream), ctypes.byref(d))), d.value


_hostfn_keepalive = []


def vcLaunchHostFunc(stream, fn, user_data=None) -> VCError:
    """`fn(user_data_address)` runs on a runtime thread once the stream reaches it."""
    cb = HOSTFN(fn)
    _hostfn_keepalive.append(cb)
    return VCError(library().vc_launch_host_func(_stream(stream), cb, _addr(user_data)))


def vcEventCreate() -> Tuple[VCError, int]:
    return _alloc(lambda p, _n: library().vc_event_create(p), 0)


def vcEventDestroy(ev) -> VCError: return VCError(library().vc_event_destroy(ev))
def vcEventRecord(ev, stream=None) -> VCError: return VCError(library().vc_event_record(ev, _stream(stream)))
def vcStreamWaitEvent(stream, ev) -> VCError: return VCError(library().vc_stream_wait_event(_stream(stream), ev))


def vcEventQuery(ev) -> Tuple[VCError, int]:
    d = ctypes.c_int(0)
    return VCError(library().vc_event_query(ev, ctypes.byref(d))), d.value


def vcEventSynchronize(ev) -> VCError: return VCError(library().vc_event_synchronize(ev))


def vcEventElapsedTime(start, end) -> Tuple[VCError, float]:
    ms = ctypes.c_float(0.0)
    return VCError(library().vc_event_elapsed_time(ctypes.byref(ms), start, end)), ms.value


def vcGraphCreate() -> Tuple[VCError, int]:
    return _alloc(lambda p, _n: library().vc_graph_create(p), 0)


def vcGraphDestroy(g) -> VCError: return VCError(library().vc_graph_destroy(g))
def vcGraphBeginRecord(g) -> VCError: return VCError(library().vc_graph_begin_record(g))
def vcGraphEndRecord(g) -> VCError: return VCError(library().vc_graph_end_record(g))
def vcGraphLaunch(g, stream=None) -> VCError: return VCError(library().vc_graph_launch(g, _stream(stream)))
def vcGraphReset(g) -> VCError: return VCError(library().vc_graph_reset(g))


def vcLoadKernel(words, entry: str) -> Tuple[VCError, int]:
    """`words`: a sequence of uint32 SPIR-V words; a missing module, one shorter
    than the 5-word header or without the SPIR-V magic is InvalidValue, as in
    the reference. vcGetKernel resolves a kernel by name without a module."""
    k = ctypes.c_void_p(0)
    if not words:
        e = library().vc_load_kernel(None, 0, entry.encode(), ctypes.byref(k))
    else:
        arr = (ctypes.c_uint32 * len(words))(*words)
        e = library().vc_load_kernel(arr, len(words), entry.encode(), ctypes.byref(k))
    return VCError(e), (k.value or 0)


def vcGetKernel(name: str) -> Tuple[VCError, int]:
    k = ctypes.c_void_p(0)
    return VCError(library().vc_get_kernel(name.encode(), ctypes.byref(k))), (k.value or 0)


def vcKernelSetConstant(kernel, name: str, value: int) -> VCError:
    return VCError(library().vc_kernel_set_constant(kernel, name.encode(), value))


def vcReleaseKernel(kernel) -> VCError: return VCError(library().vc_release_kernel(kernel))


class _Args:
    """A VCKernelArg array plus the scalar storage it points into."""

    def __init__(self, args: Sequence[Tuple[int, object]]):
        self._keep = []
        self.array = (VCKernelArg * max(1, len(args)))()
        self.count = len(args)
        for i, (kind, payload) in enumerate(args):
            if kind == VCKernelArg.POINTER:
                self.array[i] = VCKernelArg(kind, payload, 0)
            else:
                self._keep.append(payload)
                self.array[i] = VCKernelArg(kind, ctypes.addressof(payload), ctypes.sizeof(payload))


def ptr(p) -> Tuple[int, object]: return (VCKernelArg.POINTER, _addr(p))
def i32(v: int) -> Tuple[int, object]: return (VCKernelArg.SCALAR, ctypes.c_int32(int(v)))
def i64(v: int) -> Tuple[int, object]: return (VCKernelArg.SCALAR, ctypes.c_int64(int(v)))
def f32(v: float) -> Tuple[int, object]: return (VCKernelArg.SCALAR, ctypes.c_float(float(v)))


def vcLaunchKernel(kernel, grid: int, block: int, args, stream=None) -> VCError:
    a = _Args(args)
    return VCError(library().vc_launch_kernel_s(kernel, grid, block, a.array, a.count, _stream(stream)))


def vcLaunchKernel2D(kernel, gx: int, gy: int, bx: int, by: int, args, stream=None) -> VCError:
    a = _Args(args)
    return VCError(library().vc_launch_kernel_2d_s(kernel, gx, gy, bx, by, a.array, a.count,
                                                   _stream(stream)))


def vcLaunchKernelIndirect(kernel, indirect_args, offset: int, block, args, stream=None) -> VCError:
    """Workgroup counts {x, y, z} are read from the device buffer at `offset`."""
    bx, by, bz = (tuple(block) + (1, 1))[:3]
    a = _Args(args)
    return VCError(library().vc_launch_kernel_indirect_s(kernel, _addr(indirect_args), offset, bx,
                                                         by, bz, a.array, a.count,
                                                         _stream(stream)))


# Stream-taking forms of the reference header: the functions above already
# take an optional stream (None = the default stream).
vcLaunchKernelS = vcLaunchKernel
vcLaunchKernel2DS = vcLaunchKernel2D
vcLaunchKernelIndirectS = vcLaunchKernelIndirect


def vcLoadKernelFromFile(path: str, entry: str) -> Tuple[VCError, int]:
    """Load a module from a file and resolve `entry` (the library reads the
    file: whole 32-bit words, the last zero-padded)."""
    k = ctypes.c_void_p(0)
    e = library().vc_load_kernel_from_file(path.encode(), entry.encode(), ctypes.byref(k))
    return VCError(e), (k.value or 0)


def vcErrorString(err) -> str:
    return library().vc_error_string(int(err)).decode()


def kernel_error(clear: bool = True) -> int:
    """Sticky device error word of the hot kernels (0 = clean)."""
    return library().vc_kernel_error(1 if clear else 0)


def selftest_bounded_wait(timeout_us: int) -> int:
    return library().vc_selftest_bounded_wait(timeout_us)


def selftest_bounds_check() -> int:
    """Bounds-checked vadd told its output holds 1000 of 1024 elements:
    4 (kErrOutOfBounds) when the device check refused the rest."""
    return library().vc_selftest_bounds_check()


# ------------------------------------------------------------ native entries
def vadd_f32(a, b, c, n: int, stream=None) -> VCError:
    return VCError(library().vc_vadd_f32(_addr(a), _addr(b), _addr(c), n, _stream(stream)))


def sum_f32(x, n: int, out, stream=None) -> VCError:
    return VCError(library().vc_sum_f32(_addr(x), n, _addr(out), _stream(stream)))


def sum_f32_noalloc(x, n: int, out, stream=None) -> VCError:
    """vc_sum_f32 without allocating: block partials in the library's static
    device array (see include/vc_b200.h). Overlapping calls race."""
    return VCError(library().vc_sum_f32_noalloc(_addr(x), n, _addr(out), _stream(stream)))


def vadd_sum_f32(a, b, c, n: int, out, stream=None) -> VCError:
    return VCError(library().vc_vadd_sum_f32(_addr(a), _addr(b), _addr(c), n, _addr(out),
                                             _stream(stream)))


IPC_HANDLE_BYTES = 64


def peer_mailbox_alloc() -> Tuple[VCError, int]:
    """One cross-GPU exchange mailbox in the current device's memory."""
    p = ctypes.c_void_p(0)
    e = VCError(library().vc_peer_mailbox_alloc(ctypes.byref(p)))
    return e, (p.value or 0)


def peer_mailbox_free(mailbox: int) -> VCError:
    return VCError(library().vc_peer_mailbox_free(_addr(mailbox)))


def peer_ipc_get_handle(dev_ptr: int) -> Tuple[VCError, bytes]:
    """CUDA IPC handle (IPC_HANDLE_BYTES bytes) of a device allocation."""
    buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    e = VCError(library().vc_peer_ipc_get_handle(_addr(dev_ptr), buf))
    return e, buf.raw


def peer_ipc_open(handle: bytes) -> Tuple[VCError, int]:
    """Map another process's allocation (from its handle) into this one."""
    if len(handle) != IPC_HANDLE_BYTES:
        return VCError.InvalidValue, 0
    buf = ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES)
    p = ctypes.c_void_p(0)
    e = VCError(library().vc_peer_ipc_open(buf, ctypes.byref(p)))
    return e, (p.value or 0)


def peer_ipc_close(dev_ptr: int) -> VCError:
    return VCError(library().vc_peer_ipc_close(_addr(dev_ptr)))


def vadd_sum_f32_allreduce(a, b, c, n: int, out, mailboxes, rank: int, epoch: int,
                           stream=None) -> VCError:
    """c = a + b; *out = sum over all ranks of sum(c), exchanged through the
    ranks' mailboxes (all of them, in rank order) inside the kernel."""
    arr = (ctypes.c_void_p * len(mailboxes))(*[_addr(m) for m in mailboxes])
    return VCError(library().vc_vadd_sum_f32_allreduce(
        _addr(a), _addr(b), _addr(c), n, _addr(out), arr, rank, len(mailboxes), epoch,
        _stream(stream)))


def block_reduce_f32(inp, out, n: int, block: int, groups: int, stream=None) -> VCError:
    return VCError(library().vc_block_reduce_f32(_addr(inp), _addr(out), n, block, groups,
                                                 _stream(stream)))


def gemm(A, B, D, Cin, M: int, N: int, K: int, lda: int, ldb: int, ldd: int, ldc: int,
         dtype: int = Dtype.F16, b_kn: bool = True, stream=None) -> VCError:
    return VCError(library().vc_gemm(_addr(A), _addr(B), _addr(D), _addr(Cin), M, N, K, lda, ldb,
                                     ldd, ldc, int(dtype), 1 if b_kn else 0, _stream(stream)))


def flash_fwd(Q, K, V, O, BH: int, N: int, d: int, scale_log2: float, causal: bool,
              dtype: int, stream=None) -> VCError:
    return VCError(library().vc_flash_fwd(_addr(Q), _addr(K), _addr(V), _addr(O), BH, N, d,
                                          float(scale_log2), 1 if causal else 0, int(dtype),
                                          _stream(stream)))
