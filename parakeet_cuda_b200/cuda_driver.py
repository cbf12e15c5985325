"""CUDA driver API through ctypes: device memory, streams, events, pinned host
memory and stream-captured graphs, with no PyTorch.

The reference drives CUDA the same way (``parakeet_cuda/cuda_driver.py:29-118``:
``libcuda.so.1`` through ctypes, the device's primary context made current,
every nonzero ``CUresult`` raised as ``RuntimeError("{fn}: {name}: {text}
(CUDA n)")``). libpq8.so is built on the CUDA runtime, which uses the same
primary context, so the pointers and stream handles made here are the ones
its entry points take (a ``CUstream`` is a ``cudaStream_t``).

Nothing is loaded at import time: ``Driver(index)`` opens ``libcuda.so.1``.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

_P, _I, _U, _SZ, _U64 = C.c_void_p, C.c_int, C.c_uint, C.c_size_t, C.c_uint64

# CUstreamCaptureMode: capture only this thread's work into the graph
CAPTURE_THREAD_LOCAL = 1
STREAM_NON_BLOCKING = 1
EVENT_DEFAULT, EVENT_DISABLE_TIMING = 0, 2
HOST_ALLOC_PORTABLE = 1
ATTR_CC_MAJOR, ATTR_CC_MINOR, ATTR_SM_COUNT = 75, 76, 16

SIGNATURES = {
    'cuInit': [_U],
    'cuDriverGetVersion': [C.POINTER(_I)],
    'cuDeviceGetCount': [C.POINTER(_I)],
    'cuDeviceGet': [C.POINTER(_I), _I],
    'cuDeviceGetName': [C.c_char_p, _I, _I],
    'cuDeviceGetAttribute': [C.POINTER(_I), _I, _I],
    'cuDevicePrimaryCtxRetain': [C.POINTER(_P), _I],
    'cuDevicePrimaryCtxRelease_v2': [_I],
    'cuCtxSetCurrent': [_P],
    'cuCtxGetCurrent': [C.POINTER(_P)],
    'cuCtxSynchronize': [],
    'cuMemGetInfo_v2': [C.POINTER(_SZ), C.POINTER(_SZ)],
    'cuMemAlloc_v2': [C.POINTER(_U64), _SZ],
    'cuMemFree_v2': [_U64],
    'cuMemHostAlloc': [C.POINTER(_P), _SZ, _U],
    'cuMemFreeHost': [_P],
    'cuMemcpyHtoDAsync_v2': [_U64, _P, _SZ, _P],
    'cuMemcpyDtoHAsync_v2': [_P, _U64, _SZ, _P],
    'cuMemcpyDtoDAsync_v2': [_U64, _U64, _SZ, _P],
    'cuMemsetD8Async': [_U64, C.c_ubyte, _SZ, _P],
    'cuStreamCreate': [C.POINTER(_P), _U],
    'cuStreamDestroy_v2': [_P],
    'cuStreamSynchronize': [_P],
    'cuStreamWaitEvent': [_P, _P, _U],
    'cuEventCreate': [C.POINTER(_P), _U],
    'cuEventRecord': [_P, _P],
    'cuEventSynchronize': [_P],
    'cuEventElapsedTime': [C.POINTER(C.c_float), _P, _P],
    'cuEventDestroy_v2': [_P],
    'cuStreamBeginCapture_v2': [_P, _I],
    'cuStreamEndCapture': [_P, C.POINTER(_P)],
    'cuGraphInstantiateWithFlags': [C.POINTER(_P), _P, C.c_ulonglong],
    'cuGraphLaunch': [_P, _P],
    'cuGraphExecDestroy': [_P],
    'cuGraphDestroy': [_P],
    'cuModuleLoad': [C.POINTER(_P), C.c_char_p],
    'cuModuleUnload': [_P],
    'cuModuleGetFunction': [C.POINTER(_P), _P, C.c_char_p],
    'cuLaunchKernel': [_P, _U, _U, _U, _U, _U, _U, _U, _P, C.POINTER(_P), _P],
    'cuGetErrorName': [_I, C.POINTER(C.c_char_p)],
    'cuGetErrorString': [_I, C.POINTER(C.c_char_p)],
}


class CudaError(RuntimeError):
    def __init__(self, name: str, status: int, error: str, message: str):
        super().__init__(f'{name}: {error}: {message} (CUDA {status})')
        self.name, self.status = name, status


class Driver:
    """``libcuda.so.1`` with the primary context of device ``index`` made current
    on the calling thread (``cuda_driver.py:29-88`` of the reference)."""

    def __init__(self, index: int = 0, path: str = 'libcuda.so.1'):
        self.lib = C.CDLL(path)
        for name, args in SIGNATURES.items():
            fn = getattr(self.lib, name)
            fn.argtypes, fn.restype = args, _I
        self.call('cuInit', 0)
        self.index = index
        self.device = _I()
        self.call('cuDeviceGet', C.byref(self.device), index)
        self.context = _P()
        self.call('cuDevicePrimaryCtxRetain', C.byref(self.context), self.device)
        self.make_current()

    def call(self, name: str, *args) -> None:
        status = getattr(self.lib, name)(*args)
        if status:
            err, msg = C.c_char_p(), C.c_char_p()
            self.lib.cuGetErrorName(status, C.byref(err))
            self.lib.cuGetErrorString(status, C.byref(msg))
            raise CudaError(name, status, (err.value or b'?').decode(), (msg.value or b'?').decode())

    def make_current(self) -> None:
        self.call('cuCtxSetCurrent', self.context)

    def attribute(self, attr: int) -> int:
        v = _I()
        self.call('cuDeviceGetAttribute', C.byref(v), attr, self.device)
        return v.value

    def info(self) -> dict:
        name = C.create_string_buffer(256)
        self.call('cuDeviceGetName', name, len(name), self.device)
        return {'name': name.value.decode(), 'sm': self.attribute(ATTR_CC_MAJOR) * 10 + self.attribute(ATTR_CC_MINOR),
                'sms': self.attribute(ATTR_SM_COUNT)}

    def synchronize(self) -> None:
        self.call('cuCtxSynchronize')

    def mem_info(self) -> tuple[int, int]:
        free, total = _SZ(), _SZ()
        self.call('cuMemGetInfo_v2', C.byref(free), C.byref(total))
        return free.value, total.value

    # -- memory --------------------------------------------------------------
    def alloc(self, nbytes: int) -> int:
        p = _U64()
        self.call('cuMemAlloc_v2', C.byref(p), max(int(nbytes), 1))
        return p.value

    def free(self, pointer: int) -> None:
        self.call('cuMemFree_v2', pointer)

    def alloc_host(self, nbytes: int) -> int:
        """Page-locked host memory (for asynchronous copies)."""
        p = _P()
        self.call('cuMemHostAlloc', C.byref(p), max(int(nbytes), 1), HOST_ALLOC_PORTABLE)
        return p.value

    def free_host(self, pointer: int) -> None:
        self.call('cuMemFreeHost', pointer)

    def h2d(self, dst: int, src: int, nbytes: int, stream) -> None:
        self.call('cuMemcpyHtoDAsync_v2', dst, src, nbytes, _handle(stream))

    def d2h(self, dst: int, src: int, nbytes: int, stream) -> None:
        self.call('cuMemcpyDtoHAsync_v2', dst, src, nbytes, _handle(stream))

    def d2d(self, dst: int, src: int, nbytes: int, stream) -> None:
        self.call('cuMemcpyDtoDAsync_v2', dst, src, nbytes, _handle(stream))

    def memset(self, dst: int, value: int, nbytes: int, stream) -> None:
        self.call('cuMemsetD8Async', dst, value, nbytes, _handle(stream))

    # -- streams, events, graphs ----------------------------------------------
    def stream(self) -> 'Stream':
        return Stream(self)

    def event(self, timing: bool = True) -> 'Event':
        return Event(self, timing)


def _handle(obj):
    return obj.handle if hasattr(obj, 'handle') else obj


class Stream:
    def __init__(self, drv: Driver):
        self.drv = drv
        h = _P()
        drv.call('cuStreamCreate', C.byref(h), STREAM_NON_BLOCKING)
        self.handle = h

    def synchronize(self) -> None:
        self.drv.call('cuStreamSynchronize', self.handle)

    def wait(self, event: 'Event') -> None:
        self.drv.call('cuStreamWaitEvent', self.handle, event.handle, 0)

    def capture(self, enqueue) -> 'Graph':
        """Record the work ``enqueue()`` puts on this stream as a graph, ready to launch."""
        self.drv.call('cuStreamBeginCapture_v2', self.handle, CAPTURE_THREAD_LOCAL)
        graph = _P()
        try:
            enqueue()
        finally:
            self.drv.call('cuStreamEndCapture', self.handle, C.byref(graph))
        return Graph(self.drv, graph)

    def close(self) -> None:
        if self.handle:
            self.drv.call('cuStreamDestroy_v2', self.handle)
            self.handle = _P()


class Event:
    def __init__(self, drv: Driver, timing: bool = True):
        self.drv = drv
        h = _P()
        drv.call('cuEventCreate', C.byref(h), EVENT_DEFAULT if timing else EVENT_DISABLE_TIMING)
        self.handle = h

    def record(self, stream) -> 'Event':
        self.drv.call('cuEventRecord', self.handle, _handle(stream))
        return self

    def synchronize(self) -> None:
        self.drv.call('cuEventSynchronize', self.handle)

    def elapsed_ms(self, end: 'Event') -> float:
        ms = C.c_float()
        self.drv.call('cuEventElapsedTime', C.byref(ms), self.handle, end.handle)
        return ms.value

    def close(self) -> None:
        if self.handle:
            self.drv.call('cuEventDestroy_v2', self.handle)
            self.handle = _P()


class Graph:
    """An instantiated stream capture; ``launch(stream)`` replays it."""

    def __init__(self, drv: Driver, graph: C.c_void_p):
        self.drv, self.graph = drv, graph
        ex = _P()
        drv.call('cuGraphInstantiateWithFlags', C.byref(ex), graph, 0)
        self.exec = ex

    def launch(self, stream) -> None:
        self.drv.call('cuGraphLaunch', self.exec, _handle(stream))

    def close(self) -> None:
        if self.exec:
            self.drv.call('cuGraphExecDestroy', self.exec)
            self.exec = _P()
        if self.graph:
            self.drv.call('cuGraphDestroy', self.graph)
            self.graph = _P()


class PinnedArray:
    """A NumPy array over page-locked host memory (``cuMemHostAlloc``)."""

    def __init__(self, drv: Driver, shape, dtype=np.float32):
        self.drv = drv
        self.shape = (shape,) if isinstance(shape, int) else tuple(shape)
        self.dtype = np.dtype(dtype)
        self.nbytes = int(np.prod(self.shape)) * self.dtype.itemsize
        self.pointer = drv.alloc_host(self.nbytes)
        raw = (C.c_ubyte * self.nbytes).from_address(self.pointer)
        self.array = np.frombuffer(raw, np.uint8).view(self.dtype).reshape(self.shape)

    def close(self) -> None:
        if self.pointer:
            self.array = None
            self.drv.free_host(self.pointer)
            self.pointer = 0
