"""The CUDA device as a go-tensor backend.

``CudaBackend`` has the methods of Go's ``backend.Backend`` interface
(internal/backend/backend.go:130-157) with the same names, argument meaning and
error behaviour, implemented on libgotensor_cuda's C interface. It is what a
Go ``internal/cuda`` package does over cgo (the Metal backend's counterpart is
internal/mps/mps.go): storages own a device allocation that returns to the
device's stream-ordered pool when the storage is collected, every result is a
new contiguous storage of the input dtype, and misuse raises.
"""
from __future__ import annotations

import ctypes
import threading
import weakref

import numpy as np

from . import _lib
from ._lib import FLOAT32, FLOAT64, GtGeom, GtView, check

CUDA_TYPE = 1  # backend.CUDA (internal/backend/backend.go:40)
_NP = {FLOAT32: np.float32, FLOAT64: np.float64}


class Device:
    """backend.Device; equal to any device object with the same (type, index)."""
    __slots__ = ("type", "index")

    def __init__(self, type_: int, index: int):
        self.type, self.index = type_, index

    def __eq__(self, o):
        return (getattr(o, "type", None), getattr(o, "index", None)) == (self.type, self.index)

    def __hash__(self):
        return hash((self.type, self.index))

    def __repr__(self):
        return f"cuda:{self.index}"


class Context:
    """One per (process, device): gt_init's stream, pool and communicator."""

    _lock = threading.Lock()
    _by_device: dict = {}

    def __init__(self, index: int):
        self.lib = _lib.cuda_lib()
        ptr = ctypes.c_void_p()
        check(self.lib.gt_init(index, ctypes.byref(ptr)))
        self.ptr = ptr
        self.index = index

    @classmethod
    def get(cls, index: int = 0) -> "Context":
        with cls._lock:
            if index not in cls._by_device:
                cls._by_device[index] = Context(index)
            return cls._by_device[index]

    @property
    def name(self) -> str:
        return self.lib.gt_device_name(self.ptr).decode()

    @property
    def sm_count(self) -> int:
        return self.lib.gt_sm_count(self.ptr)

    def sync(self):
        check(self.lib.gt_sync(self.ptr))

    def alloc(self, nbytes: int) -> int:
        p = ctypes.c_void_p()
        check(self.lib.gt_alloc(self.ptr, nbytes, ctypes.byref(p)))
        return p.value

    def release(self, p: int):
        check(self.lib.gt_release(self.ptr, p))


def _release(ctx: Context, p: int):
    try:
        ctx.lib.gt_release(ctx.ptr, p)
    except Exception:  # interpreter shutdown
        pass


class CudaStorage:
    """backend.Storage: ``n`` contiguous elements of one dtype on one GPU."""
    __slots__ = ("ctx", "ptr", "n", "dt", "device", "__weakref__")

    def __init__(self, ctx: Context, n: int, dt: int):
        self.ctx, self.n, self.dt = ctx, n, dt
        self.device = Device(CUDA_TYPE, ctx.index)
        self.ptr = ctx.alloc(max(n, 1) * (8 if dt == FLOAT64 else 4))
        weakref.finalize(self, _release, ctx, self.ptr)

    def dtype(self) -> int:
        return self.dt

    def __len__(self):
        return self.n

    @property
    def nbytes(self) -> int:
        return self.n * (8 if self.dt == FLOAT64 else 4)


def _view(v) -> GtView:
    if isinstance(v, GtView):
        return v
    out = GtView()
    out.ndim, out.offset = v.ndim, v.offset
    for d in range(v.ndim):
        out.shape[d], out.strides[d] = v.shape[d], v.strides[d]
    return out


def _geom(g) -> GtGeom:
    if isinstance(g, GtGeom):
        return g
    out = GtGeom()
    for f, _ in GtGeom._fields_:
        setattr(out, f, getattr(g, f))
    return out


def _numel(v) -> int:
    n = 1
    for d in range(v.ndim):
        n *= v.shape[d]
    return n


class CudaBackend:
    """backend.Backend for tensor.CUDA(index)."""

    def __init__(self, index: int = 0):
        self.ctx = Context.get(index)
        self.lib = self.ctx.lib

    def device(self) -> Device:
        return Device(CUDA_TYPE, self.ctx.index)

    def _own(self, s) -> CudaStorage:
        if not isinstance(s, CudaStorage) or s.ctx is not self.ctx:
            raise TypeError(f"cuda: storage {type(s).__name__} is not on {self.device()}")
        return s

    def _same_dtype(self, *ss):
        for s in ss[1:]:
            if s.dt != ss[0].dt:
                raise TypeError("cuda: mixed dtypes")

    # -- memory
    def Zeros(self, dt: int, n: int) -> CudaStorage:
        s = CudaStorage(self.ctx, n, dt)
        check(self.lib.gt_zero(self.ctx.ptr, s.ptr, s.nbytes))
        return s

    def FromHost(self, data: np.ndarray) -> CudaStorage:
        if data.dtype == np.float32:
            dt = FLOAT32
        elif data.dtype == np.float64:
            dt = FLOAT64
        else:
            raise TypeError(f"cuda: FromHost({data.dtype})")
        data = np.ascontiguousarray(data).reshape(-1)
        s = CudaStorage(self.ctx, data.size, dt)
        check(self.lib.gt_upload(self.ctx.ptr, s.ptr, data.ctypes.data, s.nbytes))
        return s

    def ToHost(self, s) -> np.ndarray:
        s = self._own(s)
        out = np.empty(s.n, dtype=_NP[s.dt])
        check(self.lib.gt_download(self.ctx.ptr, out.ctypes.data, s.ptr, s.nbytes))
        return out

    def Cast(self, s, dt: int) -> CudaStorage:
        s = self._own(s)
        out = CudaStorage(self.ctx, s.n, dt)
        check(self.lib.gt_cast(self.ctx.ptr, s.ptr, s.dt, out.ptr, dt, s.n))
        return out

    def Write(self, dst, offset: int, src) -> None:
        dst, src = self._own(dst), self._own(src)
        self._same_dtype(dst, src)
        if offset < 0 or offset + src.n > dst.n:
            raise IndexError(f"cuda: Write of {src.n} elements at {offset} into {dst.n}")
        es = 8 if dst.dt == FLOAT64 else 4
        check(self.lib.gt_write(self.ctx.ptr, dst.ptr, offset * es, src.ptr, src.nbytes))

    def Sync(self) -> None:
        self.ctx.sync()

    # -- element-wise
    def Unary(self, op: int, scalar: float, x) -> CudaStorage:
        x = self._own(x)
        out = CudaStorage(self.ctx, x.n, x.dt)
        check(self.lib.gt_unary(self.ctx.ptr, x.dt, op, float(scalar), x.ptr, out.ptr, x.n))
        return out

    def Binary(self, op: int, a, av, b, bv) -> CudaStorage:
        a, b = self._own(a), self._own(b)
        self._same_dtype(a, b)
        va, vb = _view(av), _view(bv)
        out = CudaStorage(self.ctx, _numel(va), a.dt)
        check(self.lib.gt_binary(self.ctx.ptr, a.dt, op, a.ptr, ctypes.byref(va), b.ptr, ctypes.byref(vb), out.ptr))
        return out

    def Copy(self, src, v) -> CudaStorage:
        src = self._own(src)
        vv = _view(v)
        out = CudaStorage(self.ctx, _numel(vv), src.dt)
        check(self.lib.gt_copy(self.ctx.ptr, src.dt, src.ptr, ctypes.byref(vv), out.ptr))
        return out

    # -- reductions and linear algebra
    def Reduce(self, op: int, x, outer: int, n: int, inner: int) -> CudaStorage:
        x = self._own(x)
        out = CudaStorage(self.ctx, outer * inner, x.dt)
        check(self.lib.gt_reduce(self.ctx.ptr, x.dt, op, x.ptr, out.ptr, outer, n, inner))
        return out

    def MatMul(self, a, b, m: int, k: int, n: int, transA: bool, transB: bool) -> CudaStorage:
        a, b = self._own(a), self._own(b)
        self._same_dtype(a, b)
        out = CudaStorage(self.ctx, m * n, a.dt)
        check(self.lib.gt_matmul(self.ctx.ptr, a.dt, a.ptr, b.ptr, out.ptr, m, k, n, int(transA), int(transB)))
        return out

    # -- convolution helpers
    def Im2col(self, x, g) -> CudaStorage:
        x, gg = self._own(x), _geom(g)
        out = CudaStorage(self.ctx, gg.N * gg.OH * gg.OW * gg.C * gg.KH * gg.KW, x.dt)
        check(self.lib.gt_im2col(self.ctx.ptr, x.dt, x.ptr, out.ptr, ctypes.byref(gg)))
        return out

    def Col2im(self, cols, g) -> CudaStorage:
        cols, gg = self._own(cols), _geom(g)
        out = CudaStorage(self.ctx, gg.N * gg.C * gg.H * gg.W, cols.dt)
        check(self.lib.gt_col2im(self.ctx.ptr, cols.dt, cols.ptr, out.ptr, ctypes.byref(gg)))
        return out

    def MaxPool2d(self, x, g) -> CudaStorage:
        x, gg = self._own(x), _geom(g)
        out = CudaStorage(self.ctx, gg.N * gg.C * gg.OH * gg.OW, x.dt)
        check(self.lib.gt_maxpool_fwd(self.ctx.ptr, x.dt, x.ptr, out.ptr, ctypes.byref(gg)))
        return out

    def MaxPool2dBackward(self, x, grad, g) -> CudaStorage:
        x, grad, gg = self._own(x), self._own(grad), _geom(g)
        out = CudaStorage(self.ctx, gg.N * gg.C * gg.H * gg.W, x.dt)
        check(self.lib.gt_maxpool_bwd(self.ctx.ptr, x.dt, x.ptr, grad.ptr, out.ptr, ctypes.byref(gg)))
        return out
