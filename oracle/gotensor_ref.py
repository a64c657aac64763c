"""ORACLE — test infrastructure, not part of the product.

A restatement of go-tensor's ``tensor`` package (the layer above the
``backend.Backend`` interface) plus the CPU backend binding:

* ``CPUBackend`` binds ``liboracle_cpu.so``, the C restatement of
  ``internal/cpu`` (cpu.go, linalg.go);
* ``Tensor`` restates ``tensor/tensor.go`` (storage + shape + autograd node),
  ``tensor/autograd.go`` (tape, ``Backward``, ``NoGrad``), ``tensor/ops.go``
  (every op with its backward closure, broadcasting, ``sumTo``/``expand``) and
  ``tensor/conv.go`` (``Conv2d`` = im2col -> MatMul -> permute -> +bias,
  ``MaxPool2d``);
* the device registry of ``tensor/device.go`` so a test can register a second
  backend (a GPU) and run the same ops on both, as the reference's device
  parity tests do (``tensor/device_mps_test.go:35-66``).

Method names follow the Go API (``Add``, ``MatMul``, ``Backward``...) so that
tests read like the reference's own. Random values come from this repo's
seeded NumPy generator (the Go ``math/rand`` stream is not reproduced); like
the reference (``tensor/creation.go:74-94``) they are drawn as float64 on the
host and rounded to the tensor's dtype on upload.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from contextlib import contextmanager

import numpy as np

# ---------------------------------------------------------------------------
# internal/backend/backend.go:10-125

Float32, Float64 = 0, 1
CPU_TYPE, CUDA_TYPE, MPS_TYPE = 0, 1, 2
MAX_DIMS = 8

NEG, EXP, LOG, SQRT, ABS, RELU, SIGMOID, TANH, SIGN, STEP, ADD_SCALAR, MUL_SCALAR, POW = range(13)
ADD, SUB, MUL, DIV = range(4)
SUM, MAX = range(2)

_NP = {Float32: np.float32, Float64: np.float64}


def dtype_of(arr_dtype) -> int:
    return Float64 if np.dtype(arr_dtype) == np.float64 else Float32


class Device:
    __slots__ = ("type", "index")

    def __init__(self, type_: int, index: int = 0):
        self.type, self.index = type_, index

    def __eq__(self, o):
        return (getattr(o, "type", None), getattr(o, "index", None)) == (self.type, self.index)

    def __hash__(self):
        return hash((self.type, self.index))

    def __repr__(self):
        return {CPU_TYPE: "cpu", MPS_TYPE: "mps"}.get(self.type, f"cuda:{self.index}")


CPU = Device(CPU_TYPE)
MPS = Device(MPS_TYPE)


def CUDA(index: int) -> Device:
    return Device(CUDA_TYPE, index)


class View(ctypes.Structure):
    """backend.View (backend.go:113-117); same memory layout as gt_view."""
    _fields_ = [("ndim", ctypes.c_int32), ("_pad", ctypes.c_int32), ("offset", ctypes.c_int64),
                ("shape", ctypes.c_int64 * MAX_DIMS), ("strides", ctypes.c_int64 * MAX_DIMS)]


def make_view(shape, strides, offset=0) -> View:
    if len(shape) > MAX_DIMS:
        raise ValueError(f"at most {MAX_DIMS} dimensions are supported")
    v = View()
    v.ndim, v.offset = len(shape), offset
    for d, (s, st) in enumerate(zip(shape, strides)):
        v.shape[d], v.strides[d] = s, st
    return v


class ConvGeom(ctypes.Structure):
    """backend.ConvGeom (backend.go:120-125); same memory layout as gt_geom."""
    _fields_ = [(f, ctypes.c_int64) for f in ("N", "C", "H", "W", "KH", "KW", "OH", "OW", "stride", "pad")]


def contiguous_strides(shape):
    st, s = [0] * len(shape), 1
    for i in range(len(shape) - 1, -1, -1):
        st[i] = s
        s *= shape[i]
    return st


def numel(shape) -> int:
    n = 1
    for d in shape:
        n *= d
    return n


# ---------------------------------------------------------------------------
# CPU backend: binds the C restatement of internal/cpu.

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle_cpu.so")
_lib = None
_lib_lock = threading.Lock()


def load_library() -> ctypes.CDLL:
    global _lib
    with _lib_lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                subprocess.run(["make", "-s", "-C", _HERE], check=True)
            _lib = ctypes.CDLL(_LIB_PATH)
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


class CPUStorage:
    """backend.Storage for the CPU: a flat contiguous NumPy array."""
    __slots__ = ("data",)
    device = CPU

    def __init__(self, data: np.ndarray):
        self.data = data

    def dtype(self) -> int:
        return dtype_of(self.data.dtype)

    def __len__(self):
        return self.data.shape[0]


class CPUBackend:
    """backend.Backend over the C restatement (internal/cpu/cpu.go:26-296,
    internal/cpu/linalg.go). ``threads`` stands in for runtime.GOMAXPROCS."""

    def __init__(self, threads: int | None = None):
        self.lib = load_library()
        self.threads = threads or os.cpu_count() or 1

    def device(self):
        return CPU

    def _fn(self, name, dt):
        return getattr(self.lib, f"oc_{name}_{'f64' if dt == Float64 else 'f32'}")

    def Zeros(self, dt, n):
        return CPUStorage(np.zeros(n, dtype=_NP[dt]))

    def FromHost(self, data: np.ndarray):
        if data.dtype not in (np.float32, np.float64):
            raise TypeError(f"cpu: FromHost({data.dtype})")
        return CPUStorage(np.array(data, copy=True).reshape(-1))

    def ToHost(self, s):
        return s.data.copy()

    def Cast(self, s, dt):
        return CPUStorage(s.data.astype(_NP[dt]))

    def Write(self, dst, offset, src):
        dst.data[offset:offset + len(src)] = src.data

    def Sync(self):
        pass

    def Unary(self, op, scalar, x):
        out = np.empty_like(x.data)
        self._fn("unary", x.dtype())(ctypes.c_int(op), ctypes.c_double(scalar), _ptr(x.data), _ptr(out),
                                     ctypes.c_int64(out.size))
        return CPUStorage(out)

    def Binary(self, op, a, av: View, b, bv: View):
        out = np.empty(numel(av.shape[:av.ndim]), dtype=a.data.dtype)
        self._fn("binary", a.dtype())(ctypes.c_int(op), _ptr(a.data), ctypes.byref(av), _ptr(b.data),
                                      ctypes.byref(bv), _ptr(out))
        return CPUStorage(out)

    def Copy(self, src, v: View):
        out = np.empty(numel(v.shape[:v.ndim]), dtype=src.data.dtype)
        self._fn("copy", src.dtype())(_ptr(src.data), ctypes.byref(v), _ptr(out))
        return CPUStorage(out)

    def Reduce(self, op, x, outer, n, inner):
        out = np.empty(outer * inner, dtype=x.data.dtype)
        self._fn("reduce", x.dtype())(ctypes.c_int(op), _ptr(x.data), _ptr(out), ctypes.c_int64(outer),
                                      ctypes.c_int64(n), ctypes.c_int64(inner))
        return CPUStorage(out)

    def MatMul(self, a, b, m, k, n, transA, transB):
        out = np.empty(m * n, dtype=a.data.dtype)
        self._fn("matmul", a.dtype())(_ptr(a.data), _ptr(b.data), _ptr(out), ctypes.c_int64(m),
                                      ctypes.c_int64(k), ctypes.c_int64(n), ctypes.c_int(int(transA)),
                                      ctypes.c_int(int(transB)), ctypes.c_int(self.threads))
        return CPUStorage(out)

    def Im2col(self, x, g: ConvGeom):
        out = np.empty(g.N * g.OH * g.OW * g.C * g.KH * g.KW, dtype=x.data.dtype)
        self._fn("im2col", x.dtype())(_ptr(x.data), _ptr(out), ctypes.byref(g))
        return CPUStorage(out)

    def Col2im(self, cols, g: ConvGeom):
        out = np.empty(g.N * g.C * g.H * g.W, dtype=cols.data.dtype)
        self._fn("col2im", cols.dtype())(_ptr(cols.data), _ptr(out), ctypes.byref(g))
        return CPUStorage(out)

    def MaxPool2d(self, x, g: ConvGeom):
        out = np.empty(g.N * g.C * g.OH * g.OW, dtype=x.data.dtype)
        self._fn("maxpool", x.dtype())(_ptr(x.data), None, _ptr(out), ctypes.byref(g))
        return CPUStorage(out)

    def MaxPool2dBackward(self, x, grad, g: ConvGeom):
        out = np.empty(g.N * g.C * g.H * g.W, dtype=x.data.dtype)
        self._fn("maxpool", x.dtype())(_ptr(x.data), _ptr(grad.data), _ptr(out), ctypes.byref(g))
        return CPUStorage(out)


# ---------------------------------------------------------------------------
# tensor/device.go:157-215 — backend registry, lazily instantiated per device.

_registry_lock = threading.Lock()
_factories = {CPU_TYPE: lambda index: CPUBackend()}
_backends: dict = {}
_init_errs: dict = {}


def register_backend(device_type: int, factory) -> None:
    with _registry_lock:
        _factories[device_type] = factory
        for d in [d for d in _backends if d.type == device_type]:
            del _backends[d]
        for d in [d for d in _init_errs if d.type == device_type]:
            del _init_errs[d]


def backend_for(d: Device):
    with _registry_lock:
        if d in _backends:
            return _backends[d]
        if d in _init_errs:
            raise _init_errs[d]
        f = _factories.get(d.type)
        if f is None:
            raise RuntimeError(f"tensor: {d} support is not compiled in")
        try:
            b = f(d.index)
        except Exception as e:  # cached like tensor/device.go:187-192
            err = RuntimeError(f"tensor: {d} is unavailable: {e}")
            _init_errs[d] = err
            raise err
        _backends[d] = b
        return b


def IsAvailable(d: Device) -> bool:
    try:
        backend_for(d)
        return True
    except RuntimeError:
        return False


def Synchronize(d: Device) -> None:
    backend_for(d).Sync()


_default_dtype = Float32
_default_device = CPU


def SetDefaultDType(dt: int) -> None:
    global _default_dtype
    _default_dtype = dt


def DefaultDType() -> int:
    return _default_dtype


# ---------------------------------------------------------------------------
# tensor/creation.go — seeded host RNG (NumPy PCG64 stands in for math/rand).

_rng = np.random.default_rng(0)


def ManualSeed(seed: int) -> None:
    global _rng
    _rng = np.random.default_rng(seed)


def rng() -> np.random.Generator:
    return _rng


# ---------------------------------------------------------------------------
# tensor/autograd.go:10-18 — NoGrad is process-wide, like the reference.

_grad_disabled = False


@contextmanager
def no_grad():
    global _grad_disabled
    prev, _grad_disabled = _grad_disabled, True
    try:
        yield
    finally:
        _grad_disabled = prev


def NoGrad(fn) -> None:
    with no_grad():
        fn()


def IsGradEnabled() -> bool:
    return not _grad_disabled


class _Node:
    __slots__ = ("op", "inputs", "backward")

    def __init__(self, op, inputs, backward):
        self.op, self.inputs, self.backward = op, inputs, backward


def _from_storage(st, shape) -> "Tensor":
    return Tensor(st, list(shape))


def _new_result(st, shape, op, inputs, backward) -> "Tensor":
    """tensor/autograd.go:44-57"""
    out = _from_storage(st, shape)
    if not IsGradEnabled():
        return out
    for inp in inputs:
        if inp.requires_grad:
            out.requires_grad = True
            out.ctx = _Node(op, inputs, backward)
            break
    return out


def _check_same(op, *ts):
    """tensor/tensor.go:322-332"""
    for o in ts[1:]:
        if o.Device() != ts[0].Device():
            raise ValueError(f"tensor: {op}: expected all tensors on the same device, got {ts[0].Device()} and {o.Device()}")
        if o.DType() != ts[0].DType():
            raise ValueError(f"tensor: {op}: expected all tensors to have the same dtype")


def _contiguous_view(shape, offset=0) -> View:
    return make_view(shape, contiguous_strides(shape), offset)


def _from_host(data: np.ndarray, shape, dt, dev) -> "Tensor":
    """tensor/tensor.go:63-76: float64 host data rounded to dt, then uploaded."""
    b = backend_for(dev)
    host = np.asarray(data, dtype=np.float64).reshape(-1).astype(_NP[dt])
    return _from_storage(b.FromHost(host), shape)


class Tensor:
    """tensor/tensor.go:17-25"""
    __slots__ = ("st", "shape", "requires_grad", "grad", "ctx", "__weakref__")

    def __init__(self, st, shape):
        self.st, self.shape = st, list(shape)
        self.requires_grad, self.grad, self.ctx = False, None, None

    # -- basic properties (tensor/tensor.go:84-137)
    def be(self):
        return backend_for(self.st.device)

    def Shape(self):
        return list(self.shape)

    def Dim(self):
        return len(self.shape)

    def Numel(self):
        return len(self.st)

    def DType(self):
        return self.st.dtype()

    def Device(self):
        return self.st.device

    def Float64s(self) -> np.ndarray:
        return np.asarray(self.be().ToHost(self.st), dtype=np.float64)

    def Float32s(self) -> np.ndarray:
        return np.asarray(self.be().ToHost(self.st), dtype=np.float32)

    def Item(self) -> float:
        if self.Numel() != 1:
            raise ValueError(f"tensor: Item requires a single element, got shape {self.shape}")
        return float(self.Float64s()[0])

    def At(self, *idx) -> float:
        off = 0
        for d, i in enumerate(idx):
            off = off * self.shape[d] + i
        one = self.be().Copy(self.st, make_view([1], [1], off))
        return float(_from_storage(one, []).Float64s()[0])

    # -- device / dtype movement (tensor/tensor.go:155-216)
    def To(self, d: Device) -> "Tensor":
        if self.Device() == d:
            return self
        dst = backend_for(d)
        src = self.Device()
        return _new_result(dst.FromHost(self.be().ToHost(self.st)), self.shape, "To", [self],
                           lambda g: [g.To(src)])

    def ToDType(self, dt: int) -> "Tensor":
        if self.DType() == dt:
            return self
        src = self.DType()
        return _new_result(self.be().Cast(self.st, dt), self.shape, "ToDType", [self],
                           lambda g: [g.ToDType(src)])

    def MoveTo(self, d: Device) -> None:
        if self.ctx is not None:
            raise ValueError("tensor: MoveTo can only be called on leaf tensors")
        self.st = self.Detach().To(d).st
        if self.grad is not None:
            self.grad = self.grad.To(d)

    def CastTo(self, dt: int) -> None:
        if self.ctx is not None:
            raise ValueError("tensor: CastTo can only be called on leaf tensors")
        self.st = self.Detach().ToDType(dt).st
        if self.grad is not None:
            self.grad = self.grad.ToDType(dt)

    def CopyFrom(self, src: "Tensor") -> None:
        if src.Numel() != self.Numel():
            raise ValueError(f"tensor: CopyFrom shape {src.shape} into {self.shape}")
        src = src.Detach().ToDType(self.DType()).To(self.Device())
        self.be().Write(self.st, 0, src.st)

    def RequiresGrad(self):
        return self.requires_grad

    def SetRequiresGrad(self, b: bool) -> "Tensor":
        if self.ctx is not None:
            raise ValueError("tensor: SetRequiresGrad can only be called on leaf tensors")
        self.requires_grad = b
        return self

    def IsLeaf(self):
        return self.ctx is None

    def Grad(self):
        return self.grad

    def ZeroGrad(self):
        self.grad = None

    def Detach(self) -> "Tensor":
        return _from_storage(self.st, self.shape)

    def Clone(self) -> "Tensor":
        return _from_storage(self.be().Copy(self.st, _contiguous_view(self.shape)), self.shape)

    # -- autograd (tensor/autograd.go:59-134)
    def Backward(self, grad: "Tensor | None" = None) -> None:
        if not self.requires_grad:
            raise ValueError("tensor: Backward called on a tensor that does not require grad")
        if grad is not None:
            if list(grad.shape) != list(self.shape):
                raise ValueError("tensor: Backward grad shape does not match output shape")
            seed = grad
        else:
            if self.Numel() != 1:
                raise ValueError("tensor: grad can be implicitly created only for scalar outputs")
            seed = OnesLike(self)
        order = _topo_sort(self)
        grads = {id(self): seed}
        with no_grad():
            for v in reversed(order):
                g = grads.pop(id(v), None)
                if g is None:
                    continue
                if v.ctx is None:
                    v.grad = g.Clone() if v.grad is None else v.grad.Add(g)
                    continue
                in_grads = v.ctx.backward(g)
                for j, inp in enumerate(v.ctx.inputs):
                    if not inp.requires_grad or in_grads[j] is None:
                        continue
                    acc = grads.get(id(inp))
                    grads[id(inp)] = in_grads[j] if acc is None else acc.Add(in_grads[j])

    # -- element-wise binary ops (tensor/ops.go:13-50)
    def _binary(self, name, op, o, backward):
        _check_same(name, self, o)
        shape = _broadcast_shapes(self.shape, o.shape)
        av = make_view(shape, _broadcast_strides(self.shape, shape))
        bv = make_view(shape, _broadcast_strides(o.shape, shape))
        return _new_result(self.be().Binary(op, self.st, av, o.st, bv), shape, name, [self, o], backward)

    def Add(self, o):
        return self._binary("Add", ADD, o, lambda g: [_sum_to(g, self.shape), _sum_to(g, o.shape)])

    def Sub(self, o):
        return self._binary("Sub", SUB, o, lambda g: [_sum_to(g, self.shape), _sum_to(g.Neg(), o.shape)])

    def Mul(self, o):
        return self._binary("Mul", MUL, o, lambda g: [_sum_to(g.Mul(o), self.shape), _sum_to(g.Mul(self), o.shape)])

    def Div(self, o):
        def bw(g):
            gt = g.Div(o)
            return [_sum_to(gt, self.shape), _sum_to(gt.Mul(self).Div(o).Neg(), o.shape)]
        return self._binary("Div", DIV, o, bw)

    # -- element-wise unary ops (tensor/ops.go:52-125)
    def _unary(self, name, op, s, backward):
        st = self.be().Unary(op, s, self.st)
        y = _from_storage(st, self.shape)
        return _new_result(st, self.shape, name, [self], lambda g: [backward(g, y)])

    def _raw(self, op, s):
        return _from_storage(self.be().Unary(op, s, self.st), self.shape)

    def Neg(self):
        return self._unary("Neg", NEG, 0.0, lambda g, _: g.Neg())

    def AddScalar(self, s):
        return self._unary("AddScalar", ADD_SCALAR, s, lambda g, _: g)

    def MulScalar(self, s):
        return self._unary("MulScalar", MUL_SCALAR, s, lambda g, _: g.MulScalar(s))

    def Pow(self, p):
        return self._unary("Pow", POW, p, lambda g, _: g.Mul(self.Pow(p - 1).MulScalar(p)))

    def Exp(self):
        return self._unary("Exp", EXP, 0.0, lambda g, y: g.Mul(y))

    def Log(self):
        return self._unary("Log", LOG, 0.0, lambda g, _: g.Div(self))

    def Sqrt(self):
        return self._unary("Sqrt", SQRT, 0.0, lambda g, y: g.Div(y).MulScalar(0.5))

    def Abs(self):
        return self._unary("Abs", ABS, 0.0, lambda g, _: g.Mul(self._raw(SIGN, 0.0)))

    def ReLU(self):
        return self._unary("ReLU", RELU, 0.0, lambda g, _: g.Mul(self._raw(STEP, 0.0)))

    def Sigmoid(self):
        return self._unary("Sigmoid", SIGMOID, 0.0, lambda g, y: g.Mul(y.Mul(y.Neg().AddScalar(1))))

    def Tanh(self):
        return self._unary("Tanh", TANH, 0.0, lambda g, y: g.Mul(y.Mul(y).Neg().AddScalar(1)))

    # -- reductions (tensor/ops.go:127-192)
    def _reduce(self, op, dim, keep):
        dim = _norm_dim(dim, len(self.shape))
        st = self.be().Reduce(op, self.st, numel(self.shape[:dim]), self.shape[dim], numel(self.shape[dim + 1:]))
        return _from_storage(st, _reduced_shape(self.shape, dim, keep))

    def Sum(self):
        st = self.be().Reduce(SUM, self.st, 1, self.Numel(), 1)
        return _new_result(st, [], "Sum", [self], lambda g: [_expand(g, self.shape)])

    def Mean(self):
        return self.Sum().MulScalar(1.0 / float(self.Numel()))

    def SumDim(self, dim, keep):
        dim = _norm_dim(dim, len(self.shape))
        r = self._reduce(SUM, dim, keep)
        kept = _reduced_shape(self.shape, dim, True)
        return _new_result(r.st, r.shape, "SumDim", [self],
                           lambda g: [_expand(_from_storage(g.st, kept), self.shape)])

    def MeanDim(self, dim, keep):
        n = self.shape[_norm_dim(dim, len(self.shape))]
        return self.SumDim(dim, keep).MulScalar(1.0 / float(n))

    def MaxDim(self, dim, keep):
        return self._reduce(MAX, dim, keep)

    def Argmax(self):
        vals = self.Float64s()
        n = self.shape[-1]
        rows = len(vals) // n
        idx = []
        for r in range(rows):
            row, best = vals[r * n:(r + 1) * n], 0
            for j in range(n):
                if row[j] > row[best]:
                    best = j
            idx.append(best)
        return idx

    # -- shape ops (tensor/ops.go:194-307)
    def Reshape(self, *shape):
        shape = list(shape)
        infer, known = -1, 1
        for i, s in enumerate(shape):
            if s == -1:
                if infer >= 0:
                    raise ValueError("tensor: Reshape allows only one -1 dimension")
                infer = i
            else:
                known *= s
        if infer >= 0 and known != 0:
            shape[infer] = self.Numel() // known
        if numel(shape) != self.Numel():
            raise ValueError(f"tensor: cannot reshape {self.shape} into {shape}")
        return _new_result(self.st, shape, "Reshape", [self], lambda g: [_from_storage(g.st, self.shape)])

    def Flatten(self):
        return self.Reshape(self.shape[0], -1)

    def Permute(self, *dims):
        if len(dims) != len(self.shape):
            raise ValueError(f"tensor: Permute got {len(dims)} dims for shape {self.shape}")
        src = contiguous_strides(self.shape)
        shape, strides, inverse, seen = [0] * len(dims), [0] * len(dims), [0] * len(dims), [False] * len(dims)
        for i, d in enumerate(dims):
            d = _norm_dim(d, len(self.shape))
            if seen[d]:
                raise ValueError(f"tensor: Permute dims {dims} repeat dimension {d}")
            seen[d] = True
            shape[i], strides[i], inverse[d] = self.shape[d], src[d], i
        st = self.be().Copy(self.st, make_view(shape, strides))
        return _new_result(st, shape, "Permute", [self], lambda g: [g.Permute(*inverse)])

    def T(self):
        nd = len(self.shape)
        if nd < 2:
            raise ValueError(f"tensor: T requires at least 2 dimensions, got {self.shape}")
        dims = list(range(nd))
        dims[nd - 2], dims[nd - 1] = nd - 1, nd - 2
        return self.Permute(*dims)

    def Index(self, i):
        if len(self.shape) == 0 or i < 0 or i >= self.shape[0]:
            raise ValueError(f"tensor: Index {i} out of range for shape {self.shape}")
        inner = self.shape[1:]
        sz = numel(inner)
        v = _contiguous_view(inner, i * sz)

        def bw(g):
            d = ZerosLike(self)
            g.be().Write(d.st, i * sz, g.st)
            return [d]
        return _new_result(self.be().Copy(self.st, v), inner, "Index", [self], bw)

    # -- linear algebra (tensor/ops.go:309-329)
    def MatMul(self, o):
        _check_same("MatMul", self, o)
        if len(self.shape) != 2 or len(o.shape) != 2 or self.shape[1] != o.shape[0]:
            raise ValueError(f"tensor: MatMul shape mismatch {self.shape} @ {o.shape}")
        m, k, n = self.shape[0], self.shape[1], o.shape[1]
        b = self.be()

        def bw(g):
            gt = go = None
            if self.requires_grad:
                gt = _from_storage(b.MatMul(g.st, o.st, m, n, k, False, True), self.shape)
            if o.requires_grad:
                go = _from_storage(b.MatMul(self.st, g.st, k, m, n, True, False), o.shape)
            return [gt, go]
        return _new_result(b.MatMul(self.st, o.st, m, k, n, False, False), [m, n], "MatMul", [self, o], bw)

    # -- neural-network helpers (tensor/ops.go:331-359)
    def LogSoftmax(self):
        m = self.MaxDim(-1, True)
        shifted = self.Sub(m)
        return shifted.Sub(shifted.Exp().SumDim(-1, True).Log())

    def Softmax(self):
        return self.LogSoftmax().Exp()

    def Pick(self, index):
        if len(self.shape) != 2 or len(index) != self.shape[0]:
            raise ValueError("tensor: Pick needs a 2-D tensor and one index per row")
        c = self.shape[1]
        onehot = np.zeros(self.Numel(), dtype=np.float64)
        for i, j in enumerate(index):
            if j < 0 or j >= c:
                raise ValueError(f"tensor: Pick index {j} out of range for {c} columns")
            onehot[i * c + j] = 1
        return self.Mul(_from_host(onehot, self.shape, self.DType(), self.Device())).SumDim(1, False)

    # -- convolution helpers (tensor/conv.go:27-36)
    def _im2col(self, g: ConvGeom):
        b = self.be()
        shape = [g.N * g.OH * g.OW, g.C * g.KH * g.KW]
        return _new_result(b.Im2col(self.st, g), shape, "Im2col", [self],
                           lambda grad: [_from_storage(b.Col2im(grad.st, g), self.shape)])

    def __repr__(self):
        return f"tensor(shape={self.shape}, dtype={'float64' if self.DType() == Float64 else 'float32'}, device={self.Device()})"


def _topo_sort(root: Tensor):
    order, visited = [], set()

    def visit(t):
        if id(t) in visited or not t.requires_grad:
            return
        visited.add(id(t))
        if t.ctx is not None:
            for inp in t.ctx.inputs:
                visit(inp)
        order.append(t)
    visit(root)
    return order


def _norm_dim(dim, ndim):
    if dim < 0:
        dim += ndim
    if dim < 0 or dim >= ndim:
        raise ValueError(f"tensor: dimension {dim} out of range for {ndim}-D tensor")
    return dim


def _reduced_shape(shape, dim, keep):
    if keep:
        s = list(shape)
        s[dim] = 1
        return s
    return list(shape[:dim]) + list(shape[dim + 1:])


def _broadcast_shapes(a, b):
    """tensor/ops.go:363-391"""
    n = max(len(a), len(b))
    out = [0] * n
    for i in range(n):
        j, k = len(a) - n + i, len(b) - n + i
        da = a[j] if j >= 0 else 1
        db = b[k] if k >= 0 else 1
        if da == db:
            out[i] = da
        elif da == 1:
            out[i] = db
        elif db == 1:
            out[i] = da
        else:
            raise ValueError(f"tensor: shapes {a} and {b} are not broadcastable")
    if n > MAX_DIMS:
        raise ValueError(f"tensor: at most {MAX_DIMS} dimensions are supported, got {n}")
    return out


def _broadcast_strides(shape, target):
    st = [0] * len(target)
    off, s = len(target) - len(shape), 1
    for i in range(len(shape) - 1, -1, -1):
        if shape[i] != 1:
            st[i + off] = s
        s *= shape[i]
    return st


def _expand(t: Tensor, shape) -> Tensor:
    if list(t.shape) == list(shape):
        return t
    return _from_storage(t.be().Copy(t.st, make_view(shape, _broadcast_strides(t.shape, shape))), shape)


def _sum_to(g: Tensor, shape) -> Tensor:
    """tensor/ops.go:416-433"""
    if list(g.shape) == list(shape):
        return g
    b = g.be()
    lead = len(g.shape) - len(shape)
    if lead > 0:
        rest = g.shape[lead:]
        g = _from_storage(b.Reduce(SUM, g.st, 1, numel(g.shape[:lead]), numel(rest)), rest)
    for d in range(len(shape)):
        if shape[d] == 1 and g.shape[d] != 1:
            g = g._reduce(SUM, d, True)
    return _from_storage(g.st, shape)


# ---------------------------------------------------------------------------
# Creation (tensor/tensor.go:33-51, tensor/creation.go)

def New(data, *shape, dtype=None, device=None) -> Tensor:
    data = np.asarray(data, dtype=np.float64).reshape(-1)
    shape = list(shape) if shape else [data.size]
    if numel(shape) != data.size:
        raise ValueError(f"tensor: data length {data.size} does not match shape {shape}")
    return _from_host(data, shape, _default_dtype if dtype is None else dtype, device or _default_device)


def FromFloat32(data, *shape) -> Tensor:
    data = np.asarray(data, dtype=np.float32).reshape(-1)
    shape = list(shape) if shape else [data.size]
    return _from_storage(backend_for(CPU).FromHost(data), shape)


def FromFloat64(data, *shape) -> Tensor:
    data = np.asarray(data, dtype=np.float64).reshape(-1)
    shape = list(shape) if shape else [data.size]
    return _from_storage(backend_for(CPU).FromHost(data), shape)


def Zeros(*shape) -> Tensor:
    return _zeros(shape, _default_dtype, _default_device)


def _zeros(shape, dt, dev) -> Tensor:
    return _from_storage(backend_for(dev).Zeros(dt, numel(shape)), shape)


def Full(v, *shape) -> Tensor:
    return _from_host(np.full(numel(shape), v, dtype=np.float64), shape, _default_dtype, _default_device)


def Ones(*shape) -> Tensor:
    return Full(1.0, *shape)


def ZerosLike(t: Tensor) -> Tensor:
    return _zeros(t.shape, t.DType(), t.Device())


def OnesLike(t: Tensor) -> Tensor:
    return _from_host(np.ones(t.Numel()), t.shape, t.DType(), t.Device())


def Uniform(low, high, *shape) -> Tensor:
    data = low + (high - low) * _rng.random(numel(shape))
    return _from_host(data, shape, _default_dtype, _default_device)


def Rand(*shape) -> Tensor:
    return Uniform(0.0, 1.0, *shape)


def Randn(*shape) -> Tensor:
    return _from_host(_rng.standard_normal(numel(shape)), shape, _default_dtype, _default_device)


def Stack(ts) -> Tensor:
    """tensor/ops.go:280-307"""
    if not ts:
        raise ValueError("tensor: Stack needs at least one tensor")
    _check_same("Stack", *ts)
    inner = ts[0].shape
    sz = numel(inner)
    b = ts[0].be()
    st = b.Zeros(ts[0].DType(), len(ts) * sz)
    for i, t in enumerate(ts):
        if list(t.shape) != list(inner):
            raise ValueError(f"tensor: Stack shape mismatch {t.shape} vs {inner}")
        b.Write(st, i * sz, t.st)

    def bw(g):
        return [_from_storage(g.be().Copy(g.st, _contiguous_view(inner, i * sz)), inner) for i in range(len(ts))]
    return _new_result(st, [len(ts)] + list(inner), "Stack", list(ts), bw)


# ---------------------------------------------------------------------------
# tensor/conv.go

def conv_geom(op, shape, kh, kw, stride, padding) -> ConvGeom:
    if len(shape) != 4:
        raise ValueError(f"tensor: {op} expects input of shape (N, C, H, W), got {shape}")
    if stride < 1 or padding < 0:
        raise ValueError(f"tensor: {op} needs stride >= 1 and padding >= 0")
    g = ConvGeom(N=shape[0], C=shape[1], H=shape[2], W=shape[3], KH=kh, KW=kw, stride=stride, pad=padding)
    g.OH = (g.H + 2 * padding - kh) // stride + 1
    g.OW = (g.W + 2 * padding - kw) // stride + 1
    if g.OH <= 0 or g.OW <= 0:
        raise ValueError(f"tensor: {op} kernel {kh}x{kw} is larger than padded input {shape}")
    return g


def Conv2d(x: Tensor, weight: Tensor, bias: Tensor | None, stride: int, padding: int) -> Tensor:
    _check_same("Conv2d", x, weight)
    if len(weight.shape) != 4 or len(x.shape) != 4 or weight.shape[1] != x.shape[1]:
        raise ValueError(f"tensor: Conv2d weight {weight.shape} does not match input {x.shape}")
    o = weight.shape[0]
    if bias is not None and (len(bias.shape) != 1 or bias.shape[0] != o):
        raise ValueError(f"tensor: Conv2d bias shape {bias.shape}, want [{o}]")
    g = conv_geom("Conv2d", x.shape, weight.shape[2], weight.shape[3], stride, padding)
    k = g.C * g.KH * g.KW
    cols = x._im2col(g)
    y = cols.MatMul(weight.Reshape(o, k).T())
    out = y.Reshape(g.N, g.OH * g.OW, o).Permute(0, 2, 1).Reshape(g.N, o, g.OH, g.OW)
    if bias is not None:
        out = out.Add(bias.Reshape(o, 1, 1))
    return out


def MaxPool2d(x: Tensor, kernel: int, stride: int) -> Tensor:
    g = conv_geom("MaxPool2d", x.shape, kernel, kernel, stride, 0)
    b = x.be()
    shape = [g.N, g.C, g.OH, g.OW]
    return _new_result(b.MaxPool2d(x.st, g), shape, "MaxPool2d", [x],
                       lambda grad: [_from_storage(b.MaxPool2dBackward(x.st, grad.st, g), x.shape)])
