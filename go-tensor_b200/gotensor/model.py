"""Python handle on the native training-step runtime (include/gt_host.h).

Layers are described with the constructors of go-tensor's ``nn`` package
(``Linear(in, out)``, ``Conv2d(in, out, kernel, stride, padding)``,
``MaxPool2d(kernel, stride)``, ``ReLU()``, ``Tanh()``, ``Sigmoid()``,
``Flatten()``, ``Dropout(p)``) and compiled by the runtime into a plan of
fused kernels for one input shape. Parameters are named and ordered like
``nn.NamedParameters`` ("0.weight", "0.bias", ...).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import FLOAT32, FLOAT64, AdamCfg, GTError, Layer, SgdCfg, check
from .backend import Context

LINEAR, CONV2D, MAXPOOL2D, RELU, TANH, SIGMOID, FLATTEN, DROPOUT = range(8)
_NP = {FLOAT32: np.float32, FLOAT64: np.float64}


def Linear(in_features, out_features):
    return Layer(kind=LINEAR, in_=in_features, out=out_features)


def Conv2d(in_channels, out_channels, kernel, stride=1, padding=0):
    return Layer(kind=CONV2D, in_=in_channels, out=out_channels, kernel=kernel, stride=stride, padding=padding)


def MaxPool2d(kernel, stride=0):
    return Layer(kind=MAXPOOL2D, kernel=kernel, stride=stride)


def ReLU():
    return Layer(kind=RELU)


def Tanh():
    return Layer(kind=TANH)


def Sigmoid():
    return Layer(kind=SIGMOID)


def Flatten():
    return Layer(kind=FLATTEN)


def Dropout(p):
    return Layer(kind=DROPOUT, p=p)


class Model:
    """A Sequential model compiled for a fixed input shape on one GPU."""

    def __init__(self, layers, input_shape, dtype=FLOAT32, device=0):
        self.lib = _lib.host_lib()
        self.ctx = Context.get(device)
        self.dtype = dtype
        self.np_dtype = _NP[dtype]
        self.input_shape = list(input_shape)
        arr = (Layer * len(layers))(*layers)
        shp = (ctypes.c_int64 * len(input_shape))(*input_shape)
        p = ctypes.c_void_p()
        check(self.lib.gth_model_new(self.ctx.ptr, dtype, arr, len(layers), shp, len(input_shape), ctypes.byref(p)))
        self.ptr = p
        self.params = []  # (name, shape, offset)
        for i in range(self.lib.gth_num_tensors(self.ptr)):
            name = ctypes.create_string_buffer(64)
            shape = (ctypes.c_int64 * 4)()
            nd, off = ctypes.c_int(), ctypes.c_int64()
            check(self.lib.gth_param_info(self.ptr, i, name, 64, shape, ctypes.byref(nd), ctypes.byref(off)))
            self.params.append((name.value.decode(), [shape[d] for d in range(nd.value)], off.value))
        self.num_params = self.lib.gth_num_params(self.ptr)

    def close(self):
        """Frees the model (its captured step graph included) and leaves the
        data-parallel communicator if dp_init joined one. Every rank calls it
        after its last step."""
        p = getattr(self, "ptr", None)
        if p:
            self.ptr = None
            self.lib.gth_model_free(p)
        if getattr(self, "_dp", False):
            self._dp = False
            check(_lib.cuda_lib().gt_comm_destroy(self.ctx.ptr, 0))

    def __del__(self):
        p = getattr(self, "ptr", None)
        if p:
            try:
                self.lib.gth_model_free(p)
            except Exception:
                pass
            self.ptr = None

    # -- parameters
    def set_flat_params(self, flat: np.ndarray):
        flat = np.ascontiguousarray(flat, dtype=self.np_dtype)
        if flat.size != self.num_params:
            raise ValueError(f"expected {self.num_params} parameters, got {flat.size}")
        check(self.lib.gth_set_params(self.ptr, flat.ctypes.data))

    def flat_params(self) -> np.ndarray:
        out = np.empty(self.num_params, dtype=self.np_dtype)
        check(self.lib.gth_get_params(self.ptr, out.ctypes.data))
        return out

    def flat_grads(self) -> np.ndarray:
        out = np.empty(self.num_params, dtype=self.np_dtype)
        check(self.lib.gth_get_grads(self.ptr, out.ctypes.data))
        return out

    def _split(self, flat):
        return {name: flat[off:off + int(np.prod(shape))].reshape(shape) for name, shape, off in self.params}

    def state_dict(self) -> dict:
        return self._split(self.flat_params())

    def grads(self) -> dict:
        return self._split(self.flat_grads())

    def load_state_dict(self, sd: dict):
        """All-or-nothing, strict (nn.LoadStateDict with strict=true, nn/state.go:84-126)."""
        names = [n for n, _, _ in self.params]
        missing = [n for n in names if n not in sd]
        unexpected = sorted(k for k in sd if k not in names)
        if missing or unexpected:
            raise ValueError(f"state dict does not match model: missing {missing}, unexpected {unexpected}")
        flat = np.empty(self.num_params, dtype=self.np_dtype)
        for name, shape, off in self.params:
            v = np.asarray(sd[name])
            if list(v.shape) != list(shape):
                raise ValueError(f"{name} has shape {list(v.shape)} in the state dict but {shape} in the model")
            flat[off:off + v.size] = v.reshape(-1)
        self.set_flat_params(flat)

    # -- optimizer
    def sgd(self, lr, momentum=0.0, weight_decay=0.0):
        check(self.lib.gth_set_sgd(self.ptr, ctypes.byref(SgdCfg(lr, momentum, weight_decay))))

    def adam(self, lr=0.0, beta1=0.0, beta2=0.0, eps=0.0, weight_decay=0.0):
        check(self.lib.gth_set_adam(self.ptr, ctypes.byref(AdamCfg(lr, beta1, beta2, eps, weight_decay))))

    # -- data
    @property
    def input_device(self) -> int:
        return self.lib.gth_input_device(self.ptr)

    @property
    def labels_device(self) -> int:
        return self.lib.gth_labels_device(self.ptr)

    def set_batch(self, x: np.ndarray, labels) -> None:
        x = np.ascontiguousarray(x, dtype=self.np_dtype)
        if list(x.shape) != self.input_shape:
            raise ValueError(f"batch shape {list(x.shape)}, model expects {self.input_shape}")
        y = np.ascontiguousarray(labels, dtype=np.int32)
        if y.shape != (self.input_shape[0],):
            raise ValueError("one label per row")
        ncls = self.classes
        if y.size and (y.min() < 0 or y.max() >= ncls):
            raise ValueError(f"label out of range for {ncls} classes")  # tensor/ops.go:352-354
        lib = self.ctx.lib
        check(lib.gt_upload(self.ctx.ptr, self.input_device, x.ctypes.data, x.nbytes))
        check(lib.gt_upload(self.ctx.ptr, self.labels_device, y.ctypes.data, y.nbytes))

    def stage_batch(self, x_ptr: int, labels_ptr: int) -> None:
        """Queues the upload of the batch at host addresses x_ptr (input
        shape, model dtype) and labels_ptr (int32) on the copy stream; it
        overlaps the step in flight and is read by the next unstaged step.
        Pinned host memory (e.g. torch's pin_memory) makes it asynchronous; it
        must stay unchanged until that step has run."""
        check(self.lib.gth_stage_batch(self.ptr, x_ptr, labels_ptr))

    @property
    def classes(self) -> int:
        last = [s for _, s, _ in self.params][-1]
        return last[0]

    # -- step
    def forward_backward(self):
        check(self.lib.gth_forward_backward(self.ptr))

    def optimizer_step(self):
        check(self.lib.gth_optimizer_step(self.ptr))

    def train_step(self):
        check(self.lib.gth_train_step(self.ptr))

    def enable_graph(self, on=True):
        check(self.lib.gth_enable_graph(self.ptr, int(on)))

    def loss(self) -> float:
        out = ctypes.c_double()
        check(self.lib.gth_loss(self.ptr, ctypes.byref(out)))
        return out.value

    def forward(self) -> np.ndarray:
        out = np.empty((self.input_shape[0], self.classes), dtype=self.np_dtype)
        check(self.lib.gth_forward(self.ptr, out.ctypes.data))
        return out

    def predict(self) -> np.ndarray:
        """Forward of the current batch and Argmax of every row on the device
        (model.Forward(x).Argmax(), tensor/ops.go:176-192): int32 (batch,)."""
        out = np.empty(self.input_shape[0], dtype=np.int32)
        check(self.lib.gth_predict(self.ptr, out.ctypes.data))
        return out

    def count_correct(self) -> int:
        """Rows of the current batch whose Argmax equals their label, counted
        on the device (the accuracy loop of examples/mnist/main.go:120-133)."""
        out = ctypes.c_int64()
        check(self.lib.gth_count_correct(self.ptr, ctypes.byref(out)))
        return out.value

    @property
    def step_launches(self) -> int:
        return self.lib.gth_step_launches(self.ptr)

    def dp_init(self, rank, world, unique_id: bytes, timeout_ms=60000, bucket_bytes=25 << 20):
        check(self.lib.gth_dp_init(self.ptr, rank, world, unique_id, timeout_ms, bucket_bytes))
        self._dp = world > 1


def bucket_plan(sizes, bucket_elems):
    """The runtime's gradient bucket plan (host only): list of (lo, hi)."""
    lib = _lib.host_lib()
    n = len(sizes)
    arr = (ctypes.c_int64 * max(n, 1))(*sizes)
    bounds = (ctypes.c_int64 * (2 * max(n, 1)))()
    cnt = lib.gth_bucket_plan(arr, n, bucket_elems, bounds, max(n, 1))
    if cnt < 0:
        raise GTError("bucket plan overflow")
    return [(bounds[2 * i], bounds[2 * i + 1]) for i in range(cnt)]


def row_chunk_plan(buckets, w_off, N, K, chunks):
    """The runtime's row-chunk split of the first Linear's weight bucket (host
    only): (row boundaries, new bucket list), or ([], buckets) unchanged."""
    lib = _lib.host_lib()
    nb = len(buckets)
    flat = (ctypes.c_int64 * max(2 * nb, 1))(*[v for b in buckets for v in b])
    cap = N // 32 + 3
    rows = (ctypes.c_int64 * cap)()
    out = (ctypes.c_int64 * (2 * (nb + cap)))()
    out_nb = ctypes.c_int()
    nr = lib.gth_row_chunk_plan(flat, nb, w_off, N, K, chunks, rows, cap, out, nb + cap, ctypes.byref(out_nb))
    if nr == 0:
        return [], list(buckets)
    return list(rows[:nr]), [(out[2 * i], out[2 * i + 1]) for i in range(out_nb.value)]


def unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    check(_lib.cuda_lib().gt_comm_unique_id(buf))
    return buf.raw
