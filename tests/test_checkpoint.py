"""Checkpoints: the step runtime's native safetensors and GOTN code
(runtime/checkpoint.cpp) against the reference's formats and tests.

CPU tests pin the decoders:

* zoo.safetensors is the reference's known-answer file, one tensor of every
  dtype plus metadata (weights/safetensors/safetensors_test.go:12-21);
* corrupt files are refused (safetensors_test.go:55-71);
* the oracle's encoder round-trips (safetensors_test.go:23-53).

GPU tests (a model lives on the device) compare:

* the bytes a device model saves with the oracle's restatement of
  safetensors.Encode over nn.StateDict, F32 and F64, metadata with escapes;
* loading with LoadStateDict's checks and messages (nn/state.go:84-126);
* GOTN bytes with the oracle's nn.Save (nn/serialize.go:22-38);
* the PyTorch-written CNN weights reproducing PyTorch's forward pass
  (weights/weights_test.go:31-74).
"""
import ctypes
import json
import os
import struct

import numpy as np
import pytest

from gotensor import _lib
from gotensor._lib import GTError, check
from oracle import safetensors_ref as S

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ZOO = os.path.join(GOLDEN, "zoo.safetensors")


def native_read(path, name):
    lib = _lib.host_lib()
    numel, ndim = ctypes.c_int64(), ctypes.c_int()
    shape = (ctypes.c_int64 * 8)()
    check(lib.gth_safetensors_read(path.encode(), name.encode(), None, 0, shape, 8, ctypes.byref(ndim),
                                   ctypes.byref(numel)))
    out = (ctypes.c_double * max(numel.value, 1))()
    check(lib.gth_safetensors_read(path.encode(), name.encode(), out, numel.value, None, 0, None, None))
    return [shape[d] for d in range(ndim.value)], np.array(out[:numel.value])


def native_meta(path, key):
    buf = ctypes.create_string_buffer(256)
    n = ctypes.c_int()
    check(_lib.host_lib().gth_safetensors_metadata(path.encode(), key.encode(), buf, 256, ctypes.byref(n)))
    return buf.value.decode()


# ---- CPU: the decoders ------------------------------------------------------

def test_zoo_known_answers():
    with open(os.path.join(GOLDEN, "zoo_safetensors_expected.json")) as f:
        exp = json.load(f)
    with open(ZOO, "rb") as f:
        oracle, meta = S.decode(f.read())
    assert meta == exp["metadata"]
    for k, v in exp["metadata"].items():
        assert native_meta(ZOO, k) == v
    for name, e in exp["tensors"].items():
        want = np.asarray(e["values"], dtype=np.float64)
        shape, got = native_read(ZOO, name)
        assert shape == e["shape"], name
        assert np.array_equal(got, want, equal_nan=True), name
        assert np.array_equal(np.asarray(oracle[name][1]), want, equal_nan=True), name


def test_corrupt_files_are_refused(tmp_path):
    good = S.encode({"a": ([4], np.ones(4))}, "F32")
    cases = {"truncated": good[:-1], "huge": struct.pack("<Q", 1 << 40) + good[8:], "short": bytes([1, 2]),
             "offsets": good.replace(b"[0,16]", b"[0,12]"), "dtype": good.replace(b'"F32"', b'"F99"'),
             "json": good[:8] + b"[" + good[9:]}
    for name, b in cases.items():
        p = tmp_path / f"{name}.safetensors"
        p.write_bytes(b)
        with pytest.raises(GTError):
            native_read(str(p), "a")
        with pytest.raises(Exception):
            S.decode(b)
    p = tmp_path / "good.safetensors"
    p.write_bytes(good)
    assert native_read(str(p), "a")[1].tolist() == [1, 1, 1, 1]
    with pytest.raises(GTError, match="no tensor"):
        native_read(str(p), "b")


def test_oracle_round_trip():
    rng = np.random.default_rng(0)
    inp = {"w": ([3], np.array([1.0 / 3, -2, 1e-40])), "m": ([2, 3], rng.standard_normal(6)),
           "scalar": ([], np.array([4.0]))}
    for dt in ("F64", "F32"):
        out, meta = S.decode(S.encode(inp, dt, {"k": "v"}))
        assert meta == {"k": "v"}
        for k, (shape, vals) in inp.items():
            want = vals if dt == "F64" else vals.astype(np.float32).astype(np.float64)
            assert out[k][0] == shape and np.array_equal(out[k][1], want)


# ---- GPU: saving and loading a device model --------------------------------

CNN = [("Conv2d", (1, 2, 3, 1, 1)), ("ReLU", ()), ("MaxPool2d", (2, 0)), ("Flatten", ()), ("Linear", (32, 3))]


def cnn_model(dtype=None):
    from gotensor import FLOAT32
    from gotensor import model as gm
    layers = [getattr(gm, k)(*a) for k, a in CNN]
    return gm.Model(layers, [2, 1, 8, 8], dtype=FLOAT32 if dtype is None else dtype)


def save_st(model, path, dt, meta=None):
    lib = _lib.host_lib()
    meta = meta or {}
    keys = (ctypes.c_char_p * max(len(meta), 1))(*[k.encode("utf-8", "surrogateescape") for k in meta])
    vals = (ctypes.c_char_p * max(len(meta), 1))(*[v.encode("utf-8", "surrogateescape") for v in meta.values()])
    check(lib.gth_save_safetensors(model.ptr, str(path).encode(), dt.encode(), keys, vals, len(meta)))


def load_st(model, path, strict=True):
    check(_lib.host_lib().gth_load_safetensors(model.ptr, str(path).encode(), int(strict)))


@pytest.mark.gpu
@pytest.mark.parametrize("dt", ["F32", "F64"])
@pytest.mark.parametrize("mdt", ["f32", "f64"])
def test_save_matches_reference_encoding(tmp_path, dt, mdt):
    from gotensor import FLOAT32, FLOAT64
    model = cnn_model(FLOAT64 if mdt == "f64" else FLOAT32)
    rng = np.random.default_rng(1)
    npdt = np.float64 if mdt == "f64" else np.float32
    sd = {n: rng.standard_normal(s).astype(npdt) / 3 for n, s, _ in model.params}
    model.load_state_dict(sd)
    meta = {"note": 'a<b & c>d "q" \\ \n\t\x01\b\f', "uni": "\u00e9\u4e2d\u2028\u2029", "": "empty key",
            "bad": "x\udcffy"}  # an invalid UTF-8 byte, written through
    save_st(model, tmp_path / "m.safetensors", dt, meta)
    got = (tmp_path / "m.safetensors").read_bytes()
    want = S.encode({n: (list(v.shape), v.astype(np.float64).reshape(-1)) for n, v in sd.items()}, dt,
                    {k: v.encode("utf-8", "surrogateescape") for k, v in meta.items()})
    assert got == want
    # and it loads back (values rounded to F32 when written as F32)
    other = cnn_model(FLOAT64 if mdt == "f64" else FLOAT32)
    load_st(other, tmp_path / "m.safetensors")
    for n, v in other.state_dict().items():
        w = sd[n] if dt == "F64" else sd[n].astype(np.float32).astype(npdt)
        assert np.array_equal(v, w), n


@pytest.mark.gpu
def test_load_state_dict_semantics(tmp_path):
    from gotensor import FLOAT32
    model = cnn_model(FLOAT32)
    before = model.flat_params()
    rng = np.random.default_rng(2)
    full = {n: (s, rng.standard_normal(int(np.prod(s)))) for n, s, _ in model.params}
    # strict: a missing and an unexpected key, reported like StateDictError
    part = dict(full)
    del part["4.bias"]
    part["9.weight"] = ([2], np.zeros(2))
    p = tmp_path / "p.safetensors"
    p.write_bytes(S.encode(part, "F64"))
    with pytest.raises(GTError, match=r"nn: state dict does not match model: missing keys: 4\.bias; "
                                      r"unexpected keys: 9\.weight"):
        load_st(model, p)
    assert np.array_equal(model.flat_params(), before)  # nothing was loaded
    # not strict: the matching keys load, the rest keep their values
    load_st(model, p, strict=False)
    sd = model.state_dict()
    assert np.array_equal(sd["4.bias"], before[-3:])
    assert np.array_equal(sd["0.weight"].reshape(-1), full["0.weight"][1].astype(np.float32))
    # a shape mismatch is always an error, with the reference's message
    bad = dict(full)
    bad["4.weight"] = ([32, 3], full["4.weight"][1])
    p.write_bytes(S.encode(bad, "F64"))
    with pytest.raises(GTError, match=r"nn: 4\.weight has shape \[32 3\] in the state dict but \[3 32\] in the model"):
        load_st(model, p, strict=False)


@pytest.mark.gpu
def test_load_converts_every_dtype(tmp_path):
    """A file of F16 / BF16 / integer tensors loads into a float32 model with
    the reference's conversions (to float64, then to float32)."""
    from gotensor import FLOAT32
    model = cnn_model(FLOAT32)
    rng = np.random.default_rng(3)
    shapes = {n: s for n, s, _ in model.params}
    raw = {"0.weight": ("F16", rng.standard_normal(18).astype(np.float16).view(np.uint16).astype("<u2")),
           "0.bias": ("I8", np.array([-3, 7], dtype="i1")),
           "4.weight": ("BF16", (rng.standard_normal(96).astype(np.float32).view(np.uint32) >> 16).astype("<u2")),
           "4.bias": ("BOOL", np.array([0, 1, 2], dtype=np.uint8))}
    header, body = {}, b""
    for n in sorted(raw):
        kind, arr = raw[n]
        b = arr.tobytes()
        header[n] = {"dtype": kind, "shape": shapes[n], "data_offsets": [len(body), len(body) + len(b)]}
        body += b
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    p = tmp_path / "kinds.safetensors"
    p.write_bytes(struct.pack("<Q", len(h)) + h + body)
    load_st(model, p)
    want, _ = S.decode(p.read_bytes())
    for n, v in model.state_dict().items():
        assert np.array_equal(v.reshape(-1), want[n][1].astype(np.float32)), n


@pytest.mark.gpu
def test_pytorch_cnn_file_reproduces_pytorch_forward():
    from gotensor import FLOAT32
    with open(os.path.join(GOLDEN, "cnn_forward.json")) as f:
        fx = json.load(f)
    model = cnn_model(FLOAT32)
    load_st(model, os.path.join(GOLDEN, "cnn.safetensors"))
    for n, v in model.state_dict().items():
        assert np.array_equal(v.reshape(-1), np.asarray(fx["params"][n]["values"], dtype=np.float32)), n
    x = np.asarray(fx["input"]["values"], dtype=np.float32).reshape(fx["input"]["shape"])
    model.set_batch(x, np.zeros(2, dtype=np.int32))
    y = model.forward().astype(np.float64).reshape(-1)
    assert np.max(np.abs(y - np.asarray(fx["output"]["values"]))) <= fx["tolerance"]


@pytest.mark.gpu
def test_gotn_matches_reference_and_round_trips(tmp_path):
    import io

    from gotensor import FLOAT32
    from oracle import gotensor_ref as T
    from oracle import nn_ref as nn
    model = cnn_model(FLOAT32)
    rng = np.random.default_rng(4)
    sd = {n: rng.standard_normal(s).astype(np.float32) for n, s, _ in model.params}
    model.load_state_dict(sd)
    path = tmp_path / "m.gotn"
    check(_lib.host_lib().gth_save_gotn(model.ptr, str(path).encode()))
    ref = nn.NewSequential(nn.NewConv2d(1, 2, 3, 1, 1), nn.NewReLU(), nn.NewMaxPool2d(2, 0), nn.NewFlatten(),
                           nn.NewLinear(32, 3))
    nn.LoadStateDict(ref, {k: T.FromFloat32(v.reshape(-1), *v.shape) for k, v in sd.items()}, True)
    buf = io.BytesIO()
    nn.Save(buf, ref)
    assert path.read_bytes() == buf.getvalue()
    other = cnn_model(FLOAT32)
    check(_lib.host_lib().gth_load_gotn(other.ptr, str(path).encode()))
    assert np.array_equal(other.flat_params(), model.flat_params())
    # refusals: the reference's messages; nothing applied
    b = path.read_bytes()
    for data, msg in ((b"XOTN" + b[4:], "not a go-tensor model file"),
                      (b[:4] + struct.pack("<I", 2) + b[8:], "unsupported model file version 2"),
                      (b[:8] + struct.pack("<I", 5) + b[12:], "file has 5 parameters, module has 4"),
                      (b[:-4], "unexpected EOF")):
        path.write_bytes(data)
        before = other.flat_params()
        with pytest.raises(GTError, match=msg):
            check(_lib.host_lib().gth_load_gotn(other.ptr, str(path).encode()))
        assert np.array_equal(other.flat_params(), before)
