"""ORACLE — test infrastructure, not part of the product.

A restatement of go-tensor's safetensors reader and writer, the reference for
the native checkpoint code of the step runtime:

* ``encode`` follows weights/safetensors/safetensors.go:116-175 (``Encode``):
  tensors in sorted name order, one little-endian F32 or F64 body, a JSON
  header holding every tensor's dtype, shape and data offsets plus an
  optional ``__metadata__`` object, padded with spaces to a multiple of 8
  bytes and preceded by its length as a uint64.
* ``decode`` follows safetensors.go:55-100 (``Decode``) and
  internal/dtype/dtype.go:41-148 (element sizes, ``Decode``,
  ``HalfToFloat64``, ``BFloat16ToFloat64``, ``Numel`` with its 2^34 bound).

The header JSON is what Go's ``encoding/json`` (Go 1.23, the go.mod version)
writes for a ``map[string]any``: keys in byte order, no spaces, and strings
escaped with its HTML-safe rules. Go escapes `"` and `\\` with a backslash,
and writes `\\b \\f \\n \\r \\t` short. Other control bytes, `<`, `>` and `&`
become `\\u00XX`, U+2028 and U+2029 become `\\u2028` and `\\u2029`, and
invalid UTF-8 becomes `\\ufffd`. ``go_json_string`` restates those rules.

Only tests/ may import this module.
"""
from __future__ import annotations

import json
import struct

import numpy as np

MAX_HEADER = 100 << 20      # safetensors.go:18-19
MAX_ELEMENTS = 1 << 34      # dtype.go:130-132
SIZES = {"F64": 8, "F32": 4, "F16": 2, "BF16": 2, "I64": 8, "I32": 4, "I16": 2, "I8": 1,
         "U64": 8, "U32": 4, "U16": 2, "U8": 1, "BOOL": 1}


def go_json_string(s: str | bytes) -> str:
    """A JSON string literal as Go 1.23's json.Marshal writes it."""
    b = s.encode("utf-8", "surrogatepass") if isinstance(s, str) else s
    out = ['"']
    i = 0
    short = {0x22: '\\"', 0x5C: "\\\\", 0x08: "\\b", 0x0C: "\\f", 0x0A: "\\n", 0x0D: "\\r", 0x09: "\\t"}
    while i < len(b):
        c = b[i]
        if c < 0x80:
            if c in short:
                out.append(short[c])
            elif c < 0x20 or c in (0x3C, 0x3E, 0x26):
                out.append("\\u00%02x" % c)
            else:
                out.append(chr(c))
            i += 1
            continue
        # one UTF-8 sequence, or U+FFFD for an invalid byte
        n = 2 if c >> 5 == 0b110 else 3 if c >> 4 == 0b1110 else 4 if c >> 3 == 0b11110 else 0
        try:
            ch = b[i:i + n].decode("utf-8") if n else None
        except UnicodeDecodeError:
            ch = None
        if ch is None or len(ch) != 1:
            out.append("\\ufffd")
            i += 1
            continue
        out.append("\\u2028" if ch == "\u2028" else "\\u2029" if ch == "\u2029" else ch)
        i += n
    out.append('"')
    return "".join(out)


def encode(tensors: dict, dt: str, metadata: dict | None = None) -> bytes:
    """tensors: name -> (shape, float64 values). Returns the file's bytes."""
    if dt not in ("F32", "F64"):
        raise ValueError(f"safetensors: unsupported output dtype {dt!r}")
    if "__metadata__" in tensors:
        raise ValueError('safetensors: "__metadata__" is a reserved name')
    header = {}
    if metadata:
        header["__metadata__"] = "{" + ",".join(
            go_json_string(k) + ":" + go_json_string(v) for k, v in sorted(metadata.items(), key=lambda kv: kv[0].encode())) + "}"
    body = bytearray()
    size = 8 if dt == "F64" else 4
    for name in sorted(tensors, key=lambda k: k.encode()):
        shape, vals = tensors[name]
        vals = np.asarray(vals, dtype=np.float64).reshape(-1)
        start = len(body)
        body += vals.astype("<f8" if dt == "F64" else "<f4").tobytes()
        header[name] = ('{"dtype":"%s","shape":[%s],"data_offsets":[%d,%d]}'
                        % (dt, ",".join(str(int(d)) for d in shape), start, start + vals.size * size))
    h = ("{" + ",".join(go_json_string(k) + ":" + v for k, v in sorted(header.items(), key=lambda kv: kv[0].encode()))
         + "}").encode("utf-8", "surrogatepass")
    h += b" " * ((8 - len(h) % 8) % 8)
    return struct.pack("<Q", len(h)) + h + bytes(body)


def _half(h: int) -> float:
    """dtype.go:102-122."""
    exp, frac = (h >> 10) & 0x1F, float(h & 0x3FF)
    if exp == 0:
        v = np.ldexp(frac, -24)
    elif exp == 0x1F:
        v = float("inf") if frac == 0 else float("nan")
    else:
        v = np.ldexp(frac + 1024, exp - 25)
    return -v if h & 0x8000 else float(v)


def _decode_elems(kind: str, raw: bytes) -> np.ndarray:
    """dtype.go:57-100: elements of `kind` to float64."""
    if kind == "F64":
        return np.frombuffer(raw, "<f8").astype(np.float64)
    if kind == "F32":
        return np.frombuffer(raw, "<f4").astype(np.float64)
    if kind == "F16":
        return np.array([_half(int(h)) for h in np.frombuffer(raw, "<u2")], dtype=np.float64)
    if kind == "BF16":
        return (np.frombuffer(raw, "<u2").astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    if kind == "BOOL":
        return (np.frombuffer(raw, np.uint8) != 0).astype(np.float64)
    code = {"I64": "<i8", "I32": "<i4", "I16": "<i2", "I8": "i1", "U64": "<u8", "U32": "<u4", "U16": "<u2", "U8": "u1"}
    return np.frombuffer(raw, code[kind]).astype(np.float64)


def _numel(shape) -> int:
    n = 1
    for d in shape:
        if d < 0:
            raise ValueError(f"negative dimension in shape {shape}")
        if d != 0 and n > MAX_ELEMENTS // d:
            raise ValueError(f"shape {shape} has more than {MAX_ELEMENTS} elements")
        n *= d
    return n


def decode(b: bytes):
    """Returns (name -> (shape, float64 array), metadata dict)."""
    if len(b) < 8:
        raise ValueError("safetensors: file too short")
    (n,) = struct.unpack("<Q", b[:8])
    if n > MAX_HEADER or n > len(b) - 8:
        raise ValueError(f"safetensors: invalid header length {n}")
    raw = json.loads(b[8:8 + n].decode("utf-8"))
    body = b[8 + n:]
    meta, tensors = None, {}
    for name, h in raw.items():
        if name == "__metadata__":
            meta = dict(h)
            continue
        kind = h["dtype"]
        if kind not in SIZES:
            raise ValueError(f"safetensors: tensor {name!r} has unsupported dtype {kind}")
        numel = _numel(h["shape"])
        start, end = h["data_offsets"]
        if start < 0 or end < start or end > len(body) or end - start != numel * SIZES[kind]:
            raise ValueError(f"safetensors: tensor {name!r} has invalid data offsets {h['data_offsets']}")
        vals = _decode_elems(kind, body[start:end])
        tensors[name] = (list(h["shape"]), vals[:1] if not h["shape"] else vals)
    return tensors, meta or {}
