"""GGUF v3 writer.

Used to produce the random-init checkpoints the tests and benchmarks load
(the reference builds its fixtures with Python helpers, make_*_tiny.py, and
reads GGUF in internal/ggufload/gguf.go).  Tensor payloads can be supplied
lazily (a callable returning bytes) so a multi-GB checkpoint streams to disk
one tensor at a time.
"""
from __future__ import annotations

import os
import struct
from typing import Any, Callable, Union

import numpy as np

from .constants import GGUF_DEFAULT_ALIGNMENT, GGUF_MAGIC, GGUF_VERSION, GGMLType, ValueType, tensor_nbytes

Payload = Union[bytes, np.ndarray, Callable[[], Union[bytes, np.ndarray]]]


def _pack_string(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _infer_type(v: Any) -> ValueType:
    if isinstance(v, bool):
        return ValueType.BOOL
    if isinstance(v, int):
        return ValueType.UINT32 if 0 <= v < 2**32 else ValueType.INT64
    if isinstance(v, float):
        return ValueType.FLOAT32
    if isinstance(v, str):
        return ValueType.STRING
    if isinstance(v, (list, tuple, np.ndarray)):
        return ValueType.ARRAY
    raise TypeError(f"cannot infer GGUF type of {type(v)}")


_FMT = {
    ValueType.UINT8: "<B", ValueType.INT8: "<b", ValueType.UINT16: "<H", ValueType.INT16: "<h",
    ValueType.UINT32: "<I", ValueType.INT32: "<i", ValueType.FLOAT32: "<f", ValueType.BOOL: "<?",
    ValueType.UINT64: "<Q", ValueType.INT64: "<q", ValueType.FLOAT64: "<d",
}


def _pack_value(v: Any, vt: ValueType, elem_type: ValueType | None = None) -> bytes:
    if vt == ValueType.STRING:
        return _pack_string(v)
    if vt == ValueType.ARRAY:
        items = list(v)
        if elem_type is None:
            if items and all(isinstance(x, str) for x in items):
                elem_type = ValueType.STRING
            elif items and all(isinstance(x, float) for x in items):
                elem_type = ValueType.FLOAT32
            else:
                elem_type = ValueType.INT32
        out = [struct.pack("<IQ", int(elem_type), len(items))]
        if elem_type == ValueType.STRING:
            out.extend(_pack_string(x) for x in items)
        else:
            out.append(np.asarray(items, dtype=np.dtype(_FMT[elem_type][1:]).newbyteorder("<")).tobytes())
        return b"".join(out)
    return struct.pack(_FMT[vt], v)


class GGUFWriter:
    def __init__(self, path: str | os.PathLike, arch: str | None = None, alignment: int = GGUF_DEFAULT_ALIGNMENT):
        self.path = os.fspath(path)
        self.alignment = alignment
        self._kv: list[tuple[str, ValueType, Any, ValueType | None]] = []
        self._tensors: list[tuple[str, tuple[int, ...], GGMLType, int, Payload]] = []
        if arch is not None:
            self.add("general.architecture", arch)
        if alignment != GGUF_DEFAULT_ALIGNMENT:
            self.add("general.alignment", alignment, ValueType.UINT32)

    def add(self, key: str, value: Any, vtype: ValueType | None = None, elem_type: ValueType | None = None) -> None:
        vt = vtype if vtype is not None else _infer_type(value)
        self._kv.append((key, vt, value, elem_type))

    def add_tensor(self, name: str, shape: tuple[int, ...], ggml_type: int, payload: Payload) -> None:
        """shape in numpy order (outermost first); payload is the stored bytes."""
        t = GGMLType(ggml_type)
        n = 1
        for s in shape:
            n *= int(s)
        self._tensors.append((name, tuple(int(s) for s in shape), t, tensor_nbytes(t, n), payload))

    def write(self) -> None:
        a = self.alignment
        header = [struct.pack("<IIQQ", GGUF_MAGIC, GGUF_VERSION, len(self._tensors), len(self._kv))]
        for key, vt, v, et in self._kv:
            header.append(_pack_string(key) + struct.pack("<I", int(vt)) + _pack_value(v, vt, et))
        offsets = []
        off = 0
        for name, shape, t, nbytes, _ in self._tensors:
            off = (off + a - 1) // a * a
            offsets.append(off)
            dims = list(reversed(shape))
            header.append(_pack_string(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
                          + struct.pack("<IQ", int(t), off))
            off += nbytes
        hdr = b"".join(header)
        tmp = self.path + ".partial"
        with open(tmp, "wb") as f:
            f.write(hdr)
            pos = len(hdr)
            pad = (pos + a - 1) // a * a - pos
            f.write(b"\0" * pad)
            base = pos + pad
            for (name, shape, t, nbytes, payload), toff in zip(self._tensors, offsets):
                cur = f.tell() - base
                if cur < toff:
                    f.write(b"\0" * (toff - cur))
                data = payload() if callable(payload) else payload
                if isinstance(data, np.ndarray):
                    data = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
                    if data.size != nbytes:
                        raise ValueError(f"tensor {name}: payload has {data.size} bytes, expected {nbytes}")
                    data.tofile(f)
                else:
                    if len(data) != nbytes:
                        raise ValueError(f"tensor {name}: payload has {len(data)} bytes, expected {nbytes}")
                    f.write(data)
        os.replace(tmp, self.path)
