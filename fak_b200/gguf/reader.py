"""GGUF v2/v3 reader over a read-only memory map.

Behaviour matches the reference's GGUF opener (internal/ggufload/gguf_open.go:13-215,
internal/ggufload/gguf.go): header, metadata key/values, tensor directory, an
aligned data section, and multi-file splits (``*-00001-of-0000N.gguf``).  Tensor
payloads are returned as zero-copy ``numpy`` views of the mapping so quantized
blocks can be uploaded to the GPU unchanged.
"""
from __future__ import annotations

import dataclasses
import mmap
import os
import re
import struct
from typing import Any, Iterator

import numpy as np

from .constants import GGUF_DEFAULT_ALIGNMENT, GGUF_MAGIC, GGMLType, ValueType, tensor_nbytes

_SCALAR_FMT = {
    ValueType.UINT8: "<B", ValueType.INT8: "<b", ValueType.UINT16: "<H", ValueType.INT16: "<h",
    ValueType.UINT32: "<I", ValueType.INT32: "<i", ValueType.FLOAT32: "<f", ValueType.BOOL: "<?",
    ValueType.UINT64: "<Q", ValueType.INT64: "<q", ValueType.FLOAT64: "<d",
}
_NP_DTYPE = {
    ValueType.UINT8: np.uint8, ValueType.INT8: np.int8, ValueType.UINT16: np.uint16,
    ValueType.INT16: np.int16, ValueType.UINT32: np.uint32, ValueType.INT32: np.int32,
    ValueType.FLOAT32: np.float32, ValueType.BOOL: np.bool_, ValueType.UINT64: np.uint64,
    ValueType.INT64: np.int64, ValueType.FLOAT64: np.float64,
}


class GGUFError(ValueError):
    """Malformed or unsupported GGUF content (fail-closed, never a partial model)."""


@dataclasses.dataclass
class TensorInfo:
    name: str
    shape: tuple[int, ...]  # numpy order: outermost first (GGUF stores innermost first)
    ggml_type: GGMLType
    offset: int  # absolute byte offset into the owning file
    nbytes: int
    file_index: int = 0

    @property
    def n_elements(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n


class _Cursor:
    def __init__(self, buf: memoryview, pos: int = 0):
        self.buf = buf
        self.pos = pos

    def take(self, n: int) -> memoryview:
        if self.pos + n > len(self.buf):
            raise GGUFError(f"truncated GGUF: need {n} bytes at offset {self.pos}, file has {len(self.buf)}")
        out = self.buf[self.pos:self.pos + n]
        self.pos += n
        return out

    def scalar(self, vt: ValueType) -> Any:
        fmt = _SCALAR_FMT[vt]
        return struct.unpack(fmt, self.take(struct.calcsize(fmt)))[0]

    def u32(self) -> int:
        return struct.unpack("<I", self.take(4))[0]

    def u64(self) -> int:
        return struct.unpack("<Q", self.take(8))[0]

    def string(self) -> str:
        n = self.u64()
        if n > 1 << 30:
            raise GGUFError(f"implausible GGUF string length {n}")
        return bytes(self.take(n)).decode("utf-8", errors="replace")

    def value(self, vt: ValueType) -> Any:
        if vt == ValueType.STRING:
            return self.string()
        if vt == ValueType.ARRAY:
            et = ValueType(self.u32())
            n = self.u64()
            if et == ValueType.STRING:
                return [self.string() for _ in range(n)]
            if et == ValueType.ARRAY:
                return [self.value(ValueType.ARRAY) for _ in range(n)]
            dt = np.dtype(_NP_DTYPE[et])
            arr = np.frombuffer(self.take(n * dt.itemsize), dtype=dt).copy()
            return arr.tolist()
        return self.scalar(vt)


class GGUFFile:
    """One or more GGUF shard files presented as one model."""

    def __init__(self, path: str | os.PathLike):
        self.path = os.fspath(path)
        self.paths = self._split_paths(self.path)
        self._maps: list[mmap.mmap] = []
        self._files = []
        self.metadata: dict[str, Any] = {}
        self.tensors: dict[str, TensorInfo] = {}
        self.version = 0
        for idx, p in enumerate(self.paths):
            self._open_one(idx, p)

    @staticmethod
    def _split_paths(path: str) -> list[str]:
        m = re.match(r"^(.*)-(\d{5})-of-(\d{5})\.gguf$", path)
        if not m:
            return [path]
        stem, _, total = m.group(1), m.group(2), int(m.group(3))
        paths = [f"{stem}-{i:05d}-of-{total:05d}.gguf" for i in range(1, total + 1)]
        missing = [p for p in paths if not os.path.exists(p)]
        if missing:
            raise GGUFError(f"split GGUF is missing shards: {missing}")
        return paths

    def _open_one(self, file_index: int, path: str) -> None:
        f = open(path, "rb")
        size = os.fstat(f.fileno()).st_size
        if size < 24:
            f.close()
            raise GGUFError(f"{path}: too small to be GGUF ({size} bytes)")
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        self._files.append(f)
        self._maps.append(mm)
        cur = _Cursor(memoryview(mm))
        magic = cur.u32()
        if magic != GGUF_MAGIC:
            raise GGUFError(f"{path}: bad magic 0x{magic:08x}")
        version = cur.u32()
        if version not in (2, 3):
            raise GGUFError(f"{path}: unsupported GGUF version {version}")
        self.version = version
        n_tensors = cur.u64()
        n_kv = cur.u64()
        meta: dict[str, Any] = {}
        for _ in range(n_kv):
            key = cur.string()
            vt = ValueType(cur.u32())
            meta[key] = cur.value(vt)
        if file_index == 0:
            self.metadata.update(meta)
        align = int(meta.get("general.alignment", self.metadata.get("general.alignment", GGUF_DEFAULT_ALIGNMENT)))
        if align <= 0 or align & (align - 1):
            raise GGUFError(f"{path}: alignment {align} is not a power of two")
        infos = []
        for _ in range(n_tensors):
            name = cur.string()
            nd = cur.u32()
            if nd > 8:
                raise GGUFError(f"{path}: tensor {name} has {nd} dims")
            dims = [cur.u64() for _ in range(nd)]
            try:
                t = GGMLType(cur.u32())
            except ValueError as e:
                raise GGUFError(f"{path}: tensor {name}: unknown GGML type") from e
            off = cur.u64()
            infos.append((name, tuple(reversed(dims)), t, off))
        data_start = (cur.pos + align - 1) // align * align
        for name, shape, t, off in infos:
            n = 1
            for s in shape:
                n *= s
            nbytes = tensor_nbytes(t, n)
            abs_off = data_start + off
            if abs_off + nbytes > size:
                raise GGUFError(f"{path}: tensor {name} [{abs_off}, +{nbytes}) runs past end of file ({size})")
            if name in self.tensors:
                raise GGUFError(f"duplicate tensor {name}")
            self.tensors[name] = TensorInfo(name, shape, t, abs_off, nbytes, file_index)

    # ------------------------------------------------------------------------------------
    def raw(self, name: str) -> np.ndarray:
        """Zero-copy uint8 view of a tensor's stored bytes."""
        ti = self.tensors[name]
        mm = self._maps[ti.file_index]
        return np.frombuffer(mm, dtype=np.uint8, count=ti.nbytes, offset=ti.offset)

    def raw_rows(self, name: str) -> np.ndarray:
        """Stored bytes as [rows, row_bytes] for a 2-D (or stacked 3-D) tensor."""
        ti = self.tensors[name]
        rows = ti.n_elements // ti.shape[-1]
        return self.raw(name).reshape(rows, -1)

    def dequantize(self, name: str) -> np.ndarray:
        from .quants import dequantize
        ti = self.tensors[name]
        return dequantize(self.raw(name), ti.ggml_type, ti.shape)

    def get(self, key: str, default: Any = None) -> Any:
        return self.metadata.get(key, default)

    def __contains__(self, name: str) -> bool:
        return name in self.tensors

    def __iter__(self) -> Iterator[TensorInfo]:
        return iter(self.tensors.values())

    def close(self) -> None:
        for m in self._maps:
            try:
                m.close()
            except BufferError:
                pass  # a numpy view is still alive; the map closes when it is collected
        for f in self._files:
            f.close()
        self._maps.clear()
        self._files.clear()

    def __enter__(self) -> "GGUFFile":
        return self

    def __exit__(self, *exc) -> None:
        self.close()


def open_gguf(path: str | os.PathLike) -> GGUFFile:
    return GGUFFile(path)
