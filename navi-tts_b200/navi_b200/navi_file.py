"""The `.navi` v1 weight blob: writer and reader.

The byte layout is the drop-in boundary with the reference engine, so it is
kept identical to what the reference reads (runtime/weights/navi_file.cpp:79-148,
docs/navi-format.md:10-47) and what its converter writes (tools/convert.py:77-148):

    0   4   magic "NAVI"
    4   u32 version (1)
    8   u64 data_offset (multiple of 4096)
    16  u32 n_kv
    20  u32 n_tensors
    24  u64 file size
    32  KV entries, then tensor entries
    data_offset: tensor payloads, each starting on a 4096-byte boundary

KV entry: string key, u8 type (0 I64, 1 F64, 2 STR, 3 I64_ARRAY), value.
Tensor entry: string name, u8 dtype (0 F32, 1 F16, 2 BF16, 3 I32, 4 U8),
u8 ndim, ndim x u64 dims (outermost first), u64 offset (from data_offset),
u64 byte length.  Strings are u32 length + UTF-8 bytes.
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass, field
from pathlib import Path
from typing import Iterable

import numpy as np

VERSION = 1
PAGE = 4096

F32, F16, BF16, I32, U8 = 0, 1, 2, 3, 4
KV_I64, KV_F64, KV_STR, KV_I64_ARRAY = 0, 1, 2, 3

_NP = {F32: np.float32, F16: np.float16, I32: np.int32, U8: np.uint8}
_SIZE = {F32: 4, F16: 2, BF16: 2, I32: 4, U8: 1}


def _pstr(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<I", len(b)) + b


def _round_page(n: int) -> int:
    return (n + PAGE - 1) // PAGE * PAGE


class NaviWriter:
    """Accumulates KV entries and tensors, then writes one `.navi` file.

    Tensors are appended in insertion order; the reader and the device upload
    keep that order (plus adjacency groups), so callers that want two tensors
    adjacent on the device add them consecutively.
    """

    def __init__(self) -> None:
        self.kv: list[tuple[str, int, object]] = []
        self.tensors: list[tuple[str, int, tuple[int, ...], np.ndarray]] = []
        self._names: set[str] = set()

    def add_kv(self, key: str, value) -> None:
        if value is None:
            return
        if isinstance(value, bool):
            value = int(value)
        if isinstance(value, (int, np.integer)):
            self.kv.append((key, KV_I64, int(value)))
        elif isinstance(value, (float, np.floating)):
            self.kv.append((key, KV_F64, float(value)))
        elif isinstance(value, str):
            self.kv.append((key, KV_STR, value))
        elif isinstance(value, (list, tuple)) and all(isinstance(v, (int, np.integer)) for v in value):
            self.kv.append((key, KV_I64_ARRAY, [int(v) for v in value]))
        else:
            raise TypeError(f"{key}: a .navi KV cannot hold {type(value).__name__}")

    def add_tensor(self, name: str, dtype: int, arr: np.ndarray) -> None:
        if name in self._names:
            raise ValueError(f"duplicate tensor {name}")
        self._names.add(name)
        arr = np.ascontiguousarray(np.asarray(arr).astype(_NP[dtype], copy=False))
        self.tensors.append((name, dtype, tuple(int(d) for d in arr.shape), arr))

    def write(self, path: str | os.PathLike) -> int:
        path = Path(path)
        offsets, off = [], 0
        for _, _, _, arr in self.tensors:
            offsets.append(off)
            off += _round_page(arr.nbytes)
        table = bytearray()
        for key, kind, v in self.kv:
            table += _pstr(key) + struct.pack("<B", kind)
            if kind == KV_I64:
                table += struct.pack("<q", v)
            elif kind == KV_F64:
                table += struct.pack("<d", v)
            elif kind == KV_STR:
                table += _pstr(v)
            else:
                table += struct.pack("<I", len(v)) + b"".join(struct.pack("<q", x) for x in v)
        for (name, dtype, shape, arr), o in zip(self.tensors, offsets):
            table += _pstr(name) + struct.pack("<BB", dtype, len(shape))
            table += b"".join(struct.pack("<Q", d) for d in shape)
            table += struct.pack("<QQ", o, arr.nbytes)
        header_len = 32 + len(table)
        data_offset = _round_page(header_len)
        size = data_offset + off
        head = b"NAVI" + struct.pack("<IQIIQ", VERSION, data_offset, len(self.kv), len(self.tensors), size)
        tmp = path.with_name(path.name + ".tmp")
        with open(tmp, "wb") as f:
            f.write(head)
            f.write(table)
            f.write(b"\0" * (data_offset - header_len))
            for (name, _, _, arr), o in zip(self.tensors, offsets):
                assert f.tell() == data_offset + o, name
                f.write(arr.tobytes())
                pad = _round_page(arr.nbytes) - arr.nbytes
                if pad:
                    f.write(b"\0" * pad)
            assert f.tell() == size
        os.replace(tmp, path)
        return size


@dataclass
class TensorInfo:
    name: str
    dtype: int
    dims: tuple[int, ...]
    offset: int
    nbytes: int


@dataclass
class NaviFile:
    """Parsed `.navi` file; tensors are numpy views into a memory map."""

    path: str
    data_offset: int
    kv: dict = field(default_factory=dict)
    tensors: list[TensorInfo] = field(default_factory=list)
    _mm: np.memmap | None = None

    @staticmethod
    def open(path: str | os.PathLike) -> "NaviFile":
        path = str(path)
        mm = np.memmap(path, dtype=np.uint8, mode="r")
        raw = memoryview(mm)
        if bytes(raw[:4]) != b"NAVI":
            raise ValueError(f"{path}: bad magic; not a .navi file")
        version, data_offset, n_kv, n_t, size = struct.unpack_from("<IQIIQ", raw, 4)
        if version != VERSION:
            raise ValueError(f"{path}: .navi version {version} (this reader reads {VERSION})")
        if size != len(mm):
            raise ValueError(f"{path}: header says {size} bytes, file is {len(mm)}")
        if data_offset % PAGE or data_offset > size:
            raise ValueError(f"{path}: bad data_offset")
        p = 32

        def take(fmt):
            nonlocal p
            v = struct.unpack_from(fmt, raw, p)
            p += struct.calcsize(fmt)
            return v if len(v) > 1 else v[0]

        def pstr():
            nonlocal p
            n = take("<I")
            s = bytes(raw[p:p + n]).decode("utf-8")
            p += n
            return s

        f = NaviFile(path=path, data_offset=data_offset, _mm=mm)
        for _ in range(n_kv):
            key = pstr()
            kind = take("<B")
            if kind == KV_I64:
                f.kv[key] = take("<q")
            elif kind == KV_F64:
                f.kv[key] = take("<d")
            elif kind == KV_STR:
                f.kv[key] = pstr()
            elif kind == KV_I64_ARRAY:
                n = take("<I")
                f.kv[key] = [take("<q") for _ in range(n)]
            else:
                raise ValueError(f"{path}: kv '{key}' has unknown type {kind}")
        for _ in range(n_t):
            name = pstr()
            dtype, ndim = take("<BB")
            dims = tuple(take("<Q") for _ in range(ndim)) if ndim else ()
            if ndim == 1:
                dims = (dims,) if isinstance(dims, int) else dims
            off, nbytes = take("<QQ")
            numel = int(np.prod(dims)) if dims else 1
            if off % PAGE or data_offset + off + nbytes > size:
                raise ValueError(f"{path}: tensor '{name}' lies outside the file")
            if numel * _SIZE[dtype] != nbytes:
                raise ValueError(f"{path}: tensor '{name}' shape does not match its byte length")
            f.tensors.append(TensorInfo(name, dtype, dims, off, nbytes))
        return f

    def find(self, name: str) -> TensorInfo | None:
        for t in self.tensors:
            if t.name == name:
                return t
        return None

    def array(self, name_or_info) -> np.ndarray:
        t = name_or_info if isinstance(name_or_info, TensorInfo) else self.find(name_or_info)
        if t is None:
            raise KeyError(name_or_info)
        start = self.data_offset + t.offset
        buf = self._mm[start:start + t.nbytes]
        if t.dtype == BF16:
            u = buf.view(np.uint16).astype(np.uint32) << 16
            return u.view(np.float32).reshape(t.dims)
        return buf.view(_NP[t.dtype]).reshape(t.dims)

    def names(self) -> Iterable[str]:
        return (t.name for t in self.tensors)
