"""The `.navi` v1 weight blob: writer and reader.

The byte layout is the drop-in boundary with the reference engine, so it is
kept identical to what the reference reads (runtime/weights/navi_file.cpp:79-148,
docs/navi-format.md:10-47) and what its converter writes (tools/convert.py:106-148):

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
import tempfile
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


def _round_page(n: int) -> int:
    return -(-n // PAGE) * PAGE


def _encode_str(s: str) -> bytes:
    raw = s.encode("utf-8")
    return len(raw).to_bytes(4, "little") + raw


def _classify(value):
    """(kind, normalised value) of a hyperparameter, or None when the value is absent."""
    if value is None:
        return None
    if isinstance(value, (bool, int, np.integer)):
        return KV_I64, int(value)
    if isinstance(value, (float, np.floating)):
        return KV_F64, float(value)
    if isinstance(value, str):
        return KV_STR, value
    if isinstance(value, (list, tuple)):
        items = list(value)
        if all(isinstance(v, (bool, int, np.integer)) for v in items):
            return KV_I64_ARRAY, [int(v) for v in items]
    raise TypeError(f"a .navi hyperparameter holds an integer, a float, a string or a list of integers, "
                    f"not {type(value).__name__}")


_KV_BODY = {
    KV_I64: lambda v: struct.pack("<q", v),
    KV_F64: lambda v: struct.pack("<d", v),
    KV_STR: _encode_str,
    KV_I64_ARRAY: lambda v: struct.pack(f"<I{len(v)}q", len(v), *v),
}


class NaviBuilder:
    """Builds one `.navi` file: hyperparameters first, then tensors, laid out in one pass.

    Tensors keep the order they were put in; the reader and the device upload keep it too
    (plus the adjacency groups), so tensors wanted side by side on the device are put in
    one after the other.  `save` writes a temporary file beside the target and renames it
    into place, so a reader never sees a half-written file.
    """

    def __init__(self) -> None:
        self._hparams: dict[str, tuple[int, object]] = {}
        self._payloads: dict[str, tuple[int, np.ndarray]] = {}

    def set_kv(self, key: str, value) -> None:
        """Records a hyperparameter (None: skipped; a key set twice keeps the last value)."""
        typed = _classify(value)
        if typed is not None:
            self._hparams[key] = typed

    def put_tensor(self, name: str, dtype: int, arr) -> None:
        if name in self._payloads:
            raise ValueError(f"tensor {name!r} is already in this file")
        data = np.ascontiguousarray(np.asarray(arr), dtype=_NP[dtype])
        self._payloads[name] = (dtype, data)

    def _layout(self) -> tuple[bytes, list[int], int]:
        """The header bytes (page-padded), each payload's offset from the data region, and
        the file size."""
        offsets, cursor = [], 0
        for _, data in self._payloads.values():
            offsets.append(cursor)
            cursor += _round_page(data.nbytes)
        parts = []
        for key, (kind, value) in self._hparams.items():
            parts += [_encode_str(key), bytes([kind]), _KV_BODY[kind](value)]
        for (name, (dtype, data)), off in zip(self._payloads.items(), offsets):
            parts += [_encode_str(name), bytes([dtype, data.ndim]), struct.pack(f"<{data.ndim}Q", *data.shape),
                      struct.pack("<QQ", off, data.nbytes)]
        tables = b"".join(parts)
        data_offset = _round_page(32 + len(tables))
        total = data_offset + cursor
        preamble = b"NAVI" + struct.pack("<IQIIQ", VERSION, data_offset, len(self._hparams), len(self._payloads), total)
        header = (preamble + tables).ljust(data_offset, b"\0")
        return header, offsets, total

    def save(self, path: str | os.PathLike) -> int:
        """Writes the file; returns its size in bytes."""
        header, offsets, total = self._layout()
        target = Path(path)
        fd, tmp = tempfile.mkstemp(prefix=target.name + ".", suffix=".partial", dir=target.parent)
        try:
            with os.fdopen(fd, "wb") as out:
                out.write(header)
                for (_, data), off in zip(self._payloads.values(), offsets):
                    out.seek(len(header) + off)          # the gap to the page boundary reads as zeros
                    out.write(memoryview(data).cast("B"))
                out.truncate(total)
            os.replace(tmp, target)
        except BaseException:
            if os.path.exists(tmp):
                os.unlink(tmp)
            raise
        return total


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
