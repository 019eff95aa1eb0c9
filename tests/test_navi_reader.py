"""The C++ .navi reader and tensor-table check (navi_model_probe: NaviFile::open,
read_params, validate), on the CPU: it accepts the file the Python builder writes and reads
the same hyperparameters as the Python reader and the reference's own reader (the golden
fixture), and it refuses malformed files with NAVI_E_FORMAT and a message naming the fault
(the reference's checks, runtime/weights/navi_file.cpp:79-148 and
model/qwen3tts/params.cpp:286-303)."""
import ctypes
import json
import os
import shutil
import struct

import numpy as np
import pytest

from navi_b200 import capi, model_spec
from navi_b200.navi_file import NaviBuilder, NaviFile

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _probe(path):
    L = capi.lib()
    p = capi.Params()
    n = [ctypes.c_int(-1) for _ in range(4)]
    st = L.navi_model_probe(str(path).encode(), ctypes.byref(p), *[ctypes.byref(x) for x in n])
    return st, p, [x.value for x in n], L.navi_last_error().decode()


def test_probe_accepts_the_synthetic_model(small_navi):
    st, p, (nt, miss, mis, unused), err = _probe(small_navi)
    assert st == capi.NAVI_OK, err
    ref = json.load(open(os.path.join(GOLDEN, "navi_ref_small.json")))
    assert (miss, mis) == (0, 0) and nt == ref["n_tensors"]
    t, c = p.talker, p.cp
    assert [t.hidden, t.n_layer, t.n_head, t.n_kv_head, t.head_dim, t.ff, t.vocab] == ref["talker"]
    assert [c.hidden, c.n_layer, c.n_head, c.n_kv_head, c.head_dim, c.ff, c.vocab] == ref["cp"]
    assert p.codec_eos_id == ref["codec_eos"] and p.decoder_dim == ref["decoder_dim"]
    assert np.float32(t.rms_eps) == np.float32(ref["rms_eps"]) and t.rope_theta == ref["rope_theta"]
    f = NaviFile.open(small_navi)
    assert len(f.tensors) == nt


def _patched(src, dst, at, raw):
    shutil.copy(src, dst)
    with open(dst, "r+b") as f:
        f.seek(at)
        f.write(raw)
    return dst


def _table_entry_offset(path, name):
    """Byte offset of tensor `name`'s table entry (its name length word)."""
    blob = open(path, "rb").read(NaviFile.open(path).data_offset)
    key = struct.pack("<I", len(name)) + name.encode()
    at = blob.find(key)
    assert at > 0
    return at


@pytest.mark.parametrize("fault", ["magic", "version", "size", "data_offset", "dtype", "extent", "length", "truncated"])
def test_probe_refuses_malformed_files(small_navi, tmp_path, fault):
    dst = tmp_path / f"{fault}.navi"
    name = "talker.model.norm.weight"
    if fault == "magic":
        _patched(small_navi, dst, 0, b"NAVX")
        want = "NAVI"
    elif fault == "version":
        _patched(small_navi, dst, 4, struct.pack("<I", 2))
        want = "version 2"
    elif fault == "size":
        _patched(small_navi, dst, 24, struct.pack("<Q", os.path.getsize(small_navi) + 1))
        want = "truncated"
    elif fault == "data_offset":
        _patched(small_navi, dst, 8, struct.pack("<Q", 4097))
        want = "data offset"
    else:
        at = _table_entry_offset(small_navi, name) + 4 + len(name)
        if fault == "dtype":
            _patched(small_navi, dst, at, bytes([9]))
            want = "dtype code 9"
        elif fault == "extent":
            _patched(small_navi, dst, at + 2 + 8, struct.pack("<Q", 1 << 40))     # rank 1: dims, then offset
            want = "past the end of the file"
        elif fault == "length":
            _patched(small_navi, dst, at + 2 + 8 + 8, struct.pack("<Q", 12))      # byte length
            want = "elements but 12 bytes"
        else:
            shutil.copy(small_navi, dst)
            with open(dst, "r+b") as f:
                f.truncate(os.path.getsize(small_navi) - 4096)
            want = "truncated"
    st, _, _, err = _probe(dst)
    assert st == capi.NAVI_E_FORMAT and want in err, err


def test_probe_reports_missing_and_duplicate_tensors(tmp_path):
    c = model_spec.small_config()
    dst = tmp_path / "missing.navi"
    model_spec.write_synthetic(dst, c, include=lambda n: n != "talker.codec_head.weight")
    st, _, (nt, miss, mis, _), err = _probe(dst)
    assert st == capi.NAVI_E_FORMAT and miss == 1 and "talker.codec_head.weight" in err
    # the builder refuses a duplicate; a file that has one anyway is refused by the reader
    b = NaviBuilder()
    b.put_tensor("a", 0, np.zeros(4, np.float32))
    with pytest.raises(ValueError):
        b.put_tensor("a", 0, np.zeros(4, np.float32))
    b.put_tensor("b", 0, np.ones(4, np.float32))
    dup = tmp_path / "dup.navi"
    b.save(dup)
    raw = bytearray(open(dup, "rb").read())
    at = raw.find(struct.pack("<I", 1) + b"b")
    raw[at + 4] = ord("a")
    open(dup, "wb").write(bytes(raw))
    st, _, _, err = _probe(dup)
    assert st == capi.NAVI_E_FORMAT and "twice" in err, err


def test_builder_round_trip(tmp_path):
    b = NaviBuilder()
    b.set_kv("general.name", "x")
    b.set_kv("n", 3)
    b.set_kv("f", 0.5)
    b.set_kv("arr", [1, -2, 3])
    b.set_kv("skipped", None)
    w16 = (np.arange(12, dtype=np.float32).reshape(3, 4) / 7).astype(np.float16)
    b.put_tensor("w", 1, w16)
    b.put_tensor("v", 0, np.linspace(0, 1, 5, dtype=np.float32))
    size = b.save(tmp_path / "rt.navi")
    assert size == os.path.getsize(tmp_path / "rt.navi") and size % 4096 == 0
    f = NaviFile.open(tmp_path / "rt.navi")
    assert f.kv == {"general.name": "x", "n": 3, "f": 0.5, "arr": [1, -2, 3]}
    assert [t.name for t in f.tensors] == ["w", "v"] and all(t.offset % 4096 == 0 for t in f.tensors)
    assert np.array_equal(f.array("w"), w16) and np.array_equal(f.array("v"), np.linspace(0, 1, 5, dtype=np.float32))
