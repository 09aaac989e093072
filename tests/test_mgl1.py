"""MOSS glue files (glue.bin, "MGL1") read through hx_mgl1_tensor (CPU only).

The writer below restates moss/export_glue.py:17-23 with struct: "MGL1", int32 count, 76-byte entries
{char name[40]; int32 dtype (0 f32, 1 f16); int32 nd; int32 dims[3]; int64 offset; int64 bytes}, data at
128-byte aligned offsets."""
import struct

import numpy as np
import pytest

from hexanima_b200 import runtime as rt


def write_mgl1(tensors):
    """tensors: [(name, dtype 0|1, array)] -> file bytes."""
    hdr = 8 + len(tensors) * 76
    off = (hdr + 127) // 128 * 128
    ent, data = b"", []
    for name, dt, a in tensors:
        a = np.ascontiguousarray(a, np.float16 if dt else np.float32)
        d = list(a.shape) + [1] * (3 - a.ndim)
        ent += struct.pack("<40sii3iqq", name.encode(), dt, a.ndim, *d, off, a.nbytes)
        data.append((off, a.tobytes()))
        off = (off + a.nbytes + 127) // 128 * 128
    out = bytearray(off)
    head = b"MGL1" + struct.pack("<i", len(tensors)) + ent
    out[:len(head)] = head
    for o, b in data:
        out[o:o + len(b)] = b
    return bytes(out)


def test_mgl1_lookup():
    rng = np.random.default_rng(5)
    a = rng.standard_normal((48, 128)).astype(np.float32)
    b = rng.standard_normal(7).astype(np.float16)
    codes = np.array([1000, 968, 926, 871], np.float32)
    f = write_mgl1([("video_embedder.weight", 0, a), ("x.h", 1, b), ("step_codes", 0, codes)])
    assert np.array_equal(rt.mgl1_tensor(f, "video_embedder.weight"), a)
    assert np.array_equal(rt.mgl1_tensor(f, "x.h"), b)
    assert np.array_equal(rt.mgl1_tensor(f, "step_codes"), codes)
    with pytest.raises(rt.HxError) as e:
        rt.mgl1_tensor(f, "rope.bands")
    assert e.value.rc == rt.HX_E_RANGE


def _corrupt(f, at, fmt, value):
    g = bytearray(f)
    g[at:at + struct.calcsize(fmt)] = struct.pack(fmt, value)
    return bytes(g)


def test_mgl1_malformed_files_are_rejected():
    f = write_mgl1([("a", 0, np.ones((4, 4), np.float32))])
    bad = [b"MGL2" + f[4:],                      # magic
           f[:8 + 40],                           # entry table cut short
           _corrupt(f, 4, "<i", 1000),           # count beyond the file
           _corrupt(f, 8 + 60, "<q", len(f)),    # data offset at the end of the file
           _corrupt(f, 8 + 68, "<q", 60),        # bytes disagree with dims x dtype
           _corrupt(f, 8 + 40, "<i", 3)]         # unknown dtype
    for g in bad:
        with pytest.raises(rt.HxError) as e:
            rt.mgl1_tensor(g, "a")
        assert e.value.rc == rt.HX_E_FORMAT
