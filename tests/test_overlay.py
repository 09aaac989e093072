"""LoRA overlay files (blkNN.ovl) applied to block packs through hx_pack_apply_overlay (CPU only).

The file layout is the one moss/make_lora_overlay.py:54-56 and moss/mossrun/lorafold.cpp:284-288
write: little-endian u32 record count, then per record u64 byte offset into the pack, u32 length
and the bytes. The writer below restates it with struct, as the reference script does."""
import struct

import numpy as np
import pytest

from hexanima_b200 import runtime as rt


def _ovl(records):
    out = struct.pack("<I", len(records))
    for off, data in records:
        out += struct.pack("<QI", off, len(data)) + bytes(data)
    return out


def test_overlay_records_patch_the_pack():
    rng = np.random.default_rng(3)
    pack = bytearray(rng.integers(0, 256, 1 << 16, dtype=np.uint8).tobytes())
    recs = [(0, rng.integers(0, 256, 1152, dtype=np.uint8).tobytes()),
            (40000, rng.integers(0, 256, 4 * 1152, dtype=np.uint8).tobytes()),
            ((1 << 16) - 7, b"\x01\x02\x03\x04\x05\x06\x07"),       # ends exactly at the pack end
            (1000, b"\xaa" * 10), (1005, b"\xbb" * 10)]                  # overlapping: file order wins
    want = bytearray(pack)
    for off, data in recs:
        want[off:off + len(data)] = data
    rt.pack_apply_overlay(pack, _ovl(recs))
    assert pack == want


def test_overlay_with_no_records_is_a_no_op():
    pack = bytearray(b"\x11" * 64)
    rt.pack_apply_overlay(pack, _ovl([]))
    assert pack == bytearray(b"\x11" * 64)


@pytest.mark.parametrize("bad", [
    _ovl([(60, b"\x00" * 8)]),                       # record runs past the 64-byte pack
    _ovl([(1 << 40, b"\x00")]),                      # offset far outside
    _ovl([(0, b"\x00" * 8)])[:-3],                   # truncated data
    _ovl([(0, b"\x00" * 8)]) + b"\x00",              # trailing bytes after the last record
    struct.pack("<I", 2) + struct.pack("<QI", 0, 1) + b"\x00",   # count says 2, one present
    b"\x01\x00",                                     # shorter than the count field
])
def test_malformed_overlay_is_rejected_and_pack_untouched(bad):
    pack = bytearray(b"\x22" * 64)
    with pytest.raises(rt.HxError) as e:
        rt.pack_apply_overlay(pack, bad)
    assert e.value.rc in (rt.HX_E_FORMAT, rt.HX_E_ARG)
    assert pack == bytearray(b"\x22" * 64)
