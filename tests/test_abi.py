"""C-ABI surface of libhxdit.so without a GPU: it loads, exports every function include/hxdit.h
declares, the ctypes structs match the C layout, and the host-side helpers agree with the oracle."""
import ctypes
import os
import re
import subprocess
import tempfile

import numpy as np
import pytest
import torch

from hexanima_b200 import build, runtime as rt
from oracle import anima as oa
from oracle import moss as om

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "hxdit.h")


@pytest.fixture(scope="module", autouse=True)
def built():
    build.build()


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"HX_API\s+(?:const\s+char\*|int)\s+(hx_\w+)\s*\(", src)))


def test_every_declared_symbol_is_exported():
    names = declared()
    assert len(names) >= 20
    L = ctypes.CDLL(rt.LIB_PATH)
    for n in names:
        assert hasattr(L, n), n
    assert sorted(rt.exported_symbols()) == names


def test_struct_layouts_match_header():
    prog = r"""
#include <stdio.h>
#include <stddef.h>
#include "hxdit.h"
int main(void) {
  printf("%zu %zu %zu %zu\n", sizeof(hx_mat), sizeof(hx_weight_desc), sizeof(hx_gemm_desc), sizeof(hx_attn_desc));
  printf("%zu %zu %zu\n", offsetof(hx_gemm_desc, w), offsetof(hx_gemm_desc, vec_bstride), offsetof(hx_gemm_desc, eps));
  printf("%zu %zu\n", offsetof(hx_weight_desc, gain), offsetof(hx_attn_desc, scale));
  return 0;
}
"""
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        open(c, "w").write(prog)
        exe = os.path.join(d, "t")
        subprocess.check_call(["gcc", "-I", os.path.dirname(HEADER), c, "-o", exe])
        out = subprocess.check_output([exe]).decode().split()
    got = [int(v) for v in out]
    exp = [ctypes.sizeof(rt.hx_mat), ctypes.sizeof(rt.hx_weight_desc), ctypes.sizeof(rt.hx_gemm_desc),
           ctypes.sizeof(rt.hx_attn_desc), rt.hx_gemm_desc.w.offset, rt.hx_gemm_desc.vec_bstride.offset,
           rt.hx_gemm_desc.eps.offset, rt.hx_weight_desc.gain.offset, rt.hx_attn_desc.scale.offset]
    assert got == exp


def test_version():
    assert "sm_100a" in rt.version()


def test_blob_layout_anima():
    meta, total = rt.blob_layout(rt.MODEL_ANIMA, 1536, 256, 2, 2048, 8192, 1024)
    A = rt.A
    assert meta[A["NTOK"]] == 1536 and meta[A["NCTX"]] == 256 and meta[A["BATCH"]] == 2
    offs = [meta[A[s]] for s in ("X", "CTX", "MOD", "COS", "SIN", "H", "Q", "O", "MID", "CK")]
    assert all(o % 4096 == 0 for o in offs) and offs == sorted(offs)
    assert meta[A["CTX"]] - meta[A["X"]] >= 2 * 1536 * 2048 * 4
    assert meta[A["MID"]] + 2 * 1536 * 8192 * 2 <= meta[A["CK"]]
    assert total >= meta[A["CK"]] + 2 * 256 * 4096 * 2


def test_blob_layout_moss_and_limits():
    meta, total = rt.blob_layout(rt.MODEL_MOSS, 4608, 0, 1, 3072, 12288)
    S = rt.S
    assert meta[S["NTOK"]] == 4608 and meta[S["NVALID"]] == 4608 and meta[S["NCB"]] == 96
    assert total < 2 ** 31
    with pytest.raises(rt.HxError):
        rt.blob_layout(rt.MODEL_MOSS, 100, 0, 1, 3072, 8192)   # ntok not a multiple of 32
    with pytest.raises(rt.HxError):
        rt.blob_layout(rt.MODEL_MOSS, 6656, 0, 8, 3072, 12288)  # past the int32 byte offsets of meta[]


def test_rope_anima_matches_oracle():
    c, s = rt.rope_anima(48, 32, 10000.0, 1536)
    oc, osn = oa.make_rope(48, 32, 10000.0, 1536)
    np.testing.assert_allclose(c, oc, atol=2e-7)
    np.testing.assert_allclose(s, osn, atol=2e-7)
    c2, _ = rt.rope_anima(4, 8, 10000.0 * 4 ** (42 / 40), 64)  # NTK theta of PITFALLS:70, padded rows zero
    assert np.all(c2[32:] == 0)


def test_rope_moss_matches_oracle():
    bands = om.bands16()
    c, s = rt.rope_moss(4, 6, 16, bands.numpy(), 64)
    osin, ocos = om.rope_tables(4, 6, 16, bands)
    np.testing.assert_allclose(c[:40], ocos[:, :64].numpy(), atol=3e-6)
    np.testing.assert_allclose(s[:40], osin[:, :64].numpy(), atol=3e-6)
    assert np.all(c[40:] == 0)


def test_open_without_gpu_fails_cleanly():
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(rt.HxError):
        rt.Handle(0)
