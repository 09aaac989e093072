"""MOSS text side on the GPU through hx_weights_load + hx_mega_block: the text-refiner block (MODE 1,
moss/hexagon/mega/blk.c:237 with the bias selector of mossrun.cpp:205-209) and the text projection
(MODE 2, blk.c:229-233), on reference-format packs (export_moss.py:43-65), against the oracle fed the
packs' exact device operands. Bar: rel-L2 of the block delta <= 2e-3."""
import numpy as np
import pytest
import torch

from hexanima_b200 import runtime as rt
from oracle import moss as om
from tests.gpu_util import read_f32, rel, write_f32

pytestmark = pytest.mark.gpu
TOL = 2e-3
D, F, TW = 3072, 8192, 4096


@pytest.fixture(scope="module")
def h():
    hd = rt.Handle(0)
    yield hd
    assert hd.status() == 0
    hd.close()


def _fill_selectors(h, bfd, meta, rows):
    S = rt.S
    for slot, width in (("LQ", 384), ("LO", 128), ("LU", 128), ("LD", 128)):
        h.buf_write(bfd, meta[S[slot]], om.selector((rows,), width).half().numpy())


def test_moss_refiner_block_mode1(h):
    w = om.init_text_weights(70, D=D, F=F, blocks=1)
    pack = om.build_refiner_pack(w, 0)
    assert len(pack) == 135397376          # same size as a DiT block pack
    wfd = h.weights_load(rt.MODEL_MOSS, pack)
    mats, gain = om.pack_mats(pack)
    Tt, T = 20, 32
    g = torch.Generator().manual_seed(71)
    x = torch.randn(1, T, D, generator=g) * 2
    mod = torch.zeros(6, D)
    mod[2] = 1.0
    mod[5] = 1.0
    c, s = rt.rope_moss(0, 1, Tt, om.bands16().numpy(), T)
    meta, total = rt.blob_layout(rt.MODEL_MOSS, T, 0, 1, D, F)
    S = rt.S
    meta[S["NVALID"]] = Tt
    meta[S["MODE"]] = 1
    bfd = h.buf_alloc(total)
    write_f32(h, bfd, meta[S["X"]], x.numpy())
    write_f32(h, bfd, meta[S["COS"]], c)
    write_f32(h, bfd, meta[S["SIN"]], s)
    _fill_selectors(h, bfd, meta, T)
    h.mega_block(meta, wfd, bfd, mod=mod.numpy())
    y = torch.from_numpy(read_f32(h, bfd, meta[S["X"]], T * D).reshape(1, T, D))
    h.buf_free(bfd)
    ref = om.block_dev(x, mod, torch.from_numpy(c), torch.from_numpy(s), mats, gain, nvalid=Tt, lora=True,
                       refiner=True)
    assert rel(y[:, :Tt] - x[:, :Tt], ref[:, :Tt] - x[:, :Tt]) < TOL
    h.weights_free(wfd)


def test_moss_text_projection_mode2(h):
    w = om.init_text_weights(72, D=D, F=256, blocks=0)
    pack = om.build_proj_pack(w)
    wfd = h.weights_load(rt.MODEL_MOSS_PROJ, pack)
    Tt, T = 20, 32
    g = torch.Generator().manual_seed(73)
    txt = torch.randn(T, TW, generator=g).half()
    x0 = torch.randn(1, T, D, generator=g)           # the projection adds into whatever X holds
    mod = torch.zeros(6, D)
    mod[2] = 1.0
    meta, total = rt.blob_layout(rt.MODEL_MOSS, T, 0, 1, D, F, Cd=TW)
    S = rt.S
    meta[S["NVALID"]] = Tt
    meta[S["MODE"]] = 2
    bfd = h.buf_alloc(total)
    write_f32(h, bfd, meta[S["X"]], x0.numpy())
    h.buf_write(bfd, meta[S["H"]], txt.numpy())
    _fill_selectors(h, bfd, meta, T)
    h.mega_block(meta, wfd, bfd, mod=mod.numpy())
    y = torch.from_numpy(read_f32(h, bfd, meta[S["X"]], T * D).reshape(1, T, D))
    h.buf_free(bfd)
    m = om.proj_mat(pack)
    ref = txt.float() @ m[:, :TW].T + m[:, TW]
    assert rel(y[0] - x0[0], ref) < TOL
    # the projection weight set serves only MODE 2, a block pack never does
    meta[S["MODE"]] = 0
    bfd = h.buf_alloc(total)
    with pytest.raises(rt.HxError):
        h.mega_block(meta, wfd, bfd, mod=mod.numpy())
    h.buf_free(bfd)
    h.weights_free(wfd)
