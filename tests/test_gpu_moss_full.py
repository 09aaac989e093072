"""MOSS blocks at the full sizes of the MOSS configurations (hidden 3072, 24 heads, MLP 12288), through
hx_mega_block, against the oracle block (oracle.moss.block_dev, the staged device-weight form of
moss_ref.block / mkblk_test.py:38-55) fed the exact dequantised operands.

* 1 Mpx with q4 weights: 4096 image tokens + 512 text tokens in one joint attention (4608 tokens).
* 6144 patches + 512 text tokens with q8 weights, LoRA rank-128 slots, and a rank-64 delta (scale 1.0)
  folded into the q8 base tiles on the device first (hx_lora_fold); two images, the second compared.

Bar: rel-L2 of the block delta (x_out - x_in) over the valid tokens <= 2e-3; the folded bytes of the
o projection identical to oracle.packs.lora_fold_q8."""
import numpy as np
import pytest
import torch

from hexanima_b200 import runtime as rt
from oracle import moss as om
from oracle import packs as op
from tests.gpu_util import dev, make_mat, read_f32, rel, write_f32

pytestmark = pytest.mark.gpu
TOL = 2e-3
D, F, HEADS = 3072, 12288, 24


@pytest.fixture(scope="module")
def h():
    hd = rt.Handle(0)
    yield hd
    assert hd.status() == 0
    hd.close()


def _gain(seed):
    g = torch.Generator().manual_seed(seed)
    gain = torch.cat((1 + 0.1 * torch.randn(128, generator=g), 1 + 0.1 * torch.randn(128, generator=g),
                      1 + 0.1 * torch.randn(2 * D, generator=g)))
    gain[:128] /= np.sqrt(128.0)  # the pack folds 1/sqrt(128) into the q gain
    return gain


def _run(h, wfd, x, mod, cos, sin, nvalid):
    B, T, _ = x.shape
    meta, total = rt.blob_layout(rt.MODEL_MOSS, T, 0, B, D, F)
    S = rt.S
    meta[S["NVALID"]] = nvalid
    bfd = h.buf_alloc(total)
    write_f32(h, bfd, meta[S["X"]], x.numpy())
    write_f32(h, bfd, meta[S["COS"]], cos.numpy())
    write_f32(h, bfd, meta[S["SIN"]], sin.numpy())
    h.mega_block(meta, wfd, bfd, mod=mod.numpy())
    y = read_f32(h, bfd, meta[S["X"]], B * T * D).reshape(B, T, D)
    h.buf_free(bfd)
    return torch.from_numpy(y)


def test_moss_1mpx_q4_block(h):
    """Config: MOSS-Image at 1 Mpx (1024x1024 -> 64x64 patches) with int4 weights in groups of 32."""
    Hh, Ww, Tt = 64, 64, 512
    T = nvalid = Hh * Ww + Tt
    g = torch.Generator().manual_seed(80)
    W = {"qkv": torch.randn(3 * D, D, generator=g) * 0.02, "o": torch.randn(D, D, generator=g) * 0.02,
         "up": torch.randn(F, D, generator=g) * 0.02, "gate": torch.randn(F, D, generator=g) * 0.02,
         "dn": torch.randn(D, F, generator=g) * 0.02}
    mats, keep, deq = {}, [], {}
    for slot, name, w in ((rt.W_QKV, "qkv", W["qkv"].numpy()), (rt.W_O, "o", W["o"].numpy()),
                          (rt.W_M1, "ug", op.situ_rows(W["up"].numpy(), W["gate"].numpy())),
                          (rt.W_M2, "dn", W["dn"].numpy())):
        mats[slot], k, deq[name] = make_mat(rt.FMT_Q4, w, 32)
        keep += k
    gain = _gain(81)
    tg = gain.cuda()
    wfd = h.weights_bind(rt.MODEL_MOSS, D, F, mats, tg, lora=0, keep=keep + [tg])
    x = torch.randn(1, T, D, generator=g) * 2
    mod = torch.randn(6, D, generator=g) * 0.1
    c, s = rt.rope_moss(Hh, Ww, Tt, om.bands16().numpy(), T)
    cos, sin = torch.from_numpy(c), torch.from_numpy(s)
    y = _run(h, wfd, x, mod, cos, sin, nvalid)
    h.weights_free(wfd)
    ref = om.block_dev(x, mod, cos, sin, deq, gain, nvalid=nvalid, lora=False)
    assert rel(y - x, ref - x) < TOL


def test_moss_6144_q8_lora_fold_block(h):
    """Config: 6144 patches (e.g. 1536x1024) + 512 text tokens, q8 weights with the rank-128 LoRA slots
    (LoRA-B rows as 128 extra K columns, LoRA-A matrices), a rank-64 delta folded into every base
    matrix on the device before the block; batch 2, the second image checked."""
    Hh, Ww, Tt = 64, 96, 512
    nvalid = Hh * Ww + Tt
    T = (nvalid + 31) // 32 * 32
    B, group, rank = 2, 32, 64
    g = torch.Generator().manual_seed(90)
    shapes = {rt.W_Q: (D, D + 128), rt.W_K: (D, D + 128), rt.W_V: (D, D + 128), rt.W_O: (D, D + 128),
              rt.W_M1: (2 * F, D + 128), rt.W_M2: (D, F + 128), rt.W_AQKV: (384, D), rt.W_AO: (128, D),
              rt.W_AUG: (128, D), rt.W_ADN: (128, F)}
    mats, dv = {}, {}
    for slot, (n, k) in shapes.items():
        u, sc = op.quant_q8((torch.randn(n, k, generator=g) * 0.02).numpy(), group)
        tu, ts = dev(u), dev(sc)
        mats[slot] = rt.make_mat(rt.FMT_Q8, n, k, tu, ts, group=group)
        dv[slot] = (tu, ts)
    gain = _gain(91)
    tg = gain.cuda()
    wfd = h.weights_bind(rt.MODEL_MOSS, D, F, mats, tg, lora=1, keep=[t for p in dv.values() for t in p] + [tg])
    # rank-64 delta, scale 1.0, into the base columns of every LoRA-carrying matrix
    u_o0, s_o0 = dv[rt.W_O][0].cpu().numpy(), dv[rt.W_O][1].cpu().numpy()
    fac = {}
    for slot, k_base in ((rt.W_Q, D), (rt.W_K, D), (rt.W_V, D), (rt.W_O, D), (rt.W_M1, D), (rt.W_M2, F)):
        n = shapes[slot][0]
        fac[slot] = ((torch.randn(n, rank, generator=g) * 0.02).numpy(), (torch.randn(rank, k_base, generator=g) * 0.02).numpy())
        h.lora_fold(wfd, slot, dev(fac[slot][0]), dev(fac[slot][1]), rank, 1.0)
    h.sync()
    want_u, want_s = op.lora_fold_q8(u_o0, s_o0, group, fac[rt.W_O][0], fac[rt.W_O][1], 1.0, floor=op.F16_FLOOR_MOSS,
                                     k_base=D)
    assert np.array_equal(dv[rt.W_O][0].cpu().numpy(), want_u)
    assert np.array_equal(dv[rt.W_O][1].cpu().numpy().view(np.uint16), want_s.view(np.uint16))
    names = {rt.W_Q: "q", rt.W_K: "k", rt.W_V: "v", rt.W_O: "o", rt.W_M1: "ug", rt.W_M2: "dn", rt.W_AQKV: "aqkv",
             rt.W_AO: "ao", rt.W_AUG: "aug", rt.W_ADN: "adn"}
    deq = {names[slot]: torch.from_numpy(op.dequant_q8(dv[slot][0].cpu().numpy(), dv[slot][1].cpu().numpy(),
                                                       group).astype(np.float32)) for slot in shapes}
    x = torch.randn(B, T, D, generator=g) * 2
    mod = torch.randn(6, D, generator=g) * 0.1
    c, s = rt.rope_moss(Hh, Ww, Tt, om.bands16().numpy(), T)
    cos, sin = torch.from_numpy(c), torch.from_numpy(s)
    y = _run(h, wfd, x, mod, cos, sin, nvalid)
    h.weights_free(wfd)
    ref = om.block_dev(x[1:], mod, cos, sin, deq, gain, nvalid=nvalid, lora=True)
    assert rel(y[1:, :nvalid] - x[1:, :nvalid], ref[:, :nvalid] - x[1:, :nvalid]) < TOL
