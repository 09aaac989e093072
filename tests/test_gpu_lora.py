"""On-device LoRA fold into q8 weights (hx_lora_fold) against the oracle restatement
(oracle.packs.lora_fold_q8, the requantisation rule of moss/mossrun/lorafold.cpp:138-156).

Bars: the folded bytes and fp16 scales are identical to the oracle's; a block run on the folded
weights matches the oracle block fed the dequantised folded weights within the block bar (2e-3)."""
import numpy as np
import pytest
import torch

from hexanima_b200 import runtime as rt
from oracle import anima as oa
from oracle import moss as om
from oracle import packs as op
from tests.gpu_util import dev, rel, read_f32, write_f32

pytestmark = pytest.mark.gpu
TOL = 2e-3


@pytest.fixture(scope="module")
def h():
    hd = rt.Handle(0)
    yield hd
    assert hd.status() == 0
    hd.close()


def _factors(N, K, rank, seed, amp=0.03):
    g = torch.Generator().manual_seed(seed)
    return ((torch.randn(N, rank, generator=g) * amp).numpy(), (torch.randn(rank, K, generator=g) * amp).numpy())


def _q8(w, group):
    u, s = op.quant_q8(np.asarray(w, np.float32), group)
    tu, ts = dev(u), dev(s)
    return rt.make_mat(rt.FMT_Q8, u.shape[0], u.shape[1], tu, ts, group=group), tu, ts


def _deq(tu, ts, group):
    return torch.from_numpy(op.dequant_q8(tu.cpu().numpy(), ts.cpu().numpy(), group).astype(np.float32))


@pytest.mark.parametrize("group", [64, 32])
def test_anima_fold_bytes_and_block(h, group):
    D, F, Cd, B, T, C = 256, 512, 128, 1, 256, 64
    W, norms, modA, modB = oa.init_weights(60, D=D, F=F, Cd=Cd)
    fused = {rt.W_QKV: torch.cat((W["sq"], W["sk"], W["sv"]), 0), rt.W_O: W["so"], rt.W_CQ: W["cq"],
             rt.W_CKV: torch.cat((W["ck"], W["cv"]), 0), rt.W_CO: W["co"], rt.W_M1: W["m1"], rt.W_M2: W["m2"]}
    mats, dv = {}, {}
    for slot, w in fused.items():
        mats[slot], tu, ts = _q8(w.numpy(), group)
        dv[slot] = (tu, ts)
    gain = oa.pack_gain(norms)
    tg, tA, tB = gain.cuda(), modA.cuda().contiguous(), modB.cuda().contiguous()
    wfd = h.weights_bind(rt.MODEL_ANIMA, D, F, mats, tg, Cd=Cd, modA=tA, modB=tB,
                         keep=[t for p in dv.values() for t in p] + [tg, tA, tB])
    # (slot, rank, scale): a rank that is not a multiple of the 32-wide staging chunk, and the maximum
    for slot, rank, scale in ((rt.W_QKV, 64, 1.0), (rt.W_M1, 128, 1.0), (rt.W_M2, 7, 0.5)):
        tu, ts = dv[slot]
        u0, s0 = tu.cpu().numpy(), ts.cpu().numpy()
        N, K = u0.shape
        Bf, Af = _factors(N, K, rank, seed=slot)
        tb, ta = dev(Bf), dev(Af)
        h.lora_fold(wfd, slot, tb, ta, rank, scale)
        h.sync()
        want_u, want_s = op.lora_fold_q8(u0, s0, group, Bf, Af, scale, floor=op.F16_FLOOR_ANIMA)
        assert np.array_equal(tu.cpu().numpy(), want_u), slot
        assert np.array_equal(ts.cpu().numpy().view(np.uint16), want_s.view(np.uint16)), slot
        assert not np.array_equal(want_u, u0)  # the delta moved some weights
    # the block runs on the folded weights
    deq = {slot: _deq(*dv[slot], group) for slot in fused}
    Wd = {"sq": deq[rt.W_QKV][:D], "sk": deq[rt.W_QKV][D:2 * D], "sv": deq[rt.W_QKV][2 * D:], "so": deq[rt.W_O],
          "cq": deq[rt.W_CQ], "ck": deq[rt.W_CKV][:D], "cv": deq[rt.W_CKV][D:], "co": deq[rt.W_CO],
          "m1": deq[rt.W_M1], "m2": deq[rt.W_M2]}
    g = torch.Generator().manual_seed(61)
    x = torch.randn(B, T, D, generator=g)
    ctx = torch.randn(B, C, Cd, generator=g).half().float()
    mod = torch.randn(9, D, generator=g) * 0.1
    c, s = oa.make_rope(16, 16, ntok=T)
    cos, sin = torch.from_numpy(c), torch.from_numpy(s)
    meta, total = rt.blob_layout(rt.MODEL_ANIMA, T, C, B, D, F, Cd)
    bfd = h.buf_alloc(total)
    A = rt.A
    write_f32(h, bfd, meta[A["X"]], x.numpy())
    h.buf_write(bfd, meta[A["CTX"]], ctx.half().numpy())
    write_f32(h, bfd, meta[A["COS"]], c)
    write_f32(h, bfd, meta[A["SIN"]], s)
    h.mega_block(meta, wfd, bfd, mod=mod.numpy())
    y = torch.from_numpy(read_f32(h, bfd, meta[A["X"]], B * T * D).reshape(B, T, D))
    h.buf_free(bfd)
    ref = oa.block(x, ctx, mod, cos, sin, Wd, gain)
    assert rel(y - x, ref - x) < TOL
    h.weights_free(wfd)


def test_moss_fold_with_lora_rows_and_situ_order(h):
    """MOSS q8 matrices with the 128 LoRA-B K rows (export_moss.py:14-27): only the base columns change;
    up_gate takes B in logical [up; gate] row order and the device holds it regrouped per 256 rows."""
    D, F, B, group = 256, 256, 1, 32
    torch.manual_seed(62)
    shapes = {rt.W_Q: (D, D + 128), rt.W_K: (D, D + 128), rt.W_V: (D, D + 128), rt.W_O: (D, D + 128),
              rt.W_M1: (2 * F, D + 128), rt.W_M2: (D, F + 128), rt.W_AQKV: (384, D), rt.W_AO: (128, D),
              rt.W_AUG: (128, D), rt.W_ADN: (128, F)}
    mats, dv = {}, {}
    for slot, (N, K) in shapes.items():
        mats[slot], tu, ts = _q8((torch.randn(N, K) * 0.02).numpy(), group)
        dv[slot] = (tu, ts)
    gain = torch.cat((1 + 0.1 * torch.randn(128), 1 + 0.1 * torch.randn(128), 1 + 0.1 * torch.randn(2 * D)))
    gain[:128] /= np.sqrt(128.0)
    tg = gain.cuda()
    wfd = h.weights_bind(rt.MODEL_MOSS, D, F, mats, tg, lora=1, keep=[t for p in dv.values() for t in p] + [tg])
    for slot, k_base, rank in ((rt.W_M1, D, 64), (rt.W_Q, D, 64), (rt.W_M2, F, 33)):
        tu, ts = dv[slot]
        u0, s0 = tu.cpu().numpy(), ts.cpu().numpy()
        N = u0.shape[0]
        Bf, Af = _factors(N, k_base, rank, seed=100 + slot)      # B in logical row order
        h.lora_fold(wfd, slot, dev(Bf), dev(Af), rank, 1.0)
        h.sync()
        Bd = Bf[op.situ_logical_rows(N)] if slot == rt.W_M1 else Bf
        want_u, want_s = op.lora_fold_q8(u0, s0, group, Bd, Af, 1.0, floor=op.F16_FLOOR_MOSS, k_base=k_base)
        got_u = tu.cpu().numpy()
        assert np.array_equal(got_u, want_u), slot
        assert np.array_equal(ts.cpu().numpy().view(np.uint16), want_s.view(np.uint16)), slot
        assert np.array_equal(got_u[:, k_base:], u0[:, k_base:])   # LoRA K rows untouched
    names = {rt.W_Q: "q", rt.W_K: "k", rt.W_V: "v", rt.W_O: "o", rt.W_M1: "ug", rt.W_M2: "dn", rt.W_AQKV: "aqkv",
             rt.W_AO: "ao", rt.W_AUG: "aug", rt.W_ADN: "adn"}
    deq = {names[slot]: _deq(*dv[slot], group) for slot in shapes}
    Hh, Ww, Tt = 6, 6, 20
    nvalid = Hh * Ww + Tt
    T = 64
    g = torch.Generator().manual_seed(63)
    x = torch.randn(B, T, D, generator=g) * 2
    mod = torch.randn(6, D, generator=g) * 0.1
    c, s = rt.rope_moss(Hh, Ww, Tt, om.bands16().numpy(), T)
    meta, total = rt.blob_layout(rt.MODEL_MOSS, T, 0, B, D, F)
    S = rt.S
    meta[S["NVALID"]] = nvalid
    bfd = h.buf_alloc(total)
    write_f32(h, bfd, meta[S["X"]], x.numpy())
    write_f32(h, bfd, meta[S["COS"]], c)
    write_f32(h, bfd, meta[S["SIN"]], s)
    h.mega_block(meta, wfd, bfd, mod=mod.numpy())
    y = torch.from_numpy(read_f32(h, bfd, meta[S["X"]], B * T * D).reshape(B, T, D))
    h.buf_free(bfd)
    ref = om.block_dev(x, mod, torch.from_numpy(c), torch.from_numpy(s), deq, gain, nvalid=nvalid, lora=True)
    assert rel(y[:, :nvalid] - x[:, :nvalid], ref[:, :nvalid] - x[:, :nvalid]) < TOL
    h.weights_free(wfd)


def test_fold_rejects_bad_arguments(h):
    D, F = 256, 512
    W, norms, modA, modB = oa.init_weights(64, D=D, F=F, Cd=128)
    from tests.gpu_util import anima_bind
    wfd, _, _, keep = anima_bind(h, W, norms, modA, modB, rt.FMT_F16, 64)
    b, a = torch.zeros(3 * D, 8, device="cuda"), torch.zeros(8, D, device="cuda")
    with pytest.raises(rt.HxError) as e:
        h.lora_fold(wfd, rt.W_QKV, b, a, 8, 1.0)        # fp16 weights: nothing to requantise
    assert e.value.rc == rt.HX_E_FORMAT
    with pytest.raises(rt.HxError):
        h.lora_fold(wfd, rt.W_QKV, b, a, 0, 1.0)        # rank out of 1..128
    with pytest.raises(rt.HxError) as e:
        h.lora_fold(wfd + 1000, rt.W_QKV, b, a, 8, 1.0)
    assert e.value.rc == rt.HX_E_NOWEIGHTS
    h.weights_free(wfd)


def _deq64(tu, ts, group):
    return op.dequant_q8(tu.cpu().numpy(), ts.cpu().numpy(), group).astype(np.float64)


def test_moss_fold_into_rank128_slots(h):
    """hx_lora_fold_slots (the SVD fold of moss/mossrun/lorafold.cpp:200-284) on a MOSS q8 weight set with
    LoRA slots: for every projection, the new slots' product B'^T A' against the best rank-128
    approximation of (current slots + scale B A) from oracle.packs.fold_slots, within the q8
    requantisation error (about 0.8 %, bar 2e-2); the base columns and the other LoRA-A rows untouched;
    then a block on the folded weights against the oracle block (2e-3)."""
    D, F, B, group = 256, 256, 1, 32
    g = torch.Generator().manual_seed(70)
    shapes = {rt.W_Q: (D, D + 128), rt.W_K: (D, D + 128), rt.W_V: (D, D + 128), rt.W_O: (D, D + 128),
              rt.W_M1: (2 * F, D + 128), rt.W_M2: (D, F + 128), rt.W_AQKV: (384, D), rt.W_AO: (128, D),
              rt.W_AUG: (128, D), rt.W_ADN: (128, F)}
    mats, dv = {}, {}
    for slot, (n, k) in shapes.items():
        w = torch.randn(n, k, generator=g) * 0.02
        if slot in (rt.W_Q, rt.W_K, rt.W_V, rt.W_O, rt.W_M1, rt.W_M2):
            w[:, k - 128 + 40:] = 0  # turbo slots of effective rank 40 in the B columns
        mats[slot], tu, ts = _q8(w.numpy(), group)
        dv[slot] = (tu, ts)
    gain = torch.cat((1 + 0.1 * torch.randn(128, generator=g), 1 + 0.1 * torch.randn(128, generator=g),
                      1 + 0.1 * torch.randn(2 * D, generator=g)))
    gain[:128] /= np.sqrt(128.0)
    tg = gain.cuda()
    wfd = h.weights_bind(rt.MODEL_MOSS, D, F, mats, tg, lora=1, keep=[t for p in dv.values() for t in p] + [tg])
    table = ((rt.LORA_Q, rt.W_Q, rt.W_AQKV, 0, D, 32), (rt.LORA_K, rt.W_K, rt.W_AQKV, 128, D, 100),
             (rt.LORA_V, rt.W_V, rt.W_AQKV, 256, D, 64), (rt.LORA_O, rt.W_O, rt.W_AO, 0, D, 128),
             (rt.LORA_UG, rt.W_M1, rt.W_AUG, 0, D, 48), (rt.LORA_DN, rt.W_M2, rt.W_ADN, 0, F, 7))
    scale = 0.7
    for proj, slot, aslot, row0, kb, rank in table:
        W0, A0 = _deq64(*dv[slot], group), _deq64(*dv[aslot], group)
        u_base = dv[slot][0].cpu().numpy()[:, :kb].copy()
        a_rows = dv[aslot][0].cpu().numpy().copy()
        N = W0.shape[0]
        Bu = (torch.randn(N, rank, generator=g) * 0.02).numpy()   # logical row order
        Au = (torch.randn(rank, kb, generator=g) * 0.02).numpy()
        Bd = Bu[op.situ_logical_rows(N)] if slot == rt.W_M1 else Bu  # device row order
        BT = np.vstack((W0[:, kb:].T, scale * Bd.T.astype(np.float64)))
        AM = np.vstack((A0[row0:row0 + 128], Au.astype(np.float64)))
        P = BT.T @ AM
        U, S, Vt = np.linalg.svd(P)
        T = (U[:, :128] * S[:128]) @ Vt[:128]
        Bo, Ao = op.fold_slots(BT, AM)
        ub, sb = op.quant_q8(np.ascontiguousarray(Bo.T), group)
        ua, sa = op.quant_q8(Ao, group)
        Qo = op.dequant_q8(ub, sb, group).astype(np.float64) @ op.dequant_q8(ua, sa, group)
        h.lora_fold_slots(wfd, proj, dev(Bu), dev(Au), rank, scale)
        h.sync()
        W1, A1 = _deq64(*dv[slot], group), _deq64(*dv[aslot], group)
        Q = W1[:, kb:] @ A1[row0:row0 + 128]
        assert rel(torch.from_numpy(Q), torch.from_numpy(T)) < 2e-2, proj
        assert rel(torch.from_numpy(Q), torch.from_numpy(Qo)) < 2e-2, proj
        assert np.array_equal(dv[slot][0].cpu().numpy()[:, :kb], u_base)           # base columns untouched
        a_now = dv[aslot][0].cpu().numpy()
        others = np.ones(a_now.shape[0], bool)
        others[row0:row0 + 128] = False
        assert np.array_equal(a_now[others], a_rows[others])                      # other projections' rows
    names = {rt.W_Q: "q", rt.W_K: "k", rt.W_V: "v", rt.W_O: "o", rt.W_M1: "ug", rt.W_M2: "dn", rt.W_AQKV: "aqkv",
             rt.W_AO: "ao", rt.W_AUG: "aug", rt.W_ADN: "adn"}
    deq = {names[slot]: _deq(*dv[slot], group) for slot in shapes}
    Hh, Ww, Tt = 6, 6, 20
    nvalid = Hh * Ww + Tt
    T = 64
    x = torch.randn(B, T, D, generator=g) * 2
    mod = torch.randn(6, D, generator=g) * 0.1
    c, s = rt.rope_moss(Hh, Ww, Tt, om.bands16().numpy(), T)
    meta, total = rt.blob_layout(rt.MODEL_MOSS, T, 0, B, D, F)
    S = rt.S
    meta[S["NVALID"]] = nvalid
    bfd = h.buf_alloc(total)
    write_f32(h, bfd, meta[S["X"]], x.numpy())
    write_f32(h, bfd, meta[S["COS"]], c)
    write_f32(h, bfd, meta[S["SIN"]], s)
    h.mega_block(meta, wfd, bfd, mod=mod.numpy())
    y = torch.from_numpy(read_f32(h, bfd, meta[S["X"]], B * T * D).reshape(B, T, D))
    h.buf_free(bfd)
    ref = om.block_dev(x, mod, torch.from_numpy(c), torch.from_numpy(s), deq, gain, nvalid=nvalid, lora=True)
    assert rel(y[:, :nvalid] - x[:, :nvalid], ref[:, :nvalid] - x[:, :nvalid]) < TOL
    # a weight set without LoRA slots is refused
    with pytest.raises(rt.HxError) as e:
        W, norms, modA, modB = oa.init_weights(64, D=256, F=512, Cd=128)
        from tests.gpu_util import anima_bind
        wfd2, _, _, keep = anima_bind(h, W, norms, modA, modB, rt.FMT_Q8, 64)
        try:
            h.lora_fold_slots(wfd2, rt.LORA_Q, dev(Bu[:, :1].copy()), dev(Au[:1].copy()), 1, 1.0)
        finally:
            h.weights_free(wfd2)
    assert e.value.rc == rt.HX_E_FORMAT
    h.weights_free(wfd)
