"""The CPU oracle against the reference's golden vectors (tests/golden/make_golden.py)."""
import os

import numpy as np
import pytest
import torch

from oracle import anima as oa
from oracle import moss as om
from oracle import packs as op

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def packs():
    return np.load(os.path.join(GOLD, "packs.npz"))


@pytest.fixture(scope="module")
def mblock():
    return np.load(os.path.join(GOLD, "moss_block.npz"))


def test_wt16_bit_exact(packs):
    t = op.wt16(packs["W"])
    assert np.array_equal(np.frombuffer(t.tobytes(), np.uint8), packs["wt16"])
    assert np.array_equal(op.unwt16(t), packs["W"].astype(np.float16))


def test_q8_moss_bit_exact(packs):
    b = op.q8tiles(op.wt16(packs["W"]), op.F16_FLOOR_MOSS)
    assert np.array_equal(np.frombuffer(b, np.uint8), packs["q8_moss"])


def test_q8_anima_bit_exact(packs):
    with np.errstate(divide="ignore", invalid="ignore"):
        b = op.q8tiles(op.wt16(packs["W"]), op.F16_FLOOR_ANIMA)
    assert np.array_equal(np.frombuffer(b, np.uint8), packs["q8_anima"])


def test_q8_unpack_matches_mkblk_test(packs):
    K, N = packs["W"].shape
    w = op.unpack_q8(packs["q8_moss"].tobytes(), N // 32, K // 32)
    assert np.array_equal(w, packs["unpack_moss"])


def test_q4a_bit_exact(packs):
    b = op.q4a_tiles(packs["q4_nib"], packs["q4_S"], packs["q4_M"])
    assert np.array_equal(np.frombuffer(b, np.uint8), packs["q4a"])
    K, N = packs["W"].shape
    assert np.array_equal(op.unpack_q4a(b, N // 32, K // 32), packs["unpack_q4a"])


def test_q8_records_to_device_roundtrip(packs):
    """Device layout from records decodes to the same values as the reference unpack."""
    K, N = packs["W"].shape
    u, sc = op.q8_records_to_device(packs["q8_moss"].tobytes(), N // 32, K // 32)
    assert u.shape == (N, K) and sc.shape == (K // 32, N)
    dev = op.dequant_q8(u, sc, 32)
    ref = packs["unpack_moss"].T.astype(np.float16)
    assert np.array_equal(dev.view(np.uint16), ref.view(np.uint16))


def test_device_quantisers_roundtrip():
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    for g in (32, 64):
        u, s = op.quant_q8(w, g)
        d = op.dequant_q8(u, s, g).astype(np.float32)
        assert np.abs(d - w).max() <= np.abs(w).max() / 127 * 0.6
    p, s = op.quant_q4(w)
    assert np.array_equal(op.unpack_nibbles(op.pack_nibbles(op.unpack_nibbles(p))), op.unpack_nibbles(p))
    d = op.dequant_q4(p, s).astype(np.float32)
    assert np.abs(d - w).max() <= np.abs(w).max() / 7 * 0.6
    p, s, m = op.quant_q4a(w)
    d = op.dequant_q4a(p, s, m).astype(np.float32)
    assert np.abs(d - w).max() <= (w.max() - w.min()) / 15 * 0.6 + 1e-3


def test_rope_tables_match_moss_ref(mblock):
    sin, cos = om.rope_tables(int(mblock["H"]), int(mblock["W"]), int(mblock["T"]), torch.from_numpy(mblock["bands"]))
    np.testing.assert_allclose(sin.numpy(), mblock["sin"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(cos.numpy(), mblock["cos"], rtol=0, atol=1e-6)


@pytest.mark.parametrize("tag,rank", [("plain", 0), ("lora", 8)])
def test_moss_block_matches_moss_ref(mblock, tag, rank):
    D, F = int(mblock["D"]), int(mblock["F"])
    seed = int(mblock[f"{tag}_seed"])
    w, lora = om.init_weights(seed, D=D, F=F, lora_rank=rank)
    gen = torch.Generator().manual_seed(seed + 100)
    Nt = int(mblock["H"]) * int(mblock["W"]) + int(mblock["T"])
    x = torch.randn(Nt, D, generator=gen)
    mod = torch.randn(6, D, generator=gen) * 0.1
    # the seeded inputs are the ones the golden was computed on
    assert abs(float(x.double().sum()) - float(mblock[f"{tag}_x_sum"])) < 1e-6
    assert abs(float(sum(v.double().sum() for v in w.values())) - float(mblock[f"{tag}_w_sum"])) < 1e-6
    sin, cos = torch.from_numpy(mblock["sin"]), torch.from_numpy(mblock["cos"])
    y = om.block(x, mod, sin, cos, lambda n: w[n], 0, (lambda i, n: lora[n]) if rank else None)
    ref = torch.from_numpy(mblock[f"{tag}_out"])
    rel = float((y - ref).norm() / (ref - x).norm())
    assert rel < 1e-5, rel


def test_block_dev_matches_block_on_same_weights():
    """The staged device-operand form equals moss_ref's block when fed the same fp32 weights."""
    torch.manual_seed(0)
    D, F, Nt = 256, 256, 40
    w, lora = om.init_weights(5, D=D, F=F, lora_rank=128)
    p = "layers.0."
    s = 1.0
    mats = {}
    for n, key in (("q", "q"), ("k", "k"), ("v", "v"), ("o", "o")):
        A, B, _ = lora[n]
        mats[key] = torch.cat((w[p + f"proj.{n}.weight"], s * B), 1)
    A, B, _ = lora["ffn_up_gate"]
    ug = torch.cat((w[p + "proj.ffn_up_gate.weight"], s * B), 1)  # [2F][D+128], up rows then gate rows
    up, gate = ug[:F], ug[F:]
    mats["ug"] = torch.cat((up.view(F // 128, 128, -1), gate.view(F // 128, 128, -1)), 1).reshape(2 * F, -1)
    A, B, _ = lora["ffn_down"]
    mats["dn"] = torch.cat((w[p + "proj.ffn_down.weight"], s * B), 1)
    mats["aqkv"] = torch.cat((lora["q"][0], lora["k"][0], lora["v"][0]), 0)
    mats["ao"], mats["aug"], mats["adn"] = lora["o"][0], lora["ffn_up_gate"][0], lora["ffn_down"][0]
    gain = torch.cat((w[p + "q_norm.weight"] / np.sqrt(128.0), w[p + "k_norm.weight"], w[p + "norm1.weight"],
                      w[p + "norm2.weight"]))
    x = torch.randn(Nt, D)
    mod = torch.randn(6, D) * 0.1
    sin, cos = om.rope_tables(4, 6, 16, om.bands16())
    ref = om.block(x, mod, sin, cos, lambda n: w[n], 0, lambda i, n: lora[n], heads=D // 128)
    got = om.block_dev(x[None], mod, cos[:, :64], sin[:, :64], mats, gain)[0]
    rel = float((got - ref).norm() / (ref - x).norm())
    assert rel < 1e-5, rel


def test_anima_rope_table_formula():
    c, s = oa.make_rope(48, 32)
    assert c.shape == (1536, 64)
    assert np.all(c[:, :22] == 1) and np.all(s[:, :22] == 0)       # temporal band: angle 0
    tk = 5 * 32 + 7
    assert np.isclose(np.arccos(np.clip(c[tk, 22], -1, 1)), 5.0 % (2 * np.pi), atol=1e-5) or np.isclose(
        s[tk, 22], np.sin(5.0), atol=1e-6)
    assert np.isclose(s[tk, 43], np.sin(7.0), atol=1e-6)


def test_anima_block_small_is_finite_and_gated():
    """Gates of zero leave x unchanged (the residual update is gate-scaled at every site)."""
    W, norms, modA, modB = oa.init_weights(1, D=256, F=512, Cd=128)
    x = torch.randn(1, 64, 256)
    ctx = torch.randn(1, 32, 128)
    mod = torch.randn(9, 256) * 0.1
    mod[2] = mod[5] = mod[8] = 0
    c, s = oa.make_rope(8, 8)
    y = oa.block(x, ctx, mod, torch.from_numpy(c), torch.from_numpy(s), W, oa.pack_gain(norms))
    assert torch.equal(y, x)
    mod[2] = 1
    y = oa.block(x, ctx, mod, torch.from_numpy(c), torch.from_numpy(s), W, oa.pack_gain(norms))
    assert torch.isfinite(y).all() and not torch.equal(y, x)


def test_anima_pack_roundtrip():
    W, norms, modA, modB = oa.init_weights(2, D=2048, F=8192, Cd=1024)
    for q8 in (False, True):
        pack = oa.build_pack(W, norms, modA, modB, q8=q8)
        assert len(pack) == (83365888 if q8 else 138416128)
        Wd, gain = oa.pack_weights(pack, q8=q8)
        assert torch.allclose(gain, oa.pack_gain(norms))
        for n in oa.ORDER:
            err = (Wd[n] - W[n]).abs().max().item()
            assert err < (3e-3 if q8 else 1e-4), (n, err)


def test_sigma_schedule_matches_animad():
    sig = oa.sigma_schedule(4)
    assert abs(float(sig[0]) - 1.0) < 1e-7 and float(sig[-1]) == 0.0
    s = np.linspace(1, 0.001, 4)
    np.testing.assert_allclose(np.array(sig[:4], np.float64), 3 * s / (1 + 2 * s), rtol=1e-6)


# ---------------------------------------------------------------- MOSS text side and glue (moss_text.npz)
@pytest.fixture(scope="module")
def mtext():
    return np.load(os.path.join(GOLD, "moss_text.npz"))


def test_text_block_and_refine_match_moss_ref(mtext):
    w = om.init_text_weights(int(mtext["text_seed"]), D=3072, F=256)
    g = lambda n: w[n]
    s, c = torch.from_numpy(mtext["sin"]), torch.from_numpy(mtext["cos"])
    tb = om.text_block(torch.from_numpy(mtext["x"]), "text_embedder.blocks.0.", s, c, g)
    tr = om.text_refine(torch.from_numpy(mtext["txt"]), s, c, g)
    for got, want in ((tb, mtext["text_block"]), (tr, mtext["text_refine"])):
        want = torch.from_numpy(want)
        assert float((got - want).norm() / want.norm()) < 1e-5


def test_time_vecs_match_moss_ref(mtext):
    w = om.init_time_weights(int(mtext["time_seed"]), D=256)
    mod, head = om.time_vecs(float(mtext["t_code"]), lambda n: w[n])
    assert np.allclose(mod.numpy(), mtext["mod"], rtol=1e-5, atol=1e-6)
    assert np.allclose(head.numpy(), mtext["head"], rtol=1e-5, atol=1e-6)


def test_refiner_pack_mode1_form_matches_text_block():
    """A refiner pack (biases in LoRA row 0) run in the device-operand form with the MODE 1 bias selector
    equals text_block on the same dequantised weights."""
    D, F, T = 3072, 256, 32
    w = om.init_text_weights(31, D=D, F=F)
    pack = om.build_refiner_pack(w, 0)
    mats, gain = om.pack_mats(pack, D=D, F=F)
    # the text_block weights as the pack holds them
    ug = mats["ug"].view(F // 128, 2, 128, -1)
    up, gate = ug[:, 0].reshape(F, -1), ug[:, 1].reshape(F, -1)
    p = "text_embedder.blocks.0."
    wd = {p + "qkv.weight": torch.cat([mats[n][:, :D] for n in "qkv"], 0),
          p + "qkv.bias": torch.cat([mats[n][:, D] for n in "qkv"]),
          p + "proj.weight": mats["o"][:, :D], p + "proj.bias": mats["o"][:, D],
          p + "ffn_up.weight": up[:, :D], p + "ffn_up.bias": up[:, D],
          p + "ffn_gate.weight": gate[:, :D], p + "ffn_gate.bias": gate[:, D],
          p + "ffn_down.weight": mats["dn"][:, :F], p + "ffn_down.bias": mats["dn"][:, F],
          p + "q_norm.weight": gain[:128] * np.sqrt(128.0), p + "k_norm.weight": gain[128:256],
          p + "norm1.weight": gain[256:256 + D], p + "norm2.weight": gain[256 + D:256 + 2 * D]}
    sin, cos = om.rope_tables(0, 1, T, om.bands16())
    x = torch.randn(T, D, generator=torch.Generator().manual_seed(32))
    ref = om.text_block(x, p, sin, cos, lambda n: wd[n])
    mod = torch.zeros(6, D)
    mod[2] = 1.0
    mod[5] = 1.0
    got = om.block_dev(x[None], mod, cos[:, :64], sin[:, :64], mats, gain, lora=True, refiner=True)[0]
    assert float((got - ref).norm() / ref.norm()) < 1e-5


def test_proj_pack_bias_row():
    w = om.init_text_weights(33, D=3072, F=256, blocks=0)
    pack = om.build_proj_pack(w)
    assert len(pack) == 135397376
    m = om.proj_mat(pack)
    assert m.shape == (3072, 4224)
    b = w["text_embedder.proj.bias"]
    assert float((m[:, 4096] - b).abs().max()) < 1e-3 * float(b.abs().max())
    assert float(m[:, 4097:].abs().max()) == 0.0
