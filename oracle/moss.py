"""MOSS-Image DiT block oracle in torch fp32 — test infrastructure, see oracle/__init__.py.

Restates moss/moss_ref.py (pinned against it by tests/golden/moss_block.npz):
  rms          moss_ref.py:21-22   x * rsqrt(mean x^2 + eps) * w
  situ         moss_ref.py:24-25   4 tanh(g/4) sigmoid(g) * 25 tanh(h/25)
  rope_tables  moss_ref.py:27-35   image (0, T, y-(H-1)/2, x-(W-1)/2), text (0, i, 0, 0); angle c[d//16] * bands[d%16]
  rotate       moss_ref.py:37-39   split-half rotation with duplicated halves of the tables
  attn         moss_ref.py:41-46   per-head rms(q|k) * gain, rotate, softmax(q k^T / sqrt(128)) v
  lin          moss_ref.py:48-54   x W^T (+ b) (+ s (x A^T) B^T)
  block        moss_ref.py:56-67   mod rows: shift_a, scale_a, gate_a, shift_f, scale_f, gate_f
  text_block   moss_ref.py:81-89   refiner block: rms, qkv + bias, attn, proj + bias, rms, SiTU(up, gate) + biases
  text_refine  moss_ref.py:91-94   text_embedder.proj (4096 -> D) + bias, then two text blocks
  time_vecs    moss_ref.py:96-105  cos|sin(t * 10000^(-i/128)), silu MLP, shared block / head modulation
(pinned by tests/golden/moss_text.npz) and the q8-pack-aware staged form of mkblk_test.py:38-55 (LoRA as extra K tiles: [x | x A] @ [W ; s B^T],
attention scale 1.0 with the q gain pre-divided by sqrt(128)).
"""
import math

import numpy as np
import torch

HD = 128


def rms(x, w, eps=1e-6):
    return x * torch.rsqrt(x.square().mean(-1, keepdim=True) + eps) * w


def situ(h, g):
    return (4.0 * torch.tanh(g / 4.0) * torch.sigmoid(g)) * (25.0 * torch.tanh(h / 25.0))


def rope_tables(H, W, T, bands):
    """-> sin, cos [H*W + T][128] (halves duplicated)."""
    yy, xx = torch.meshgrid(torch.arange(H), torch.arange(W), indexing="ij")
    img = torch.zeros(H * W, 4)
    img[:, 1] = T
    img[:, 2] = yy.flatten().float() - (H - 1) / 2
    img[:, 3] = xx.flatten().float() - (W - 1) / 2
    txt = torch.zeros(T, 4)
    txt[:, 1] = torch.arange(T).float()
    coords = torch.cat((img, txt), 0)                                  # [N, 4]
    ang = (coords[:, :, None] * bands[None, None, :]).reshape(-1, 64)  # angle d = c[d//16] * bands[d%16]
    s, c = torch.sin(ang), torch.cos(ang)
    return torch.cat((s, s), -1), torch.cat((c, c), -1)


def rotate(x, sin, cos):
    """x [N, H, 128]; sin/cos [N, 128]"""
    a, b = x[..., :64], x[..., 64:]
    return x * cos[:, None] + torch.cat((-b, a), -1) * sin[:, None]


def attn(q, k, v, sin, cos, qn, kn, heads, scale=None, nvalid=None):
    N = q.shape[0]
    q = rotate(rms(q.view(N, heads, -1), qn), sin, cos)
    k = rotate(rms(k.view(N, heads, -1), kn), sin, cos)
    v = v.view(N, heads, -1)
    sc = (1.0 / math.sqrt(q.shape[-1])) if scale is None else scale
    s = torch.einsum("qhd,khd->hqk", q, k) * sc
    if nvalid is not None and nvalid < N:
        s[..., nvalid:] = float("-inf")
    o = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v)
    return o.reshape(N, -1)


def lin(x, w, b=None, lora=None):
    y = x @ w.T
    if b is not None:
        y = y + b
    if lora is not None:
        A, B, s = lora
        y = y + s * ((x @ A.T) @ B.T)
    return y


def block(x, mod, sin, cos, g, i, lora=None, heads=24):
    """moss_ref.block: x [N, D]; g(name) -> [out][in] weights; lora(i, n) -> (A, B, s) or None."""
    p = f"layers.{i}."
    sa, ca, ga, sf, cf, gf = mod
    L = (lambda n: lora(i, n)) if lora else (lambda n: None)
    y = rms(x, g(p + "norm1.weight")) * (1 + ca) + sa
    q = lin(y, g(p + "proj.q.weight"), lora=L("q"))
    k = lin(y, g(p + "proj.k.weight"), lora=L("k"))
    v = lin(y, g(p + "proj.v.weight"), lora=L("v"))
    a = attn(q, k, v, sin, cos, g(p + "q_norm.weight"), g(p + "k_norm.weight"), heads)
    x = x + lin(a, g(p + "proj.o.weight"), lora=L("o")) * ga
    y = rms(x, g(p + "norm2.weight")) * (1 + cf) + sf
    h, gt = lin(y, g(p + "proj.ffn_up_gate.weight"), lora=L("ffn_up_gate")).chunk(2, -1)
    return x + lin(situ(h, gt), g(p + "proj.ffn_down.weight"), lora=L("ffn_down")) * gf


def selector(shape_lead, width):
    """The MODE 1 bias selector of an L buffer: 1.0 in column 0 of every 128-column part (mossrun.cpp:205-209)."""
    t = torch.zeros(*shape_lead, width)
    t[..., 0::128] = 1.0
    return t


def block_dev(x, mod, cos64, sin64, mats, gain, nvalid=None, lora=True, heads=None, refiner=False):
    """Staged, device-weight form (mkblk_test.py:38-55): every matrix is the [N][K'] operand the GPU
    multiplies (LoRA-B rows appended along K when lora), A matrices [r][K]; gain = [q/sqrt(128), k,
    norm1, norm2]; up_gate rows grouped per 256 (128 up, 128 gate). x [B, T, D]; cos64/sin64 [T][64].
    refiner: MODE 1 (moss/hexagon/mega/blk.c:237) - the L operands are the bias selector, not y A^T."""
    B, T, D = x.shape
    H = heads or D // HD
    sa, ca, ga, sf, cf, gf = mod
    qg, kg, n1, n2 = gain[:128], gain[128:256], gain[256:256 + D], gain[256 + D:256 + 2 * D]
    cat = lambda a, b: torch.cat((a, b), -1)
    if refiner:
        sel = {k: (lambda y, n=n: selector(y.shape[:-1], n)) for k, n in (("aqkv", 384), ("ao", 128), ("aug", 128),
                                                                          ("adn", 128))}
        mats = dict(mats)
        for k in sel:
            mats[k] = None
    else:
        sel = {}
    LA = lambda y, name: sel[name](y) if name in sel else y @ mats[name].T
    y = rms(x, n1) * (1 + ca) + sa
    if lora:
        Lq = LA(y, "aqkv")
        q = cat(y, Lq[..., 0:128]) @ mats["q"].T
        k = cat(y, Lq[..., 128:256]) @ mats["k"].T
        v = cat(y, Lq[..., 256:384]) @ mats["v"].T
    else:
        qkv = y @ mats["qkv"].T
        q, k, v = qkv[..., :D], qkv[..., D:2 * D], qkv[..., 2 * D:]
    c = torch.cat((cos64, cos64), -1)[None, :, None, :]
    s = torch.cat((sin64, sin64), -1)[None, :, None, :]
    rot = lambda t: t * c + torch.cat((-t[..., 64:], t[..., :64]), -1) * s
    q = rot(rms(q.view(B, T, H, HD), qg))
    k = rot(rms(k.view(B, T, H, HD), kg))
    v = v.view(B, T, H, HD)
    # attention in groups of heads (the same per-head math; bounds host memory at the large configs)
    a = torch.empty(B, T, H, HD, dtype=q.dtype)
    for h0 in range(0, H, 4):
        sc = torch.einsum("bqhd,bkhd->bhqk", q[:, :, h0:h0 + 4], k[:, :, h0:h0 + 4])
        if nvalid is not None and nvalid < T:
            sc[..., nvalid:] = float("-inf")
        a[:, :, h0:h0 + 4] = torch.einsum("bhqk,bkhd->bqhd", torch.softmax(sc, -1), v[:, :, h0:h0 + 4])
    a = a.reshape(B, T, D)
    o = (cat(a, LA(a, "ao")) if lora else a) @ mats["o"].T
    x = x + o * ga
    y2 = rms(x, n2) * (1 + cf) + sf
    ug = (cat(y2, LA(y2, "aug")) if lora else y2) @ mats["ug"].T  # [B, T, 2F], grouped per 256
    F = ug.shape[-1] // 2
    g4 = ug.view(B, T, F // 128, 2, 128)
    mid = situ(g4[:, :, :, 0], g4[:, :, :, 1]).reshape(B, T, F)
    dn = (cat(mid, LA(mid, "adn")) if lora else mid) @ mats["dn"].T
    return x + dn * gf


def init_weights(seed, D=3072, F=8192, std=0.02, lora_rank=0):
    """Seeded synthetic MOSS block in moss_ref naming (layer 0): g(name) dict of [out][in] tensors."""
    gen = torch.Generator().manual_seed(seed)
    n = lambda *s: torch.randn(*s, generator=gen) * std
    p = "layers.0."
    w = {p + "norm1.weight": 1 + n(D), p + "norm2.weight": 1 + n(D), p + "q_norm.weight": 1 + n(HD),
         p + "k_norm.weight": 1 + n(HD), p + "proj.q.weight": n(D, D), p + "proj.k.weight": n(D, D),
         p + "proj.v.weight": n(D, D), p + "proj.o.weight": n(D, D), p + "proj.ffn_up_gate.weight": n(2 * F, D),
         p + "proj.ffn_down.weight": n(D, F)}
    lora = {}
    if lora_rank:
        for name, (o, i) in {"q": (D, D), "k": (D, D), "v": (D, D), "o": (D, D), "ffn_up_gate": (2 * F, D),
                             "ffn_down": (D, F)}.items():
            lora[name] = (n(lora_rank, i) * 10, n(o, lora_rank) * 10, 1.0)
    return w, lora


def bands16(theta=10000.0):
    """RoPE bands 1/theta^(i/16) (pipeline_moss_image.py:158-160)."""
    return torch.tensor([1.0 / theta ** (i / 16.0) for i in range(16)], dtype=torch.float32)


def build_pack(w, lora, i=0):
    """MOSS blkNN.bin bytes (export_moss.py:29-41): q8 tiles of [W^T ; s B^T] (up_gate interleaved per 32
    columns), the LoRA-A matrices, gains [q/sqrt(128), k, norm1, norm2] padded to 8192 floats."""
    from .packs import F16_FLOOR_MOSS, interleave32, q8tiles, wt16
    p = f"layers.{i}."

    def mat(w_oi, lr, inter=False):
        wk = w_oi.T.contiguous()
        if inter:
            h = wk.shape[1] // 2
            wk = torch.from_numpy(interleave32(wk[:, :h].numpy(), wk[:, h:].numpy()))
        A, Bm, s = lr
        b = (s * Bm.T).contiguous()
        if inter:
            h = b.shape[1] // 2
            b = torch.from_numpy(interleave32(b[:, :h].numpy(), b[:, h:].numpy()))
        return q8tiles(wt16(torch.cat((wk, b), 0).numpy()), F16_FLOOR_MOSS)

    out = [mat(w[p + f"proj.{n}.weight"], lora[n]) for n in ("q", "k", "v", "o")]
    out.append(mat(w[p + "proj.ffn_up_gate.weight"], lora["ffn_up_gate"], True))
    out.append(mat(w[p + "proj.ffn_down.weight"], lora["ffn_down"]))
    At = lambda n: lora[n][0].T
    out.append(q8tiles(wt16(torch.cat((At("q"), At("k"), At("v")), 1).numpy()), F16_FLOOR_MOSS))
    for n in ("o", "ffn_up_gate", "ffn_down"):
        out.append(q8tiles(wt16(At(n).contiguous().numpy()), F16_FLOOR_MOSS))
    gain = np.concatenate([w[p + "q_norm.weight"].numpy() / np.sqrt(128.0), w[p + "k_norm.weight"].numpy(),
                           w[p + "norm1.weight"].numpy(), w[p + "norm2.weight"].numpy()]).astype(np.float32)
    out.append(gain.tobytes() + bytes(8192 * 4 - gain.nbytes))
    return b"".join(out)


def pack_mats(pack, D=3072, F=8192):
    """Device-operand view of a MOSS pack: {name: [N][K'] fp32 of fp16(q*s)}, gain [256 + 2D]."""
    from .packs import dequant_q8_f16
    specs = [("q", D, D + 128), ("k", D, D + 128), ("v", D, D + 128), ("o", D, D + 128), ("ug_pack", 2 * F, D + 128),
             ("dn", D, F + 128), ("aqkv", 384, D), ("ao", 128, D), ("aug", 128, D), ("adn", 128, F)]
    mats, off = {}, 0
    for name, N, K in specs:
        size = (N // 32) * (K // 32) * 1152
        w = dequant_q8_f16(pack[off:off + size], N // 32, K // 32).astype(np.float32)  # [K][N]
        mats[name] = torch.from_numpy(np.ascontiguousarray(w.T))
        off += size
    ug = mats.pop("ug_pack")  # rows: pack column order, 32-row blocks (up_j, gate_j)
    blocks = ug.view(2 * F // 64, 2, 32, -1)
    up, gate = blocks[:, 0].reshape(F, -1), blocks[:, 1].reshape(F, -1)
    mats["ug"] = torch.cat((up.view(F // 128, 128, -1), gate.view(F // 128, 128, -1)), 1).reshape(2 * F, -1)
    gain = torch.from_numpy(np.frombuffer(pack[off:off + (256 + 2 * D) * 4], np.float32).copy())
    return mats, gain


# ---------------------------------------------------------------- text side and sampler glue
def text_block(x, p, sin, cos, g, heads=24):
    """moss_ref.text_block: x [N, D]; weights g(p + name) with biases."""
    h = rms(x, g(p + "norm1.weight"))
    q, k, v = lin(h, g(p + "qkv.weight"), g(p + "qkv.bias")).chunk(3, -1)
    a = attn(q, k, v, sin, cos, g(p + "q_norm.weight"), g(p + "k_norm.weight"), heads)
    x = x + lin(a, g(p + "proj.weight"), g(p + "proj.bias"))
    y = rms(x, g(p + "norm2.weight"))
    up = lin(y, g(p + "ffn_up.weight"), g(p + "ffn_up.bias"))
    gate = lin(y, g(p + "ffn_gate.weight"), g(p + "ffn_gate.bias"))
    return x + lin(situ(up, gate), g(p + "ffn_down.weight"), g(p + "ffn_down.bias"))


def text_refine(txt, sin_t, cos_t, g, heads=24):
    """moss_ref.text_refine: txt [T, 4096] -> [T, D]."""
    x = lin(txt, g("text_embedder.proj.weight"), g("text_embedder.proj.bias"))
    for i in range(2):
        x = text_block(x, f"text_embedder.blocks.{i}.", sin_t, cos_t, g, heads)
    return x


def time_vecs(t, g):
    """moss_ref.time_vecs: -> mod [6, D], head [2, D] (code t; embedding in float64 then float32)."""
    half = 128
    freq = 10000 ** (-torch.arange(half, dtype=torch.float64) / half)
    ph = float(t) * freq
    e = torch.cat((ph.cos(), ph.sin())).float()
    a = torch.nn.functional.silu(e @ g("time_embedding.0.weight").T + g("time_embedding.0.bias"))
    tm = a @ g("time_embedding.2.weight").T + g("time_embedding.2.bias")
    mod = tm @ g("shared_block_modulation.weight").T + g("shared_block_modulation.bias")
    head = tm @ g("video_head_modulation.weight").T + g("video_head_modulation.bias")
    return mod.view(6, -1), head.view(2, -1)


def init_text_weights(seed, D=3072, F=256, TW=4096, std=0.02, blocks=2):
    """Seeded synthetic text_embedder (moss_ref naming): proj TW -> D and `blocks` refiner blocks."""
    gen = torch.Generator().manual_seed(seed)
    n = lambda *s: torch.randn(*s, generator=gen) * std
    w = {"text_embedder.proj.weight": n(D, TW), "text_embedder.proj.bias": n(D)}
    for i in range(blocks):
        p = f"text_embedder.blocks.{i}."
        w.update({p + "norm1.weight": 1 + n(D), p + "norm2.weight": 1 + n(D), p + "q_norm.weight": 1 + n(HD),
                  p + "k_norm.weight": 1 + n(HD), p + "qkv.weight": n(3 * D, D), p + "qkv.bias": n(3 * D),
                  p + "proj.weight": n(D, D), p + "proj.bias": n(D), p + "ffn_up.weight": n(F, D),
                  p + "ffn_up.bias": n(F), p + "ffn_gate.weight": n(F, D), p + "ffn_gate.bias": n(F),
                  p + "ffn_down.weight": n(D, F), p + "ffn_down.bias": n(D)})
    return w


def init_time_weights(seed, D=3072, std=0.02):
    """Seeded synthetic time_embedding / modulation weights (moss_ref naming)."""
    gen = torch.Generator().manual_seed(seed)
    n = lambda *s: torch.randn(*s, generator=gen) * std
    return {"time_embedding.0.weight": n(D, 256), "time_embedding.0.bias": n(D),
            "time_embedding.2.weight": n(D, D), "time_embedding.2.bias": n(D),
            "shared_block_modulation.weight": n(6 * D, D), "shared_block_modulation.bias": n(6 * D),
            "video_head_modulation.weight": n(2 * D, D), "video_head_modulation.bias": n(2 * D)}


def build_refiner_pack(w, i):
    """Refiner block pack (export_moss.py:43-59 `pack_refiner`): the block layout of build_pack with the
    biases in row 0 of the 128 LoRA K rows (scale 1) and zero LoRA-A matrices."""
    p = f"text_embedder.blocks.{i}."
    D = w[p + "norm1.weight"].shape[0]
    qkv, qkvb = w[p + "qkv.weight"], w[p + "qkv.bias"]

    def bias_lora(b, fan_in):
        B = torch.zeros(b.shape[0], 128)
        B[:, 0] = b
        return (torch.zeros(128, fan_in), B, 1.0)

    F = w[p + "ffn_up.weight"].shape[0]
    blk = {"layers.0.proj.q.weight": qkv[:D], "layers.0.proj.k.weight": qkv[D:2 * D],
           "layers.0.proj.v.weight": qkv[2 * D:], "layers.0.proj.o.weight": w[p + "proj.weight"],
           "layers.0.proj.ffn_up_gate.weight": torch.cat((w[p + "ffn_up.weight"], w[p + "ffn_gate.weight"]), 0),
           "layers.0.proj.ffn_down.weight": w[p + "ffn_down.weight"],
           "layers.0.q_norm.weight": w[p + "q_norm.weight"], "layers.0.k_norm.weight": w[p + "k_norm.weight"],
           "layers.0.norm1.weight": w[p + "norm1.weight"], "layers.0.norm2.weight": w[p + "norm2.weight"]}
    lora = {"q": bias_lora(qkvb[:D], D), "k": bias_lora(qkvb[D:2 * D], D), "v": bias_lora(qkvb[2 * D:], D),
            "o": bias_lora(w[p + "proj.bias"], D),
            "ffn_up_gate": bias_lora(torch.cat((w[p + "ffn_up.bias"], w[p + "ffn_gate.bias"])), D),
            "ffn_down": bias_lora(w[p + "ffn_down.bias"], F)}
    return build_pack(blk, lora)


def build_proj_pack(w, pad_to=135397376):
    """Text projection pack (export_moss.py:61-65 `pack_proj`): q8 tiles of [Wp^T ; bias, 127 zero rows]
    ([D/32 nb][(TW+128)/32 kb]) padded with zeros to the block-pack size."""
    from .packs import F16_FLOOR_MOSS, q8tiles, wt16
    Wp, b = w["text_embedder.proj.weight"], w["text_embedder.proj.bias"]
    B = torch.zeros(128, Wp.shape[0])
    B[0] = b
    d = q8tiles(wt16(torch.cat((Wp.T, B), 0).numpy()), F16_FLOOR_MOSS)
    return d + bytes(max(0, pad_to - len(d)))


def proj_mat(pack, D=3072, TW=4096):
    """Device-operand view of a projection pack: [D][TW + 128] fp32 of fp16(q*s)."""
    from .packs import dequant_q8_f16
    size = (D // 32) * ((TW + 128) // 32) * 1152
    w = dequant_q8_f16(pack[:size], D // 32, (TW + 128) // 32).astype(np.float32)   # [K][N]
    return torch.from_numpy(np.ascontiguousarray(w.T))


def sample_dev(z, x0, tx, glue, blocks, codes, cos64, sin64, ntok):
    """MOSS sampler in device-operand form: sample_ref.py:15-20 around moss_ref.dit_forward (moss_ref.py:
    107-120) with the text rows `tx` already refined. z, x0 [B, 128, Ni]; tx [T, D]; glue: moss_ref-named
    tensors holding the values the device multiplies (fp16-rounded matrices; video_embedder.bias rounded to
    fp16 because it rides in the embedder GEMM's K column); blocks: [(mats, gain, lora)] for block_dev.
    The embedder input and the final-layer input are rounded to fp16 as the device GEMMs take them."""
    B, C, Ni = z.shape
    T, D = tx.shape
    g = lambda n: glue[n]
    for code in codes:
        xin = z + torch.einsum("oc,bct->bot", g("latent_mix.Q"), x0)
        rows = xin.transpose(1, 2).half().float() @ g("video_embedder.weight").T + g("video_embedder.bias")
        x = torch.zeros(B, ntok, D)
        x[:, :Ni] = rows
        x[:, Ni:Ni + T] = tx
        mod, head = time_vecs(code, g)
        for mats, gain, lora in blocks:
            x = block_dev(x, mod, cos64, sin64, mats, gain, nvalid=Ni + T, lora=lora)
        hf = (rms(x, g("final_norm_video.weight")) * (1 + head[1]) + head[0]).half().float()
        v = (hf @ g("final_linear_video.weight").T)[:, :Ni]           # [B, Ni, 128]
        x0 = z - v.transpose(1, 2)
    return x0


def init_glue_weights(seed, D, std=0.02):
    """Seeded synthetic sampler glue (moss_ref names), matrices already fp16-rounded as the device holds them."""
    w = init_time_weights(seed, D=D, std=std)
    gen = torch.Generator().manual_seed(seed + 1)
    n = lambda *s: torch.randn(*s, generator=gen) * std
    w.update({"video_embedder.weight": n(D, 128) * 5, "video_embedder.bias": n(D),
              "final_norm_video.weight": 1 + n(D), "final_linear_video.weight": n(128, D),
              "latent_mix.Q": n(128, 128) * 10})
    for k in ("time_embedding.0.weight", "time_embedding.2.weight", "shared_block_modulation.weight",
              "video_head_modulation.weight", "video_embedder.weight", "video_embedder.bias",
              "final_linear_video.weight"):
        w[k] = w[k].half().float()
    return w
