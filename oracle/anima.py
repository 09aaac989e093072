"""Anima DiT block oracle in torch fp32 — test infrastructure, see oracle/__init__.py.

Restates hexagon/mega/blk.c:148-175 (the reference ships no runnable Anima block in Python):
  site 0: h = LNmod(x); q, k, v = h W; q, k = RoPE(RMS(q|k) * gain); o = attn(q, k, v); x += gate * o Wo
  site 1: h = LNmod(x); q = RMS(h Wcq) * gain; ck = RMS(ctx Wck) * gain; cv = ctx Wcv;
          o = attn(q, ck, cv) over all context rows (zero-padded rows are NOT masked, PITFALLS:71);
          x += gate * o Wco
  site 2: h = LNmod(x); x += gate * GELU(h Wm1) Wm2
with
  LNmod   kern.c:38-65   y = (x - mu) / sqrt(E[x^2] - mu^2 + 1e-6) * (1 + scale) + shift (no affine)
  RMS     kern.c:199-232 per 128-wide head: x / sqrt(mean x^2 + 1e-6) * gain
  RoPE    kern.c:213-222 split-half pairs (d, d+64): lo = a c - b s, hi = b c + a s
  gains   export_all.py:31-32  [q/sqrt(128), k, cq/sqrt(128), ck]; attention scale 1.0
  GELU    ktest.c:63     exact erf form
  tables  megarun.cpp:77-90   angles d<22: 0; d<43: row * th^(-2i/42); else col * th^(-2i/42)
  mod     megarun.cpp:158-171 per site: B (A silu(emb)) + lora; chunks shift, scale, gate
Weights are [out][in] (torch Linear layout); the pack stores their transposes as W[K][N] tiles.
"""
import math

import numpy as np
import torch

HD = 128
ORDER = ["sq", "sk", "sv", "so", "cq", "ck", "cv", "co", "m1", "m2"]  # export_all.py:9 order


def ln_mod(x, shift, scale, eps=1e-6):
    mu = x.mean(-1, keepdim=True)
    var = (x * x).mean(-1, keepdim=True) - mu * mu
    return (x - mu) * torch.rsqrt(var.clamp_min(0) + eps) * (1 + scale) + shift


def rms_head(x, gain, eps=1e-6):
    """x [..., H, 128]"""
    return x * torch.rsqrt(x.square().mean(-1, keepdim=True) + eps) * gain


def rope(x, cos, sin):
    """x [B, T, H, 128]; cos, sin [T, 64]"""
    a, b = x[..., :64], x[..., 64:]
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    return torch.cat((a * c - b * s, b * c + a * s), -1)


def attention(q, k, v, scale=1.0, nvalid=None):
    """q [B, Tq, H, d], k, v [B, Tk, H, d] -> [B, Tq, H, d]; keys >= nvalid masked."""
    s = torch.einsum("bqhd,bkhd->bhqk", q, k) * scale
    if nvalid is not None and nvalid < k.shape[1]:
        s[..., nvalid:] = float("-inf")
    p = torch.softmax(s, -1)
    return torch.einsum("bhqk,bkhd->bqhd", p, v)


def gelu(x):
    return 0.5 * x * (1 + torch.erf(x / math.sqrt(2.0)))


def make_rope(gh, gw, theta=10000.0, ntok=None):
    """cos, sin float32 [ntok][64]."""
    ntok = ntok or gh * gw
    dim_h = 128 // 6 * 2
    nt, nh = (128 - 2 * dim_h) // 2, dim_h // 2
    fh = 1.0 / np.power(float(theta), 2.0 * np.arange(nh) / dim_h)
    tk = np.arange(gh * gw)
    hh, ww = tk // gw, tk % gw
    ang = np.zeros((gh * gw, 64))
    ang[:, nt:nt + nh] = hh[:, None] * fh[None, :]
    ang[:, nt + nh:] = ww[:, None] * fh[None, :]
    cos = np.zeros((ntok, 64), np.float32)
    sin = np.zeros((ntok, 64), np.float32)
    cos[: gh * gw] = np.cos(ang)
    sin[: gh * gw] = np.sin(ang)
    return cos, sin


def modulation(modA, modB, emb, lora):
    """modA [3][256][D], modB [3][3D][256] (fp16 values), emb [D], lora [3D] -> mod [9][D] fp32."""
    s = emb * torch.sigmoid(emb)
    out = []
    for site in range(3):
        h1 = modA[site].float() @ s
        out.append(modB[site].float() @ h1 + lora)
    D = emb.shape[0]
    return torch.cat(out).view(9, D)


def block(x, ctx, mod, cos, sin, W, gain, heads=None):
    """x [B, T, D] fp32, ctx [B, C, Cd], mod [9][D], cos/sin [T][64], W[name] [out][in], gain [512] -> new x."""
    B, T, D = x.shape
    H = heads or D // HD
    x = x.clone()
    lin = lambda a, n: a @ W[n].T
    for site in range(3):
        sh, sc, gt = mod[3 * site], mod[3 * site + 1], mod[3 * site + 2]
        h = ln_mod(x, sh, sc)
        if site == 0:
            q = rope(rms_head(lin(h, "sq").view(B, T, H, HD), gain[0:128]), cos, sin)
            k = rope(rms_head(lin(h, "sk").view(B, T, H, HD), gain[128:256]), cos, sin)
            v = lin(h, "sv").view(B, T, H, HD)
            o = attention(q, k, v).reshape(B, T, D)
            x = x + gt * lin(o, "so")
        elif site == 1:
            C = ctx.shape[1]
            q = rms_head(lin(h, "cq").view(B, T, H, HD), gain[256:384])
            ck = rms_head(lin(ctx, "ck").view(B, C, H, HD), gain[384:512])
            cv = lin(ctx, "cv").view(B, C, H, HD)
            o = attention(q, ck, cv).reshape(B, T, D)
            x = x + gt * lin(o, "co")
        else:
            x = x + gt * lin(gelu(lin(h, "m1")), "m2")
    return x


def init_weights(seed, D=2048, F=8192, Cd=1024, std=0.02):
    """Seeded synthetic block: weights ~N(0, std), norm gains 1 + N(0, std), mod weights ~N(0, std)."""
    g = torch.Generator().manual_seed(seed)
    n = lambda *s: torch.randn(*s, generator=g) * std
    W = {"sq": n(D, D), "sk": n(D, D), "sv": n(D, D), "so": n(D, D), "cq": n(D, D), "ck": n(D, Cd), "cv": n(D, Cd),
         "co": n(D, D), "m1": n(F, D), "m2": n(D, F)}
    norms = {k: 1 + n(HD) for k in ("q", "k", "cq", "ck")}
    modA = n(3, 256, D).half()
    modB = n(3, 3 * D, 256).half()
    return W, norms, modA, modB


def pack_gain(norms):
    """[q/sqrt(128), k, cq/sqrt(128), ck] fp32 (export_all.py:31-32)."""
    sc = 1.0 / math.sqrt(HD)
    return torch.cat([norms["q"] * sc, norms["k"], norms["cq"] * sc, norms["ck"]]).float()


def build_pack(W, norms, modA, modB, q8=False):
    """blkNN.bin bytes (export_all.py main loop): 10 matrices as tiles of W^T, gains padded to 4096 B, mod weights."""
    from .packs import F16_FLOOR_ANIMA, q8tiles, wt16
    parts = []
    for name in ORDER:
        t = wt16(W[name].T.contiguous().numpy())
        parts.append(q8tiles(t, F16_FLOOR_ANIMA) if q8 else t.tobytes())
    g = pack_gain(norms).numpy().astype(np.float32)
    parts.append(g.tobytes() + bytes(4096 - g.nbytes))
    for site in range(3):
        parts.append(modA[site].numpy().astype(np.float16).tobytes())
        parts.append(modB[site].numpy().astype(np.float16).tobytes())
    return b"".join(parts)


def pack_weights(pack, D=2048, F=8192, Cd=1024, q8=False):
    """The fp32 [out][in] weights the device multiplies after loading `pack` (fp16 values or fp16(q*s))."""
    from .packs import dequant_q8_f16, unwt16
    dims = {"sq": (D, D), "sk": (D, D), "sv": (D, D), "so": (D, D), "cq": (D, D), "ck": (Cd, D), "cv": (Cd, D),
            "co": (D, D), "m1": (D, F), "m2": (F, D)}  # (K, N)
    W, off = {}, 0
    for name in ORDER:
        K, N = dims[name]
        nb, kb = N // 32, K // 32
        if q8:
            size = nb * kb * 1152
            w = dequant_q8_f16(pack[off:off + size], nb, kb)
        else:
            size = nb * kb * 2048
            t = np.frombuffer(pack[off:off + size], np.float16).reshape(nb, kb, 16, 32, 2)
            w = unwt16(t)
        W[name] = torch.from_numpy(w.astype(np.float32).T.copy())
        off += size
    gain = torch.from_numpy(np.frombuffer(pack[off:off + 2048], np.float32).copy())
    return W, gain


# ---------------------------------------------------------------- per-step glue (animad.cpp:423-492)
def sigma_schedule(steps):
    """animad.cpp:397-399: s = linspace(1, 0.001), sigma = 3s / (1 + 2s), final 0."""
    sig = []
    for i in range(steps):
        sv = 1.0 - (1.0 - 0.001) * i / (steps - 1) if steps > 1 else 1.0
        sig.append(np.float32(3 * sv / (1 + 2 * sv)))
    return sig + [np.float32(0.0)]


def timestep_embedding(t, D, w_norm):
    """animad.cpp:424-427 in float32: tp = [cos(t f_i) | sin(t f_i)], f_i = exp(-ln(1e4) i / (D/2)); emb = rms(tp) * w."""
    half = D // 2
    i = np.arange(half, dtype=np.float32)
    f = np.exp(-np.log(np.float32(10000.0)) * i / np.float32(half)).astype(np.float32)
    a = (np.float32(t) * f).astype(np.float32)
    tp = torch.from_numpy(np.concatenate([np.cos(a), np.sin(a)]).astype(np.float32))
    emb = tp / torch.sqrt(tp.square().mean() + 1e-6) * w_norm.float()
    return tp, emb


def glue_init(seed, D=2048, std=0.02):
    g = torch.Generator().manual_seed(seed)
    n = lambda *s: (torch.randn(*s, generator=g) * std).half()
    return {"t_norm": (1 + torch.randn(D, generator=g) * std).half(), "t_lin1": n(D, D), "t_lin2": n(3 * D, D),
            "x_emb": n(D, 68), "f_modA": n(256, D), "f_modB": n(2 * D, 256), "f_lin": n(64, D)}


def patchify(lat):
    """[B][16][H][W] -> [B][T][68] with feature c*4 + a*2 + b and a zero 17th channel (animad.cpp:447-449)."""
    B, C, H, W = lat.shape
    p = lat.view(B, C, H // 2, 2, W // 2, 2).permute(0, 2, 4, 1, 3, 5).reshape(B, (H // 2) * (W // 2), C * 4)
    return torch.cat((p, torch.zeros(B, p.shape[1], 4)), -1)


def unpatchify(y, H, W, C=16):
    """[B][T][64] with feature (a*2+b)*16 + c -> [B][16][H][W] (animad.cpp:490-492)."""
    B = y.shape[0]
    return y.view(B, H // 2, W // 2, 2, 2, C).permute(0, 5, 1, 3, 2, 4).reshape(B, C, H, W)


def sample_step(lat, sig_i, sig_next, ctx, cos, sin, blocks, glue):
    """One Euler denoising step of animad.cpp:423-492 at sigma sig_i: timestep embedding, t_embedder,
    patchify + x_embedder, every block with its modulation, final layer, unpatchify,
    lat + (sig_next - sig_i) * v. Returns the new latent."""
    B, C, H, Wd = lat.shape
    D = glue["t_lin1"].shape[0]
    tp, emb = timestep_embedding(sig_i, D, glue["t_norm"])
    lora = glue["t_lin2"].float() @ torch.nn.functional.silu(glue["t_lin1"].float() @ tp)
    x = patchify(lat) @ glue["x_emb"].float().T
    for (W, gain, modA, modB) in blocks:
        x = block(x, ctx, modulation(modA, modB, emb, lora), cos, sin, W, gain)
    fm = glue["f_modB"].float() @ (glue["f_modA"].float() @ torch.nn.functional.silu(emb)) + lora[: 2 * D]
    h = ln_mod(x, fm[:D], fm[D:])
    v = unpatchify(h @ glue["f_lin"].float().T, H, Wd)
    return lat + (float(sig_next) - float(sig_i)) * v


def sample(lat, ctx, cos, sin, blocks, glue, steps=4, sigmas=None):
    """Full Euler sample of animad.cpp:423-492: blocks = [(W, gain, modA, modB)] (iterated once per
    step), glue = glue_init dict. lat [B][16][H][W] fp32 -> denoised latent."""
    sig = sigmas if sigmas is not None else sigma_schedule(steps)
    lat = lat.clone()
    for i in range(steps):
        lat = sample_step(lat, sig[i], sig[i + 1], ctx, cos, sin, blocks, glue)
    return lat


# ---------------------------------------------------------------- LLM adapter (text side)
ADAPTER_DIM, ADAPTER_HEADS, ADAPTER_HD, ADAPTER_FF, ADAPTER_BLOCKS, ADAPTER_CTX = 1024, 16, 64, 4096, 6, 512
ADAPTER_BLOCK_KEYS = ("norm_sa", "sa_q", "sa_k", "sa_v", "sa_o", "sa_qn", "sa_kn", "norm_ca", "ca_q", "ca_k", "ca_v",
                      "ca_o", "ca_qn", "ca_kn", "norm_mlp", "mlp0_w", "mlp0_b", "mlp2_w", "mlp2_b")


def adapter_rope(n, hd=ADAPTER_HD):
    """1D split-half RoPE tables [n][hd/2] (phone/animad.cpp:130-137 `rope1d`): angle i / 10000^(2j/hd),
    in float64, rounded to float32."""
    j = np.arange(hd // 2, dtype=np.float64)
    a = np.arange(n, dtype=np.float64)[:, None] / np.power(10000.0, 2.0 * j / hd)[None, :]
    return torch.from_numpy(np.cos(a).astype(np.float32)), torch.from_numpy(np.sin(a).astype(np.float32))


def _adapter_rms(x, g, eps=1e-6):
    return x * torch.rsqrt((x.double() ** 2).mean(-1, keepdim=True).float() + eps) * g


def _adapter_rope(t, c, s):
    """t [n, heads, 64]: pairs (j, j+32) rotated (animad.cpp:138-148 `rope_apply`)."""
    a, b = t[..., :32], t[..., 32:]
    c, s = c[:, None, :], s[:, None, :]
    return torch.cat((a * c - b * s, a * s + b * c), -1)


def adapter(hidden, ids, wts, W):
    """The Anima LLM adapter (phone/animad.cpp:179-218): T5 token ids [L] and LLM hidden states
    hidden [S][1024] -> cross-attention context [512][1024] (rows >= L zero). Six blocks of
    RMS -> self-attention (16 heads x 64, per-head RMS on q/k, 1D RoPE) -> RMS -> cross-attention to
    hidden (keys roped with their own positions) -> RMS -> MLP 1024 -> 4096 (GELU erf) -> 1024, each
    adding into x; then out_proj, RMS (norm) and a per-token weight. Float32 math on fp16 weights;
    W holds fp32 copies of the fp16 weights: "embed", "blocks" (list of dicts with ADAPTER_BLOCK_KEYS),
    "out_w", "out_b", "norm"."""
    L, S = len(ids), hidden.shape[0]
    H, hd = ADAPTER_HEADS, ADAPTER_HD
    x = W["embed"][torch.as_tensor(ids, dtype=torch.long)].clone()
    tc, ts = adapter_rope(L)
    sc, ss = adapter_rope(S)

    def attn(Bw, pre, xq, xkv, cross):
        q = (xq @ Bw[pre + "_q"].T).view(-1, H, hd)
        k = (xkv @ Bw[pre + "_k"].T).view(-1, H, hd)
        v = (xkv @ Bw[pre + "_v"].T).view(-1, H, hd)
        q = _adapter_rope(_adapter_rms(q, Bw[pre + "_qn"]), tc, ts)
        k = _adapter_rope(_adapter_rms(k, Bw[pre + "_kn"]), sc if cross else tc, ss if cross else ts)
        p = torch.softmax(torch.einsum("qhd,khd->hqk", q, k) * 0.125, -1)
        o = torch.einsum("hqk,khd->qhd", p, v).reshape(-1, H * hd)
        return o @ Bw[pre + "_o"].T

    for Bw in W["blocks"]:
        h = _adapter_rms(x, Bw["norm_sa"])
        x = x + attn(Bw, "sa", h, h, False)
        h = _adapter_rms(x, Bw["norm_ca"])
        x = x + attn(Bw, "ca", h, hidden, True)
        h = _adapter_rms(x, Bw["norm_mlp"])
        m = gelu(h @ Bw["mlp0_w"].T + Bw["mlp0_b"])
        x = x + (m @ Bw["mlp2_w"].T + Bw["mlp2_b"])
    y = _adapter_rms(x @ W["out_w"].T + W["out_b"], W["norm"]) * torch.as_tensor(wts, dtype=torch.float32)[:, None]
    out = torch.zeros(ADAPTER_CTX, ADAPTER_DIM)
    out[:L] = y
    return out


def adapter_init(seed, vocab=1000, std=0.02):
    """Seeded synthetic adapter weights, fp16-representable (returned as fp16 tensors)."""
    g = torch.Generator().manual_seed(seed)
    D, F = ADAPTER_DIM, ADAPTER_FF
    n = lambda *s: (torch.randn(*s, generator=g) * std).half()
    gn = lambda d: (1 + 0.1 * torch.randn(d, generator=g)).half()
    blocks = []
    for _ in range(ADAPTER_BLOCKS):
        b = {}
        for pre in ("sa", "ca"):
            for m in ("q", "k", "v", "o"):
                b[f"{pre}_{m}"] = n(D, D)
            b[f"{pre}_qn"], b[f"{pre}_kn"] = gn(ADAPTER_HD), gn(ADAPTER_HD)
        b["norm_sa"], b["norm_ca"], b["norm_mlp"] = gn(D), gn(D), gn(D)
        b["mlp0_w"], b["mlp0_b"], b["mlp2_w"], b["mlp2_b"] = n(F, D), n(F), n(D, F), n(D)
        blocks.append(b)
    return {"embed": (torch.randn(vocab, D, generator=g)).half(), "blocks": blocks, "out_w": n(D, D), "out_b": n(D),
            "norm": gn(D)}


def adapter_f32(W16):
    """fp32 copies of fp16 adapter weights (the arithmetic the reference does on them)."""
    return {"embed": W16["embed"].float(), "blocks": [{k: v.float() for k, v in b.items()} for b in W16["blocks"]],
            "out_w": W16["out_w"].float(), "out_b": W16["out_b"].float(), "norm": W16["norm"].float()}
