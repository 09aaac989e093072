"""Seeded synthetic Anima weight sets generated on the device, shared by bench.py and the GPU tests.

Distributions follow the benchmark configs: q8 weights as int8 values uniform in [-127, 127] (stored
offset binary, u = q + 128 in [1, 255]) with fp16 scales |N(0, 0.02)| / 127 per group of `group` along
K; fp16 weights ~N(0, 0.02); norm gains 1 + N(0, 0.02) with the q and cross-q gains pre-scaled by
1/sqrt(128) (hexagon/mega/export_all.py:31-32); modulation weights fp16 ~N(0, 0.02) in the pack's
[3][256][D] / [3][3D][256] layout (hexagon/mega/blk_wlayout.h:14). Block i draws from its own
generator (seed + i), so any block can be regenerated alone.
"""
import torch

from . import runtime as rt


def anima_shapes(D, F, Cd):
    """Fused weight slots of an Anima block: (N, K) per slot, W[N][K]."""
    return {rt.W_QKV: (3 * D, D), rt.W_O: (D, D), rt.W_CQ: (D, D), rt.W_CKV: (2 * D, Cd), rt.W_CO: (D, D),
            rt.W_M1: (F, D), rt.W_M2: (D, F)}


def anima_block_tensors(seed, fmt, D=2048, F=8192, Cd=1024, group=64, device="cuda"):
    """One block's device tensors: {"mats": {slot: (w, scale|None)}, "gain", "modA", "modB"}."""
    g = torch.Generator(device=device).manual_seed(seed)
    mats = {}
    for slot, (n, k) in anima_shapes(D, F, Cd).items():
        if fmt == rt.FMT_F16:
            mats[slot] = ((0.02 * torch.randn(n, k, device=device, generator=g)).half(), None)
        elif fmt == rt.FMT_Q8:
            u = torch.randint(1, 256, (n, k), dtype=torch.uint8, device=device, generator=g)
            s = (torch.randn(k // group, n, device=device, generator=g).abs() * (0.02 / 127)).half()
            mats[slot] = (u, s)
        else:
            raise ValueError("synthetic Anima blocks are fp16 or q8")
    gain = 1 + 0.02 * torch.randn(512, device=device, generator=g)
    gain[:128] /= 128 ** 0.5
    gain[256:384] /= 128 ** 0.5
    modA = (0.02 * torch.randn(3, 256, D, device=device, generator=g)).half()
    modB = (0.02 * torch.randn(3, 3 * D, 256, device=device, generator=g)).half()
    return {"mats": mats, "gain": gain, "modA": modA, "modB": modB}


def bind_anima_block(h, t, fmt, D=2048, F=8192, Cd=1024, group=64):
    """Bind one block's tensors (anima_block_tensors) to the handle; returns the weight-set fd."""
    mats, keep = {}, []
    for slot, (w, s) in t["mats"].items():
        n, k = w.shape
        mats[slot] = rt.make_mat(fmt, n, k, w, s, group=group) if fmt == rt.FMT_Q8 else rt.make_mat(fmt, n, k, w)
        keep += [w] if s is None else [w, s]
    keep += [t["gain"], t["modA"], t["modB"]]
    return h.weights_bind(rt.MODEL_ANIMA, D, F, mats, t["gain"], Cd=Cd, modA=t["modA"], modB=t["modB"], keep=keep)


def anima_blocks(h, n, fmt, seed, D=2048, F=8192, Cd=1024, group=64, device="cuda"):
    """n blocks bound to the handle: (wfds, tensors per block)."""
    wfds, ts = [], []
    for i in range(n):
        t = anima_block_tensors(seed + i, fmt, D, F, Cd, group, device)
        wfds.append(bind_anima_block(h, t, fmt, D, F, Cd, group))
        ts.append(t)
    return wfds, ts


def anima_glue(D, seed, device="cuda"):
    """Glue weights of the sampler (t_embedder, x_embedder, final layer), fp16 ~N(0, 0.02)."""
    g = torch.Generator(device=device).manual_seed(seed)
    n = lambda *s: (0.02 * torch.randn(*s, device=device, generator=g)).half()
    return {"t_norm": (1 + 0.02 * torch.randn(D, device=device, generator=g)).half(), "t_lin1": n(D, D),
            "t_lin2": n(3 * D, D), "x_emb": n(D, 68), "f_modA": n(256, D), "f_modB": n(2 * D, 256), "f_lin": n(64, D)}


def load_glue(h, D, glue):
    return h.glue_load(D, glue["t_norm"], glue["t_lin1"], glue["t_lin2"], glue["x_emb"], glue["f_modA"],
                       glue["f_modB"], glue["f_lin"])
