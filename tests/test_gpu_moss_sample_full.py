"""The MOSS sampler at the full width and token count of the 1 Mpx configuration: hidden 3072, 24 heads,
MLP 12288, q4 weights in groups of 32, a 64x64 latent of 128 channels (4096 image tokens) plus 512 text
tokens in one joint attention (4608 tokens), the four rapid-moss steps (hx_moss_sample as one CUDA graph:
time vectors, latent mix, video embedder, block chain, head, x0 update; moss/sample_ref.py:15-22,
moss/mossrun/mossrun.cpp:316-333) against oracle.moss.sample_dev fed the device's operand values.

Two blocks instead of 42 keep the CPU oracle at about 20 s; every kernel runs at its real shape.
Bar (north_star): rel-L2 <= 1e-2 of the final x0 and of its velocity part after the 4-step sample."""
import math

import numpy as np
import pytest
import torch

from hexanima_b200 import runtime as rt
from oracle import moss as om
from oracle import packs as op
from tests.gpu_util import dev, rel

pytestmark = pytest.mark.gpu
D, F, LH, LW, T, B, NBLK = 3072, 12288, 64, 64, 512, 1, 2
CODES = [1000.0, 968.0, 926.0, 871.0]   # the rapid-moss step codes


def test_moss_1mpx_sample_matches_oracle():
    h = rt.Handle(0)
    try:
        gdev = torch.Generator(device="cuda").manual_seed(4400)
        wfds, blocks, keep = [], [], []
        shapes = {rt.W_QKV: ("qkv", 3 * D, D), rt.W_O: ("o", D, D), rt.W_M1: ("ug", 2 * F, D), rt.W_M2: ("dn", D, F)}
        for i in range(NBLK):
            mats, deq = {}, {}
            for slot, (name, n, k) in shapes.items():
                p = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device="cuda", generator=gdev)
                s = (torch.randn(k // 32, n, device="cuda", generator=gdev).abs() * (0.02 / 7)).half()
                mats[slot] = rt.make_mat(rt.FMT_Q4, n, k, p, s, group=32)
                keep += [p, s]
                deq[name] = torch.from_numpy(op.dequant_q4(p.cpu().numpy(), s.cpu().numpy(), 32).astype(np.float32))
            g = torch.Generator().manual_seed(4500 + i)
            gain = torch.cat((1 + 0.1 * torch.randn(128, generator=g), 1 + 0.1 * torch.randn(128, generator=g),
                              1 + 0.1 * torch.randn(2 * D, generator=g)))
            gain[:128] /= math.sqrt(128.0)
            tg = gain.cuda()
            keep.append(tg)
            wfds.append(h.weights_bind(rt.MODEL_MOSS, D, F, mats, tg, lora=0, keep=keep))
            blocks.append((deq, gain, False))
        glue = om.init_glue_weights(4600, D)
        t16 = lambda k: dev(glue[k].half().numpy())
        t32 = lambda k: dev(glue[k].float().numpy())
        gfd = h.moss_glue_load(D, t_lin0=t16("time_embedding.0.weight"), t_b0=t32("time_embedding.0.bias"),
                               t_lin2=t16("time_embedding.2.weight"), t_b2=t32("time_embedding.2.bias"),
                               mod_w=t16("shared_block_modulation.weight"), mod_b=t32("shared_block_modulation.bias"),
                               head_w=t16("video_head_modulation.weight"), head_b=t32("video_head_modulation.bias"),
                               emb_w=t16("video_embedder.weight"), emb_b=t32("video_embedder.bias"),
                               fin_norm=t32("final_norm_video.weight"), fin_w=t16("final_linear_video.weight"),
                               mix_q=t32("latent_mix.Q"))
        Ni = LH * LW
        ntok = Ni + T
        g = torch.Generator().manual_seed(4601)
        z = torch.randn(B, 128, Ni, generator=g)
        tx = torch.randn(T, D, generator=g)
        meta, total = rt.blob_layout(rt.MODEL_MOSS, ntok, 0, B, D, F)
        bfd = h.buf_alloc(total)
        c, s = rt.rope_moss(LH, LW, T, om.bands16().numpy(), ntok)
        S = rt.S
        h.buf_write(bfd, meta[S["COS"]], c)
        h.buf_write(bfd, meta[S["SIN"]], s)
        x0d = torch.zeros(B, 128, Ni, device="cuda")
        h.moss_sample(gfd, meta, wfds, bfd, z.cuda(), x0d, LH, LW, tx.cuda(), T, CODES, use_graph=True)
        h.sync()
        got = x0d.cpu()
        assert h.status() == 0
        h.buf_free(bfd)
        for w in wfds:
            h.weights_free(w)
        torch.set_grad_enabled(False)
        ref = om.sample_dev(z, torch.zeros(B, 128, Ni), tx, glue, blocks, CODES, torch.from_numpy(c),
                            torch.from_numpy(s), ntok)
        assert torch.isfinite(got).all()
        e_x0, e_v = rel(got, ref), rel(got - z, ref - z)
        print(f"MOSS 1 Mpx q4 sample, {NBLK} blocks: rel-L2 x0 {e_x0:.3e}, velocity part {e_v:.3e}")
        assert e_x0 < 1e-2
        assert e_v < 1e-2
    finally:
        h.close()
