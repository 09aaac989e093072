"""The MOSS sampler on the GPU (hx_moss_glue_load + hx_moss_sample: time vectors, latent mix, video
embedder, block chain, head, x0 update as one CUDA graph) against oracle.moss.sample_dev on the same
device operands. Bar (north_star): rel-L2 of the final x0 <= 1e-2 after the full 4-step sample."""
import numpy as np
import pytest
import torch

from hexanima_b200 import runtime as rt
from oracle import moss as om
from tests.gpu_util import dev, make_mat, rel

pytestmark = pytest.mark.gpu
D, F, LH, LW, T, B = 512, 256, 4, 6, 8, 2
CODES = [1000.0, 968.0, 926.0, 871.0]   # the rapid-moss step codes


@pytest.fixture(scope="module")
def h():
    hd = rt.Handle(0)
    yield hd
    assert hd.status() == 0
    hd.close()


def _blocks(h, n):
    from oracle import packs as op
    out, wfds, keep = [], [], []
    for i in range(n):
        g = torch.Generator().manual_seed(80 + i)
        qkv = torch.randn(3 * D, D, generator=g) * 0.02
        o = torch.randn(D, D, generator=g) * 0.02
        up, gate = torch.randn(F, D, generator=g) * 0.02, torch.randn(F, D, generator=g) * 0.02
        dn = torch.randn(D, F, generator=g) * 0.02
        mats, deq = {}, {}
        for slot, name, w in ((rt.W_QKV, "qkv", qkv), (rt.W_O, "o", o),
                              (rt.W_M1, "ug", torch.from_numpy(op.situ_rows(up.numpy(), gate.numpy()))),
                              (rt.W_M2, "dn", dn)):
            m, k, d = make_mat(rt.FMT_Q8, w.numpy(), 32)
            mats[slot], deq[name] = m, d
            keep += k
        gain = torch.cat((1 + 0.1 * torch.randn(128, generator=g), 1 + 0.1 * torch.randn(128, generator=g),
                          1 + 0.1 * torch.randn(2 * D, generator=g)))
        gain[:128] /= np.sqrt(128.0)
        tg = gain.cuda()
        keep.append(tg)
        wfds.append(h.weights_bind(rt.MODEL_MOSS, D, F, mats, tg, lora=0, keep=keep))
        out.append((deq, gain, False))
    return wfds, out


def test_moss_sample_matches_oracle(h):
    wfds, blocks = _blocks(h, 2)
    glue = om.init_glue_weights(90, D)
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
    ntok = 32
    g = torch.Generator().manual_seed(91)
    z = torch.randn(B, 128, Ni, generator=g)
    tx = torch.randn(T, D, generator=g)
    meta, total = rt.blob_layout(rt.MODEL_MOSS, ntok, 0, B, D, F)
    bfd = h.buf_alloc(total)
    c, s = rt.rope_moss(LH, LW, T, om.bands16().numpy(), ntok)
    S = rt.S
    h.buf_write(bfd, meta[S["COS"]], c)
    h.buf_write(bfd, meta[S["SIN"]], s)
    zd, txd = z.cuda(), tx.cuda()
    results = []
    for use_graph in (True, False):
        x0d = torch.zeros(B, 128, Ni, device="cuda")
        h.moss_sample(gfd, meta, wfds, bfd, zd, x0d, LH, LW, txd, T, CODES, use_graph=use_graph)
        h.sync()
        results.append(x0d.cpu())
    assert torch.equal(results[0], results[1])        # graph replay == direct launches
    ref = om.sample_dev(z, torch.zeros(B, 128, Ni), tx, glue, blocks, CODES, torch.from_numpy(c), torch.from_numpy(s),
                        ntok)
    assert rel(results[0], ref) < 1e-2
    assert rel(results[0] - z, ref - z) < 1e-2          # the velocity part itself, not just z
    # the same glue read from a glue.bin file (export_glue.py dtypes: fp32 except the two modulation matrices)
    from tests.test_mgl1 import write_mgl1
    f16 = ("shared_block_modulation.weight", "video_head_modulation.weight")
    f = write_mgl1([(k, 1 if k in f16 else 0, v.numpy()) for k, v in glue.items()] +
                   [("step_codes", 0, np.array(CODES, np.float32)), ("rope.bands", 0, om.bands16().numpy())])
    gfd2 = h.moss_glue_load_mgl1(f)
    x0d = torch.zeros(B, 128, Ni, device="cuda")
    h.moss_sample(gfd2, meta, wfds, bfd, zd, x0d, LH, LW, txd, T, rt.mgl1_tensor(f, "step_codes"))
    h.sync()
    assert torch.equal(x0d.cpu(), results[0])
    h.buf_free(bfd)
    for w in wfds:
        h.weights_free(w)
