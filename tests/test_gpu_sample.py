"""Full 4-step Anima sample on the GPU (hx_anima_sample) against the oracle sampler.

Bar (north_star): rel-L2 <= 1e-2 on the latent update after the full sample."""
import numpy as np
import pytest
import torch

from hexanima_b200 import runtime as rt
from oracle import anima as oa
from tests.gpu_util import anima_bind, rel, write_f32

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def h():
    hd = rt.Handle(0)
    yield hd
    assert hd.status() == 0
    hd.close()


@pytest.mark.parametrize("fmt,use_graph", [(rt.FMT_F16, True), (rt.FMT_Q8, False)])
def test_anima_sample_matches_oracle(h, fmt, use_graph):
    D, F, Cd, B, C, nblk, steps = 256, 512, 128, 2, 64, 2, 4
    LH, LW = 16, 24
    T = (LH // 2) * (LW // 2)
    sets = [oa.init_weights(70 + i, D=D, F=F, Cd=Cd) for i in range(nblk)]
    bound = [anima_bind(h, *s, fmt=fmt, group=64) for s in sets]
    glue = oa.glue_init(77, D=D)
    gt = {k: v.cuda() for k, v in glue.items()}
    gfd = h.glue_load(D, gt["t_norm"], gt["t_lin1"], gt["t_lin2"], gt["x_emb"], gt["f_modA"], gt["f_modB"], gt["f_lin"])
    g = torch.Generator().manual_seed(78)
    lat = torch.randn(B, 16, LH, LW, generator=g)
    ctx = torch.randn(B, C, Cd, generator=g).half()
    cos, sin = rt.rope_anima(LH // 2, LW // 2, 10000.0, T)
    meta, total = rt.blob_layout(rt.MODEL_ANIMA, T, C, B, D, F, Cd)
    bfd = h.buf_alloc(total)
    A = rt.A
    h.buf_write(bfd, meta[A["CTX"]], ctx.numpy())
    write_f32(h, bfd, meta[A["COS"]], cos)
    write_f32(h, bfd, meta[A["SIN"]], sin)
    lat_dev = lat.clone().cuda()
    h.anima_sample(gfd, meta, [b[0] for b in bound], bfd, lat_dev, LH, LW, steps, use_graph=use_graph)
    h.sync()
    got = lat_dev.cpu()
    blocks = [(bound[i][1], bound[i][2], sets[i][2], sets[i][3]) for i in range(nblk)]
    ref = oa.sample(lat, ctx.float(), torch.from_numpy(cos), torch.from_numpy(sin), blocks, glue, steps)
    assert torch.isfinite(got).all()
    assert rel(got - lat, ref - lat) < 1e-2
    if use_graph:  # a second call replays the captured graph from a fresh latent and gives the same bits
        lat_dev.copy_(lat.cuda())
        h.anima_sample(gfd, meta, [b[0] for b in bound], bfd, lat_dev, LH, LW, steps, use_graph=True)
        h.sync()
        assert torch.equal(lat_dev.cpu(), got)
    h.buf_free(bfd)
    for b in bound:
        h.weights_free(b[0])

