"""Parity of the benchmarked workloads at their full shapes, end to end.

The sample (hx_anima_sample: timestep embedding, x_embedder, per-block AdaLN modulation, the block chain,
final layer, unpatchify and Euler, phone/animad.cpp:397-399,423-492; blocks hexagon/mega/blk.c:148-175)
runs at the real Anima shape: hidden 2048, 16 heads, 1536 image tokens of a 512x768 image, 256 text tokens
of width 1024, MLP 8192, 4 steps, on the synthetic weights bench.py times (hexanima_b200.synth). The
oracle (oracle.anima.sample, torch fp32 on the CPU) is fed the exact operand values the device multiplies:
the fp16 weights, or fp16(q*s) of the q8 records, rebuilt block by block from the device copies.

Bars (north_star): rel-L2 <= 1e-2 on the latent update after the full 4-step sample; <= 2e-3 on the delta
of one block.
  * config 3: 36 q8-g64 blocks, 2 images (3072 rows: the weight-expansion path with look-ahead on the
    side stream that the bench runs from two images up), each image checked on its own;
  * config 2: 28 fp16 blocks, 1 image;
  * one q8-g64 block at 8 images (12288 rows, the bench's per-GPU load at one GPU) through hx_mega_block.
"""
import pytest
import torch

from hexanima_b200 import runtime as rt
from hexanima_b200 import synth
from oracle import anima as oa
from tests.gpu_util import LazyAnimaBlocks, dequant_q8_torch, read_f32, rel, write_f32

D, F, Cd, T, C, LH, LW = 2048, 8192, 1024, 1536, 256, 64, 96
SAMPLE_TOL, BLOCK_TOL = 1e-2, 2e-3


@pytest.fixture(scope="module")
def h():
    hd = rt.Handle(0)
    yield hd
    assert hd.status() == 0
    hd.close()


def _blob(h, B, ctx, cos, sin):
    meta, total = rt.blob_layout(rt.MODEL_ANIMA, T, C, B, D, F, Cd)
    bfd = h.buf_alloc(total)
    A = rt.A
    h.buf_write(bfd, meta[A["CTX"]], ctx.numpy())
    write_f32(h, bfd, meta[A["COS"]], cos)
    write_f32(h, bfd, meta[A["SIN"]], sin)
    return meta, bfd


def test_dequant_helper_matches_oracle_codec():
    import numpy as np
    from oracle import packs as op
    g = torch.Generator().manual_seed(3)
    u = torch.randint(1, 256, (64, 256), dtype=torch.uint8, generator=g)
    s = (torch.randn(4, 64, generator=g).abs() * (0.02 / 127)).half()
    ref = op.dequant_q8(u.numpy(), s.numpy(), 64).astype(np.float32)
    assert np.array_equal(dequant_q8_torch(u, s, 64).numpy(), ref)


@pytest.mark.gpu
@pytest.mark.parametrize("name,fmt,nblk,B", [("config3-q8g64-36blk-2img", rt.FMT_Q8, 36, 2),
                                             ("config2-f16-28blk-1img", rt.FMT_F16, 28, 1)])
def test_full_sample_matches_oracle(h, name, fmt, nblk, B):
    seed = 5000 if fmt == rt.FMT_Q8 else 6000
    wfds, ts = synth.anima_blocks(h, nblk, fmt, seed, D, F, Cd, 64)
    glue = synth.anima_glue(D, seed + 999)
    gfd = synth.load_glue(h, D, glue)
    g = torch.Generator().manual_seed(seed + 7)
    lat = torch.randn(B, 16, LH, LW, generator=g)
    ctx = torch.randn(B, C, Cd, generator=g).half()
    cos, sin = rt.rope_anima(LH // 2, LW // 2, 10000.0, T)
    meta, bfd = _blob(h, B, ctx, cos, sin)
    lat_dev = lat.clone().cuda()
    h.anima_sample(gfd, meta, wfds, bfd, lat_dev, LH, LW, 4, use_graph=True)
    h.sync()
    got = lat_dev.cpu()
    assert h.status() == 0
    h.buf_free(bfd)
    torch.set_grad_enabled(False)
    ref = oa.sample(lat, ctx.float(), torch.from_numpy(cos), torch.from_numpy(sin), LazyAnimaBlocks(ts, fmt, D),
                    {k: v.cpu() for k, v in glue.items()}, 4)
    for w in wfds:
        h.weights_free(w)
    del ts
    assert torch.isfinite(got).all()
    errs = [rel(got[b] - lat[b], ref[b] - lat[b]) for b in range(B)]
    err = rel(got - lat, ref - lat)
    print(f"{name}: rel-L2 of the latent update {err:.3e} (per image {', '.join(f'{e:.3e}' for e in errs)})")
    assert err < SAMPLE_TOL
    assert max(errs) < SAMPLE_TOL


@pytest.mark.gpu
def test_q8_block_at_eight_images(h):
    B = 8
    wfds, ts = synth.anima_blocks(h, 1, rt.FMT_Q8, 7100, D, F, Cd, 64)
    g = torch.Generator().manual_seed(7101)
    x = torch.randn(B, T, D, generator=g)
    ctx = torch.randn(B, C, Cd, generator=g).half()
    mod = torch.randn(9, D, generator=g) * 0.1
    cos, sin = oa.make_rope(LH // 2, LW // 2, ntok=T)
    meta, bfd = _blob(h, B, ctx, cos, sin)
    write_f32(h, bfd, meta[rt.A["X"]], x.numpy())
    h.mega_block(meta, wfds[0], bfd, mod=mod.numpy())
    y = torch.from_numpy(read_f32(h, bfd, meta[rt.A["X"]], B * T * D).reshape(B, T, D))
    assert h.status() == 0
    h.buf_free(bfd)
    W, gain, _, _ = LazyAnimaBlocks(ts, rt.FMT_Q8, D).weights(0)
    h.weights_free(wfds[0])
    torch.set_grad_enabled(False)
    ref = oa.block(x, ctx.float(), mod, torch.from_numpy(cos), torch.from_numpy(sin), W, gain)
    errs = [rel(y[b] - x[b], ref[b] - x[b]) for b in range(B)]
    print(f"q8-g64 block, 8 images: rel-L2 of the block delta per image max {max(errs):.3e}")
    assert max(errs) < BLOCK_TOL
