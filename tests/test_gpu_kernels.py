"""Kernel-level parity on the GPU, through the C ABI (hx_gemm / hx_attention / hx_lnmod / hx_rmsmod).

Tolerances: dequantisation bit-exact; GEMM / attention outputs within fp16-output rounding of an
fp32 reference computed from the same fp16 operands (rel-L2 <= 2e-3 per output tensor)."""
import math

import numpy as np
import pytest
import torch

from hexanima_b200 import runtime as rt
from oracle import anima as oa
from oracle import moss as om
from tests.gpu_util import make_mat, rel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def h():
    hd = rt.Handle(0)
    yield hd
    assert hd.status() == 0
    hd.close()


TILES = [1, 2]  # single-CTA 128x256 tiles, CTA-pair 256x256 tiles (cta_group::2)
TILES3 = [1, 2, 3, 4]  # + q8 weights dequantised into TMEM; quantised weights expanded to fp16 first
TILE224 = 5  # CTA-pair 256x224 tiles (112 weight rows per CTA): GELU / store epilogues, fp16 or q8 weights


def _onehot_dequant(h, fmt, w, group, tile):
    """out = I * W^T reproduces the device's dequantised operand exactly (one fp32 product per output)."""
    N, K = w.shape
    mat, keep, deq = make_mat(fmt, w, group)
    A = torch.eye(K, dtype=torch.float16, device="cuda")
    out = torch.zeros(K, N, dtype=torch.float16, device="cuda")
    h.gemm(A, K, mat, rt.EPI_STORE, lda=K, out=out, ldo=N, tile=tile)
    h.sync()
    return out.cpu().T.contiguous(), deq


@pytest.mark.parametrize("tile", TILES3 + [TILE224])
@pytest.mark.parametrize("fmt,group", [(rt.FMT_F16, 64), (rt.FMT_Q8, 32), (rt.FMT_Q8, 64), (rt.FMT_Q4, 32),
                                       (rt.FMT_Q4A, 32)])
def test_dequant_bit_exact(h, fmt, group, tile):
    if tile == 3 and fmt != rt.FMT_Q8:
        pytest.skip("the TMEM-weight kernel takes q8 weights")
    if tile == TILE224 and fmt not in (rt.FMT_F16, rt.FMT_Q8):
        pytest.skip("224-column pair tiles take fp16 or q8 weights")
    rng = np.random.default_rng(7)
    N, K = (512 if tile == 3 else 320), 256
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    w[3] *= 1e-3     # small scales: subnormal fp16 products
    w[7] *= 300.0    # large values
    w[11] = 0.0
    got, deq = _onehot_dequant(h, fmt, w, group, tile)
    ref = deq.half()
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), int((got != ref).sum())


def _ref_gemm(A16, Wd):
    return A16.float().cpu() @ Wd.T


@pytest.mark.parametrize("tile", TILES3 + [TILE224])
@pytest.mark.parametrize("fmt", [rt.FMT_F16, rt.FMT_Q8, rt.FMT_Q4])
def test_gemm_store_and_gelu(h, fmt, tile):
    if tile == 3 and fmt != rt.FMT_Q8:
        pytest.skip("the TMEM-weight kernel takes q8 weights")
    if tile == TILE224 and fmt == rt.FMT_Q4:
        pytest.skip("224-column pair tiles take fp16 or q8 weights")
    torch.manual_seed(1)
    M, K, N = 300, 512, (512 if tile == 3 else 544)
    A = torch.randn(M, K).half()
    mat, keep, Wd = make_mat(fmt, (torch.randn(N, K) * 0.05).numpy(), 32)
    ref = _ref_gemm(A, Wd)
    for epi, f in ((rt.EPI_STORE, lambda t: t), (rt.EPI_GELU, oa.gelu)):
        out = torch.zeros(M, N, dtype=torch.float16, device="cuda")
        Ad = A.cuda()
        torch.cuda.synchronize()  # torch's stream and the handle's (non-blocking) stream are not ordered
        h.gemm(Ad, M, mat, epi, lda=K, out=out, ldo=N, tile=tile)
        h.sync()
        assert rel(out.float(), f(ref)) < 2e-3


@pytest.mark.parametrize("tile", TILES)
def test_gelu_epilogue_ulps(h, tile):
    """The GELU epilogue's polynomial erfc (csrc/hx_gelu.cuh) on exactly known inputs: a one-hot GEMM
    passes fp16 weights spanning [-10, 10] through unchanged, so out = fp16(gelu(w)); against the exact
    erf GELU rounded to fp16: at most one ulp apart, and on at most 2 % of the values."""
    import scipy.special as sp
    K, N = 256, 512
    rng = np.random.default_rng(11)
    w = np.concatenate((np.linspace(-10, 10, N * K // 2), rng.uniform(-6, 6, N * K // 2))).astype(np.float16)
    rng.shuffle(w)
    w = w.reshape(N, K)
    mat, keep, _ = make_mat(rt.FMT_F16, w.astype(np.float32))
    A = torch.eye(K, dtype=torch.float16, device="cuda")
    out = torch.zeros(K, N, dtype=torch.float16, device="cuda")
    h.gemm(A, K, mat, rt.EPI_GELU, lda=K, out=out, ldo=N, tile=tile)
    h.sync()
    got = out.cpu().numpy().T.copy()
    x = w.astype(np.float64)
    ref = (0.5 * x * (1 + sp.erf(x / np.sqrt(2)))).astype(np.float16)
    d = np.abs(got.view(np.int16).astype(np.int32) - ref.view(np.int16).astype(np.int32))
    d = np.where((got == 0) & (ref == 0), 0, d)  # +0 / -0
    assert d.max() <= 1 and (d > 0).mean() <= 0.02, (int(d.max()), float((d > 0).mean()))


@pytest.mark.parametrize("tile", TILES3)
def test_gemm_large_k_and_lora_a2(h, tile):
    torch.manual_seed(2)
    M, K1, N = 256, 8192, 512
    A = torch.randn(M, K1).half() * 0.5
    L = torch.randn(M, 384).half()
    W = torch.randn(N, K1 + 128) * 0.02
    mat, keep, Wd = make_mat(rt.FMT_Q8, W.numpy(), 32)
    out = torch.zeros(M, N, dtype=torch.float16, device="cuda")
    Lc = L.cuda()
    # extra K columns come from columns 128..255 of L (the k slice of the fused LoRA-A output)
    h.gemm(A.cuda(), M, mat, rt.EPI_STORE, lda=K1, k1=K1, a2=Lc.data_ptr() + 128 * 2, lda2=384, out=out, ldo=N,
           tile=tile)
    h.sync()
    ref = torch.cat((A.float(), L[:, 128:256].float()), 1) @ Wd.T
    assert rel(out.float(), ref) < 2e-3


@pytest.mark.parametrize("tile", TILES3)
def test_gemm_residual(h, tile):
    torch.manual_seed(3)
    B, T, K, N = 2, 160, 256, 512
    M = B * T
    A = torch.randn(M, K).half()
    mat, keep, Wd = make_mat(rt.FMT_Q8, (torch.randn(N, K) * 0.05).numpy(), 64)
    x0 = torch.randn(M, N)
    gate = torch.randn(B, N)
    x = x0.cuda()
    g = gate.cuda()
    h.gemm(A.cuda(), M, mat, rt.EPI_RESID, lda=K, x=x, ldx=N, gate=g, vec_bstride=N, rows_per_img=T, tile=tile)
    h.sync()
    ref = x0 + gate.repeat_interleave(T, 0) * _ref_gemm(A, Wd)
    assert rel(x.cpu() - x0, ref - x0) < 2e-3


@pytest.mark.parametrize("M,K", [(1536, 8192), (3072, 2048)])
def test_gemm_residual_split_k(h, M, K):
    """One / two images of the residual down- and o-projection shapes: the automatic choice splits K over
    CTA-pair work units that reduce-add partial sums into x (fp32 sums in an unfixed order)."""
    torch.manual_seed(31)
    N, T = 2048, 1536
    A = (torch.randn(M, K) * 0.5).half()
    mat, keep, Wd = make_mat(rt.FMT_Q8, (torch.randn(N, K) * 0.02).numpy(), 64)
    x0 = torch.randn(M, N)
    gate = torch.randn(M // T, N)
    x = x0.cuda()
    h.gemm(A.cuda(), M, mat, rt.EPI_RESID, lda=K, x=x, ldx=N, gate=gate.cuda(), vec_bstride=N, rows_per_img=T)
    h.sync()
    ref = x0 + gate.repeat_interleave(T, 0) * _ref_gemm(A, Wd)
    assert rel(x.cpu() - x0, ref - x0) < 2e-3


@pytest.mark.parametrize("tile", TILES3)
def test_gemm_large_a_operand(h, tile):
    """A larger than L2 (134 MB) with small weights: the launch walks the N tiles of each A block
    consecutively; sampled rows against fp32 math."""
    torch.manual_seed(41)
    M, K, N = 8192, 8192, 512
    Ad = (torch.randn(M, K, device="cuda") * 0.5).half()
    mat, keep, Wd = make_mat(rt.FMT_Q8, (torch.randn(N, K) * 0.02).numpy(), 64)
    out = torch.zeros(M, N, dtype=torch.float16, device="cuda")
    h.gemm(Ad, M, mat, rt.EPI_STORE, lda=K, out=out, ldo=N, tile=tile)
    h.sync()
    rows = torch.cat((torch.arange(0, 256), torch.randint(256, M, (256,), generator=torch.Generator().manual_seed(42))))
    ref = Ad[rows.cuda()].float().cpu() @ Wd.T
    assert rel(out[rows.cuda()].float().cpu(), ref) < 2e-3


@pytest.mark.parametrize("tile", TILES3)
def test_gemm_rms_rope_segments(h, tile):
    torch.manual_seed(4)
    T, K, D = 192, 256, 256  # 2 heads per segment; q | k | v = 768 columns
    A = torch.randn(T, K).half()
    fmt = rt.FMT_Q8 if tile in (3, 4) else rt.FMT_F16
    mat, keep, Wd = make_mat(fmt, (torch.randn(3 * D, K) * 0.05).numpy(), 64)
    gq, gk = 1 + 0.1 * torch.randn(128), 1 + 0.1 * torch.randn(128)
    ang = torch.rand(T, 64) * 6.0
    cos, sin = torch.cos(ang), torch.sin(ang)
    out = torch.zeros(T, 3 * D, dtype=torch.float16, device="cuda")
    gqc, gkc, cc, sc = gq.cuda(), gk.cuda(), cos.cuda(), sin.cuda()
    h.gemm(A.cuda(), T, mat, rt.EPI_RMS, lda=K, out=out, ldo=3 * D, gain0=gqc, gain1=gkc, seg1=D, seg2=2 * D,
           rope0=1, rope1=1, cos_t=cc, sin_t=sc, rows_per_img=T, tile=tile)
    h.sync()
    ref = _ref_gemm(A, Wd)
    H = D // 128
    q = oa.rope(oa.rms_head(ref[:, :D].view(1, T, H, 128), gq), cos, sin).reshape(T, D)
    k = oa.rope(oa.rms_head(ref[:, D:2 * D].view(1, T, H, 128), gk), cos, sin).reshape(T, D)
    o = out.float().cpu()
    assert rel(o[:, :D], q) < 2e-3 and rel(o[:, D:2 * D], k) < 2e-3 and rel(o[:, 2 * D:], ref[:, 2 * D:]) < 2e-3


@pytest.mark.parametrize("tile", [1, 2, 4])
def test_gemm_situ(h, tile):
    torch.manual_seed(5)
    M, K, F = 200, 256, 512
    A = torch.randn(M, K).half()
    up, gate = torch.randn(F, K) * 0.1, torch.randn(F, K) * 0.1
    from oracle import packs as op
    w = op.situ_rows(up.numpy(), gate.numpy())
    mat, keep, Wd = make_mat(rt.FMT_Q8, w, 32)
    out = torch.zeros(M, F, dtype=torch.float16, device="cuda")
    h.gemm(A.cuda(), M, mat, rt.EPI_SITU, lda=K, out=out, ldo=F, tile=tile)
    h.sync()
    ug = _ref_gemm(A, Wd).view(M, F // 128, 2, 128)
    ref = om.situ(ug[:, :, 0], ug[:, :, 1]).reshape(M, F)
    assert rel(out.float(), ref) < 2e-3


@pytest.mark.parametrize("fmt,group", [(rt.FMT_Q8, 64), (rt.FMT_Q8, 32), (rt.FMT_Q4, 32), (rt.FMT_Q4A, 32)])
def test_expanded_weights_same_bits(h, fmt, group):
    """From 3072 rows up the automatic choice expands quantised weights to fp16 in the handle's scratch and
    runs the fp16 kernel: the same operand values and k order as the CTA-pair kernel's own dequantisers,
    so the outputs agree bit for bit (store epilogue, with LoRA extra K columns)."""
    torch.manual_seed(12)
    M, K1, N = 3072, 1024, 512
    A = (torch.randn(M, K1, device="cuda") * 0.5).half()
    L = torch.randn(M, 128, device="cuda").half()
    mat, keep, Wd = make_mat(fmt, (torch.randn(N, K1 + 128) * 0.05).numpy(), group)
    outs = [torch.zeros(M, N, dtype=torch.float16, device="cuda") for _ in range(3)]
    torch.cuda.synchronize()  # the fills (torch's stream) complete before the handle's stream writes
    for tile, o in zip((2, 0, 4), outs):
        h.gemm(A, M, mat, rt.EPI_STORE, lda=K1, k1=K1, a2=L.data_ptr(), lda2=128, out=o, ldo=N, tile=tile)
    h.sync()
    ref = torch.cat((A.float().cpu(), L.float().cpu()), 1) @ Wd.T
    assert rel(outs[0].float().cpu(), ref) < 2e-3
    for o in outs[1:]:
        assert torch.equal(o.view(torch.int16), outs[0].view(torch.int16)), int((o != outs[0]).sum())


@pytest.mark.parametrize("fmt", [rt.FMT_F16, rt.FMT_Q8, rt.FMT_Q4A])
def test_gemm_pair_tiles_large(h, fmt):
    """A shape where the automatic choice takes CTA pairs (many 256x256 tiles) against the single-CTA result."""
    torch.manual_seed(9)
    M, K, N = 4096, 1024, 2048
    A = torch.randn(M, K, device="cuda").half()
    mat, keep, Wd = make_mat(fmt, (torch.randn(N, K) * 0.05).numpy(), 32)
    o1 = torch.zeros(M, N, dtype=torch.float16, device="cuda")
    o2 = torch.zeros(M, N, dtype=torch.float16, device="cuda")
    h.gemm(A, M, mat, rt.EPI_GELU, lda=K, out=o1, ldo=N, tile=1)
    h.gemm(A, M, mat, rt.EPI_GELU, lda=K, out=o2, ldo=N, tile=0)
    h.sync()
    ref = oa.gelu(A.float().cpu() @ Wd.T)
    assert rel(o1.float(), ref) < 2e-3 and rel(o2.float(), ref) < 2e-3
    assert rel(o1.float(), o2.float()) < 1e-3


@pytest.mark.parametrize("fmt,group,M,N", [(rt.FMT_F16, 64, 1536, 8192), (rt.FMT_Q8, 64, 1536, 8192),
                                           (rt.FMT_Q8, 32, 1536, 8192), (rt.FMT_Q8, 64, 3072, 8192),
                                           (rt.FMT_F16, 64, 600, 1024), (rt.FMT_Q8, 32, 600, 1024)])
def test_gemm_pair_224_tiles(h, fmt, group, M, N):
    """256x224 pair tiles (tile 5, and the automatic choice for mlp.layer1 at one and two images) against
    fp32 math on the same operands and against the 256x256 pair tiles: the accumulation order over K is the
    same, so the outputs agree to fp16 rounding of equal sums. N = 8192 makes 37 tiles per band, the last
    128 wide; N = 1024 makes 5, the last 128 wide. At 3072 rows the automatic choice expands the q8 weights
    and runs the fp16 kernel with 224-column tiles."""
    torch.manual_seed(21)
    K = 2048 if M >= 1536 else 512
    A = torch.randn(M, K, device="cuda").half()
    mat, keep, Wd = make_mat(fmt, (torch.randn(N, K) * 0.03).numpy(), group)
    outs = {t: torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda") for t in (TILE224, 2, 0)}
    torch.cuda.synchronize()  # the NaN fills (torch's stream) complete before the handle's stream writes
    for tile, o in outs.items():
        h.gemm(A, M, mat, rt.EPI_GELU, lda=K, out=o, ldo=N, tile=tile)
    h.sync()
    ref = oa.gelu(A.float().cpu() @ Wd.T)
    for tile, o in outs.items():
        oc = o.float().cpu()
        assert torch.isfinite(oc).all(), tile
        assert rel(oc, ref) < 2e-3, tile
    assert rel(outs[TILE224].float(), outs[2].float()) < 1e-3


@pytest.mark.parametrize("B,H,Tq,Tk,nvalid,amp", [(2, 2, 200, 333, 300, 0.6), (1, 3, 256, 256, 0, 0.6),
                                                   (2, 16, 1536, 1536, 0, 0.6), (1, 2, 130, 70, 0, 0.6),
                                                   (1, 2, 256, 520, 70, 2.5), (1, 4, 384, 1024, 0, 2.5)])
def test_attention(h, B, H, Tq, Tk, nvalid, amp):
    """amp 2.5 gives scaled logits with a standard deviation near 6, so the running maximum moves from
    tile to tile and most probabilities are tiny; nvalid 70 of 520 leaves whole key tiles masked."""
    torch.manual_seed(6)
    D = 128 * H
    # q lives in a fused [q | k | v] row buffer, k and v in a separate one, exercising column offsets
    qbuf = (torch.randn(B, Tq, 3 * D) * amp).half()
    kv = (torch.randn(B, Tk, 2 * D) * amp).half()
    out = torch.zeros(B, Tq, D, dtype=torch.float16, device="cuda")
    scale = 1.0 / math.sqrt(128)
    qc, kvc = qbuf.cuda(), kv.cuda()
    h.attention(qc, kvc, kvc, out, B, H, Tq, Tk, 3 * D, 2 * D, 2 * D, D, q_col0=D, k_col0=0, v_col0=D,
                nvalid=nvalid, scale=scale)
    h.sync()
    q = qbuf[..., D:2 * D].float().view(B, Tq, H, 128)
    k = kv[..., :D].float().view(B, Tk, H, 128)
    v = kv[..., D:].float().view(B, Tk, H, 128)
    ref = oa.attention(q, k, v, scale=scale, nvalid=nvalid or None).reshape(B, Tq, D)
    assert rel(out.float(), ref) < 2e-3


@pytest.mark.parametrize("B,H,Tq,Tk,nvalid,amp", [(8, 16, 1536, 256, 0, 0.6), (1, 16, 1536, 256, 0, 2.5),
                                                   (2, 3, 200, 256, 250, 0.6), (1, 2, 130, 70, 0, 2.5),
                                                   (3, 5, 64, 200, 130, 0.6), (1, 1, 1000, 129, 0, 0.6)])
def test_attention_short_keys(h, B, H, Tq, Tk, nvalid, amp):
    """The short-key kernel (kernel 2: at most 256 keys, K and V resident per (image, head), one exact
    softmax step) against the fp32 reference and against the general kernel (kernel 1) on the same inputs:
    the Anima cross-attention at 8 and 1 images (T 1536, C 256), partial query tiles, masked keys (nvalid),
    fewer than 128 keys, and CTAs whose query-tile range spans several (image, head) groups."""
    torch.manual_seed(16)
    D = 128 * H
    qbuf = (torch.randn(B, Tq, 3 * D) * amp).half()
    kv = (torch.randn(B, Tk, 2 * D) * amp).half()
    outs = {kn: torch.full((B, Tq, D), float("nan"), dtype=torch.float16, device="cuda") for kn in (2, 1, 0)}
    scale = 1.0 / math.sqrt(128)
    qc, kvc = qbuf.cuda(), kv.cuda()
    torch.cuda.synchronize()  # the fills and copies (torch's stream) complete before the handle's stream runs
    for kn, o in outs.items():
        h.attention(qc, kvc, kvc, o, B, H, Tq, Tk, 3 * D, 2 * D, 2 * D, D, q_col0=D, k_col0=0, v_col0=D,
                    nvalid=nvalid, scale=scale, kernel=kn)
    h.sync()
    q = qbuf[..., D:2 * D].float().view(B, Tq, H, 128)
    k = kv[..., :D].float().view(B, Tk, H, 128)
    v = kv[..., D:].float().view(B, Tk, H, 128)
    ref = oa.attention(q, k, v, scale=scale, nvalid=nvalid or None).reshape(B, Tq, D)
    for kn, o in outs.items():
        oc = o.float().cpu()
        assert torch.isfinite(oc).all(), kn
        assert rel(oc, ref) < 2e-3, kn
    assert rel(outs[2].float(), outs[1].float()) < 2e-3


@pytest.mark.parametrize("D", [1024, 2048, 3072])
def test_lnmod_rmsmod(h, D):
    torch.manual_seed(8)
    B, T = 2, 96
    x = torch.randn(B * T, D) * 3 + 0.5
    sh, sc, w = torch.randn(B, D) * 0.1, torch.randn(B, D) * 0.1, 1 + torch.randn(D) * 0.1
    out = torch.zeros(B * T, D, dtype=torch.float16, device="cuda")
    h.lnmod(x.cuda(), out, B * T, D, sh.cuda(), sc.cuda(), vec_bstride=D, rows_per_img=T)
    h.sync()
    ref = oa.ln_mod(x.view(B, T, D), sh[:, None], sc[:, None]).reshape(B * T, D)
    assert rel(out.float(), ref) < 1e-3
    h.rmsmod(x.cuda(), out, B * T, D, w.cuda(), sh.cuda(), sc.cuda(), vec_bstride=D, rows_per_img=T)
    h.sync()
    ref = (om.rms(x.view(B, T, D), w) * (1 + sc[:, None]) + sh[:, None]).reshape(B * T, D)
    assert rel(out.float(), ref) < 1e-3


def test_bad_arguments_are_rejected(h):
    mat, keep, _ = make_mat(rt.FMT_F16, np.zeros((64, 100), np.float32))  # K not a multiple of 64
    A = torch.zeros(64, 100, dtype=torch.float16, device="cuda")
    out = torch.zeros(64, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(rt.HxError):
        h.gemm(A, 64, mat, rt.EPI_STORE, lda=100, out=out, ldo=64)
    with pytest.raises(rt.HxError):
        h.attention(A, A, A, out, 1, 1, 64, 64, 100, 100, 100, 64)  # row pitch not 16-byte aligned
    m2, keep2, _ = make_mat(rt.FMT_F16, np.zeros((256, 128), np.float32))
    A2 = torch.zeros(64, 128, dtype=torch.float16, device="cuda")
    x = torch.zeros(64, 256, device="cuda")
    g = torch.zeros(256, device="cuda")
    q3 = torch.zeros(1, 128, 128, dtype=torch.float16, device="cuda")
    kv3 = torch.zeros(1, 300, 128, dtype=torch.float16, device="cuda")
    with pytest.raises(rt.HxError):  # the short-key kernel takes at most 256 keys
        h.attention(q3, kv3, kv3, q3, 1, 1, 128, 300, 128, 128, 128, 128, scale=1.0, kernel=2)
    with pytest.raises(rt.HxError):  # 224-column pair tiles take the GELU and store epilogues only
        h.gemm(A2, 64, m2, rt.EPI_RESID, lda=128, x=x, ldx=256, gate=g, tile=5)
