"""Block-level parity on the GPU through the per-block operator (hx_mega_block) and the chain (hx_chain).

Bar: rel-L2 of the block output delta (x_out - x_in) against the oracle <= 2e-3, with the oracle fed
the exact operands the device multiplies (fp16 weights, or the bit-exact fp16 dequantised values)."""
import numpy as np
import pytest
import torch

from hexanima_b200 import runtime as rt
from oracle import anima as oa
from oracle import moss as om
from tests.gpu_util import anima_bind, make_mat, read_f32, rel, write_f32

pytestmark = pytest.mark.gpu
TOL = 2e-3


@pytest.fixture(scope="module")
def h():
    hd = rt.Handle(0)
    yield hd
    assert hd.status() == 0
    hd.close()


def _anima_inputs(B, T, C, D, Cd, gh, gw, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, D, generator=g)
    ctx = torch.randn(B, C, Cd, generator=g).half().float()  # the blob holds ctx in fp16
    mod = torch.randn(9, D, generator=g) * 0.1
    cos, sin = oa.make_rope(gh, gw, ntok=T)
    return x, ctx, mod, torch.from_numpy(cos), torch.from_numpy(sin)


def _anima_run(h, wfd, x, ctx, mod, cos, sin, D, F, Cd):
    B, T, _ = x.shape
    C = ctx.shape[1]
    meta, total = rt.blob_layout(rt.MODEL_ANIMA, T, C, B, D, F, Cd)
    bfd = h.buf_alloc(total)
    A = rt.A
    write_f32(h, bfd, meta[A["X"]], x.numpy())
    h.buf_write(bfd, meta[A["CTX"]], ctx.half().numpy())
    write_f32(h, bfd, meta[A["COS"]], cos.numpy())
    write_f32(h, bfd, meta[A["SIN"]], sin.numpy())
    times = h.mega_block(meta, wfd, bfd, mod=mod.numpy(), ntimes=25)
    y = read_f32(h, bfd, meta[A["X"]], B * T * D).reshape(B, T, D)
    h.buf_free(bfd)
    return torch.from_numpy(y), times


@pytest.mark.parametrize("fmt,group", [(rt.FMT_F16, 64), (rt.FMT_Q8, 64), (rt.FMT_Q8, 32), (rt.FMT_Q4, 32)])
def test_anima_block_bind_small(h, fmt, group):
    D, F, Cd, B, T, C = 256, 512, 128, 2, 256, 64
    W, norms, modA, modB = oa.init_weights(10, D=D, F=F, Cd=Cd)
    wfd, Wd, gain, keep = anima_bind(h, W, norms, modA, modB, fmt, group)
    x, ctx, mod, cos, sin = _anima_inputs(B, T, C, D, Cd, 16, 16)
    y, times = _anima_run(h, wfd, x, ctx, mod, cos, sin, D, F, Cd)
    ref = oa.block(x, ctx, mod, cos, sin, Wd, gain)
    assert rel(y - x, ref - x) < TOL
    assert times[0] > 0
    h.weights_free(wfd)


@pytest.mark.parametrize("q8", [False, True])
def test_anima_block_reference_pack(h, q8):
    """A reference blkNN.bin (fp16 or q8, export_all.py layout) at the real block shape, one 512x768 image."""
    D, F, Cd, B, T, C = 2048, 8192, 1024, 1, 1536, 256
    W, norms, modA, modB = oa.init_weights(20, D=D, F=F, Cd=Cd)
    pack = oa.build_pack(W, norms, modA, modB, q8=q8)
    wfd = h.weights_load(rt.MODEL_ANIMA, pack)
    Wd, gain = oa.pack_weights(pack, q8=q8)
    x, ctx, mod, cos, sin = _anima_inputs(B, T, C, D, Cd, 32, 48, seed=3)
    y, _ = _anima_run(h, wfd, x, ctx, mod, cos, sin, D, F, Cd)
    torch.set_num_threads(max(1, torch.get_num_threads()))
    ref = oa.block(x, ctx, mod, cos, sin, Wd, gain)
    assert rel(y - x, ref - x) < TOL
    h.weights_free(wfd)


def test_anima_chain_graph_matches_sequential_and_modulation(h):
    D, F, Cd, B, T, C, n = 256, 512, 128, 1, 128, 32, 3
    sets = [oa.init_weights(30 + i, D=D, F=F, Cd=Cd) for i in range(n)]
    bound = [anima_bind(h, *s) for s in sets]
    wfds = [b[0] for b in bound]
    x, ctx, _, cos, sin = _anima_inputs(B, T, C, D, Cd, 8, 16, seed=5)
    emb = torch.randn(D)
    lora = torch.randn(3 * D) * 0.1
    meta, total = rt.blob_layout(rt.MODEL_ANIMA, T, C, B, D, F, Cd)
    A = rt.A
    bfd = h.buf_alloc(total)

    def load():
        write_f32(h, bfd, meta[A["X"]], x.numpy())
        h.buf_write(bfd, meta[A["CTX"]], ctx.half().numpy())
        write_f32(h, bfd, meta[A["COS"]], cos.numpy())
        write_f32(h, bfd, meta[A["SIN"]], sin.numpy())

    e, l = emb.cuda(), lora.cuda()
    # modulation against the oracle (megarun.cpp:158-171)
    md = torch.zeros(9 * D + 768, device="cuda")
    h.modulation(wfds[0], e, l, md)
    h.sync()
    mref = oa.modulation(sets[0][2], sets[0][3], emb, lora)
    assert rel(md[:9 * D].cpu().view(9, D), mref) < 1e-5
    # chain with graph replay, twice (second call replays), against per-block calls
    load()
    h.chain(meta, wfds, bfd, emb_dev=e, lora_dev=l, use_graph=True)
    load()
    h.chain(meta, wfds, bfd, emb_dev=e, lora_dev=l, use_graph=True)
    y_graph = read_f32(h, bfd, meta[A["X"]], B * T * D)
    load()
    for i, w in enumerate(wfds):
        mi = oa.modulation(sets[i][2], sets[i][3], emb, lora)
        h.mega_block(meta, w, bfd, mod=mi.numpy())
    y_seq = read_f32(h, bfd, meta[A["X"]], B * T * D)
    assert rel(torch.from_numpy(y_graph), torch.from_numpy(y_seq)) < 1e-5
    # and the whole chain against the oracle
    xr = x.clone()
    for i in range(n):
        Wd, gain = bound[i][1], bound[i][2]
        xr = oa.block(xr, ctx, oa.modulation(sets[i][2], sets[i][3], emb, lora), cos, sin, Wd, gain)
    assert rel(torch.from_numpy(y_graph).view(B, T, D) - x, xr - x) < TOL
    # skipmask: skipping every block leaves x untouched
    load()
    h.chain(meta, wfds, bfd, emb_dev=e, lora_dev=l, skipmask=0b111, use_graph=False)
    assert np.array_equal(read_f32(h, bfd, meta[A["X"]], B * T * D), x.numpy().ravel())
    h.buf_free(bfd)
    for w in wfds:
        h.weights_free(w)


def test_anima_chain_weights_expanded_ahead(h):
    """Two 1536-token images (3072 rows): the chain expands each q8 matrix to fp16 on a side stream ahead of
    its GEMM (two buffers in turn, the last GEMM of a block issuing the next block's q|k|v). Graph replay,
    eager per-block calls and the oracle agree."""
    D, F, Cd, B, T, C, n = 256, 512, 128, 2, 1536, 64, 3
    sets = [oa.init_weights(70 + i, D=D, F=F, Cd=Cd) for i in range(n)]
    bound = [anima_bind(h, *s, fmt=rt.FMT_Q8, group=64) for s in sets]
    wfds = [b[0] for b in bound]
    x, ctx, _, cos, sin = _anima_inputs(B, T, C, D, Cd, 32, 48, seed=7)
    emb = torch.randn(D)
    lora = torch.randn(3 * D) * 0.1
    meta, total = rt.blob_layout(rt.MODEL_ANIMA, T, C, B, D, F, Cd)
    A = rt.A
    bfd = h.buf_alloc(total)

    def load():
        write_f32(h, bfd, meta[A["X"]], x.numpy())
        h.buf_write(bfd, meta[A["CTX"]], ctx.half().numpy())
        write_f32(h, bfd, meta[A["COS"]], cos.numpy())
        write_f32(h, bfd, meta[A["SIN"]], sin.numpy())

    e, l = emb.cuda(), lora.cuda()
    ys = []
    for _ in range(2):  # capture, then replay
        load()
        h.chain(meta, wfds, bfd, emb_dev=e, lora_dev=l, use_graph=True)
        ys.append(read_f32(h, bfd, meta[A["X"]], B * T * D))
    assert np.array_equal(ys[0], ys[1])
    load()
    for i, w in enumerate(wfds):
        h.mega_block(meta, w, bfd, mod=oa.modulation(sets[i][2], sets[i][3], emb, lora).numpy())
    y_seq = read_f32(h, bfd, meta[A["X"]], B * T * D)
    assert rel(torch.from_numpy(ys[0]), torch.from_numpy(y_seq)) < 1e-5
    xr = x.clone()
    for i in range(n):
        Wd, gain = bound[i][1], bound[i][2]
        xr = oa.block(xr, ctx, oa.modulation(sets[i][2], sets[i][3], emb, lora), cos, sin, Wd, gain)
    assert rel(torch.from_numpy(ys[0]).view(B, T, D) - x, xr - x) < TOL
    h.buf_free(bfd)
    for w in wfds:
        h.weights_free(w)
    assert h.status() == 0


def _moss_run(h, wfd, x, mod, cos, sin, D, F, nvalid):
    B, T, _ = x.shape
    meta, total = rt.blob_layout(rt.MODEL_MOSS, T, 0, B, D, F)
    S = rt.S
    meta[S["NVALID"]] = nvalid
    bfd = h.buf_alloc(total)
    write_f32(h, bfd, meta[S["X"]], x.numpy())
    write_f32(h, bfd, meta[S["COS"]], cos.numpy())
    write_f32(h, bfd, meta[S["SIN"]], sin.numpy())
    h.mega_block(meta, wfd, bfd, mod=mod.numpy())
    y = read_f32(h, bfd, meta[S["X"]], B * T * D).reshape(B, T, D)
    h.buf_free(bfd)
    return torch.from_numpy(y)


def test_moss_block_reference_pack_lora(h):
    """A MOSS q8 pack with LoRA-B rows as extra K tiles (export_moss.py layout), masked joint attention."""
    D, F = 3072, 8192
    w, lora = om.init_weights(40, D=D, F=F, lora_rank=128)
    pack = om.build_pack(w, lora)
    assert len(pack) == 135397376
    wfd = h.weights_load(rt.MODEL_MOSS, pack)
    mats, gain = om.pack_mats(pack)
    Hh, Ww, Tt = 4, 8, 18
    nvalid = Hh * Ww + Tt
    T = (nvalid + 31) // 32 * 32
    g = torch.Generator().manual_seed(41)
    x = torch.randn(1, T, D, generator=g) * 4
    mod = torch.randn(6, D, generator=g) * 0.1
    c, s = rt.rope_moss(Hh, Ww, Tt, om.bands16().numpy(), T)
    cos, sin = torch.from_numpy(c), torch.from_numpy(s)
    y = _moss_run(h, wfd, x, mod, cos, sin, D, F, nvalid)
    ref = om.block_dev(x, mod, cos, sin, mats, gain, nvalid=nvalid, lora=True)
    assert rel(y[:, :nvalid] - x[:, :nvalid], ref[:, :nvalid] - x[:, :nvalid]) < TOL
    h.weights_free(wfd)


@pytest.mark.parametrize("fmt", [rt.FMT_Q4, rt.FMT_Q8])
def test_moss_block_bind_no_lora(h, fmt):
    D, F, B = 384, 512, 2
    torch.manual_seed(50)
    qkv = torch.randn(3 * D, D) * 0.02
    up, gate, dn, o = (torch.randn(F, D) * 0.02, torch.randn(F, D) * 0.02, torch.randn(D, F) * 0.02,
                       torch.randn(D, D) * 0.02)
    from oracle import packs as op
    mats, keep, deq = {}, [], {}
    for slot, name, wt in ((rt.W_QKV, "qkv", qkv), (rt.W_O, "o", o), (rt.W_M1, "ug", torch.from_numpy(
            op.situ_rows(up.numpy(), gate.numpy()))), (rt.W_M2, "dn", dn)):
        m, k, d = make_mat(fmt, wt.numpy(), 32)
        mats[slot], deq[name] = m, d
        keep += k
    gain = torch.cat((1 + 0.1 * torch.randn(128), 1 + 0.1 * torch.randn(128), 1 + 0.1 * torch.randn(2 * D)))
    gain[:128] /= np.sqrt(128.0)
    tg = gain.cuda()
    wfd = h.weights_bind(rt.MODEL_MOSS, D, F, mats, tg, lora=0, keep=keep + [tg])
    Hh, Ww, Tt = 6, 6, 20
    nvalid = Hh * Ww + Tt
    T = 64
    x = torch.randn(B, T, D) * 2
    mod = torch.randn(6, D) * 0.1
    c, s = rt.rope_moss(Hh, Ww, Tt, om.bands16().numpy(), T)
    cos, sin = torch.from_numpy(c), torch.from_numpy(s)
    y = _moss_run(h, wfd, x, mod, cos, sin, D, F, nvalid)
    ref = om.block_dev(x, mod, cos, sin, deq, gain, nvalid=nvalid, lora=False)
    assert rel(y[:, :nvalid] - x[:, :nvalid], ref[:, :nvalid] - x[:, :nvalid]) < TOL
    h.weights_free(wfd)


def test_meta_errors(h):
    D, F, Cd = 256, 512, 128
    W, norms, modA, modB = oa.init_weights(60, D=D, F=F, Cd=Cd)
    wfd, Wd, gain, keep = anima_bind(h, W, norms, modA, modB)
    meta, total = rt.blob_layout(rt.MODEL_ANIMA, 64, 32, 1, D, F, Cd)
    small = h.buf_alloc(total // 2)
    with pytest.raises(rt.HxError) as e:
        h.mega_block(meta, wfd, small, mod=np.zeros(9 * D, np.float32))
    assert e.value.rc == rt.HX_E_RANGE
    with pytest.raises(rt.HxError) as e:
        h.mega_block(meta, 12345, small)
    assert e.value.rc == rt.HX_E_NOWEIGHTS
    with pytest.raises(rt.HxError) as e:
        h.mega_block(meta, wfd, 999)
    assert e.value.rc == rt.HX_E_NOBLOB
    h.buf_free(small)
    h.weights_free(wfd)
