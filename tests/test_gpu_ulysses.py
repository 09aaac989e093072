"""Ulysses sequence-parallel MOSS block on 2 GPUs through the C ABI (hx_sp_init + meta SP), against
the oracle block on the full sequence. Needs 2 visible GPUs; each rank is a spawned process."""
import multiprocessing as mp
import queue

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

D, F, T, NVALID, WORLD = 512, 512, 256, 230, 2


def _weights():
    torch.manual_seed(123)
    from oracle import packs as op
    qkv = torch.randn(3 * D, D) * 0.02
    o = torch.randn(D, D) * 0.02
    up, gate = torch.randn(F, D) * 0.02, torch.randn(F, D) * 0.02
    dn = torch.randn(D, F) * 0.02
    gain = torch.cat((1 + 0.1 * torch.randn(128), 1 + 0.1 * torch.randn(128), 1 + 0.1 * torch.randn(2 * D)))
    gain[:128] /= np.sqrt(128.0)
    return {"qkv": qkv.numpy(), "o": o.numpy(), "ug": op.situ_rows(up.numpy(), gate.numpy()), "dn": dn.numpy()}, gain


def _inputs():
    g = torch.Generator().manual_seed(321)
    x = torch.randn(1, T, D, generator=g) * 2
    mod = torch.randn(6, D, generator=g) * 0.1
    return x, mod


def _worker(rank, uid, q):
    try:
        torch.cuda.set_device(rank)
        from hexanima_b200 import runtime as rt
        from oracle import moss as om
        from tests.gpu_util import make_mat
        W, gain = _weights()
        x, mod = _inputs()
        h = rt.Handle(rank)
        h.sp_init(WORLD, rank, uid)
        mats, keep = {}, []
        for slot, name in ((rt.W_QKV, "qkv"), (rt.W_O, "o"), (rt.W_M1, "ug"), (rt.W_M2, "dn")):
            m, k, _ = make_mat(rt.FMT_Q8, W[name], 32)
            mats[slot] = m
            keep += k
        tg = gain.cuda()
        wfd = h.weights_bind(rt.MODEL_MOSS, D, F, mats, tg, lora=0, keep=keep + [tg])
        Tl = T // WORLD
        c, s = rt.rope_moss(8, 24, 64, om.bands16().numpy(), T)  # 192 image + 64 text tokens
        meta, total = rt.blob_layout(rt.MODEL_MOSS, Tl, 0, 1, D, F)
        S = rt.S
        meta[S["NVALID"]] = NVALID
        meta[S["SP"]] = WORLD
        bfd = h.buf_alloc(total)
        lo, hi = rank * Tl, (rank + 1) * Tl
        h.buf_write(bfd, meta[S["X"]], x[0, lo:hi].numpy())
        h.buf_write(bfd, meta[S["COS"]], np.ascontiguousarray(c[lo:hi]))
        h.buf_write(bfd, meta[S["SIN"]], np.ascontiguousarray(s[lo:hi]))
        h.mega_block(meta, wfd, bfd, mod=mod.numpy())
        y = np.frombuffer(h.buf_read(bfd, meta[S["X"]], Tl * D * 4).tobytes(), np.float32).reshape(Tl, D).copy()
        st = h.status()
        h.close()
        q.put((rank, y, st, None))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, None, None, repr(e)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_moss_block_ulysses_two_gpus():
    from hexanima_b200 import runtime as rt
    from oracle import moss as om
    from tests.gpu_util import make_mat, rel
    uid = rt.sp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, uid, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(WORLD):
            rank, y, st, err = q.get(timeout=240)
            assert err is None, err
            assert st == 0
            res[rank] = y
    except queue.Empty:
        pytest.fail("a rank did not report within 240 s")
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
    got = torch.from_numpy(np.concatenate([res[0], res[1]], 0))[None]
    W, gain = _weights()
    x, mod = _inputs()
    deq = {n: make_mat(rt.FMT_Q8, W[n], 32)[2] for n in ("qkv", "o", "ug", "dn")}
    c, s = rt.rope_moss(8, 24, 64, om.bands16().numpy(), T)
    ref = om.block_dev(x, mod, torch.from_numpy(c), torch.from_numpy(s), deq, gain, nvalid=NVALID, lora=False)
    assert rel(got[:, :NVALID] - x[:, :NVALID], ref[:, :NVALID] - x[:, :NVALID]) < 2e-3
