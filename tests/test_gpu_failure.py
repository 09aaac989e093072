"""Failure detection without a GPU fault: the bounded device wait and its rc path.

The reference reports a failed device check as rc -77 and keeps serving (moss/hexagon/mega/blk.c:112-118,
149-155; rc contract hexagon/mega/blk.c:110-127). Here every pipeline wait is an mbarrier wait bounded
by a time limit; on expiry the kernel records a code in the handle's status word and returns, and the
host answers HX_E_TIMEOUT. hx_wait_selftest runs that same wait with a run-time limit of 1 ms on a
barrier nobody arrives on (nothing else in flight), so the test exercises the expiry path without
hanging or faulting the GPU; afterwards a normal block call on the same handle and on a fresh one
still matches the oracle."""
import pytest
import torch

from hexanima_b200 import runtime as rt
from oracle import anima as oa
from tests.gpu_util import anima_bind, read_f32, rel, write_f32

pytestmark = pytest.mark.gpu


def _small_block_ok(h):
    D, F, Cd, B, T, C = 256, 512, 128, 1, 128, 64
    W, norms, modA, modB = oa.init_weights(321, D=D, F=F, Cd=Cd)
    wfd, Wd, gain, keep = anima_bind(h, W, norms, modA, modB, fmt=rt.FMT_Q8, group=64)
    g = torch.Generator().manual_seed(9)
    x = torch.randn(B, T, D, generator=g)
    ctx = torch.randn(B, C, Cd, generator=g).half()
    mod = torch.randn(9, D, generator=g) * 0.1
    cos, sin = oa.make_rope(8, 16, ntok=T)
    meta, total = rt.blob_layout(rt.MODEL_ANIMA, T, C, B, D, F, Cd)
    bfd = h.buf_alloc(total)
    A = rt.A
    write_f32(h, bfd, meta[A["X"]], x.numpy())
    h.buf_write(bfd, meta[A["CTX"]], ctx.numpy())
    write_f32(h, bfd, meta[A["COS"]], cos)
    write_f32(h, bfd, meta[A["SIN"]], sin)
    h.mega_block(meta, wfd, bfd, mod=mod.numpy())
    y = torch.from_numpy(read_f32(h, bfd, meta[A["X"]], B * T * D).reshape(B, T, D))
    h.buf_free(bfd)
    h.weights_free(wfd)
    ref = oa.block(x, ctx.float(), mod, torch.from_numpy(cos), torch.from_numpy(sin), Wd, gain)
    return rel(y - x, ref - x) < 2e-3 and h.status() == 0


def test_bounded_wait_expires_with_timeout_rc_and_handle_survives():
    h = rt.Handle(0)
    try:
        assert h.wait_selftest(1_000_000, arrive=True) == rt.HX_OK          # someone arrives: the wait completes
        assert h.wait_selftest(1_000_000, arrive=False) == rt.HX_E_TIMEOUT  # nobody arrives: expires after 1 ms
        assert h.status() == 0                                              # the status word was read and cleared
        assert h.wait_selftest(1_000_000, arrive=True) == rt.HX_OK
        with pytest.raises(rt.HxError) as e:                                # limits outside 1 us .. 2 s are refused
            h.wait_selftest(10, arrive=False)
        assert e.value.rc == rt.HX_E_ARG
        assert _small_block_ok(h)                                           # the same handle keeps working
    finally:
        h.close()
    h2 = rt.Handle(0)
    try:
        assert _small_block_ok(h2)                                          # and a fresh handle too
    finally:
        h2.close()
