"""The Anima LLM adapter on the GPU (hx_adapter_load + hx_anima_adapter) against the oracle restatement of
phone/animad.cpp:179-218 (oracle.anima.adapter, float32 on the same fp16 weights). The GPU rounds the
activations entering each projection to fp16 (measured effect on the output: 3.5e-4 rel-L2 at L=77);
bar: rel-L2 of the context rows <= 2e-3, padding rows exactly zero."""
import numpy as np
import pytest
import torch

from hexanima_b200 import runtime as rt
from oracle import anima as oa
from tests.gpu_util import rel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def h():
    hd = rt.Handle(0)
    yield hd
    assert hd.status() == 0
    hd.close()


def _dev(W16):
    return {"embed": W16["embed"].cuda(), "blocks": [{k: v.cuda() for k, v in b.items()} for b in W16["blocks"]],
            "out_w": W16["out_w"].cuda(), "out_b": W16["out_b"].cuda(), "norm": W16["norm"].cuda()}


@pytest.mark.parametrize("L,S", [(77, 200), (512, 33), (1, 1)])
def test_adapter_matches_oracle(h, L, S):
    W16 = oa.adapter_init(5, vocab=1000)
    afd = h.adapter_load(_dev(W16))
    g = torch.Generator().manual_seed(6 + L)
    ids = torch.randint(0, 1000, (L,), generator=g).numpy()
    wts = (0.5 + torch.rand(L, generator=g)).numpy()
    hidden = torch.randn(S, 1024, generator=g)
    out = torch.full((512, 1024), float("nan"), device="cuda")
    h.anima_adapter(afd, hidden.cuda(), ids, wts, out)
    h.sync()
    got = out.cpu()
    ref = oa.adapter(hidden, ids, wts, oa.adapter_f32(W16))
    assert torch.equal(got[L:], torch.zeros(512 - L, 1024))
    assert rel(got[:L], ref[:L]) < 2e-3


def test_adapter_rejects_bad_ids(h):
    W16 = oa.adapter_init(7, vocab=50)
    afd = h.adapter_load(_dev(W16))
    out = torch.zeros(512, 1024, device="cuda")
    hidden = torch.zeros(4, 1024, device="cuda")
    with pytest.raises(rt.HxError) as e:
        h.anima_adapter(afd, hidden, np.array([3, 50], np.int32), np.ones(2, np.float32), out)
    assert e.value.rc == rt.HX_E_ARG
    with pytest.raises(rt.HxError):
        h.anima_adapter(afd, hidden, np.zeros(513, np.int32), np.ones(513, np.float32), out)  # more than 512 tokens
