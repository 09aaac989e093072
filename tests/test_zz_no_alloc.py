"""hx_modulation_noalloc: the allocation-free modulation entry point, for callers that cannot call
cudaMalloc (a thread running while another captures a CUDA graph in the global mode, hosts with a fixed
memory pool, callers without a handle). Its scratch is a static device array shared by every call.

Checked through the C ABI against the handle-based hx_modulation on the same inputs, two calls in a row
(the second must not see the first one's scratch). This file is collected last on purpose."""
import pytest
import torch

from hexanima_b200 import runtime as rt
from tests.gpu_util import anima_bind, rel
from oracle import anima as oa

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("D", [256, 2048])
def test_modulation_noalloc_matches_handle_version(D):
    h = rt.Handle(0)
    try:
        W, norms, modA, modB = oa.init_weights(90 + D, D=D, F=512, Cd=128)
        wfd, _, _, keep = anima_bind(h, W, norms, modA, modB)
        tA, tB = modA.cuda().contiguous(), modB.cuda().contiguous()
        stream = h.stream()
        g = torch.Generator().manual_seed(D)
        for call in range(2):
            emb = torch.randn(D, generator=g).cuda()
            lora = (0.1 * torch.randn(3 * D, generator=g)).cuda()
            ref = torch.zeros(9 * D + 3 * 256, device="cuda")
            h.modulation(wfd, emb, lora, ref)
            got = torch.full((9 * D,), float("nan"), device="cuda")
            rt.modulation_noalloc(tA, tB, emb, lora, got, 3, D, stream)
            h.sync()
            assert torch.isfinite(got).all(), call
            assert rel(got, ref[:9 * D]) < 1e-5, call
        with pytest.raises(rt.HxError) as e:  # 17 sites need 17*256 floats, over the 4096 of the static scratch
            rt.modulation_noalloc(tA, tB, emb, lora, got, 17, D, stream)
        assert e.value.rc == rt.HX_E_SCRATCH
        h.weights_free(wfd)
        assert h.status() == 0
    finally:
        h.close()
