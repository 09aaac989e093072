"""hx_modulation_noalloc: the allocation-free modulation entry point, for callers that cannot call
cudaMalloc (a thread running while another captures a CUDA graph in the global mode, hosts with a fixed
memory pool, callers without a handle). Its scratch is a static device array shared by every call.

Checked through the C ABI against the handle-based hx_modulation and against the oracle's modulation
(megarun.cpp:158-171) on the same inputs, two calls in a row (the second must not see the first one's
scratch); that free device memory does not move across further calls; and that the host rejects a
misaligned weight pointer and an oversized request before launching anything. This file is collected
last on purpose."""
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
            emb = torch.randn(D, generator=g)
            lora = 0.1 * torch.randn(3 * D, generator=g)
            e, l = emb.cuda(), lora.cuda()
            ref = torch.zeros(9 * D + 3 * 256, device="cuda")
            h.modulation(wfd, e, l, ref)
            got = torch.full((9 * D,), float("nan"), device="cuda")
            rt.modulation_noalloc(tA, tB, e, l, got, 3, D, stream)
            h.sync()
            assert torch.isfinite(got).all(), call
            assert rel(got, ref[:9 * D]) < 1e-5, call
            assert rel(got.cpu().view(9, D), oa.modulation(modA, modB, emb, lora)) < 1e-5, call
        # further calls allocate nothing: free device memory is unchanged (both kernels are loaded by now)
        h.sync()
        free0 = torch.cuda.mem_get_info()[0]
        for _ in range(4):
            rt.modulation_noalloc(tA, tB, e, l, got, 3, D, stream)
        h.sync()
        assert torch.cuda.mem_get_info()[0] == free0
        with pytest.raises(rt.HxError) as e1:  # 17 sites need 17*256 floats, over the 4096 of the static scratch
            rt.modulation_noalloc(tA, tB, e, l, got, 17, D, stream)
        assert e1.value.rc == rt.HX_E_SCRATCH
        with pytest.raises(rt.HxError) as e2:  # 2 bytes off a 16-byte boundary: refused on the host, no launch
            rt.modulation_noalloc(tA.data_ptr() + 2, tB, e, l, got, 3, D, stream)
        assert e2.value.rc == rt.HX_E_ARG
        h.weights_free(wfd)
        assert h.status() == 0
    finally:
        h.close()
