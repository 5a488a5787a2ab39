"""The allocation-free router entry point (moe_router_topk_noalloc), for callers that cannot allocate device memory
(a host runtime that owns all device memory and has no workspace to pass): called through the C ABI twice in a
row, it must give the same logits, indices and weights as the workspace entry point moe_router_topk. Collected
last so that a failure here leaves every other test already run; passes alone in a fresh process too."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("decode_only")]


@pytest.mark.parametrize("T", [1, 16, 21])
def test_noalloc_router_matches_workspace_router(T):
    import mvcc_b200 as m
    s = O.Shape(H=1024, E=32, TOPK=8, I=512, Is=512, G=64)
    L = O.make_layer(s, 71)
    t = {n: torch.from_numpy(a if a.dtype == np.uint8 else a.view(np.int16)).cuda() for n, a in L.items()}
    layer = m.MoeLayer(m.MoeShape(H=s.H, E=s.E, TOPK=s.TOPK, I=s.I, Is=s.Is, G=s.G), t)
    x = torch.from_numpy(O.f32_to_bf16(O.normal(72, T, T * s.H)).reshape(T, s.H).view(np.int16)).cuda()

    def outs():
        return (torch.zeros(T, s.E, device="cuda"), torch.zeros(T, s.TOPK, dtype=torch.int32, device="cuda"),
                torch.zeros(T, s.TOPK, device="cuda"))

    ref = outs()
    m.MoeBlock(layer, T).router_topk(x, *ref)
    for _ in range(2):  # two calls in a row share (and reuse) the static scratch
        got = outs()
        rc = m._lib.moe_router_topk_noalloc(ctypes.byref(layer.c), ctypes.c_void_p(x.data_ptr()),
                                            ctypes.c_void_p(got[0].data_ptr()), ctypes.c_void_p(got[1].data_ptr()),
                                            ctypes.c_void_p(got[2].data_ptr()), T,
                                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0
        torch.cuda.synchronize()
        assert O.max_rel_err(got[0].cpu().numpy(), ref[0].cpu().numpy()) < 1e-5
        assert np.array_equal(got[1].cpu().numpy(), ref[1].cpu().numpy())
        assert np.allclose(got[2].cpu().numpy(), ref[2].cpu().numpy(), rtol=1e-5, atol=1e-7)
