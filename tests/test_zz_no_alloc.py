"""The allocation-free router entry point (moe_router_topk_noalloc), for callers that cannot allocate device memory
(a host runtime that owns all device memory and has no workspace to pass): called through the C ABI twice in a
row, it must give the same logits, indices and weights as the workspace entry point moe_router_topk when both take
the decode kernels, and agree within the router's tolerance where moe_router_topk takes the tensor-core router.
Collected last so that a failure here leaves every other test already run; passes alone in a fresh process too."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O

SHAPES = {"h1024_e32": O.Shape(H=1024, E=32, TOPK=8, I=512, Is=512, G=64),
          "qwen_e256": O.Shape(H=2048, E=256, TOPK=8, I=512, Is=512, G=64)}


def _noalloc(m, layer, x, outs, T):
    return m._lib.moe_router_topk_noalloc(ctypes.byref(layer.c), ctypes.c_void_p(x.data_ptr()),
                                          ctypes.c_void_p(outs[0].data_ptr()), ctypes.c_void_p(outs[1].data_ptr()),
                                          ctypes.c_void_p(outs[2].data_ptr()), T,
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _setup(name, T, seed):
    import mvcc_b200 as m
    s = SHAPES[name]
    L = O.make_layer(s, 71) if s.E <= 32 else None
    if L is None:  # full geometry: the router only needs the router matrix; the other tensors are not read
        layer = m.synth_layer(m.MoeShape(), seed=71)
    else:
        t = {n: torch.from_numpy(a if a.dtype == np.uint8 else a.view(np.int16)).cuda() for n, a in L.items()}
        layer = m.MoeLayer(m.MoeShape(H=s.H, E=s.E, TOPK=s.TOPK, I=s.I, Is=s.Is, G=s.G), t)
    x = torch.from_numpy(O.f32_to_bf16(O.normal(seed, T, T * s.H)).reshape(T, s.H).view(np.int16)).cuda()

    def outs():
        return (torch.zeros(T, s.E, device="cuda"), torch.zeros(T, s.TOPK, dtype=torch.int32, device="cuda"),
                torch.zeros(T, s.TOPK, device="cuda"))
    return m, s, layer, x, outs


@pytest.mark.gpu
@pytest.mark.usefixtures("decode_only")
@pytest.mark.parametrize("name,T", [("h1024_e32", 1), ("h1024_e32", 16), ("h1024_e32", 21), ("qwen_e256", 1),
                                    ("qwen_e256", 16), ("qwen_e256", 40)])
def test_noalloc_router_matches_workspace_router(name, T):
    m, s, layer, x, outs = _setup(name, T, 72)
    ref = outs()
    m.MoeBlock(layer, T).router_topk(x, *ref)
    for _ in range(2):  # two calls in a row share (and reuse) the static scratch
        got = outs()
        assert _noalloc(m, layer, x, got, T) == 0
        torch.cuda.synchronize()
        assert O.max_rel_err(got[0].cpu().numpy(), ref[0].cpu().numpy()) < 1e-5
        assert np.array_equal(got[1].cpu().numpy(), ref[1].cpu().numpy())
        assert np.allclose(got[2].cpu().numpy(), ref[2].cpu().numpy(), rtol=1e-5, atol=1e-7)
        assert m.router_topk_noalloc_error() == 0  # the scratch error word, read back and cleared


@pytest.mark.gpu
@pytest.mark.parametrize("T", [16, 300])
def test_noalloc_router_at_the_default_threshold(T):
    """At the default prefill threshold moe_router_topk takes the tensor-core router (fp32 sums of the same bf16
    products in another order): logits agree to 1e-5 relative, indices wherever the 8th/9th margin exceeds the
    logit difference, and the rule applied to the allocation-free call's own logits reproduces its indices."""
    m, s, layer, x, outs = _setup("qwen_e256", T, 73)
    ref = outs()
    m.MoeBlock(layer, T).router_topk(x, *ref)
    got = outs()
    assert _noalloc(m, layer, x, got, T) == 0
    torch.cuda.synchronize()
    gl, rl = got[0].cpu().numpy(), ref[0].cpu().numpy()
    assert O.max_rel_err(gl, rl) < 1e-5
    idx_c, _ = O.Oracle().topk(gl, s.TOPK)
    assert np.array_equal(idx_c, got[1].cpu().numpy())
    srt = np.sort(rl, axis=1)[:, ::-1]
    ok = srt[:, s.TOPK - 1] - srt[:, s.TOPK] > 2 * np.abs(gl - rl).max(axis=1) + 1e-6
    assert ok.mean() >= 0.9
    assert np.array_equal(got[1].cpu().numpy()[ok], ref[1].cpu().numpy()[ok])


def test_noalloc_router_rejects_bad_shapes_before_any_device_call():
    """Shape checks come first: an unsupported geometry is refused with cudaErrorInvalidValue (1) without touching
    the device (this runs without a GPU)."""
    import mvcc_b200 as m
    w = m.MoeLayerWeights()
    w.router = 16
    w.H, w.E, w.TOPK, w.I, w.Is, w.G, w.eps = 2048, 300, 8, 512, 512, 64, 1e-6  # E above the top-k limit of 256
    buf = ctypes.c_void_p(16)
    assert m._lib.moe_router_topk_noalloc(ctypes.byref(w), buf, buf, buf, buf, 1, None) == 1
    w.E = 256
    assert m._lib.moe_router_topk_noalloc(ctypes.byref(w), buf, buf, buf, buf, 0, None) == 1  # T < 1
