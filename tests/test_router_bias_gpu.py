"""The optional per-expert router bias (moe_layer_weights.router_bias, the prefill benchmark's Zipf-skewed expert
load) through every path: fused decode (T < 8), the three-kernel decode path, and the prefill path, against the
oracle with the same bias added to its fp32 logits."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.test_decode_gpu import TOL_BF16, check_routing, host16, mb, stable_rows, to_dev16, upload

pytestmark = pytest.mark.gpu


def biased_layer(s, seed):
    m = mb()
    L = O.make_layer(s, seed)
    layer = upload(s, L)
    bias = m.zipf_bias(s.E, seed=0)
    t = dict(layer.t)
    t["router_bias"] = torch.from_numpy(bias).cuda()
    L = dict(L)
    L["router_bias"] = bias
    return L, m.MoeLayer(layer.shape, t)


@pytest.mark.parametrize("T,path", [(1, "fused"), (5, "fused"), (16, "decode"), (300, "prefill")])
def test_block_with_router_bias(orc, T, path):
    m = mb()
    s = O.Shape(H=1024, E=32, TOPK=8, I=512, Is=512, G=64)
    L, layer = biased_layer(s, 29)
    hidden, attn = O.make_activations(s, T, 300 + T)
    if path == "decode":
        m.set_prefill_min_tokens(1 << 30)
    try:
        blk = m.MoeBlock(layer, T)
        h = torch.from_numpy(np.ascontiguousarray(hidden, np.float32)).cuda()
        normed = torch.zeros(T, s.H, dtype=torch.int16, device="cuda")
        blk.forward(h, to_dev16(attn), normed)
        torch.cuda.synchronize()
        tr = blk.trace(T)
        gl = tr["logits"].cpu().numpy()
        gi = tr["idx"].cpu().numpy()
        gw = tr["wts"].cpu().numpy()
    finally:
        m.set_prefill_min_tokens(0)
    ref = orc.block_forward(s, L, hidden, attn, mode=1 if path == "prefill" else 0)
    check_routing(orc, s, gl, gi, gw, ref["logits"], ref["idx"], ref["wts"], logit_tol=2e-3)
    ok = stable_rows(s, ref["logits"], gpu_logits=gl)
    assert O.max_rel_err(h.cpu().numpy()[ok], ref["hidden"][ok]) < TOL_BF16
    assert O.max_rel_err(O.bf16_to_f32(host16(normed)[ok]), O.bf16_to_f32(ref["normed"][ok])) < TOL_BF16
    # the bias skews the load: the most-biased experts take more than their even share of the picks
    if T >= 16:
        order = np.argsort(-L["router_bias"])
        share = np.isin(gi, order[:4]).mean()
        assert share > 4.0 / s.E


def test_router_bias_shape_is_checked():
    m = mb()
    s = O.Shape(H=1024, E=32, TOPK=8, I=512, Is=512, G=64)
    layer = upload(s, O.make_layer(s, 29))
    t = dict(layer.t)
    t["router_bias"] = torch.zeros(s.E + 1, device="cuda")
    with pytest.raises(ValueError):
        m.MoeLayer(layer.shape, t)
