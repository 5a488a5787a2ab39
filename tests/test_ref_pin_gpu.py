"""Pins the oracle and the B200 kernels to the reference itself: the reference's own CUDA kernels
(examples/qwen/kernels.cuh compiled for sm_100a into oracle/_ref/libqk_ref.so) run on the same seeded inputs.
The reference's geometry limits apply (group size 128, H % 1024 == 0, I % 512 == 0)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import parity

pytestmark = pytest.mark.gpu

SHAPE = O.Shape(H=1024, E=32, TOPK=8, I=512, Is=512, G=128)


@pytest.fixture(scope="module")
def ref():
    from oracle import ref_kernels as R
    if not R.available():
        pytest.fail("oracle/_ref/libqk_ref.so is missing: build it with "
                    "`make -C oracle ref REF=<reference checkout>` before shipping")
    return R


@pytest.fixture(scope="module")
def layer():
    return O.make_layer(SHAPE, 9)


@pytest.mark.parametrize("T,with_next", [(1, False), (3, True), (8, False), (40, True)])
def test_oracle_matches_reference_kernels(orc, ref, layer, T, with_next):
    s = SHAPE
    hidden, attn = O.make_activations(s, T, 200 + T)
    nr = O.f32_to_bf16(1.0 + 0.1 * O.normal(200, T, s.H)) if with_next else None
    r = ref.block_forward(s, layer, hidden, attn, next_rms1=nr)
    o = orc.block_forward(s, layer, hidden, attn, next_rms1=nr, mode=-1)  # the reference's path choice by T
    # logits differ only through one-ulp bf16 flips of normed (RMSNorm summation order and rsqrt)
    assert O.max_rel_err(o["logits"], r["logits"]) < 2e-3
    margin = parity.topk_margin(o["logits"], s.TOPK)
    ok = parity.keep_stable(margin > 2 * np.abs(o["logits"] - r["logits"]).max(axis=1) + 1e-6, margin)
    assert np.array_equal(o["idx"][ok], r["idx"][ok])
    assert O.max_rel_err(o["routed"][ok], r["routed"][ok]) < 2e-2
    assert O.max_rel_err(O.bf16_to_f32(o["sout"]), O.bf16_to_f32(r["sout"])) < 1e-2
    assert O.max_rel_err(o["hidden"][ok], r["hidden"][ok]) < 1e-2
    assert O.max_rel_err(O.bf16_to_f32(o["normed"][ok]), O.bf16_to_f32(r["normed"][ok])) < 1e-2


@pytest.mark.parametrize("T", [1, 4])
def test_b200_decode_matches_reference_decode_kernels(ref, layer, T):
    """At T < 8 both take decode kernels with the same lane-order reductions: routing must agree bit for bit."""
    import mvcc_b200 as m
    s = SHAPE
    hidden, attn = O.make_activations(s, T, 300 + T)
    r = ref.block_forward(s, layer, hidden, attn)
    t = {n: torch.from_numpy(a if a.dtype == np.uint8 else a.view(np.int16)).cuda() for n, a in layer.items()}
    lay = m.MoeLayer(m.MoeShape(H=s.H, E=s.E, TOPK=s.TOPK, I=s.I, Is=s.Is, G=s.G), t)
    blk = m.MoeBlock(lay, T)
    h = torch.from_numpy(hidden).cuda()
    a = torch.from_numpy(attn.view(np.int16)).cuda()
    n = torch.zeros(T, s.H, dtype=torch.int16, device="cuda")
    blk.forward(h, a, n)
    torch.cuda.synchronize()
    tr = blk.trace(T)
    assert np.array_equal(tr["idx"].cpu().numpy(), r["idx"])
    assert O.max_rel_err(tr["logits"].cpu().numpy(), r["logits"]) < 1e-5
    assert O.max_rel_err(tr["routed"].cpu().numpy(), r["routed"]) < 1e-4
    assert O.max_rel_err(h.cpu().numpy(), r["hidden"]) < 1e-3
