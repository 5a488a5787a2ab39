"""Live pin of the decode stack on a B200: the reference's own attention and LM-head kernels (oracle/_ref/libqk_ref.so,
built from examples/qwen/kernels.cuh), this library's kernels and the CPU oracle (oracle/decode_stack.py) on the same
seeded inputs (tests/golden/make_golden_stack.py's generator). Bars as in tests/test_golden_stack.py; the library's
attention output agrees with the reference's within 1e-2 and its argmax equals the reference's."""
import importlib.util
import os

import numpy as np
import pytest
import torch

from oracle import decode_stack as S
from oracle import oracle as O

pytestmark = pytest.mark.gpu
HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _gen():
    spec = importlib.util.spec_from_file_location("make_golden_stack", os.path.join(HERE, "make_golden_stack.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


G = _gen()


@pytest.fixture(scope="module", autouse=True)
def ref_lib():
    from oracle import ref_kernels as R
    if not R.available():
        pytest.fail("oracle/_ref/libqk_ref.so is missing: build it with "
                    "`make -C oracle ref REF=<reference checkout>` before shipping")


def _rel(a, b):
    return O.max_rel_err(S.bf16_f(a), S.bf16_f(b))


@pytest.mark.parametrize("name,T,pos0,seed", G.ATTN_CASES)
def test_attention_three_ways(name, T, pos0, seed):
    from mvcc_b200 import stack as st
    a = G.ATTN
    layer, kc, vc, normed = G.attn_inputs(T, seed)
    r_out, _, r_kc, r_vc = G.ref_attention(layer, kc, vc, normed, T, pos0)
    o_kc, o_vc = kc.copy(), vc.copy()
    o_out = S.attention_layer(normed, layer, a["Hq"], a["Hkv"], a["D"], a["rope_dim"], a["theta"], pos0, a["eps"],
                              o_kc, o_vc, a["gate"])
    shape = st.AttnShape(H=a["H"], Hq=a["Hq"], Hkv=a["Hkv"], D=a["D"], rope_dim=a["rope_dim"], theta=a["theta"],
                         eps=a["eps"], gate=a["gate"])
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).cuda()  # noqa: E731
    lay = st.AttnLayer(shape, {k: dev(v) for k, v in layer.items()})
    blk = st.AttnBlock(lay, a["ctx"], max_T=T, caches=(dev(kc), dev(vc)))
    out = torch.zeros(T, a["H"], dtype=torch.int16, device="cuda")
    blk.forward(dev(normed), out, pos0)
    torch.cuda.synchronize()
    b_out = out.cpu().numpy().view(np.uint16)
    assert _rel(o_out, r_out) < 1e-2      # oracle vs reference
    assert _rel(b_out, r_out) < 1e-2      # library vs reference
    assert _rel(b_out, o_out) < 1e-2      # library vs oracle
    new = slice(pos0, pos0 + T)
    b_kc, b_vc = blk.kc.cpu().numpy().view(np.uint16), blk.vc.cpu().numpy().view(np.uint16)
    assert np.array_equal(b_vc[:, new], r_vc[:, new]) and np.array_equal(o_vc[:, new], r_vc[:, new])
    assert _rel(b_kc[:, new], r_kc[:, new]) < 1e-2 and _rel(o_kc[:, new], r_kc[:, new]) < 1e-2


def test_lm_head_three_ways():
    from mvcc_b200 import stack as st
    hidden, fnorm, head = G.lm_inputs()
    r_logits, r_next, r_normed = G.ref_lm_head(hidden, fnorm, head)
    o_logits, o_next = S.lm_head_argmax(hidden, fnorm, head, G.LM["eps"])
    hd = torch.from_numpy(hidden[None, :].copy()).cuda()
    nrm = torch.zeros(1, G.LM["H"], dtype=torch.int16, device="cuda")
    st.rmsnorm(hd, torch.from_numpy(fnorm.view(np.int16)).cuda(), nrm, G.LM["eps"])
    lm = st.LmHead(torch.from_numpy(head.view(np.int16)).cuda())
    nxt = torch.zeros(1, dtype=torch.int32, device="cuda")
    logits = torch.zeros(G.LM["V"], device="cuda")
    lm.argmax(nrm[0], nxt, logits=logits)
    torch.cuda.synchronize()
    b_logits = logits.cpu().numpy()
    scale = np.abs(r_logits).max()
    assert np.abs(o_logits - r_logits).max() < 1e-3 * scale
    assert np.abs(b_logits - r_logits).max() < 1e-3 * scale
    assert o_next == r_next == int(nxt.item())
    assert np.array_equal(nrm.cpu().numpy().view(np.uint16)[0], r_normed) or _rel(nrm.cpu().numpy().view(np.uint16)[0], r_normed) < 1e-2
