"""Pins the decode-stack oracle (oracle/decode_stack.py) to golden vectors produced by the reference's own CUDA
kernels (attention branch and LM head of examples/qwen, run on a B200 by tests/golden/make_golden_stack.py). Inputs
are regenerated from the committed seeds and checked against the stored SHA-256 first. Bars: attention output, q and
the new k rows within max relative error 1e-2 (bf16; the reference uses fast-math exp/pow/sincos and a split-K
summation order), the new v rows bit for bit (a copy), logits within 1e-3 of the largest, the argmax equal."""
import importlib.util
import json
import os

import numpy as np
import pytest

from oracle import decode_stack as S
from oracle import oracle as O

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
META_PATH = os.path.join(HERE, "ref_stack_meta.json")
pytestmark = pytest.mark.skipif(not os.path.exists(META_PATH), reason="decode-stack golden vectors not generated")


def _gen():
    spec = importlib.util.spec_from_file_location("make_golden_stack", os.path.join(HERE, "make_golden_stack.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


G = _gen()


def _meta():
    return json.load(open(META_PATH))


def _rel(a, b):
    return O.max_rel_err(S.bf16_f(a), S.bf16_f(b))


@pytest.mark.parametrize("name", [c[0] for c in G.ATTN_CASES])
def test_attention_oracle_matches_reference_kernels(name):
    meta = _meta()
    case = meta["cases"][name]
    a = meta["attn"]
    T, pos0 = case["T"], case["pos0"]
    layer, kc, vc, normed = G.attn_inputs(T, case["seed"])
    assert G.digest(*[layer[k] for k in sorted(layer)], kc, vc, normed) == case["inputs_sha256"], \
        "input generator drifted from the golden vectors"
    ref = dict(np.load(os.path.join(HERE, f"ref_stack_{name}.npz")))
    out = S.attention_layer(normed, layer, a["Hq"], a["Hkv"], a["D"], a["rope_dim"], a["theta"], pos0, a["eps"], kc,
                            vc, a["gate"])
    assert _rel(out, ref["attn_out"]) < 1e-2
    assert np.array_equal(vc[:, pos0:pos0 + T], ref["v_new"])
    assert _rel(kc[:, pos0:pos0 + T], ref["k_new"]) < 1e-2


def test_lm_head_oracle_matches_reference_kernels():
    meta = _meta()
    hidden, fnorm, head = G.lm_inputs()
    assert G.digest(hidden, fnorm, head) == meta["lm_sha256"], "input generator drifted from the golden vectors"
    ref = dict(np.load(os.path.join(HERE, "ref_stack_lm.npz")))
    logits, idx = S.lm_head_argmax(hidden, fnorm, head, meta["lm"]["eps"])
    assert np.abs(logits - ref["logits"]).max() < 1e-3 * np.abs(ref["logits"]).max()
    assert idx == int(ref["next"])
    assert np.array_equal(S.rmsnorm(hidden[None, :].astype(np.float64), fnorm, meta["lm"]["eps"])[0], ref["normed"]) or \
        _rel(S.rmsnorm(hidden[None, :].astype(np.float64), fnorm, meta["lm"]["eps"])[0], ref["normed"]) < 1e-2
