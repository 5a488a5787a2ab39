"""CPU tests of the oracle (the parity checker): numeric helpers, the top-k rule, the stable permutation, and a
cross-check of the C restatement against an independent float64 numpy restatement of the block."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

SMALL = O.Shape(H=1024, E=32, TOPK=8, I=512, Is=512, G=128)
SMALL64 = O.Shape(H=512, E=16, TOPK=4, I=256, Is=256, G=64)


@pytest.fixture(scope="module")
def layer_small():
    return O.make_layer(SMALL, 7)


def test_bf16_rounding_matches_torch(orc):
    x = (O.normal(1, 2, 100_000) * np.float32(3.7)).astype(np.float32)
    x[:4] = [0.0, -0.0, 1e-40, 3.4e38]
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(O.f32_to_bf16(x), ref)
    assert np.array_equal(orc.to_bf16(x), ref)
    assert orc.lib.orc_f32_to_bf16(np.float32(1.00390625)) == 0x3F80  # tie rounds to even


def test_f16_decode(orc):
    bits = np.arange(0, 65536, 7, dtype=np.uint16)
    want = bits.view(np.float16).astype(np.float32)
    got = np.array([orc.lib.orc_f16_to_f32(int(b)) for b in bits], np.float32)
    finite = np.isfinite(want)
    assert np.array_equal(got[finite], want[finite])


def test_topk_rule_value_desc_index_asc(orc):
    """router_topk_kernel (kernels.cuh:774-809): ties go to the lower expert index."""
    lg = np.array([[1.0, 3.0, 3.0, 2.0, 3.0, -1.0, 2.0, 0.5]], np.float32)
    idx, wts = orc.topk(lg, 4)
    assert idx.tolist() == [[1, 2, 4, 3]]
    e = np.exp(np.array([3, 3, 3, 2], np.float64) - 3)
    assert np.allclose(wts[0], e / e.sum(), rtol=1e-6)
    rng = np.random.default_rng(0)
    lg = rng.integers(-3, 4, (64, 256)).astype(np.float32)  # many exact ties
    idx, wts = orc.topk(lg, 8)
    for t in range(64):
        order = sorted(range(256), key=lambda e: (-lg[t, e], e))[:8]
        assert idx[t].tolist() == order
    assert np.allclose(wts.sum(1), 1.0, atol=1e-6)


def test_sort_is_stable_bijection(orc):
    rng = np.random.default_rng(3)
    idx = rng.integers(0, 256, (4096, 8)).astype(np.int32)
    off, srt = orc.sort(idx, 256)
    flat = idx.reshape(-1)
    assert off[0] == 0 and off[-1] == flat.size
    assert np.array_equal(np.sort(srt), np.arange(flat.size))  # bijection
    want = np.argsort(flat, kind="stable")  # by expert, ascending pair index within an expert
    assert np.array_equal(srt, want)
    assert np.array_equal(np.diff(off), np.bincount(flat, minlength=256))


def test_quantizer_c_matches_numpy_and_bounds(orc):
    w = O.bf16_to_f32(O.f32_to_bf16(0.02 * O.normal(5, 5, 128 * 512))).reshape(128, 512)
    for G in (32, 64, 128):
        q1, s1 = O.quantize_int4(w, G)
        q2, s2 = orc.quantize_int4(w, G)
        assert np.array_equal(q1, q2) and np.array_equal(s1, s2)
        d = O.dequant_int4(q1, s1, G)
        sc = np.repeat(O.f16_to_f32(s1), G, axis=1)
        assert np.all(np.abs(d - w) <= 0.5 * sc * (1 + 1e-3) + 1e-12)


def _np_block(shape, L, hidden, attn, next_rms1, mode):
    """Independent float64 restatement of qwen.cu:429-448 with the reference's bf16 rounding points."""
    s = shape
    b2f = lambda a: O.bf16_to_f32(a).astype(np.float64)
    rb = lambda a: O.bf16_to_f32(O.f32_to_bf16(np.asarray(a, np.float32))).astype(np.float64)
    h = hidden.astype(np.float64) + b2f(attn)
    inv = 1.0 / np.sqrt((h * h).mean(1, keepdims=True) + s.eps)
    x = rb(h * inv * b2f(L["rms2"]))
    logits = x @ b2f(L["router"]).T
    T = x.shape[0]
    idx = np.argsort(-logits, axis=1, kind="stable")[:, : s.TOPK]
    pv = np.take_along_axis(logits, idx, 1)
    w = np.exp(pv - pv.max(1, keepdims=True))
    w /= w.sum(1, keepdims=True)
    wg = O.dequant_int4(L["exp_gu_q"].reshape(-1, s.H // 2), L["exp_gu_s"].reshape(-1, s.H // s.G), s.G)
    wd = O.dequant_int4(L["exp_dn_q"].reshape(-1, s.I // 2), L["exp_dn_s"].reshape(-1, s.I // s.G), s.G)
    if mode == 1:
        wg, wd = rb(wg), rb(wd)
    wg = wg.reshape(s.E, 2 * s.I, s.H)
    wd = wd.reshape(s.E, s.H, s.I)
    routed = np.zeros((T, s.H))
    for t in range(T):
        for k in range(s.TOPK):
            e = idx[t, k]
            g = wg[e, : s.I] @ x[t]
            u = wg[e, s.I:] @ x[t]
            inter = rb(g / (1 + np.exp(-g)) * u)
            routed[t] += w[t, k] * (wd[e] @ inter)
    sgu = rb(x @ b2f(L["shared_gate_up"]).T)
    sinter = rb(sgu[:, : s.Is] / (1 + np.exp(-sgu[:, : s.Is])) * sgu[:, s.Is:])
    sout = rb(sinter @ b2f(L["shared_down"]).T)
    gate = 1 / (1 + np.exp(-(x @ b2f(L["shared_gate"]))))
    hout = h + routed + gate[:, None] * sout
    out = {"logits": logits, "idx": idx, "routed": routed, "sout": sout, "hidden": hout, "x": x}
    if next_rms1 is not None:
        inv = 1.0 / np.sqrt((hout * hout).mean(1, keepdims=True) + s.eps)
        out["normed"] = rb(hout * inv * b2f(next_rms1))
    return out


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("T", [3, 8])
def test_oracle_matches_float64_restatement(orc, layer_small, mode, T):
    """The C oracle against the float64 restatement with the same bf16 rounding points: what is left is the fp32
    accumulation and the bf16 roundings it flips by one ulp. Measured at these inputs: with the router input equal,
    logits within 3e-7; one router-input element one ulp apart (T = 8) moves them by 9.6e-5; routed within 6.1e-4;
    sout and the next layer's normed within one bf16 ulp (2^-8 relative); hidden within 1.3e-4. The bars keep a few
    times that: fp32 accumulation takes at most 1/6 of the int4 outputs' parity tolerance (2e-2) and 1/10 of the
    fp32 hidden's (1e-2)."""
    s = SMALL
    hidden, attn = O.make_activations(s, T, 8 + T)
    nr = O.f32_to_bf16(1.0 + 0.1 * O.normal(3, 3, s.H))
    got = orc.block_forward(s, layer_small, hidden, attn, next_rms1=nr, mode=mode)
    ref = _np_block(s, layer_small, hidden, attn, nr, mode)
    assert O.max_rel_err(got["logits"], ref["logits"]) < 5e-4
    # routing identical wherever the 8th/9th margin exceeds twice the logit difference
    lerr = np.abs(got["logits"] - ref["logits"]).max(axis=1)
    srt = np.sort(ref["logits"], axis=1)[:, ::-1]
    margin = srt[:, s.TOPK - 1] - srt[:, s.TOPK]
    for t in range(T):
        if margin[t] > 2 * lerr[t] + 1e-6:
            assert sorted(got["idx"][t]) == sorted(ref["idx"][t])
    assert O.max_rel_err(got["routed"], ref["routed"]) < 3e-3
    assert O.max_rel_err(O.bf16_to_f32(got["sout"]), ref["sout"]) < 2 ** -8 + 1e-6
    assert O.max_rel_err(got["hidden"], ref["hidden"]) < 1e-3
    assert O.max_rel_err(O.bf16_to_f32(got["normed"]), ref["normed"]) < 2 ** -8 + 1e-6


def test_decode_and_tile_numerics_agree(orc, layer_small):
    s = SMALL
    hidden, attn = O.make_activations(s, 2, 12)
    a = orc.block_forward(s, layer_small, hidden, attn, mode=0)
    b = orc.block_forward(s, layer_small, hidden, attn, mode=1)
    assert np.array_equal(a["idx"], b["idx"])
    assert O.max_rel_err(b["routed"], a["routed"]) < 2e-2


def test_exact_inputs_give_exact_dots(orc):
    """With exact-valued inputs every fp32 dot is exact, so decode and tile numerics give identical inter."""
    s = SMALL64
    L = O.make_layer(s, 5, exact=True)
    x = O.exact_normed(s, 4, 5)
    logits, idx, wts = orc.router(s, L, x)
    want = O.bf16_to_f32(x).astype(np.float64) @ O.bf16_to_f32(L["router"]).astype(np.float64).T
    assert np.array_equal(logits, want.astype(np.float32))
    i0, r0 = orc.routed(s, L, x, idx, wts, mode=0)
    i1, r1 = orc.routed(s, L, x, idx, wts, mode=1)
    assert np.array_equal(i0, i1)
    assert O.max_rel_err(r1, r0) < 1e-6


def test_threaded_oracle_is_deterministic(orc, layer_small):
    s = SMALL
    hidden, attn = O.make_activations(s, 4, 13)
    a = orc.block_forward(s, layer_small, hidden, attn)
    orc.set_threads(4)
    try:
        b = orc.block_forward(s, layer_small, hidden, attn)
    finally:
        orc.set_threads(1)
    for k in ("hidden", "routed", "sout", "idx"):
        assert np.array_equal(a[k], b[k])


def test_router_bias_is_added_to_fp32_logits(orc):
    """The optional per-expert bias shifts the oracle's logits exactly (one fp32 add after the sum) and the top-k
    and weights follow the biased logits, in the router and in the whole block."""
    s = O.Shape(H=512, E=16, TOPK=4, I=256, Is=256, G=32)
    L = O.make_layer(s, 3)
    x = O.f32_to_bf16(O.normal(5, 4, 4 * s.H)).reshape(4, s.H)
    l0, _, _ = orc.router(s, L, x)
    Lb = dict(L)
    Lb["router_bias"] = np.linspace(-1, 1, s.E).astype(np.float32)
    l1, i1, w1 = orc.router(s, Lb, x)
    assert np.array_equal(l1, (l0 + Lb["router_bias"][None, :]).astype(np.float32))
    ic, wc = orc.topk(l1, s.TOPK)
    assert np.array_equal(ic, i1) and np.array_equal(wc, w1)
    h, a = O.make_activations(s, 3, 7)
    rb = orc.block_forward(s, Lb, h, a, mode=0)
    r0 = orc.block_forward(s, L, h, a, mode=0)
    assert np.allclose(rb["logits"] - r0["logits"], Lb["router_bias"][None, :], atol=1e-6)


def test_ep_oracle_one_rank_equals_block_and_ranks_only_reorder_sums(orc):
    """The expert-parallel restatement with one rank is the tile-numerics block with its routed row rounded to bf16
    (the row that crosses the return exchange); with W ranks it differs further only by the per-rank roundings and
    the fp32 order of the routed sum (per rank in slot order, then over ranks)."""
    s = O.Shape(H=512, E=32, TOPK=4, I=256, Is=256, G=32)
    L = O.make_layer(s, 5)
    h, a = O.make_activations(s, 6, 9)
    ref = orc.block_forward(s, L, h, a, mode=1)
    one = orc.ep_block_forward(s, L, h, a, 1)
    assert np.array_equal(one["routed"], O.bf16_to_f32(O.f32_to_bf16(ref["routed"])))
    assert O.max_rel_err(one["hidden"], ref["hidden"]) < 2.0 ** -8
    for world in (2, 4):
        ep = orc.ep_block_forward(s, L, h, a, world)
        assert O.max_rel_err(ep["routed"], ref["routed"]) < 2.0 ** -8
        assert O.max_rel_err(ep["hidden"], ref["hidden"]) < 2.0 ** -8
    nr = O.f32_to_bf16(1.0 + 0.1 * O.normal(7, 1, s.H))
    ref_n = orc.block_forward(s, L, h, a, next_rms1=nr, mode=1)
    one_n = orc.ep_block_forward(s, L, h, a, 1, next_rms1=nr)
    assert O.max_rel_err(one_n["hidden"], ref_n["hidden"]) < 2.0 ** -8
    assert O.max_rel_err(O.bf16_to_f32(one_n["normed"]), O.bf16_to_f32(ref_n["normed"])) < 1e-2
