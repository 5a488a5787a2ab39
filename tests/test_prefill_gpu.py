"""GPU parity tests of the prefill path (T >= 8: router GEMM + top-k, stable expert sort, tcgen05 grouped INT4
GEMMs, shared-expert GEMMs, slot-order combine) through the C ABI, against the oracle's tile numerics (mode 1, the
reference's moe() path for T >= 8, qwen.cu:345-363) on the same seeded inputs. Bars as for the decode path: router
top-k bit-exact (the rule on the GPU's logits; end to end beyond the logit tolerance), the expert sort bit-exact
(stable order by pair index), int4 outputs within 2e-2, bf16 within 1e-2 max relative error."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.test_decode_gpu import (TOL_BF16, TOL_INT4, check_routing, host16, mb, stable_rows, to_dev16,
                                   upload)

pytestmark = pytest.mark.gpu

SHAPES = {
    "h1024_g128": O.Shape(H=1024, E=32, TOPK=8, I=512, Is=512, G=128),
    "h1024_g64": O.Shape(H=1024, E=32, TOPK=8, I=512, Is=512, G=64),
    "h512_g32_k4": O.Shape(H=512, E=16, TOPK=4, I=256, Is=256, G=32),
}

PREFILL_T = 4096
_cache = {}


def layer_for(name):
    if name not in _cache:
        s = SHAPES[name]
        L = O.make_layer(s, 23)
        _cache[name] = (s, L, upload(s, L))
    return _cache[name]


def rand_x(s, T, seed):
    return O.f32_to_bf16(O.normal(seed, T, T * s.H)).reshape(T, s.H)


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("T", [8, 40, 300])
def test_router_gemm_topk(orc, name, T):
    """dense(router) on the tcgen05 GEMM + the top-k rule: fp32 logits of exact bf16 products, summation order
    aside, so the logit tolerance is 1e-5."""
    s, L, layer = layer_for(name)
    m = mb()
    blk = m.MoeBlock(layer, T)
    x = rand_x(s, T, 131 + T)
    logits = torch.zeros(T, s.E, device="cuda")
    idx = torch.zeros(T, s.TOPK, dtype=torch.int32, device="cuda")
    wts = torch.zeros(T, s.TOPK, device="cuda")
    blk.router_topk(to_dev16(x), logits, idx, wts)
    torch.cuda.synchronize()
    rl, ri, rw = orc.router(s, L, x)
    check_routing(orc, s, logits.cpu().numpy(), idx.cpu().numpy(), wts.cpu().numpy(), rl, ri, rw)


def test_router_gemm_exact_inputs_bit_exact(orc):
    """Small-integer activations and power-of-two weights: every partial sum is exact, so the tensor-core logits
    equal the oracle's bit for bit."""
    s = O.Shape(H=1024, E=32, TOPK=8, I=512, Is=512, G=64)
    L = O.make_layer(s, 21, exact=True)
    layer = upload(s, L)
    m = mb()
    T = 136
    blk = m.MoeBlock(layer, T)
    x = O.exact_normed(s, T, 45)
    logits = torch.zeros(T, s.E, device="cuda")
    idx = torch.zeros(T, s.TOPK, dtype=torch.int32, device="cuda")
    wts = torch.zeros(T, s.TOPK, device="cuda")
    blk.router_topk(to_dev16(x), logits, idx, wts)
    torch.cuda.synchronize()
    rl, ri, _ = orc.router(s, L, x)
    assert np.array_equal(logits.cpu().numpy(), rl)
    assert np.array_equal(idx.cpu().numpy(), ri)


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("T", [8, 33, 300])
def test_routed_experts_prefill(orc, name, T):
    s, L, layer = layer_for(name)
    m = mb()
    blk = m.MoeBlock(layer, T)
    x = rand_x(s, T, 141 + T)
    _, idx, wts = orc.router(s, L, x)
    routed = torch.zeros(T, s.H, device="cuda")
    inter = torch.zeros(T, s.TOPK, s.I, dtype=torch.int16, device="cuda")
    blk.routed_experts(to_dev16(x), torch.from_numpy(idx).cuda(), torch.from_numpy(wts).cuda(), routed, inter)
    torch.cuda.synchronize()
    ri, rr = orc.routed(s, L, x, idx, wts, mode=1)
    gi = host16(inter)
    # g and u are 2*H-term fp32 sums in another order than the oracle's, so an inter value from a cancelling sum
    # can move by several bf16 ulps; relative to the tensor and in the bulk it stays within one ulp
    assert O.max_rel_err(O.bf16_to_f32(gi), O.bf16_to_f32(ri)) < TOL_BF16
    assert np.mean(np.abs(gi.astype(np.int32) - ri.astype(np.int32)) <= 1) >= 0.999
    assert O.max_rel_err(routed.cpu().numpy(), rr) < TOL_INT4
    assert blk.error_word() == 0


def test_routed_duplicate_and_invalid_indices(orc):
    """Caller routing may repeat an expert within a token (each pair still counts) and may hold an out-of-range
    index (flagged in the error word, the pair dropped, never a fault); other tokens are unaffected."""
    s, L, layer = layer_for("h1024_g64")
    m = mb()
    T = 24
    blk = m.MoeBlock(layer, T)
    x = rand_x(s, T, 151)
    _, idx, wts = orc.router(s, L, x)
    idx[3, 1] = idx[3, 0]
    idx[5] = 7
    idx[9, 2] = 999
    routed = torch.zeros(T, s.H, device="cuda")
    blk.routed_experts(to_dev16(x), torch.from_numpy(idx).cuda(), torch.from_numpy(wts).cuda(), routed)
    torch.cuda.synchronize()
    assert blk.error_word() == 1
    keep = np.ones(T, bool)
    keep[9] = False
    _, rr = orc.routed(s, L, x[keep], idx[keep], wts[keep], mode=1)
    assert O.max_rel_err(routed.cpu().numpy()[keep], rr) < TOL_INT4


@pytest.mark.parametrize("name", ["h1024_g64", "h512_g32_k4"])
@pytest.mark.parametrize("T", [8, 130])
def test_shared_expert_prefill(orc, name, T):
    s, L, layer = layer_for(name)
    m = mb()
    blk = m.MoeBlock(layer, T)
    x = rand_x(s, T, 161 + T)
    sout = torch.zeros(T, s.H, dtype=torch.int16, device="cuda")
    blk.shared_expert(to_dev16(x), sout)
    torch.cuda.synchronize()
    _, rs = orc.shared(s, L, x)
    assert O.max_rel_err(O.bf16_to_f32(host16(sout)), O.bf16_to_f32(rs)) < TOL_BF16


def run_block(s, layer, hidden, attn, next_rms1=None):
    m = mb()
    T = hidden.shape[0]
    blk = m.MoeBlock(layer, T)
    h = torch.from_numpy(np.ascontiguousarray(hidden, np.float32)).cuda()
    a = to_dev16(attn)
    normed = torch.zeros(T, s.H, dtype=torch.int16, device="cuda")
    nr = None if next_rms1 is None else to_dev16(next_rms1)
    blk.forward(h, a, normed, next_rms1=nr)
    torch.cuda.synchronize()
    return blk, h.cpu().numpy(), host16(normed)


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("T,with_next", [(8, False), (40, True), (300, False), (300, True)])
def test_block_prefill(orc, name, T, with_next):
    s, L, layer = layer_for(name)
    hidden, attn = O.make_activations(s, T, 170 + T)
    nr = O.f32_to_bf16(1.0 + 0.1 * O.normal(171, 1, s.H)) if with_next else None
    blk, gh, gn = run_block(s, layer, hidden, attn, nr)
    ref = orc.block_forward(s, L, hidden, attn, next_rms1=nr, mode=1)
    tr = blk.trace(T)
    gl = tr["logits"].cpu().numpy()
    check_routing(orc, s, gl, tr["idx"].cpu().numpy(), tr["wts"].cpu().numpy(), ref["logits"], ref["idx"],
                  ref["wts"], logit_tol=2e-3)
    ok = stable_rows(s, ref["logits"], gpu_logits=gl)
    assert O.max_rel_err(gh[ok], ref["hidden"][ok]) < TOL_BF16
    assert O.max_rel_err(O.bf16_to_f32(gn[ok]), O.bf16_to_f32(ref["normed"][ok])) < TOL_BF16
    assert O.max_rel_err(tr["routed"].cpu().numpy()[ok], ref["routed"][ok]) < TOL_INT4
    assert O.max_rel_err(O.bf16_to_f32(host16(tr["sout"])), O.bf16_to_f32(ref["sout"])) < TOL_BF16
    assert np.allclose(tr["gate"].cpu().numpy()[ok], ref["gate"][ok], rtol=2e-3)
    assert blk.error_word() == 0


@pytest.mark.parametrize("T", [8, 300, 1000])
def test_expert_sort_is_stable_and_bit_exact(orc, T):
    """The permutation equals the oracle's stable counting sort of the GPU's own routing, bit for bit."""
    s, L, layer = layer_for("h1024_g64")
    hidden, attn = O.make_activations(s, T, 180 + T)
    blk, _, _ = run_block(s, layer, hidden, attn)
    tr = blk.trace(T)
    off, srt = orc.sort(tr["idx"].cpu().numpy(), s.E)
    assert np.array_equal(tr["offsets"].cpu().numpy(), off)
    assert np.array_equal(tr["sorted"].cpu().numpy(), srt)


def test_block_prefill_deterministic():
    s, L, layer = layer_for("h1024_g128")
    hidden, attn = O.make_activations(s, 257, 190)
    _, h1, n1 = run_block(s, layer, hidden, attn)
    _, h2, n2 = run_block(s, layer, hidden, attn)
    assert np.array_equal(h1, h2) and np.array_equal(n1, n2)


@pytest.mark.parametrize("T", [512, 4096])
def test_full_size_prefill_rows_against_oracle(orc, T):
    """BASELINE geometry (H=2048, E=256, top-8, I=Is=512, G=64) on the device generator. Each token's outputs depend
    on that token alone, so the oracle runs a sample of 24 tokens of the same batch; the sort is checked whole."""
    m = mb()
    ms = m.MoeShape()
    layer = m.synth_layer(ms, seed=9)
    hid, att = m.synth_activations(ms, T, 11)
    torch.cuda.synchronize()
    s = O.Shape()
    L = {n: (v.cpu().numpy() if v.dtype == torch.uint8 else v.cpu().numpy().view(np.uint16))
         for n, v in layer.t.items()}
    hidden = hid.cpu().numpy()
    attn = att.cpu().numpy().view(np.uint16)
    blk = m.MoeBlock(layer, T)
    normed = torch.zeros(T, ms.H, dtype=torch.int16, device="cuda")
    blk.forward(hid, att, normed)
    torch.cuda.synchronize()
    tr = blk.trace(T)
    gidx = tr["idx"].cpu().numpy()
    off, srt = orc.sort(gidx, s.E)
    assert np.array_equal(tr["sorted"].cpu().numpy(), srt)
    rows = np.random.default_rng(T).choice(T, 24, replace=False)
    ref = orc.block_forward(s, L, hidden[rows], attn[rows], mode=1)
    gl = tr["logits"].cpu().numpy()[rows]
    check_routing(orc, s, gl, gidx[rows], tr["wts"].cpu().numpy()[rows], ref["logits"], ref["idx"], ref["wts"],
                  logit_tol=2e-3)
    ok = stable_rows(s, ref["logits"], gpu_logits=gl)
    assert O.max_rel_err(tr["routed"].cpu().numpy()[rows][ok], ref["routed"][ok]) < TOL_INT4
    assert O.max_rel_err(hid.cpu().numpy()[rows][ok], ref["hidden"][ok]) < TOL_BF16
    assert blk.error_word() == 0


def test_config4_zipf_full_geometry_against_oracle(orc):
    """BASELINE config 4 exactly as benchmarked: H=2048, E=256, top-8, I=Is=512, INT4 G=64, 4096 tokens, router
    logits plus the Zipf(1.1) per-expert bias, so one expert takes nearly every token. The expert sort (offsets and
    permutation) is checked whole and bit for bit; every token's outputs are compared with the oracle's tile
    numerics, all the pairs of the hottest expert included."""
    m = mb()
    ms = m.MoeShape()
    T = PREFILL_T
    base = m.synth_layer(ms, seed=2000)
    bias = m.zipf_bias(ms.E, seed=0)
    t = dict(base.t)
    t["router_bias"] = torch.from_numpy(bias).cuda()
    layer = m.MoeLayer(ms, t)
    hid, att = m.synth_activations(ms, T, 17)
    torch.cuda.synchronize()
    hidden = hid.cpu().numpy()
    attn = att.cpu().numpy().view(np.uint16)
    blk = m.MoeBlock(layer, T)
    normed = torch.zeros(T, ms.H, dtype=torch.int16, device="cuda")
    blk.forward(hid, att, normed)
    torch.cuda.synchronize()
    tr = blk.trace(T)
    gidx = tr["idx"].cpu().numpy()
    off, srt = orc.sort(gidx, ms.E)
    assert np.array_equal(tr["offsets"].cpu().numpy(), off)
    assert np.array_equal(tr["sorted"].cpu().numpy(), srt)
    load = np.bincount(gidx.ravel(), minlength=ms.E)
    hot = int(load.argmax())
    assert load[hot] > T // 2  # the skew the benchmark measures
    s = O.Shape()
    L = {n: (v.cpu().numpy() if v.dtype == torch.uint8 else v.cpu().numpy().view(np.uint16))
         for n, v in base.t.items()}
    L["router_bias"] = bias
    del base, t
    ref = orc.block_forward(s, L, hidden, attn, mode=1)
    gl = tr["logits"].cpu().numpy()
    check_routing(orc, s, gl, gidx, tr["wts"].cpu().numpy(), ref["logits"], ref["idx"], ref["wts"], logit_tol=2e-3)
    ok = stable_rows(s, ref["logits"], gpu_logits=gl)
    on_hot = (gidx == hot).any(axis=1)
    assert (ok & on_hot).sum() >= 0.9 * on_hot.sum()
    assert O.max_rel_err(tr["routed"].cpu().numpy()[ok], ref["routed"][ok]) < TOL_INT4
    assert O.max_rel_err(tr["routed"].cpu().numpy()[ok & on_hot], ref["routed"][ok & on_hot]) < TOL_INT4
    assert O.max_rel_err(O.bf16_to_f32(host16(tr["sout"])), O.bf16_to_f32(ref["sout"])) < TOL_BF16
    assert O.max_rel_err(hid.cpu().numpy()[ok], ref["hidden"][ok]) < TOL_BF16
    assert O.max_rel_err(O.bf16_to_f32(host16(normed)[ok]), O.bf16_to_f32(ref["normed"][ok])) < TOL_BF16
    assert blk.error_word() == 0
