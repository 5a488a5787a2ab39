"""GPU parity tests of the decode-stack pieces (include/moe_stack.h) through the C ABI against the CPU oracle
oracle/decode_stack.py on the same inputs: the attention layer (qkv, per-head norm + RoPE, cache append, split-K
attention, optional sigmoid gate, o), the LM head with fused argmax (ties to the lowest index, NaN never wins), and a
two-layer decode step end to end. Bars: bf16 outputs within max relative error 1e-2, the new V rows in the caches
bit for bit, logits within 1e-3 of the largest, argmax exact wherever the top-2 margin exceeds the logit error."""
import numpy as np
import pytest
import torch

from oracle import decode_stack as S
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL_BF16 = 1e-2


def host(t):
    return t.cpu().numpy().view(np.uint16) if t.dtype == torch.int16 else t.cpu().numpy()


def attn_host(layer):
    return {n: host(v) for n, v in layer.t.items() if v is not None}


def rel(a, b):
    return O.max_rel_err(S.bf16_f(a), S.bf16_f(b))


@pytest.mark.parametrize("gate", [False, True])
@pytest.mark.parametrize("ctx,pos0,T", [(1024, 0, 1), (1024, 700, 1), (1024, 517, 3), (4096, 4095, 1)])
def test_attention_layer_against_oracle(gate, ctx, pos0, T):
    from mvcc_b200 import stack as st
    a = st.AttnShape(gate=gate)
    layer = st.synth_attn_layer(a, seed=11 + ctx + pos0)
    gen = torch.Generator(device="cuda").manual_seed(5)
    kc = (torch.randn(a.Hkv, ctx, a.D, generator=gen, device="cuda")).to(torch.bfloat16).view(torch.int16)
    vc = (torch.randn(a.Hkv, ctx, a.D, generator=gen, device="cuda")).to(torch.bfloat16).view(torch.int16)
    blk = st.AttnBlock(layer, ctx, max_T=T, caches=(kc, vc))
    normed = torch.from_numpy(S.bf16_bits(np.random.default_rng(7).standard_normal((T, a.H))).view(np.int16)).cuda()
    kc0, vc0 = host(kc).copy(), host(vc).copy()
    out = torch.zeros(T, a.H, dtype=torch.int16, device="cuda")
    blk.forward(normed, out, pos0)
    torch.cuda.synchronize()
    L = attn_host(layer)
    kr, vr = kc0.copy(), vc0.copy()
    ref = S.attention_layer(host(normed), L, a.Hq, a.Hkv, a.D, a.rope_dim, a.theta, pos0, a.eps, kr, vr, gate)
    assert rel(host(out), ref) < TOL_BF16
    kg, vg = host(kc), host(vc)
    new = slice(pos0, pos0 + T)
    assert np.array_equal(vg[:, new], vr[:, new])  # v rows are copied
    assert rel(kg[:, new], kr[:, new]) < TOL_BF16  # k rows: normed + rotated
    keep = np.ones(ctx, bool)
    keep[new] = False
    assert np.array_equal(kg[:, keep], kc0[:, keep]) and np.array_equal(vg[:, keep], vc0[:, keep])
    assert blk.error_word() == 0


def test_attention_rejects_bad_shapes():
    import mvcc_b200 as m
    from mvcc_b200 import stack as st
    layer = st.synth_attn_layer(st.AttnShape(), seed=3)
    blk = st.AttnBlock(layer, 64, max_T=1)
    x = torch.zeros(1, 2048, dtype=torch.int16, device="cuda")
    with pytest.raises(m.MoeError):
        blk.forward(x, x.clone(), 64)  # pos0 + T > ctx
    with pytest.raises(m.MoeError):
        blk.forward(torch.zeros(5, 2048, dtype=torch.int16, device="cuda"), x, 0, T=5)  # T > 4


@pytest.mark.parametrize("V", [4096, 151936])
def test_lm_head_logits_and_argmax(V):
    from mvcc_b200 import stack as st
    H = 2048
    gen = torch.Generator(device="cuda").manual_seed(V)
    w = (0.02 * torch.randn(V, H, generator=gen, device="cuda")).to(torch.bfloat16).view(torch.int16)
    x = torch.from_numpy(S.bf16_bits(np.random.default_rng(9).standard_normal(H)).view(np.int16)).cuda()
    head = st.LmHead(w)
    nxt = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    logits = torch.zeros(V, device="cuda")
    for _ in range(2):  # the ticket returns to zero: a second call is as good as the first
        head.argmax(x, nxt, logits=logits)
        torch.cuda.synchronize()
        ref = (S.bf16_f(host(w)).astype(np.float32) @ S.bf16_f(host(x)).astype(np.float32)).astype(np.float32)
        gl = logits.cpu().numpy()
        err = np.abs(gl - ref).max()
        assert err < 1e-3 * np.abs(ref).max()
        top2 = np.sort(ref)[-2:]
        if top2[1] - top2[0] > 2 * err:
            assert int(nxt.item()) == int(np.argmax(ref))
        assert int(nxt.item()) == S.argmax_lowest(gl)


def _best_ms(fn, reps=5):
    """Best of `reps` CUDA-event timings of fn() on the current stream, after one warm-up call."""
    fn()
    best = float("inf")
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    return best


def test_lm_head_streams_at_the_copy_bandwidth():
    """A bandwidth gate in the manner of the reference's attention test (tests/kernels/qwen_attention.cu:70-108,
    at least 70 % of the device-to-device copy's GB/s): the 2048 x 151936 LM head GEMV with its argmax reads its
    622 MB of weights at no less than half the rate a plain device copy of the same bytes moves them (read + write),
    timed in the same process. The weights exceed the 126 MB L2, so neither side is served from cache."""
    from mvcc_b200 import stack as st
    V, H = 151936, 2048
    w = torch.zeros(V, H, dtype=torch.int16, device="cuda")
    x = torch.zeros(H, dtype=torch.int16, device="cuda")
    head = st.LmHead(w)
    nxt = torch.zeros(1, dtype=torch.int32, device="cuda")
    gemv_ms = _best_ms(lambda: head.argmax(x, nxt))
    dst = torch.empty_like(w)
    copy_ms = _best_ms(lambda: dst.copy_(w))
    nbytes = w.numel() * 2
    gemv_gbs, copy_gbs = nbytes / gemv_ms / 1e6, 2 * nbytes / copy_ms / 1e6
    assert gemv_gbs >= 0.5 * copy_gbs, (gemv_gbs, copy_gbs)


def test_lm_head_ties_go_to_the_lowest_index_and_nan_never_wins():
    from mvcc_b200 import stack as st
    V, H = 8192, 256
    rng = np.random.default_rng(3)
    wf = 0.02 * rng.standard_normal((V, H))
    x = np.abs(rng.standard_normal(H))
    wf[5000] = 0.05  # the largest logit, shared by rows 5000 and 7000 (identical rows)
    wf[7000] = 0.05
    wb = S.bf16_bits(wf)
    wb[100] = 0x7FC0  # a NaN row: its logit is NaN and must not win
    w = torch.from_numpy(wb.view(np.int16)).cuda()
    xb = torch.from_numpy(S.bf16_bits(x).view(np.int16)).cuda()
    head = st.LmHead(w)
    nxt = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    logits = torch.zeros(V, device="cuda")
    head.argmax(xb, nxt, logits=logits)
    torch.cuda.synchronize()
    assert np.isnan(logits[100].item())
    assert int(nxt.item()) == 5000
    # all NaN: nothing beats the start value, the result is 0 (argmax_partial_kernel's initial index)
    wn = torch.full((64, H), 0x7FC0, dtype=torch.int16, device="cuda")
    st.LmHead(wn).argmax(xb, nxt)
    torch.cuda.synchronize()
    assert int(nxt.item()) == 0


def _stack_host(stk, moe_host):
    return {"attn": [attn_host(b.layer) for b in stk.attn], "kc": [host(b.kc).copy() for b in stk.attn],
            "vc": [host(b.vc).copy() for b in stk.attn], "rms1": [host(r) for r in stk.rms1],
            "final": host(stk.final_norm), "head": host(stk.head.w), "moe": moe_host}


@pytest.mark.parametrize("T", [1, 3])
def test_attention_with_fused_input_norm_matches_the_separate_norm(T):
    """moe_attn_forward_rms (the input RMSNorm computed by every CTA of the qkv GEMV) against moe_rmsnorm followed by
    moe_attn_forward, on the same caches: the normed rows agree to the last bit except where the two sum-of-squares
    orders round rsqrt differently, so the outputs agree within the bf16 bar and the cache rows written are equal."""
    from mvcc_b200 import stack as st
    a = st.AttnShape()
    layer = st.synth_attn_layer(a, seed=77)
    gen = torch.Generator(device="cuda").manual_seed(9)
    kc = (torch.randn(a.Hkv, 1024, a.D, generator=gen, device="cuda")).to(torch.bfloat16).view(torch.int16)
    vc = (torch.randn(a.Hkv, 1024, a.D, generator=gen, device="cuda")).to(torch.bfloat16).view(torch.int16)
    rms1 = (1.0 + 0.1 * torch.randn(a.H, generator=gen, device="cuda")).to(torch.bfloat16).view(torch.int16)
    hidden = 3.0 * torch.randn(T, a.H, generator=gen, device="cuda")
    b1 = st.AttnBlock(layer, 1024, max_T=T, caches=(kc.clone(), vc.clone()))
    b2 = st.AttnBlock(layer, 1024, max_T=T, caches=(kc.clone(), vc.clone()))
    normed = torch.zeros(T, a.H, dtype=torch.int16, device="cuda")
    o1 = torch.zeros(T, a.H, dtype=torch.int16, device="cuda")
    o2 = torch.zeros(T, a.H, dtype=torch.int16, device="cuda")
    st.rmsnorm(hidden, rms1, normed, a.eps)
    b1.forward(normed, o1, 600, T=T)
    b2.forward_rms(hidden, rms1, o2, 600, T=T)
    torch.cuda.synchronize()
    assert rel(host(o2), host(o1)) < TOL_BF16
    new = slice(600, 600 + T)
    assert np.array_equal(host(b2.vc)[:, new], host(b1.vc)[:, new])
    assert rel(host(b2.kc)[:, new], host(b1.kc)[:, new]) < TOL_BF16


def test_two_layer_decode_step_against_oracle(orc):
    """(attention with its input RMSNorm fused into the qkv GEMV, MoE block) x 2, the last block applying the final
    norm -> LM head argmax, against the oracle's composition of the same steps (rmsnorm, attention, the block with the
    next layer's norm; decode numerics for the T = 1 MoE block)."""
    import mvcc_b200 as m
    from mvcc_b200 import stack as st
    ms = O.Shape(H=2048, E=32, TOPK=8, I=512, Is=512, G=64)
    moe_host = [O.make_layer(ms, 40 + i) for i in range(2)]
    layers = []
    for L in moe_host:
        t = {n: torch.from_numpy(a if a.dtype == np.uint8 else a.view(np.int16)).cuda() for n, a in L.items()}
        layers.append(m.MoeLayer(m.MoeShape(H=ms.H, E=ms.E, TOPK=ms.TOPK, I=ms.I, Is=ms.Is, G=ms.G), t))
    ctx, pos0, V = 256, 255, 4096
    stk = st.DecodeStack(L=2, ctx=ctx, vocab=V, moe=m.MoeShape(H=ms.H, E=ms.E, TOPK=ms.TOPK, I=ms.I, Is=ms.Is, G=ms.G),
                         seed=2, moe_layers=layers)
    hs = _stack_host(stk, moe_host)
    hidden0, _ = O.make_activations(ms, 1, 8)
    hidden = torch.from_numpy(hidden0.copy()).cuda()
    logits = torch.zeros(V, device="cuda")
    stk.step(hidden, pos0, logits=logits)
    torch.cuda.synchronize()
    # oracle
    a = stk.attn_shape
    h = hidden0.astype(np.float32).copy()
    normed = S.rmsnorm(h, hs["rms1"][0], a.eps)
    margins = []
    for i in range(2):
        attn_out = S.attention_layer(normed, hs["attn"][i], a.Hq, a.Hkv, a.D, a.rope_dim, a.theta, pos0, a.eps,
                                     hs["kc"][i], hs["vc"][i], a.gate)
        nxt = hs["rms1"][i + 1] if i + 1 < 2 else hs["final"]
        r = orc.block_forward(ms, moe_host[i], h, attn_out, next_rms1=nxt, mode=0)
        srt = np.sort(r["logits"], axis=1)[:, ::-1]
        margins.append(float(srt[0, ms.TOPK - 1] - srt[0, ms.TOPK]))
        h, normed = r["hidden"], r["normed"]
    assert min(margins) > 1e-3, margins  # the seed keeps routing away from near ties
    assert O.max_rel_err(hidden.cpu().numpy(), h) < TOL_BF16
    assert rel(host(stk.normed[:1]), normed) < TOL_BF16
    ref_logits = (S.bf16_f(hs["head"]).astype(np.float32) @ S.bf16_f(normed[0]).astype(np.float32))
    gl = logits.cpu().numpy()
    err = np.abs(gl - ref_logits).max()
    assert err < 2e-2 * np.abs(ref_logits).max()
    top2 = np.sort(ref_logits)[-2:]
    if top2[1] - top2[0] > 2 * err:
        assert int(stk.next.item()) == int(np.argmax(ref_logits))
    assert int(stk.next.item()) == S.argmax_lowest(gl)
