"""CPU tests of oracle/decode_stack.py, the checker for the attention layers and LM head of a decode step: the
restated math against the reference's own algorithm structure (split-K online softmax, kernels.cuh:665-761, with the
split count of qwen.cu:61) and against cases with known answers."""
import numpy as np
import pytest

from oracle import decode_stack as S


def _bits(rng, *shape, scale=1.0):
    return S.bf16_bits(scale * rng.standard_normal(shape))


def split_k_attention(q, k, v, nsplit):
    """The reference's two kernels in float32: per split an online softmax over its keys (running max, rescaled sum
    and accumulator), then the merge of the splits' (acc, m, l) -- kernels.cuh:665-761."""
    n = k.shape[0]
    chunk = (n + nsplit - 1) // nsplit
    parts = []
    for sp in range(nsplit):
        m, l, acc = np.float32(-1e30), np.float32(0), np.zeros(q.shape[0], np.float32)
        for j in range(sp * chunk, min(n, sp * chunk + chunk)):
            sc = np.float32(np.dot(q, k[j]))
            m_new = max(m, sc)
            corr, p = np.float32(np.exp(m - m_new)), np.float32(np.exp(sc - m_new))
            l = l * corr + p
            acc = acc * corr + p * v[j]
            m = m_new
        parts.append((acc, m, l))
    gm = max(p[1] for p in parts)
    gl, out = np.float32(0), np.zeros_like(parts[0][0])
    for acc, m, l in parts:
        c = np.float32(np.exp(m - gm)) if l > 0 else np.float32(0)
        gl += l * c
        out += acc * c
    return out / gl


@pytest.mark.parametrize("n,nsplit", [(1, 1), (7, 1), (40, 2), (300, 10), (1000, 32)])
def test_attention_equals_split_k_online_softmax(n, nsplit):
    rng = np.random.default_rng(n)
    D, Hq, Hkv = 256, 4, 2
    kc = np.zeros((Hkv, n, D), np.uint16)
    vc = np.zeros((Hkv, n, D), np.uint16)
    kc[:] = _bits(rng, Hkv, n, D)
    vc[:] = _bits(rng, Hkv, n, D)
    q = _bits(rng, 1, Hq, D)
    out = S.attention(q, kc, vc, Hq, Hkv, pos0=n - 1)
    for h in range(Hq):
        qf = (S.bf16_f(q[0, h]) / np.sqrt(D)).astype(np.float32)
        ref = split_k_attention(qf, S.bf16_f(kc[h // 2]).astype(np.float32), S.bf16_f(vc[h // 2]).astype(np.float32),
                                nsplit)
        got = S.bf16_f(out[0, h])
        assert np.max(np.abs(got - ref)) <= np.max(np.abs(ref)) * 2 ** -7 + 1e-6


def test_attention_known_answers():
    rng = np.random.default_rng(1)
    D = 256
    kc = np.zeros((1, 8, D), np.uint16)
    vc = _bits(rng, 1, 8, D)
    q = _bits(rng, 2, 2, D)
    out = S.attention(q, kc, vc, Hq=2, Hkv=1, pos0=4)
    # token 0 sees keys 0..4, token 1 keys 0..5; all keys are zero, so the weights are uniform
    assert np.array_equal(out[0, 0], S.bf16_bits(S.bf16_f(vc[0, :5]).mean(axis=0)))
    assert np.array_equal(out[1, 1], S.bf16_bits(S.bf16_f(vc[0, :6]).mean(axis=0)))
    one = S.attention(q[:1], kc, vc, Hq=2, Hkv=1, pos0=0)  # a single key: softmax weight 1
    assert np.array_equal(one[0, 1], vc[0, 0])


def test_qk_norm_rope_and_cache_writes():
    rng = np.random.default_rng(2)
    Hq, Hkv, D, rope_dim, T, ctx, pos0 = 4, 2, 256, 64, 2, 16, 5
    qkv = _bits(rng, T, (Hq + 2 * Hkv) * D)
    ones = S.bf16_bits(np.ones(D))
    kc = np.zeros((Hkv, ctx, D), np.uint16)
    vc = np.zeros((Hkv, ctx, D), np.uint16)
    q = S.qk_norm_rope(qkv, ones, ones, Hq, Hkv, D, rope_dim, 1e7, pos0, 1e-6, kc, vc)
    heads = S.bf16_f(qkv).reshape(T, Hq + 2 * Hkv, D)
    for t in range(T):
        pos = pos0 + t
        for j in range(Hkv):
            assert np.array_equal(vc[j, pos], S.bf16_bits(heads[t, Hq + Hkv + j]))  # v rows copied
        for h in range(Hq):
            x = heads[t, h] / np.sqrt((heads[t, h] ** 2).mean() + 1e-6)
            got = S.bf16_f(q[t, h])
            # dims past rope_dim are only normalised; each rotated pair keeps its length
            assert np.allclose(got[rope_dim:], x[rope_dim:], rtol=2 ** -7, atol=1e-6)
            half = rope_dim // 2
            r_got = got[:half] ** 2 + got[half:rope_dim] ** 2
            r_x = x[:half] ** 2 + x[half:rope_dim] ** 2
            assert np.allclose(r_got, r_x, rtol=2 ** -6, atol=1e-5)
    assert not kc[:, :pos0].any() and kc[:, pos0:pos0 + T].any()
    # position 0 rotates nothing
    kc0 = np.zeros_like(kc)
    q0 = S.qk_norm_rope(qkv[:1], ones, ones, Hq, Hkv, D, rope_dim, 1e7, 0, 1e-6, kc0, np.zeros_like(vc))
    x0 = heads[0, 0] / np.sqrt((heads[0, 0] ** 2).mean() + 1e-6)
    assert np.array_equal(q0[0, 0], S.bf16_bits(x0))


def test_attention_layer_with_gate_shapes_and_rounding():
    rng = np.random.default_rng(3)
    H, Hq, Hkv, D, T = 128, 2, 1, 256, 3
    layer = {"qkv": _bits(rng, (Hq + 2 * Hkv) * D, H, scale=0.05), "gate": _bits(rng, Hq * D, H, scale=0.05),
             "o": _bits(rng, H, Hq * D, scale=0.05), "q_norm": S.bf16_bits(np.ones(D)),
             "k_norm": S.bf16_bits(np.ones(D))}
    normed = _bits(rng, T, H)
    kc = np.zeros((Hkv, 8, D), np.uint16)
    vc = np.zeros((Hkv, 8, D), np.uint16)
    out = S.attention_layer(normed, layer, Hq, Hkv, D, 64, 1e7, 0, 1e-6, kc, vc, attn_gate=True)
    assert out.shape == (T, H) and out.dtype == np.uint16
    assert kc[:, :T].any() and not kc[:, T:].any()
    no_gate = S.attention_layer(normed, layer, Hq, Hkv, D, 64, 1e7, 0, 1e-6, np.zeros_like(kc), np.zeros_like(vc),
                                attn_gate=False)
    assert not np.array_equal(out, no_gate)


def test_argmax_ties_nan_and_floor():
    assert S.argmax_lowest(np.array([1.0, 3.0, 3.0, 2.0], np.float32)) == 1
    assert S.argmax_lowest(np.array([np.nan, 0.5, 0.5], np.float32)) == 1
    assert S.argmax_lowest(np.array([np.nan, np.nan], np.float32)) == 0
    assert S.argmax_lowest(np.array([-np.inf, -np.inf], np.float32)) == 0  # nothing beats the -1e30 start


def test_lm_head_argmax():
    rng = np.random.default_rng(4)
    H, V = 64, 1000
    W = _bits(rng, V, H)
    h = rng.standard_normal(H)
    norm = S.bf16_bits(np.ones(H))
    logits, idx = S.lm_head_argmax(h, norm, W, 1e-6)
    x = S.bf16_f(S.rmsnorm(h[None], norm, 1e-6)[0])
    assert np.allclose(logits, x @ S.bf16_f(W).T, rtol=1e-6, atol=1e-6)
    assert idx == int(np.argmax(logits))
    W2 = W.copy()
    W2[idx + 1 if idx + 1 < V else idx - 1] = W[idx]  # a duplicate row ties: the lower index wins
    _, idx2 = S.lm_head_argmax(h, norm, W2, 1e-6)
    assert idx2 == min(idx, idx + 1 if idx + 1 < V else idx - 1)
