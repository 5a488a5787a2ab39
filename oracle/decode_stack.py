"""CPU oracle (TEST INFRASTRUCTURE, not the product) for the non-MoE pieces of one decode step of examples/qwen's
attention layers and the LM head: the parity checker for a decode-stack implementation.

Each function restates one reference kernel or host step, with its rounding points, in float64 numpy followed by the
reference's rounding to bf16 where it stores bf16; the reference's fast-math intrinsics (__expf, __powf, __sincosf,
rsqrtf) and its split-K summation order are therefore matched within tolerance, not bit for bit:
  * rmsnorm            kernels.cuh:83-93        y = bf16(x * rsqrt(mean(x^2) + eps) * w)
  * dense              qwen.cu:297-319          y = x . W^T, fp32 accumulate, stored as the output type (bf16 here)
  * qk_norm_rope       kernels.cuh:608-663      per-head RMSNorm (weights with 1 + w folded in), rotate-half RoPE
                                                over the first rope_dim dims at position pos0 + t, bf16; K and V rows
                                                into the caches at that position
  * attention          kernels.cuh:665-761,     causal softmax(q . k / sqrt(D)) . v over keys [0, pos0 + t], GQA:
                       qwen.cu:52-64            query head h reads kv head h // (Hq / Hkv); bf16 output
  * sigmoid_gate       kernels.cuh:765-769      o = bf16(o * sigmoid(g))
  * attention_layer    qwen.cu:413-425          the attention branch of forward() up to attn_out
  * lm_head_argmax     qwen.cu:451-456,         final RMSNorm of the last token, logits = x . W^T (fp32), argmax
                       kernels.cuh:1124-1164    with ties to the lowest index (NaN never wins; all-NaN gives 0)

Pinning: the reference's tests hold no golden vectors for these kernels and its CPU loops for attention
(tests/kernels/qwen_attention.cu) live inside a GPU test program, so the pin comes from the reference's own kernels:
tests/golden/make_golden_stack.py ran its attention branch and LM head (examples/qwen/kernels.cuh built by
oracle/Makefile's `ref` target, launched in qwen.cu's order by oracle/ref/qk_ref_shim.cu) on seeded inputs on a B200,
and tests/test_golden_stack.py checks this module against those outputs (tests/test_stack_ref_pin_gpu.py repeats the
comparison live).
"""
import numpy as np


def bf16_bits(x):
    """float -> bf16 bit patterns (uint16), round to nearest even (the reference's f2bf)."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, np.float32))
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, np.uint16(0x7FC0), r)


def bf16_f(bits):
    """bf16 bit patterns -> float64 values."""
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def round_bf16(x):
    return bf16_f(bf16_bits(x))


def rmsnorm(x, w_bits, eps):
    """kernels.cuh:83-93: x fp32 [T, H] (float64 here), w bf16 bits [H] -> bf16 bits [T, H]."""
    x = np.asarray(x, np.float64)
    inv = 1.0 / np.sqrt((x * x).mean(axis=-1, keepdims=True) + eps)
    return bf16_bits(x * inv * bf16_f(w_bits))


def dense(x_bits, w_bits):
    """qwen.cu:297-319 with a bf16 output: bf16 x [T, K] . bf16 W [N, K]^T accumulated exactly, rounded to bf16."""
    return bf16_bits(bf16_f(x_bits) @ bf16_f(w_bits).T)


def rope_angles(pos, rope_dim, theta):
    """Angles of dims d < rope_dim / 2 at position pos: pos * theta^(-2d / rope_dim) (kernels.cuh:644-651)."""
    d = np.arange(rope_dim // 2, dtype=np.float64)
    return pos * theta ** (-2.0 * d / rope_dim)


def qk_norm_rope(qkv_bits, q_norm, k_norm, Hq, Hkv, D, rope_dim, theta, pos0, eps, kc, vc):
    """kernels.cuh:608-663. qkv bf16 bits [T, (Hq + 2 Hkv) D] (q heads, then k heads, then v heads). Returns q bf16
    bits [T, Hq, D]; writes k (normed + rotated) and v (copied) into the bf16 caches kc, vc [Hkv, ctx, D] at rows
    pos0 + t."""
    T = qkv_bits.shape[0]
    heads = bf16_f(qkv_bits).reshape(T, Hq + 2 * Hkv, D)
    half = rope_dim // 2
    q_out = np.zeros((T, Hq, D), np.uint16)
    for t in range(T):
        pos = pos0 + t
        ang = rope_angles(pos, rope_dim, theta)
        c, s = np.cos(ang), np.sin(ang)
        for hh in range(Hq + Hkv):
            v = heads[t, hh].copy()
            w = q_norm if hh < Hq else k_norm
            v = v / np.sqrt((v * v).mean() + eps) * bf16_f(w)
            a, b = v[:half].copy(), v[half:rope_dim].copy()
            v[:half] = a * c - b * s
            v[half:rope_dim] = b * c + a * s
            if hh < Hq:
                q_out[t, hh] = bf16_bits(v)
            else:
                kc[hh - Hq, pos] = bf16_bits(v)
        for j in range(Hkv):
            vc[j, pos] = bf16_bits(heads[t, Hq + Hkv + j])
    return q_out


def attention(q_bits, kc, vc, Hq, Hkv, pos0):
    """kernels.cuh:665-761 + qwen.cu:52-64: for token t and query head h, softmax over keys [0, pos0 + t] of
    q . k / sqrt(D), times v, from kv head h // (Hq / Hkv); bf16 bits [T, Hq, D]."""
    T, _, D = q_bits.shape
    G = Hq // Hkv
    q = bf16_f(q_bits)
    out = np.zeros((T, Hq, D), np.uint16)
    for t in range(T):
        n = pos0 + t + 1
        for h in range(Hq):
            k = bf16_f(kc[h // G, :n])
            v = bf16_f(vc[h // G, :n])
            sc = k @ q[t, h] / np.sqrt(D)
            p = np.exp(sc - sc.max())
            out[t, h] = bf16_bits((p @ v) / p.sum())
    return out


def sigmoid_gate(o_bits, g_bits):
    """kernels.cuh:765-769: o = bf16(o * sigmoid(g))."""
    g = bf16_f(g_bits)
    return bf16_bits(bf16_f(o_bits) / (1.0 + np.exp(-g)))


def attention_layer(normed_bits, layer, Hq, Hkv, D, rope_dim, theta, pos0, eps, kc, vc, attn_gate):
    """The attention branch of forward(), qwen.cu:413-425: qkv = dense(normed), optional gate = dense(normed),
    per-head norm + RoPE into the caches, attention, optional sigmoid gate, attn_out = dense(o). `layer` holds bf16
    bits: qkv [(Hq + 2 Hkv) D, H], gate [Hq D, H] (if attn_gate), o [H, Hq D], q_norm [D], k_norm [D]."""
    T = normed_bits.shape[0]
    qkv = dense(normed_bits, layer["qkv"])
    q = qk_norm_rope(qkv, layer["q_norm"], layer["k_norm"], Hq, Hkv, D, rope_dim, theta, pos0, eps, kc, vc)
    o = attention(q, kc, vc, Hq, Hkv, pos0).reshape(T, Hq * D)
    if attn_gate:
        o = sigmoid_gate(o, dense(normed_bits, layer["gate"]))
    return dense(o, layer["o"])


def argmax_lowest(logits):
    """kernels.cuh:1124-1164: index of the largest value, ties to the lowest index; NaN never wins; if nothing beats
    the -1e30 start value the result is 0."""
    x = np.asarray(logits, np.float32)
    best_v, best_i = np.float32(-1e30), 0
    ok = ~np.isnan(x)
    if ok.any():
        m = x[ok].max()
        if m > best_v:
            best_i = int(np.flatnonzero(ok & (x == m))[0])
    return best_i


def lm_head_argmax(hidden_last, final_norm_bits, lm_head_bits, eps):
    """qwen.cu:451-456: RMSNorm of the last token's fp32 residual, fp32 logits = x . W^T, argmax (lowest index on
    ties). Returns (logits float32 [V], index)."""
    x = rmsnorm(np.asarray(hidden_last, np.float64)[None, :], final_norm_bits, eps)[0]
    logits = (bf16_f(x) @ bf16_f(lm_head_bits).T).astype(np.float32)
    return logits, argmax_lowest(logits)
