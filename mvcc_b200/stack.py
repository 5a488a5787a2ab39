"""Decode stack around the MoE block: the attention layers, the first layer's input norm and the LM head of a
Qwen3.5-MoE decode step (include/moe_stack.h), and a whole step over L layers.

The reference's decode step is forward() at examples/qwen/qwen.cu:372-457: per layer the attention branch
(qwen.cu:413-425), then the MoE block (qwen.cu:429-448, include/moe_block.h) whose combine applies the next layer's
input RMSNorm, and after the last layer the final RMSNorm and the LM head with argmax (qwen.cu:451-456). Here each
piece is one or a few launches of libmoe_b200.so; `DecodeStack.step` issues the whole sequence on one stream, so a
caller can capture it in one CUDA graph per token (the reference's tests capture its step the same way,
tests/kernels/qwen_attention.cu:148-175). torch is used for device memory and streams only.
"""
import ctypes
import dataclasses

import torch

from . import (MoeAttnWeights, MoeBlock, MoeLayer, MoeShape, _check, _lib, _ptr, _stream, synth_activations,
               synth_layer)


@dataclasses.dataclass
class AttnShape:
    """Geometry of one attention layer (the pack config's q_heads, kv_heads, head_dim, rope_dim, rope_theta,
    attn_gate; convert.py:317-334). Defaults: BASELINE config 3 (H 2048, 16 q heads, 2 kv heads, head_dim 256)."""

    H: int = 2048
    Hq: int = 16
    Hkv: int = 2
    D: int = 256
    rope_dim: int = 64
    theta: float = 1.0e7
    eps: float = 1e-6
    gate: bool = False

    def weight_bytes(self):
        nq = self.Hq * self.D
        return 2 * self.H * ((self.Hq + 2 * self.Hkv) * self.D + nq + (nq if self.gate else 0))


class AttnLayer:
    """Device tensors of one attention layer in the pack layout (bf16 bits as int16): qkv [(Hq + 2 Hkv) D, H],
    gate [Hq D, H] (if shape.gate), o [H, Hq D], q_norm and k_norm [D]."""

    NAMES = ("qkv", "gate", "o", "q_norm", "k_norm")

    def __init__(self, shape: AttnShape, tensors: dict):
        s = shape
        self.shape = s
        self.t = dict(tensors)
        nq, nqkv = s.Hq * s.D, (s.Hq + 2 * s.Hkv) * s.D
        expect = {"qkv": (nqkv, s.H), "o": (s.H, nq), "q_norm": (s.D,), "k_norm": (s.D,)}
        if s.gate:
            expect["gate"] = (nq, s.H)
        for n, shp in expect.items():
            v = self.t[n]
            if tuple(v.shape) != shp or v.dtype != torch.int16 or not v.is_contiguous() or not v.is_cuda:
                raise ValueError(f"{n}: expected contiguous cuda int16 {shp}, got {v.dtype} {tuple(v.shape)}")
        self.c = MoeAttnWeights(*[ctypes.c_void_p(self.t[n].data_ptr()) if self.t.get(n) is not None else None
                                  for n in self.NAMES], s.H, s.Hq, s.Hkv, s.D, s.rope_dim, s.theta, s.eps)


class AttnBlock:
    """Workspace and caches for one attention layer: bf16 K and V caches [Hkv][ctx][D] and the caller-owned
    workspace of moe_attn_forward for up to max_T tokens."""

    def __init__(self, layer: AttnLayer, ctx: int, max_T: int = 1, caches=None):
        s = layer.shape
        self.layer, self.ctx, self.max_T = layer, ctx, max_T
        n = _lib.moe_attn_workspace_bytes(ctypes.byref(layer.c), max_T, ctx)
        if n == 0:
            raise ValueError("unsupported attention geometry")
        self.ws = torch.zeros(n, dtype=torch.uint8, device=layer.t["qkv"].device)
        if caches is None:
            caches = (torch.zeros(s.Hkv, ctx, s.D, dtype=torch.int16, device=self.ws.device),
                      torch.zeros(s.Hkv, ctx, s.D, dtype=torch.int16, device=self.ws.device))
        self.kc, self.vc = caches

    def forward(self, normed, attn_out, pos0, T=None, stream=None):
        """qwen.cu:413-425 for T tokens at positions pos0 .. pos0 + T - 1 (normed, attn_out bf16 bits [T,H])."""
        T = normed.shape[0] if T is None else T
        _check(_lib.moe_attn_forward(ctypes.byref(self.layer.c), _ptr(self.kc), _ptr(self.vc), self.ctx, pos0,
                                     _ptr(normed), _ptr(attn_out), T, _ptr(self.ws), self.ws.numel(),
                                     _stream(stream)), "moe_attn_forward")

    def error_word(self, stream=None):
        """Reads and clears the workspace's error word (MOE_ERR_TIMEOUT: a cache-copy wait gave up)."""
        rc = _lib.moe_attn_workspace_error(_ptr(self.ws), self.ws.numel(), _stream(stream))
        if rc < 0:
            raise RuntimeError(f"moe_attn_workspace_error failed: cudaError {-rc}")
        return rc

    def forward_rms(self, hidden, rms1, attn_out, pos0, T=None, stream=None):
        """forward() with the layer's input RMSNorm fused in: hidden fp32 [T,H] normalised with rms1 (bf16 bits [H])
        inside the first GEMV (moe_attn_forward_rms)."""
        T = hidden.shape[0] if T is None else T
        _check(_lib.moe_attn_forward_rms(ctypes.byref(self.layer.c), _ptr(rms1), _ptr(hidden), _ptr(self.kc),
                                         _ptr(self.vc), self.ctx, pos0, _ptr(attn_out), T, _ptr(self.ws),
                                         self.ws.numel(), _stream(stream)), "moe_attn_forward_rms")


def rmsnorm(x, w, y, eps=1e-6, stream=None):
    """y = bf16(x * rsqrt(mean(x^2) + eps) * w) per row (rmsnorm_kernel, kernels.cuh:83-93)."""
    _check(_lib.moe_rmsnorm(_ptr(x), _ptr(w), _ptr(y), x.shape[0], x.shape[1], eps, _stream(stream)), "moe_rmsnorm")


class LmHead:
    """The LM head with fused argmax (moe_lm_head_argmax): weight bf16 bits [V,H] and its workspace."""

    def __init__(self, weight):
        self.w = weight
        self.V, self.H = weight.shape
        n = _lib.moe_lm_head_workspace_bytes(self.V, self.H)
        if n == 0:
            raise ValueError("unsupported LM head geometry")
        self.ws = torch.zeros(n, dtype=torch.uint8, device=weight.device)

    def argmax(self, normed, next_token, logits=None, stream=None):
        """next_token (int32 [1] device) = argmax of normed [H] . W^T; logits fp32 [V] written when given."""
        _check(_lib.moe_lm_head_argmax(_ptr(normed), _ptr(self.w), self.V, self.H, _ptr(logits), _ptr(next_token),
                                       _ptr(self.ws), self.ws.numel(), _stream(stream)), "moe_lm_head_argmax")


def _normal_bf16(shape, gen, std, mean=0.0, device="cuda"):
    return (mean + std * torch.randn(*shape, generator=gen, device=device)).to(torch.bfloat16).view(torch.int16)


def synth_attn_layer(shape: AttnShape, seed: int, device="cuda", std=0.02) -> AttnLayer:
    """Seeded attention layer on the device: bf16 N(0, std) projections, per-head norm weights 1 + N(0, 0.1)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    s = shape
    nq, nqkv = s.Hq * s.D, (s.Hq + 2 * s.Hkv) * s.D
    t = {"qkv": _normal_bf16((nqkv, s.H), gen, std, device=device), "o": _normal_bf16((s.H, nq), gen, std, device=device),
         "q_norm": _normal_bf16((s.D,), gen, 0.1, 1.0, device=device),
         "k_norm": _normal_bf16((s.D,), gen, 0.1, 1.0, device=device),
         "gate": _normal_bf16((nq, s.H), gen, std, device=device) if s.gate else None}
    return AttnLayer(s, t)


class DecodeStack:
    """L layers of (attention, MoE block), the first layer's input norm, the final norm and the LM head: one decode
    step of BASELINE config 3 per call of `step`. Weights, KV caches (bf16 N(0,1) at every position, as if ctx
    tokens had been decoded) and norm vectors are seeded synthetic tensors on the device."""

    def __init__(self, L=40, ctx=4096, vocab=151936, attn=None, moe=None, seed=0, device="cuda", max_T=1,
                 std=0.02, moe_layers=None):
        self.attn_shape = attn or AttnShape()
        self.moe_shape = moe or MoeShape()
        a, m = self.attn_shape, self.moe_shape
        if a.H != m.H:
            raise ValueError("attention and MoE layers must share H")
        self.L, self.ctx, self.V, self.max_T = L, ctx, vocab, max_T
        dev = torch.device(device)
        gen = torch.Generator(device=dev).manual_seed(seed)
        self.attn, self.moe, self.rms1 = [], [], []
        for i in range(L):
            layer = synth_attn_layer(a, seed * 1000 + 2 * i, device=dev, std=std)
            caches = (_normal_bf16((a.Hkv, ctx, a.D), gen, 1.0, device=dev),
                      _normal_bf16((a.Hkv, ctx, a.D), gen, 1.0, device=dev))
            self.attn.append(AttnBlock(layer, ctx, max_T, caches))
            ml = moe_layers[i] if moe_layers is not None else synth_layer(m, seed * 1000 + 2 * i + 1, device=dev,
                                                                          std=std)
            self.moe.append(MoeBlock(ml, max_T))
            self.rms1.append(_normal_bf16((a.H,), gen, 0.1, 1.0, device=dev))
        self.final_norm = _normal_bf16((a.H,), gen, 0.1, 1.0, device=dev)
        self.head = LmHead(_normal_bf16((vocab, a.H), gen, std, device=dev))
        self.normed = torch.zeros(max_T, a.H, dtype=torch.int16, device=dev)
        self.attn_out = torch.zeros(max_T, a.H, dtype=torch.int16, device=dev)
        self.next = torch.zeros(1, dtype=torch.int32, device=dev)

    def weight_bytes(self):
        """Bytes one batch-1 step must read at least: per layer the attention weights, the K and V caches up to the
        new position and the MoE block (router, the routed experts' weights and scales for top-k distinct
        experts, shared expert, norms); the LM head."""
        a, m = self.attn_shape, self.moe_shape
        kv = 2 * a.Hkv * self.ctx * a.D * 2
        moe = m.E * m.H * 2 + m.TOPK * m.expert_bytes() + 3 * m.Is * m.H * 2 + 2 * m.H * 2
        return self.L * (a.weight_bytes() + kv + moe) + self.V * a.H * 2

    def step(self, hidden, pos0, T=1, stream=None, logits=None):
        """One decode step for T tokens whose fp32 residual is `hidden` [T,H] (updated in place) at positions
        pos0 .. pos0 + T - 1; the next token of the last one lands in self.next."""
        # each layer's input norm runs inside its first GEMV (moe_attn_forward_rms); the last MoE block applies the
        # final norm for the LM head
        for i in range(self.L):
            self.attn[i].forward_rms(hidden[:T], self.rms1[i], self.attn_out[:T], pos0, T=T, stream=stream)
            nxt = self.final_norm if i + 1 == self.L else None
            self.moe[i].forward(hidden, self.attn_out[:T], self.normed[:T], next_rms1=nxt, T=T, stream=stream)
        self.head.argmax(self.normed[T - 1], self.next, logits=logits, stream=stream)


def main(argv=None):
    """`python -m mvcc_b200.stack [--steps N] [--layers L]`: N plain decode steps (no CUDA graph) of BASELINE config 3
    on cuda:0 -- seeded synthetic weights and a 4096-token cache, each step at position 4095 from the same residual --
    printing the next token of each. Used to capture the step's kernel launch list with a profiler."""
    import argparse
    ap = argparse.ArgumentParser(prog="python -m mvcc_b200.stack")
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--layers", type=int, default=40)
    args = ap.parse_args(argv)
    s = torch.cuda.Stream()
    stk = DecodeStack(L=args.layers, ctx=4096, vocab=151936, seed=5)
    h0, _ = synth_activations(stk.moe_shape, 1, seed=41, stream=s)
    h = h0.clone()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        for _ in range(args.steps):
            h.copy_(h0)
            stk.step(h, 4095, stream=s)
            s.synchronize()
            print("next token", int(stk.next.item()), flush=True)


if __name__ == "__main__":
    main()
