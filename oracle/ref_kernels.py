"""ref_kernels.py -- runs the reference's own CUDA kernels (examples/qwen/kernels.cuh, built into
oracle/_ref/libqk_ref.so by `make -C oracle ref REF=<reference checkout>`) on numpy inputs.

TEST INFRASTRUCTURE, NOT PRODUCT CODE: used by the GPU pinning tests and by tests/golden/make_golden.py to
produce golden vectors from the reference itself. torch provides the device buffers. The reference's limits
apply: group size 128 only (kernels.cuh:842, 1020), H % 1024 == 0 (kernels.cuh:825), I % 512 == 0
(kernels.cuh:863); activation buffers read by its tensor-core GEMMs are padded to round_up(T, 128) rows
(qwen.cu:259).
"""
import ctypes
import os

import numpy as np
import torch

from . import oracle as O

_lib = None


def available():
    return os.path.exists(O.REF_LIB_PATH)


def lib():
    global _lib
    if _lib is None:
        if not available():
            raise FileNotFoundError(f"{O.REF_LIB_PATH} missing: build it with "
                                    "`make -C oracle ref REF=<reference checkout>`")
        _lib = ctypes.CDLL(O.REF_LIB_PATH)
    return _lib


class _Layer(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("rms2", "router", "exp_gu_q", "exp_gu_s", "exp_dn_q", "exp_dn_s",
                                               "shared_gate_up", "shared_down", "shared_gate")] + \
               [(n, ctypes.c_int32) for n in ("H", "E", "TOPK", "I", "Is")] + [("eps", ctypes.c_float)]


class _Work(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("logits_r", "topk_i", "topk_w", "inter", "routed", "moe_off",
                                               "moe_sorted", "slot_out", "sgu", "sinter", "sout")]


def _dev(a):
    a = np.ascontiguousarray(a)
    return torch.from_numpy(a if a.dtype == np.uint8 else a.view(np.int16)).cuda()


def _vp(t):
    return ctypes.c_void_p(t.data_ptr())


def block_forward(shape, layer, hidden, attn_out, next_rms1=None):
    """The reference's MoE block (qwen.cu:429-448) on the GPU. Returns numpy outputs and intermediates."""
    s = shape
    if s.G != 128:
        raise ValueError("the reference kernels hard-code group size 128")
    T = hidden.shape[0]
    Tp = (T + 127) // 128 * 128
    d = {n: _dev(layer[n]) for n in layer}
    L = _Layer(*[_vp(d[n]) for n, _ in _Layer._fields_[:9]], s.H, s.E, s.TOPK, s.I, s.Is, s.eps)
    f32, i16, i32 = torch.float32, torch.int16, torch.int32
    z = dict(device="cuda")
    buf = {
        "logits_r": torch.zeros(Tp, s.E, dtype=f32, **z), "topk_i": torch.zeros(Tp, s.TOPK, dtype=i32, **z),
        "topk_w": torch.zeros(Tp, s.TOPK, dtype=f32, **z), "inter": torch.zeros(Tp, s.TOPK, s.I, dtype=i16, **z),
        "routed": torch.zeros(Tp, s.H, dtype=f32, **z), "moe_off": torch.zeros(s.E + 1, dtype=i32, **z),
        "moe_sorted": torch.zeros(Tp * s.TOPK, dtype=i32, **z),
        "slot_out": torch.zeros(Tp * s.TOPK, s.H, dtype=f32, **z), "sgu": torch.zeros(Tp, 2 * s.Is, dtype=i16, **z),
        "sinter": torch.zeros(Tp, s.Is, dtype=i16, **z), "sout": torch.zeros(Tp, s.H, dtype=i16, **z),
    }
    W = _Work(*[_vp(buf[n]) for n, _ in _Work._fields_])
    h = torch.zeros(Tp, s.H, dtype=f32, **z)
    h[:T] = torch.from_numpy(np.ascontiguousarray(hidden, np.float32))
    a = torch.zeros(Tp, s.H, dtype=i16, **z)
    a[:T] = torch.from_numpy(np.ascontiguousarray(attn_out).view(np.int16))
    normed = torch.zeros(Tp, s.H, dtype=i16, **z)
    nr = None if next_rms1 is None else _dev(next_rms1)
    lb = lib()
    lb.qkref_block_forward.restype = ctypes.c_int
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lb.qkref_block_forward(ctypes.byref(L), ctypes.byref(W), _vp(h), _vp(a), _vp(normed),
                                None if nr is None else _vp(nr), ctypes.c_int(T), stream)
    torch.cuda.synchronize()
    if rc != 0:
        raise RuntimeError(f"reference block failed: cudaError {rc}")

    def np_(t, dt):
        return t[:T].cpu().numpy().view(dt)

    return {
        "hidden": np_(h, np.float32), "normed": np_(normed, np.uint16),
        "logits": np_(buf["logits_r"], np.float32), "idx": np_(buf["topk_i"], np.int32),
        "wts": np_(buf["topk_w"], np.float32), "inter": np_(buf["inter"], np.uint16),
        "routed": np_(buf["routed"], np.float32), "sinter": np_(buf["sinter"], np.uint16),
        "sout": np_(buf["sout"], np.uint16),
    }
