"""oracle.py -- ctypes front end of the CPU oracle (moe_oracle.c) and the seeded numpy input generator.

Inputs for CPU-checked tests come from numpy's PCG64 generator (make_layer / make_activations); full-size GPU
tests and the benchmark generate on the device instead (mvcc_b200.synth_layer) and copy to the host for checks.

TEST INFRASTRUCTURE, NOT PRODUCT CODE: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference legs use this module, as the checker. Arrays follow the reference's pack layout (convert.py:6-20):
bf16 / fp16 values are carried as uint16 bit patterns, INT4 rows as packed uint8 (low nibble = even k).
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmoe_oracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libqk_ref.so")


def build(ref=False):
    """Compile the oracle (and, with ref=True and the reference tree present, the reference shim)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if ref:
        subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)


# ------------------------------------------------------------------ numeric helpers (numpy)

def f32_to_bf16(a):
    """Round-to-nearest-even float32 -> bf16 bits (uint16), as __float2bfloat16."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
    nan = (u & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000)
    if nan.any():
        r[nan] = ((u[nan] >> np.uint32(16)) | np.uint32(0x40)).astype(np.uint16)
    return r


def bf16_to_f32(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f16_to_f32(h):
    return np.asarray(h, dtype=np.uint16).view(np.float16).astype(np.float32)


def normal(seed, sid, n):
    """n float32 samples of N(0,1) from numpy's PCG64 generator seeded with (seed, sid)."""
    return np.random.default_rng([int(seed), int(sid)]).standard_normal(int(n), dtype=np.float32)


def quantize_int4(w, G):
    """bf16-valued float32 weights [N, K] -> (packed uint8 [N, K/2], fp16-bits scales [N, K/G]).
    scale = fp16(absmax / 7) per group of G along K; q = clamp(rint(w / scale), -7, 7) + 8."""
    N, K = w.shape
    g = w.reshape(N, K // G, G).astype(np.float32)
    amax = np.abs(g).max(axis=2)
    s16 = (amax / np.float32(7.0)).astype(np.float32).astype(np.float16)
    s = s16.astype(np.float32)[:, :, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(s > 0, np.rint(g / np.where(s > 0, s, 1)), 0)
    q = (np.clip(q, -7, 7) + 8).astype(np.uint8).reshape(N, K)
    packed = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
    return packed, s16.view(np.uint16)


def dequant_int4(packed, scales_bits, G):
    """Inverse view for checks: float32 [N, K] = (q - 8) * scale."""
    lo = (packed & 0xF).astype(np.int32)
    hi = (packed >> 4).astype(np.int32)
    q = np.stack([lo, hi], axis=-1).reshape(packed.shape[0], -1) - 8
    s = np.repeat(f16_to_f32(scales_bits), G, axis=1)
    return q.astype(np.float32) * s


class Shape:
    def __init__(self, H=2048, E=256, TOPK=8, I=512, Is=512, G=64, eps=1e-6):
        self.H, self.E, self.TOPK, self.I, self.Is, self.G, self.eps = H, E, TOPK, I, Is, G, eps

    def as_tuple(self):
        return (self.H, self.E, self.TOPK, self.I, self.Is, self.G, self.eps)


def make_layer(shape, seed, std=0.02, exact=False):
    """Seeded layer in pack layout. exact=True draws exact-valued weights (small integers times powers of two,
    nibbles uniform, power-of-two scales) so that fp32 dot products are exact in any summation order, in the
    style of the reference's warp_tile exact case (tests/kernels/warp_tile.cu:59-61)."""
    s = shape
    rng = np.random.default_rng(seed)
    L = {}
    if exact:
        L["rms2"] = f32_to_bf16(np.ones(s.H, np.float32))
        L["router"] = f32_to_bf16(rng.integers(-8, 9, (s.E, s.H)).astype(np.float32) / 64.0)
        L["shared_gate_up"] = f32_to_bf16(rng.integers(-4, 5, (2 * s.Is, s.H)).astype(np.float32) / 256.0)
        L["shared_down"] = f32_to_bf16(rng.integers(-4, 5, (s.H, s.Is)).astype(np.float32) / 256.0)
        L["shared_gate"] = f32_to_bf16(rng.integers(-4, 5, (s.H,)).astype(np.float32) / 256.0)

        def qrows(n, k):
            q = rng.integers(0, 16, (n, k)).astype(np.uint8)
            packed = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
            sc = (2.0 ** -rng.integers(6, 9, (n, k // s.G))).astype(np.float16).view(np.uint16)
            return packed, sc
        gq, gs = qrows(s.E * 2 * s.I, s.H)
        dq, ds = qrows(s.E * s.H, s.I)
    else:
        orc = Oracle()

        def nb(sid, shp, mean=0.0, sd=std):
            return orc.to_bf16((mean + sd * normal(seed, sid, int(np.prod(shp)))).astype(np.float32)).reshape(shp)
        L["rms2"] = f32_to_bf16(np.ones(s.H, np.float32))
        L["router"] = nb(2, (s.E, s.H))
        L["shared_gate_up"] = nb(3, (2 * s.Is, s.H))
        L["shared_down"] = nb(4, (s.H, s.Is))
        L["shared_gate"] = nb(5, (s.H,))
        gq, gs = orc.quantize_int4(bf16_to_f32(nb(6, (s.E * 2 * s.I, s.H))), s.G)
        dq, ds = orc.quantize_int4(bf16_to_f32(nb(7, (s.E * s.H, s.I))), s.G)
    L["exp_gu_q"] = gq.reshape(s.E, 2 * s.I, s.H // 2)
    L["exp_gu_s"] = gs.reshape(s.E, 2 * s.I, s.H // s.G)
    L["exp_dn_q"] = dq.reshape(s.E, s.H, s.I // 2)
    L["exp_dn_s"] = ds.reshape(s.E, s.H, s.I // s.G)
    return {k: np.ascontiguousarray(v) for k, v in L.items()}


def gemv_i8(x_bits, q8, s8):
    """gemv_i8_kernel (kernels.cuh:215-274): y[t, n] = sum over 32-input chunks c of s8[n, c * 32 / group] times the
    chunk's dot of the raw int8 row values with x (bf16 bits); float64 here, so the kernel's fp32 summation order is
    matched within tolerance. q8 int8 [N, K], s8 fp16 [N, K / group]."""
    x = bf16_to_f32(np.asarray(x_bits, np.uint16)).astype(np.float64)
    q = np.asarray(q8, np.int8).astype(np.float64)
    sc = np.asarray(s8).view(np.float16).astype(np.float64)
    N, K = q.shape
    group = K // sc.shape[1]
    chunks = (x[:, None, :] * q[None, :, :]).reshape(x.shape[0], N, K // 32, 32).sum(axis=3)
    return (chunks * np.repeat(sc, group // 32, axis=1)[None, :, :]).sum(axis=2)


def shared_i8(shape, q8_gu, s8_gu, q8_dn, s8_dn, normed):
    """The shared expert on int8 weights with the reference's GEMV numerics (qwen.cu:436-438 with --dense int8): sgu
    = bf16(gemv_i8(normed)), sinter = bf16(silu(g) * u), sout = bf16(gemv_i8(sinter)). Returns (sinter, sout) bf16
    bits."""
    s = shape
    sgu = f32_to_bf16(gemv_i8(normed, q8_gu, s8_gu).astype(np.float32))
    g = bf16_to_f32(sgu[:, :s.Is]).astype(np.float64)
    u = bf16_to_f32(sgu[:, s.Is:]).astype(np.float64)
    sinter = f32_to_bf16((g / (1.0 + np.exp(-g)) * u).astype(np.float32))
    sout = f32_to_bf16(gemv_i8(sinter, q8_dn, s8_dn).astype(np.float32))
    return sinter, sout


def make_activations(shape, T, seed, exact=False):
    """hidden fp32 [T,H] and attn_out bf16 [T,H], seeded (N(0,1), or small exact values)."""
    if exact:
        rng = np.random.default_rng(seed + 1000)
        hidden = (rng.integers(-4, 5, (T, shape.H)) / 4.0).astype(np.float32)
        attn = f32_to_bf16((rng.integers(-4, 5, (T, shape.H)) / 4.0).astype(np.float32))
        return hidden, attn
    hidden = bf16_to_f32(f32_to_bf16(normal(seed, 101, T * shape.H).astype(np.float32))).reshape(T, shape.H).copy()
    attn = f32_to_bf16(normal(seed, 102, T * shape.H).astype(np.float32)).reshape(T, shape.H)
    return hidden, attn


def exact_normed(shape, T, seed):
    """Exact-valued bf16 activations for kernel-level KATs: multiples of 1/4 in [-2, 2]."""
    rng = np.random.default_rng(seed + 2000)
    return f32_to_bf16((rng.integers(-8, 9, (T, shape.H)) / 4.0).astype(np.float32))


# ------------------------------------------------------------------ ctypes binding of moe_oracle.c

class _Weights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("rms2", "router", "exp_gu_q", "exp_gu_s", "exp_dn_q", "exp_dn_s",
                                               "shared_gate_up", "shared_down", "shared_gate")] + \
               [(n, ctypes.c_int32) for n in ("H", "E", "TOPK", "I", "Is", "G")] + [("eps", ctypes.c_float),
                                                                              ("router_bias", ctypes.c_void_p)]


class _Trace(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("logits", "idx", "wts", "inter", "routed", "sgu", "sinter", "sout",
                                               "gate")]


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


class Oracle:
    def __init__(self):
        if not os.path.exists(LIB_PATH):
            build()
        self.lib = ctypes.CDLL(LIB_PATH)
        self.lib.orc_moe_block_forward.restype = ctypes.c_int
        self.lib.orc_f32_to_bf16.restype = ctypes.c_uint16
        self.lib.orc_f32_to_bf16.argtypes = [ctypes.c_float]
        self.lib.orc_bf16_to_f32.restype = ctypes.c_float
        self.lib.orc_bf16_to_f32.argtypes = [ctypes.c_uint16]
        self.lib.orc_f16_to_f32.restype = ctypes.c_float
        self.lib.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        self.lib.orc_max_threads.restype = ctypes.c_int
        self.lib.orc_set_threads.argtypes = [ctypes.c_int]

    def to_bf16(self, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(x.shape, np.uint16)
        self.lib.orc_f32_to_bf16_n(_p(x), _p(y), ctypes.c_int64(x.size))
        return y

    def quantize_int4(self, w, G):
        """C twin of quantize_int4(): (packed uint8 [N, K/2], fp16-bits scales [N, K/G])."""
        w = np.ascontiguousarray(w, np.float32)
        N, K = w.shape
        q = np.empty((N, K // 2), np.uint8)
        sc = np.empty((N, K // G), np.uint16)
        self.lib.orc_quantize_int4_rows(_p(w), ctypes.c_int64(N), K, G, _p(q), _p(sc))
        return q, sc

    def set_threads(self, n):
        self.lib.orc_set_threads(int(n))

    def max_threads(self):
        return self.lib.orc_max_threads()

    def block_forward(self, shape, layer, hidden, attn_out, next_rms1=None, mode=-1):
        """Runs the block on copies of hidden; returns dict with hidden, normed and the trace intermediates."""
        s = shape
        T = hidden.shape[0]
        keep = [np.ascontiguousarray(layer[n]) for n, _ in _Weights._fields_[:9]]
        bias = layer.get("router_bias")
        bias = None if bias is None else np.ascontiguousarray(bias, np.float32)
        w = _Weights(*[_p(a) for a in keep], s.H, s.E, s.TOPK, s.I, s.Is, s.G, s.eps, _p(bias))
        h = np.ascontiguousarray(hidden, dtype=np.float32).copy()
        a = np.ascontiguousarray(attn_out, dtype=np.uint16)
        normed = np.zeros((T, s.H), np.uint16)
        out = {
            "logits": np.zeros((T, s.E), np.float32), "idx": np.zeros((T, s.TOPK), np.int32),
            "wts": np.zeros((T, s.TOPK), np.float32), "inter": np.zeros((T, s.TOPK, s.I), np.uint16),
            "routed": np.zeros((T, s.H), np.float32), "sgu": np.zeros((T, 2 * s.Is), np.uint16),
            "sinter": np.zeros((T, s.Is), np.uint16), "sout": np.zeros((T, s.H), np.uint16),
            "gate": np.zeros((T,), np.float32),
        }
        tr = _Trace(*[_p(out[n]) for n, _ in _Trace._fields_])
        nr = None if next_rms1 is None else np.ascontiguousarray(next_rms1, dtype=np.uint16)
        rc = self.lib.orc_moe_block_forward(ctypes.byref(w), _p(h), _p(a), _p(normed), _p(nr), ctypes.c_int(T),
                                            ctypes.c_int(mode), ctypes.byref(tr))
        if rc != 0:
            raise ValueError("oracle rejected the shape")
        out["hidden"] = h
        out["normed"] = normed
        return out

    def router(self, shape, layer, normed):
        s = shape
        T = normed.shape[0]
        logits = np.zeros((T, s.E), np.float32)
        idx = np.zeros((T, s.TOPK), np.int32)
        wts = np.zeros((T, s.TOPK), np.float32)
        x = np.ascontiguousarray(normed, np.uint16)
        r = np.ascontiguousarray(layer["router"])
        self.lib.orc_dense_bf16_f32(_p(x), _p(r), _p(logits), T, s.E, s.H)
        if layer.get("router_bias") is not None:  # fp32 add after the sum, as the block does
            logits = (logits + np.asarray(layer["router_bias"], np.float32)[None, :]).astype(np.float32)
        self.lib.orc_topk(_p(logits), _p(idx), _p(wts), T, s.E, s.TOPK)
        return logits, idx, wts

    def topk(self, logits, K):
        T, E = logits.shape
        idx = np.zeros((T, K), np.int32)
        wts = np.zeros((T, K), np.float32)
        lg = np.ascontiguousarray(logits, np.float32)
        self.lib.orc_topk(_p(lg), _p(idx), _p(wts), T, E, K)
        return idx, wts

    def routed(self, shape, layer, normed, idx, wts, mode=0):
        """moe() on given routing: returns (inter bf16 [T,K,I], routed fp32 [T,H])."""
        s = shape
        T = normed.shape[0]
        x = np.ascontiguousarray(normed, np.uint16)
        ix = np.ascontiguousarray(idx, np.int32)
        wt = np.ascontiguousarray(wts, np.float32)
        inter = np.zeros((T, s.TOPK, s.I), np.uint16)
        routed = np.zeros((T, s.H), np.float32)
        gq, gs, dq, ds = (np.ascontiguousarray(layer[n]) for n in ("exp_gu_q", "exp_gu_s", "exp_dn_q", "exp_dn_s"))
        if mode == 0:
            self.lib.orc_moe_gate_up_int4(_p(x), _p(gq), _p(gs), _p(ix), _p(inter), T, s.TOPK, s.I, s.H, s.G)
            self.lib.orc_moe_down_int4(_p(inter), _p(dq), _p(ds), _p(ix), _p(wt), _p(routed), T, s.TOPK, s.H, s.I,
                                       s.G)
        else:
            slot = np.zeros((T * s.TOPK, s.H), np.float32)
            self.lib.orc_moe_gate_up_tile(_p(x), _p(gq), _p(gs), _p(ix), _p(inter), T, s.TOPK, s.I, s.H, s.G)
            self.lib.orc_moe_down_tile(_p(inter), _p(dq), _p(ds), _p(ix), _p(wt), _p(slot), T, s.TOPK, s.H, s.I, s.G)
            self.lib.orc_moe_slot_reduce(_p(slot), _p(routed), T, s.TOPK, s.H)
        return inter, routed

    def slot_partials(self, shape, layer, normed, idx, wts):
        """The tile path's per-slot partials (kernels.cuh:942-1057): slot [T, TOPK, H] fp32 = w * down(inter)."""
        s = shape
        T = normed.shape[0]
        x = np.ascontiguousarray(normed, np.uint16)
        ix = np.ascontiguousarray(idx, np.int32)
        wt = np.ascontiguousarray(wts, np.float32)
        inter = np.zeros((T, s.TOPK, s.I), np.uint16)
        slot = np.zeros((T, s.TOPK, s.H), np.float32)
        gq, gs, dq, ds = (np.ascontiguousarray(layer[n]) for n in ("exp_gu_q", "exp_gu_s", "exp_dn_q", "exp_dn_s"))
        self.lib.orc_moe_gate_up_tile(_p(x), _p(gq), _p(gs), _p(ix), _p(inter), T, s.TOPK, s.I, s.H, s.G)
        self.lib.orc_moe_down_tile(_p(inter), _p(dq), _p(ds), _p(ix), _p(wt), _p(slot), T, s.TOPK, s.H, s.I, s.G)
        return slot

    def shared_gate_combine(self, shape, layer, hidden_res, routed, sout, normed, next_rms1=None):
        """shared_gate_combine(_rmsnorm)_kernel (kernels.cuh:1081-1121) on the residual-added hidden: returns
        (hidden, normed_out, gate)."""
        s = shape
        T = hidden_res.shape[0]
        h = np.ascontiguousarray(hidden_res, np.float32).copy()
        nout = np.zeros((T, s.H), np.uint16)
        gate = np.zeros((T,), np.float32)
        nr = None if next_rms1 is None else np.ascontiguousarray(next_rms1, np.uint16)
        self.lib.orc_shared_gate_combine(_p(h), _p(np.ascontiguousarray(routed, np.float32)),
                                         _p(np.ascontiguousarray(sout, np.uint16)),
                                         _p(np.ascontiguousarray(normed, np.uint16)),
                                         _p(np.ascontiguousarray(layer["shared_gate"])), _p(nr), _p(nout), _p(gate),
                                         T, s.H, ctypes.c_float(s.eps))
        return h, nout, gate

    def ep_routed(self, shape, layer, normed, idx, wts, world):
        """Routed output of the expert-parallel layer over `world` ranks (rank d owns experts [d*E/world,
        (d+1)*E/world)): per rank the partial of its slots summed in slot order in fp32 and rounded to bf16 (the row
        that crosses the return exchange), then the partials summed in rank order in fp32 (mvcc_b200/csrc/moe_ep.cu
        and the source-side combine of moe_prefill.cu)."""
        s = shape
        slot = self.slot_partials(shape, layer, normed, idx, wts)
        El = s.E // world
        T = normed.shape[0]
        routed = np.zeros((T, s.H), np.float32)
        owner = np.asarray(idx) // El
        for d in range(world):
            part = np.zeros((T, s.H), np.float32)
            for k in range(s.TOPK):
                on = owner[:, k] == d
                part[on] = part[on] + slot[on, k]
            sent = (owner == d).any(axis=1)
            routed[sent] = routed[sent] + bf16_to_f32(f32_to_bf16(part[sent]))
        return routed

    def ep_block_forward(self, shape, layer, hidden, attn_out, world, next_rms1=None):
        """The block with its routed experts split over `world` ranks (tile numerics otherwise): returns the
        block_forward dict with routed / hidden / normed of the expert-parallel summation order."""
        s = shape
        base = self.block_forward(shape, layer, hidden, attn_out, mode=1)
        normed0 = base["normed"]
        routed = self.ep_routed(shape, layer, normed0, base["idx"], base["wts"], world)
        hres = (np.asarray(hidden, np.float32) + bf16_to_f32(np.asarray(attn_out, np.uint16))).astype(np.float32)
        h, nout, _ = self.shared_gate_combine(s, layer, hres, routed, base["sout"], normed0, next_rms1)
        out = dict(base)
        out["routed"] = routed
        out["hidden"] = h
        out["normed"] = nout if next_rms1 is not None else normed0
        return out

    def shared(self, shape, layer, normed):
        """Shared expert: returns (sinter bf16 [T,Is], sout bf16 [T,H])."""
        s = shape
        T = normed.shape[0]
        x = np.ascontiguousarray(normed, np.uint16)
        sgu = np.zeros((T, 2 * s.Is), np.uint16)
        sinter = np.zeros((T, s.Is), np.uint16)
        sout = np.zeros((T, s.H), np.uint16)
        self.lib.orc_dense_bf16_bf16(_p(x), _p(np.ascontiguousarray(layer["shared_gate_up"])), _p(sgu), T, 2 * s.Is,
                                     s.H)
        self.lib.orc_silu_mul(_p(sgu), _p(sinter), T, s.Is)
        self.lib.orc_dense_bf16_bf16(_p(sinter), _p(np.ascontiguousarray(layer["shared_down"])), _p(sout), T, s.H,
                                     s.Is)
        return sinter, sout

    def sort(self, idx, E):
        flat = np.ascontiguousarray(idx, np.int32).reshape(-1)
        offsets = np.zeros(E + 1, np.int32)
        srt = np.zeros(flat.size, np.int32)
        self.lib.orc_moe_sort(_p(flat), flat.size, E, _p(offsets), _p(srt))
        return offsets, srt


def max_rel_err(y, r):
    """max_i |y_i - r_i| / max_i |r_i| (the tolerance metric of the block's parity bar)."""
    y = np.asarray(y, np.float64)
    r = np.asarray(r, np.float64)
    den = np.max(np.abs(r))
    return float(np.max(np.abs(y - r)) / den) if den > 0 else float(np.max(np.abs(y - r)))
