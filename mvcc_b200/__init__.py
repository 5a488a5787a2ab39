"""mvcc_b200 -- B200-native MoE block of mvcc's examples/qwen behind its C ABI (include/moe_block.h).

The compute path is libmoe_b200.so (hand-written sm_100a CUDA, built in-tree by mvcc_b200/build.py). This module
is the host-side mirror of the reference's launch interface for the block: `MoeLayer` carries the fields of the
reference's `Layer`/`Model` (qwen.cu:99-124) plus the INT4 group size, and `MoeBlock` owns the workspace the
reference's `Work` held (qwen.cu:227-293) and issues the calls forward() makes at qwen.cu:429-448.
PyTorch is used only for device memory and streams. There is no CPU fallback: if the library is missing the
import fails, and every call raises on a non-zero cudaError_t.
"""
import ctypes
import dataclasses
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmoe_b200.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: build it with `python mvcc_b200/build.py` (nvcc, sm_100a)")
_lib = ctypes.CDLL(LIB_PATH)


class MoeLayerWeights(ctypes.Structure):
    """ctypes mirror of `moe_layer_weights` (include/moe_block.h)."""

    _fields_ = [
        ("rms2", ctypes.c_void_p),
        ("router", ctypes.c_void_p),
        ("exp_gu_q", ctypes.c_void_p),
        ("exp_gu_s", ctypes.c_void_p),
        ("exp_dn_q", ctypes.c_void_p),
        ("exp_dn_s", ctypes.c_void_p),
        ("shared_gate_up", ctypes.c_void_p),
        ("shared_down", ctypes.c_void_p),
        ("shared_gate", ctypes.c_void_p),
        ("H", ctypes.c_int32),
        ("E", ctypes.c_int32),
        ("TOPK", ctypes.c_int32),
        ("I", ctypes.c_int32),
        ("Is", ctypes.c_int32),
        ("G", ctypes.c_int32),
        ("eps", ctypes.c_float),
        ("router_bias", ctypes.c_void_p),
        ("shared_gate_up_q8", ctypes.c_void_p),
        ("shared_gate_up_s8", ctypes.c_void_p),
        ("shared_down_q8", ctypes.c_void_p),
        ("shared_down_s8", ctypes.c_void_p),
        ("shared_group", ctypes.c_int32),
    ]


class MoeAttnWeights(ctypes.Structure):
    """ctypes mirror of `moe_attn_weights` (include/moe_stack.h)."""

    _fields_ = [(n, ctypes.c_void_p) for n in ("qkv", "gate", "o", "q_norm", "k_norm")] + \
               [(n, ctypes.c_int32) for n in ("H", "Hq", "Hkv", "D", "rope_dim")] + \
               [("theta", ctypes.c_float), ("eps", ctypes.c_float)]


class MoeTrace(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("logits", "idx", "wts", "routed", "sout", "gate", "sorted",
                                               "offsets")]


class MoeStats(ctypes.Structure):
    """ctypes mirror of `moe_stats` (include/moe_block.h)."""

    _fields_ = [("launches", ctypes.c_uint64), ("block_calls", ctypes.c_uint64), ("pack_bytes", ctypes.c_uint64)]


_P = ctypes.c_void_p
_I = ctypes.c_int
_W = ctypes.POINTER(MoeLayerWeights)
_SIGS = {
    "moe_check_shape": (_I, [_W]),
    "moe_workspace_bytes": (ctypes.c_size_t, [_W, _I]),
    "moe_workspace_init": (_I, [_P, ctypes.c_size_t, _P]),
    "moe_workspace_error": (_I, [_P, ctypes.c_size_t, _P]),
    "moe_block_forward": (_I, [_W, _P, ctypes.c_size_t, _P, _P, _P, _P, _I, _P]),
    "moe_block_forward_events": (_I, [_W, _P, ctypes.c_size_t, _P, _P, _P, _P, _I, ctypes.POINTER(_P), _P]),
    "moe_event_create": (_I, [ctypes.POINTER(_P)]),
    "moe_event_destroy": (_I, [_P]),
    "moe_event_elapsed_ms": (_I, [_P, _P, ctypes.POINTER(ctypes.c_float)]),
    "moe_router_topk": (_I, [_W, _P, ctypes.c_size_t, _P, _P, _P, _P, _I, _P]),
    "moe_router_topk_noalloc": (_I, [_W, _P, _P, _P, _P, _I, _P]),
    "moe_router_topk_noalloc_error": (_I, [_P]),
    "moe_routed_experts": (_I, [_W, _P, ctypes.c_size_t, _P, _P, _P, _P, _P, _I, _P]),
    "moe_shared_expert": (_I, [_W, _P, ctypes.c_size_t, _P, _P, _I, _P]),
    "moe_workspace_trace": (_I, [_W, _P, ctypes.c_size_t, _I, ctypes.POINTER(MoeTrace)]),
    "moe_set_prefill_min_tokens": (_I, [_I]),
    "moe_synth_normal_bf16": (_I, [_P, ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float,
                                   ctypes.c_float, _P]),
    "moe_synth_int4_rows": (_I, [_P, _P, ctypes.c_int64, _I, _I, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float,
                                 _P]),
    "moe_version": (ctypes.c_char_p, []),
    "moe_stats_get": (None, [ctypes.POINTER(MoeStats)]),
    "moe_stats_reset": (None, []),
    # expert-parallel stages (include/moe_ep.h)
    "moe_ep_record_bytes": (ctypes.c_size_t, [_W]),
    "moe_ep_dispatch": (_I, [_W, _P, ctypes.c_size_t, _P, _P, _P, _I, _I, _P, _P, _P, _P]),
    "moe_ep_experts": (_I, [_W, _P, ctypes.c_size_t, _P, _I, _P, _P]),
    "moe_ep_combine": (_I, [_W, _P, ctypes.c_size_t, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P]),
    "moe_ep_recv_bytes": (ctypes.c_size_t, [_W, _I, _I]),
    "moe_ep_ret_bytes": (ctypes.c_size_t, [_W, _I, _I]),
    "moe_ep_rcount_offset": (ctypes.c_size_t, [_W, _I, _I]),
    "moe_ep_dispatch_peers": (_I, [_W, _P, ctypes.c_size_t, _P, _P, _P, _I, _I, _P, _P, _P, _P]),
    "moe_ep_experts_peers": (_I, [_W, _P, ctypes.c_size_t, _I, _P, _P]),
    "moe_device_alloc": (_I, [ctypes.c_size_t, ctypes.POINTER(_P)]),
    "moe_device_free": (_I, [_P]),
    "moe_ipc_handle": (_I, [_P, _P]),
    "moe_ipc_open": (_I, [_P, ctypes.POINTER(_P)]),
    "moe_ipc_close": (_I, [_P]),
    # attention layer, first-layer norm and LM head of a decode step (include/moe_stack.h)
    "moe_attn_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(MoeAttnWeights), _I, _I]),
    "moe_attn_workspace_error": (_I, [_P, ctypes.c_size_t, _P]),
    "moe_attn_forward": (_I, [ctypes.POINTER(MoeAttnWeights), _P, _P, _I, _I, _P, _P, _I, _P, ctypes.c_size_t, _P]),
    "moe_attn_forward_rms": (_I, [ctypes.POINTER(MoeAttnWeights), _P, _P, _P, _P, _I, _I, _P, _I, _P, ctypes.c_size_t,
                                  _P]),
    "moe_rmsnorm": (_I, [_P, _P, _P, _I, _I, ctypes.c_float, _P]),
    "moe_lm_head_workspace_bytes": (ctypes.c_size_t, [_I, _I]),
    "moe_lm_head_argmax": (_I, [_P, _P, _I, _I, _P, _P, _P, ctypes.c_size_t, _P]),
    # weight pack reader (include/moe_pack.h); the structures are declared in mvcc_b200/pack.py
    "moe_pack_open": (_P, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]),
    "moe_pack_close": (None, [_P]),
    "moe_pack_last_error": (ctypes.c_char_p, [_P]),
    "moe_pack_geometry_get": (_I, [_P, _P]),
    "moe_pack_tensor_count": (_I, [_P]),
    "moe_pack_tensor": (_I, [_P, ctypes.c_char_p, _P]),
    "moe_pack_tensor_name": (ctypes.c_char_p, [_P, _I]),
    "moe_pack_layer_host": (_I, [_P, _I, _W]),
    "moe_pack_layer_bytes": (ctypes.c_size_t, [_P, _I]),
    "moe_pack_upload_layer": (_I, [_P, _I, _P, ctypes.c_size_t, _W, _P]),
}
for _name, (_res, _args) in _SIGS.items():
    _fn = getattr(_lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args

EXPORTED = tuple(_SIGS)


class MoeError(RuntimeError):
    pass


def _check(rc, what):
    if rc != 0:
        raise MoeError(f"{what} failed: cudaError {rc}")


def version():
    return _lib.moe_version().decode()


def stats():
    """The library's counters (moe_stats_get): kernel launches issued (a launch captured into a CUDA graph counts
    once, at capture), block calls, bytes the pack loader copied to the device."""
    st = MoeStats()
    _lib.moe_stats_get(ctypes.byref(st))
    return {"launches": st.launches, "block_calls": st.block_calls, "pack_bytes": st.pack_bytes}


def reset_stats():
    _lib.moe_stats_reset()


def tensor_stats(t, bf16=None):
    """The reference's `--debug` statistics of one tensor (qwen.cu:66-89): element count, mean and rms over all
    elements with the non-finite ones left out of the sums, absmax of the finite ones, the count of NaN/inf values and
    the first four values. `bf16` (default: int16 or uint16 storage) decodes bf16 bits. Synchronises the device the
    tensor lives on and copies it to the host."""
    x = t.detach()
    if bf16 is None:
        bf16 = x.dtype in (torch.int16, torch.uint16)
    x = x.contiguous().reshape(-1)
    x = x.view(torch.bfloat16) if bf16 else x
    x = x.to("cpu", torch.float64)
    n = x.numel()
    fin = torch.isfinite(x)
    v = torch.where(fin, x, torch.zeros_like(x))
    return {"n": n, "mean": float(v.sum()) / n if n else 0.0, "rms": float((v * v).sum() / n) ** 0.5 if n else 0.0,
            "absmax": float(v.abs().max()) if n else 0.0, "nonfinite": int(n - int(fin.sum())),
            "head": [float(a) for a in x[:4]]}


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


class Event:
    """A CUDA timing event owned by libmoe_b200 (recordable inside graph capture through forward_events)."""

    def __init__(self):
        h = ctypes.c_void_p()
        _check(_lib.moe_event_create(ctypes.byref(h)), "moe_event_create")
        self.handle = h

    def elapsed_ms(self, later):
        ms = ctypes.c_float()
        _check(_lib.moe_event_elapsed_ms(self.handle, later.handle, ctypes.byref(ms)), "moe_event_elapsed_ms")
        return ms.value

    def __del__(self):
        if getattr(self, "handle", None) and _lib is not None:
            _lib.moe_event_destroy(self.handle)
            self.handle = None


@dataclasses.dataclass(frozen=True)
class MoeShape:
    """Geometry of one MoE layer (the reference's pack config, convert.py:327-334) plus the INT4 group size."""

    H: int = 2048
    E: int = 256
    TOPK: int = 8
    I: int = 512
    Is: int = 512
    G: int = 64
    eps: float = 1e-6

    def expert_bytes(self):
        """Weight + scale bytes of one routed expert (the reference's decode_weight_bytes term, qwen.cu:470)."""
        return 2 * self.I * self.H // 2 + self.H * self.I // 2 + 2 * (2 * self.I * (self.H // self.G)
                                                                     + self.H * (self.I // self.G))


class MoeLayer:
    """Device tensors of one layer in the reference's pack layout (convert.py:6-20, 388-415)."""

    NAMES = ("rms2", "router", "exp_gu_q", "exp_gu_s", "exp_dn_q", "exp_dn_s", "shared_gate_up", "shared_down",
             "shared_gate")
    INT8_NAMES = ("shared_gate_up_q8", "shared_gate_up_s8", "shared_down_q8", "shared_down_s8")

    def __init__(self, shape: MoeShape, tensors: dict):
        self.shape = shape
        self.t = dict(tensors)
        s = shape
        expect = {
            "rms2": ((s.H,), torch.int16), "router": ((s.E, s.H), torch.int16),
            "exp_gu_q": ((s.E, 2 * s.I, s.H // 2), torch.uint8),
            "exp_gu_s": ((s.E, 2 * s.I, s.H // s.G), torch.int16),
            "exp_dn_q": ((s.E, s.H, s.I // 2), torch.uint8),
            "exp_dn_s": ((s.E, s.H, s.I // s.G), torch.int16),
            "shared_gate_up": ((2 * s.Is, s.H), torch.int16), "shared_down": ((s.H, s.Is), torch.int16),
            "shared_gate": ((s.H,), torch.int16),
        }
        for n, (shp, dt) in expect.items():
            v = self.t[n]
            if tuple(v.shape) != shp or v.dtype != dt or not v.is_contiguous() or not v.is_cuda:
                raise ValueError(f"{n}: expected contiguous cuda {dt} {shp}, got {v.dtype} {tuple(v.shape)}")
        bias = self.t.get("router_bias")
        if bias is not None and (tuple(bias.shape) != (s.E,) or bias.dtype != torch.float32 or not bias.is_cuda
                                 or not bias.is_contiguous()):
            raise ValueError(f"router_bias: expected contiguous cuda float32 ({s.E},)")
        self.c = MoeLayerWeights(*[ctypes.c_void_p(self.t[n].data_ptr()) for n in self.NAMES],
                                 s.H, s.E, s.TOPK, s.I, s.Is, s.G, s.eps,
                                 None if bias is None else ctypes.c_void_p(bias.data_ptr()))
        # optional int8 shared expert (--dense int8 packs): int8 rows and fp16 group scales as stored
        i8 = [self.t.get(n) for n in self.INT8_NAMES]
        if any(v is not None for v in i8):
            gq, gs, dq, ds = i8
            if any(v is None for v in i8):
                raise ValueError("int8 shared expert: all of " + ", ".join(self.INT8_NAMES) + " are needed")
            g8 = s.H // gs.shape[1] if gs.dim() == 2 and gs.shape[1] else 0
            want = {"shared_gate_up_q8": ((2 * s.Is, s.H), torch.int8),
                    "shared_gate_up_s8": ((2 * s.Is, s.H // max(g8, 1)), torch.int16),
                    "shared_down_q8": ((s.H, s.Is), torch.int8),
                    "shared_down_s8": ((s.H, s.Is // max(g8, 1)), torch.int16)}
            for n, (shp, dt) in want.items():
                v = self.t[n]
                if tuple(v.shape) != shp or v.dtype != dt or not v.is_contiguous() or not v.is_cuda:
                    raise ValueError(f"{n}: expected contiguous cuda {dt} {shp}, got {v.dtype} {tuple(v.shape)}")
            self.c.shared_gate_up_q8 = gq.data_ptr()
            self.c.shared_gate_up_s8 = gs.data_ptr()
            self.c.shared_down_q8 = dq.data_ptr()
            self.c.shared_down_s8 = ds.data_ptr()
            self.c.shared_group = g8
        _check(_lib.moe_check_shape(ctypes.byref(self.c)), "moe_check_shape")


class MoeBlock:
    """Workspace owner and launcher for one layer's MoE block (the reference's Work + forward() steps)."""

    def __init__(self, layer: MoeLayer, max_T: int):
        self.layer = layer
        self.max_T = max_T
        nbytes = _lib.moe_workspace_bytes(ctypes.byref(layer.c), max_T)
        if nbytes == 0:
            raise MoeError("moe_workspace_bytes rejected the shape")
        self.ws_bytes = nbytes
        dev = layer.t["router"].device
        self.ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        _check(_lib.moe_workspace_init(_ptr(self.ws), nbytes, _stream(None)), "moe_workspace_init")
        # The zeroing is stream-ordered; wait for it so the block may be used from any stream afterwards.
        torch.cuda.current_stream(dev).synchronize()

    def _args(self):
        return ctypes.byref(self.layer.c), _ptr(self.ws), self.ws_bytes

    def forward(self, hidden, attn_out, normed, next_rms1=None, T=None, stream=None):
        """qwen.cu:429-448 for T tokens: hidden (fp32 [T,H], in/out), attn_out (bf16 bits [T,H]), normed (out)."""
        T = hidden.shape[0] if T is None else T
        _check(_lib.moe_block_forward(*self._args(), _ptr(hidden), _ptr(attn_out), _ptr(normed), _ptr(next_rms1),
                                      T, _stream(stream)), "moe_block_forward")

    def forward_events(self, hidden, attn_out, normed, events, next_rms1=None, T=None, stream=None):
        """forward() that records the 4 Event handles before the block and after each of its kernels."""
        T = hidden.shape[0] if T is None else T
        arr = (ctypes.c_void_p * 4)(*[e.handle for e in events])
        _check(_lib.moe_block_forward_events(*self._args(), _ptr(hidden), _ptr(attn_out), _ptr(normed),
                                             _ptr(next_rms1), T, arr, _stream(stream)), "moe_block_forward_events")

    def router_topk(self, normed, logits, idx, wts, T=None, stream=None):
        T = normed.shape[0] if T is None else T
        _check(_lib.moe_router_topk(*self._args(), _ptr(normed), _ptr(logits), _ptr(idx), _ptr(wts), T,
                                    _stream(stream)), "moe_router_topk")

    def routed_experts(self, normed, idx, wts, routed, inter=None, T=None, stream=None):
        T = normed.shape[0] if T is None else T
        _check(_lib.moe_routed_experts(*self._args(), _ptr(normed), _ptr(idx), _ptr(wts), _ptr(routed), _ptr(inter),
                                       T, _stream(stream)), "moe_routed_experts")

    def shared_expert(self, normed, sout, T=None, stream=None):
        T = normed.shape[0] if T is None else T
        _check(_lib.moe_shared_expert(*self._args(), _ptr(normed), _ptr(sout), T, _stream(stream)),
               "moe_shared_expert")

    def error_word(self, stream=None):
        rc = _lib.moe_workspace_error(_ptr(self.ws), self.ws_bytes, _stream(stream))
        if rc < 0:
            raise MoeError(f"moe_workspace_error failed: cudaError {-rc}")
        return rc

    def trace(self, T):
        """Device views of the last forward's intermediates (logits, idx, wts, routed, sout, gate)."""
        tr = MoeTrace()
        _check(_lib.moe_workspace_trace(*self._args(), T, ctypes.byref(tr)), "moe_workspace_trace")
        s = self.layer.shape
        base = self.ws.data_ptr()

        def view(ptr, n, dtype):
            off = ptr - base
            nb = n * torch.empty((), dtype=dtype).element_size()
            return self.ws[off:off + nb].view(dtype)

        out = {
            "logits": view(tr.logits, T * s.E, torch.float32).view(T, s.E),
            "idx": view(tr.idx, T * s.TOPK, torch.int32).view(T, s.TOPK),
            "wts": view(tr.wts, T * s.TOPK, torch.float32).view(T, s.TOPK),
            "routed": view(tr.routed, T * s.H, torch.float32).view(T, s.H),
            "sout": view(tr.sout, T * s.H, torch.int16).view(T, s.H),
            "gate": view(tr.gate, T, torch.float32),
        }
        if tr.sorted:  # prefill path: the stable expert sort
            out["sorted"] = view(tr.sorted, T * s.TOPK, torch.int32)
            out["offsets"] = view(tr.offsets, s.E + 1, torch.int32)
        return out

    def debug_stats(self, T, hidden=None, normed=None):
        """The reference's `--debug` report for the last forward of T tokens (qwen.cu:382-449 print the same
        statistics per stage): tensor_stats of every traced intermediate, plus hidden and normed when given."""
        tr = self.trace(T)
        out = {n: tensor_stats(v, bf16=(n == "sout")) for n, v in tr.items() if n not in ("idx", "sorted", "offsets")}
        if hidden is not None:
            out["hidden"] = tensor_stats(hidden)
        if normed is not None:
            out["normed"] = tensor_stats(normed, bf16=True)
        return out


def set_prefill_min_tokens(T: int):
    """Process-wide token count from which calls take the prefill path (0 = default 8; a huge value keeps every
    call on the decode kernels)."""
    _check(_lib.moe_set_prefill_min_tokens(int(T)), "moe_set_prefill_min_tokens")


def router_topk_noalloc(layer: MoeLayer, normed, logits, idx, wts, T=None, stream=None):
    """Router + top-k with no workspace (moe_router_topk_noalloc): for callers that cannot allocate device memory.
    Calls that overlap on the GPU share the library's fixed scratch and must be serialised."""
    T = normed.shape[0] if T is None else T
    _check(_lib.moe_router_topk_noalloc(ctypes.byref(layer.c), _ptr(normed), _ptr(logits), _ptr(idx), _ptr(wts), T,
                                        _stream(stream)), "moe_router_topk_noalloc")


def router_topk_noalloc_error(stream=None):
    """Reads and clears the allocation-free router's error word on the current device (moe_router_topk_noalloc_error)."""
    rc = _lib.moe_router_topk_noalloc_error(_stream(stream))
    if rc < 0:
        raise MoeError(f"moe_router_topk_noalloc_error failed: cudaError {-rc}")
    return rc


def synth_layer(shape: MoeShape, seed: int, device="cuda", std=0.02, stream=None) -> MoeLayer:
    """Seeded synthetic layer on the device (weights bf16 N(0, std); experts INT4 with absmax/7 group scales)."""
    s = shape
    dev = torch.device(device)
    st = _stream(stream)
    t = {}

    def normal(name, shp, sid, mean, sd):
        x = torch.empty(shp, dtype=torch.int16, device=dev)
        _check(_lib.moe_synth_normal_bf16(_ptr(x), x.numel(), seed, sid, mean, sd, st), "moe_synth_normal_bf16")
        t[name] = x

    normal("rms2", (s.H,), 1, 1.0, 0.0)
    normal("router", (s.E, s.H), 2, 0.0, std)
    normal("shared_gate_up", (2 * s.Is, s.H), 3, 0.0, std)
    normal("shared_down", (s.H, s.Is), 4, 0.0, std)
    normal("shared_gate", (s.H,), 5, 0.0, std)
    t["exp_gu_q"] = torch.empty((s.E, 2 * s.I, s.H // 2), dtype=torch.uint8, device=dev)
    t["exp_gu_s"] = torch.empty((s.E, 2 * s.I, s.H // s.G), dtype=torch.int16, device=dev)
    t["exp_dn_q"] = torch.empty((s.E, s.H, s.I // 2), dtype=torch.uint8, device=dev)
    t["exp_dn_s"] = torch.empty((s.E, s.H, s.I // s.G), dtype=torch.int16, device=dev)
    _check(_lib.moe_synth_int4_rows(_ptr(t["exp_gu_q"]), _ptr(t["exp_gu_s"]), s.E * 2 * s.I, s.H, s.G, seed, 6, std,
                                    st), "moe_synth_int4_rows")
    _check(_lib.moe_synth_int4_rows(_ptr(t["exp_dn_q"]), _ptr(t["exp_dn_s"]), s.E * s.H, s.I, s.G, seed, 7, std, st),
           "moe_synth_int4_rows")
    return MoeLayer(shape, t)


def zipf_bias(E: int, seed: int = 0, s: float = 1.1):
    """Per-expert router bias b_e = -s * ln(1 + pi(e)), pi a seeded permutation of 0..E-1: the Zipf(s) expert-load
    skew of the prefill benchmark (fp32 numpy array, host)."""
    import numpy as np
    perm = np.random.default_rng(seed).permutation(E)
    return (-s * np.log1p(perm.astype(np.float64))).astype(np.float32)


def synth_activations(shape: MoeShape, T: int, seed: int, device="cuda", stream=None):
    """hidden fp32 [T,H] ~ N(0,1) (via bf16) and attn_out bf16 [T,H] ~ N(0,1), seeded."""
    dev = torch.device(device)
    st = _stream(stream)
    h16 = torch.empty((T, shape.H), dtype=torch.int16, device=dev)
    a16 = torch.empty((T, shape.H), dtype=torch.int16, device=dev)
    _check(_lib.moe_synth_normal_bf16(_ptr(h16), h16.numel(), seed, 101, 0.0, 1.0, st), "moe_synth_normal_bf16")
    _check(_lib.moe_synth_normal_bf16(_ptr(a16), a16.numel(), seed, 102, 0.0, 1.0, st), "moe_synth_normal_bf16")
    hidden = (h16.to(torch.int32) << 16).view(torch.float32).contiguous()
    return hidden, a16
