"""The .mvccq weight pack: reading one layer's MoE block into HBM (include/moe_pack.h), and writing packs.

`MoePack` wraps the library's reader: the file is mapped read-only, its header parsed and checked, and
`MoePack.layer(i)` copies layer i's nine block tensors into one device buffer and returns a `MoeLayer` over it --
what the reference's `Model::load` does for these tensors (qwen.cu:158-166, 181-190), except that the weights land
in HBM instead of a zero-copy host mapping (pack.hpp:140-149).

`write_pack` writes the same format as the reference's converter (convert.py:175-211): "MVCCQ001", a little-endian
u64 header length, the compact JSON header {"config", "tensors"} inside a fixed header slot (1 MiB by default),
then each blob at the next 64-byte boundary. It exists so packs of synthetic layers (group 64 included, which no
GPTQ checkpoint can be repacked to) can be written and read back through the same path as converted checkpoints.
"""
import ctypes
import json
import os
import struct

import numpy as np
import torch

from . import MoeError, MoeLayer, MoeLayerWeights, MoeShape, _lib, _stream

MAGIC = b"MVCCQ001"
HEADER_SLOT = 1 << 20
BLOB_ALIGN = 64

# Block tensor names inside a layer (convert.py:370-415) for each MoeLayer field, with the stored dtype.
BLOCK_TENSORS = (
    ("rms2", "rms2", "bf16"),
    ("router", "router", "bf16"),
    ("exp_gu_q", "exp.gate_up.q", "u8"),
    ("exp_gu_s", "exp.gate_up.s", "f16"),
    ("exp_dn_q", "exp.down.q", "u8"),
    ("exp_dn_s", "exp.down.s", "f16"),
    ("shared_gate_up", "shared.gate_up", "bf16"),
    ("shared_down", "shared.down", "bf16"),
    ("shared_gate", "shared.gate", "bf16"),
)
_NUMPY = {"bf16": np.uint16, "f16": np.float16, "f32": np.float32, "u8": np.uint8, "i8": np.int8}
_TORCH = {"bf16": torch.int16, "f16": torch.int16, "f32": torch.float32, "u8": torch.uint8, "i8": torch.int8}


class MoePackGeometry(ctypes.Structure):
    """ctypes mirror of `moe_pack_geometry` (include/moe_pack.h)."""

    _fields_ = [(n, ctypes.c_int32) for n in ("H", "L", "E", "TOPK", "I", "Is", "G")] + [("eps", ctypes.c_float)]


class MoePackTensorInfo(ctypes.Structure):
    """ctypes mirror of `moe_pack_tensor_info` (include/moe_pack.h)."""

    _fields_ = [("off", ctypes.c_uint64), ("nbytes", ctypes.c_uint64), ("host", ctypes.c_void_p),
                ("ndim", ctypes.c_int32), ("shape", ctypes.c_int64 * 6), ("dtype", ctypes.c_char * 8)]


class PackError(MoeError):
    def __init__(self, rc, msg):
        super().__init__(f"{msg} (cudaError {rc})")
        self.rc = rc


class MoePack:
    """A mapped .mvccq pack. Use as a context manager or call close(); tensors read from it are copies."""

    def __init__(self, path):
        err = ctypes.create_string_buffer(512)
        h = _lib.moe_pack_open(os.fsencode(path), err, len(err))
        if not h:
            raise PackError(1, err.value.decode(errors="replace"))
        self._h = ctypes.c_void_p(h)
        self.path = path
        g = MoePackGeometry()
        self._check(_lib.moe_pack_geometry_get(self._h, ctypes.byref(g)))
        self.geometry = g
        self.shape = MoeShape(H=g.H, E=g.E, TOPK=g.TOPK, I=g.I, Is=g.Is, G=g.G, eps=g.eps)
        self.layers = g.L

    def _check(self, rc):
        if rc != 0:
            raise PackError(rc, _lib.moe_pack_last_error(self._h).decode(errors="replace"))

    def close(self):
        if getattr(self, "_h", None):
            _lib.moe_pack_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        if _lib is not None:
            self.close()

    def names(self):
        return [_lib.moe_pack_tensor_name(self._h, i).decode() for i in range(_lib.moe_pack_tensor_count(self._h))]

    def info(self, name):
        inf = MoePackTensorInfo()
        self._check(_lib.moe_pack_tensor(self._h, name.encode(), ctypes.byref(inf)))
        return inf

    def tensor(self, name):
        """A host copy of one tensor (bf16 as uint16 bits, f16 as float16)."""
        inf = self.info(name)
        raw = ctypes.string_at(inf.host, inf.nbytes)
        dt = inf.dtype.decode()
        arr = np.frombuffer(raw, dtype=_NUMPY.get(dt, np.uint8))
        shape = tuple(inf.shape[:inf.ndim])
        return arr.reshape(shape) if dt in _NUMPY else arr

    def block_shapes(self):
        """Shape of each block tensor (keyed by MoeLayer field) at this pack's geometry."""
        s = self.shape
        return {"rms2": (s.H,), "router": (s.E, s.H), "exp_gu_q": (s.E, 2 * s.I, s.H // 2),
                "exp_gu_s": (s.E, 2 * s.I, s.H // s.G), "exp_dn_q": (s.E, s.H, s.I // 2),
                "exp_dn_s": (s.E, s.H, s.I // s.G), "shared_gate_up": (2 * s.Is, s.H),
                "shared_down": (s.H, s.Is), "shared_gate": (s.H,)}

    def layer_host(self, layer):
        """Layer `layer`'s block tensors as host copies keyed by MoeLayer field, checked as for layer() (an int8
        shared expert comes back as its dequantised bf16 rows, the values layer() uploads)."""
        w = MoeLayerWeights()
        self._check(_lib.moe_pack_layer_host(self._h, layer, ctypes.byref(w)))
        out = {}
        for (field, _, dt), shape in zip(BLOCK_TENSORS, self.block_shapes().values()):
            n = int(np.prod(shape)) * np.dtype(_NUMPY[dt]).itemsize
            out[field] = np.frombuffer(ctypes.string_at(getattr(w, field), n), dtype=_NUMPY[dt]).reshape(shape)
        return out

    def layer_bytes(self, layer):
        n = _lib.moe_pack_layer_bytes(self._h, layer)
        if n == 0:  # the same checks again, for their error code
            self._check(_lib.moe_pack_layer_host(self._h, layer, ctypes.byref(MoeLayerWeights())) or 1)
        return n

    def layer(self, layer, device="cuda", stream=None) -> MoeLayer:
        """Copies layer `layer`'s block into one device buffer (moe_pack_upload_layer) and returns its MoeLayer.
        The copies are ordered on `stream` (default: the current stream)."""
        nbytes = self.layer_bytes(layer)
        buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        w = MoeLayerWeights()
        self._check(_lib.moe_pack_upload_layer(self._h, layer, ctypes.c_void_p(buf.data_ptr()), nbytes,
                                               ctypes.byref(w), _stream(stream)))
        base = buf.data_ptr()
        t = {}
        for (field, _, dt), shape in zip(BLOCK_TENSORS, self.block_shapes().values()):
            off = getattr(w, field) - base
            n = int(np.prod(shape)) * np.dtype(_NUMPY[dt]).itemsize
            t[field] = buf[off:off + n].view(_TORCH[dt]).view(shape)
        if w.shared_gate_up_q8:  # the int8 shared expert as stored, beside its bf16 rows
            s, g8 = self.shape, w.shared_group
            for field, shape, dtype in (("shared_gate_up_q8", (2 * s.Is, s.H), torch.int8),
                                        ("shared_gate_up_s8", (2 * s.Is, s.H // g8), torch.int16),
                                        ("shared_down_q8", (s.H, s.Is), torch.int8),
                                        ("shared_down_s8", (s.H, s.Is // g8), torch.int16)):
                off = getattr(w, field) - base
                n = int(np.prod(shape)) * torch.empty((), dtype=dtype).element_size()
                t[field] = buf[off:off + n].view(dtype).view(shape)
        ml = MoeLayer(self.shape, t)
        ml.storage = buf  # the tensors are views of this buffer
        return ml


def quantize_int8_rows(w_bf16, group=128):
    """Symmetric int8 rows with fp16 group scales, as the reference's converter makes them for --dense int8
    (quant_int8_rows, convert.py:162-169): per (row, group of `group` inputs) scale = absmax / 127 (1 where the
    group is all zero), q = clip(rint(w / scale), -127, 127) computed with the fp32 scale, the scale stored as fp16.
    w_bf16: uint16 bf16 bit patterns [N, K]. Returns (int8 [N, K], float16 [N, K / group])."""
    w = np.ascontiguousarray(w_bf16, dtype=np.uint16)
    N, K = w.shape
    f = (w.astype(np.uint32) << 16).view(np.float32).reshape(N, K // group, group)
    amax = np.abs(f).max(axis=2, keepdims=True)
    scale = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(f / scale), -127, 127).astype(np.int8).reshape(N, K)
    return q, scale.reshape(N, K // group).astype(np.float16)


def dequantize_int8_rows(q, scales):
    """bf16 bit patterns of q * scale (the product is exact in fp32; one round to nearest even), the values the
    loader puts on the device for an int8 shared expert."""
    q = np.asarray(q, np.int8)
    N, K = q.shape
    g = K // scales.shape[1]
    f = q.astype(np.float32) * np.repeat(np.asarray(scales, np.float16).astype(np.float32), g, axis=1)
    u = f.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def block_entries(layer_index, tensors, shared_int8_group=None):
    """(name, dtype, array) pack entries for one layer's block from MoeLayer-keyed host arrays (bf16 and f16 as
    16-bit patterns, INT4 packed as uint8), in the order the reference's converter writes them
    (convert.py:372-415: norms, router, shared expert, routed experts). With shared_int8_group, the shared expert's
    two matrices are written as int8 rows + fp16 scales (quantize_int8_rows), as convert.py --dense int8 does."""
    order = ("rms2", "router", "shared_gate_up", "shared_down", "shared_gate", "exp_gu_q", "exp_gu_s", "exp_dn_q",
             "exp_dn_s")
    by_field = {f: (sub, dt) for f, sub, dt in BLOCK_TENSORS}
    out = []
    for f in order:
        sub, dt = by_field[f]
        a = np.ascontiguousarray(tensors[f])
        if dt in ("bf16", "f16"):
            a = a.view(np.uint16) if a.dtype != np.float16 else a
        if shared_int8_group and f in ("shared_gate_up", "shared_down"):
            q, sc = quantize_int8_rows(a, shared_int8_group)
            out += [(f"L{layer_index}.{sub}.q8", "i8", q), (f"L{layer_index}.{sub}.s8", "f16", sc)]
            continue
        out.append((f"L{layer_index}.{sub}", dt, a))
    return out


def pack_config(shape: MoeShape, layers, **extra):
    """The "config" keys the reader needs (convert.py:327-333 names), plus any others the caller passes."""
    cfg = {"hidden": shape.H, "layers": layers, "experts": shape.E, "topk": shape.TOPK, "inter": shape.I,
           "shared_inter": shape.Is, "eps": shape.eps, "group": shape.G}
    cfg.update(extra)
    return cfg


def write_pack(path, config, entries, header_slot=HEADER_SLOT):
    """Writes a .mvccq pack: `entries` is a sequence of (name, dtype, array) written in that order."""
    tensors = {}
    blobs = []
    off = header_slot
    for name, dtype, arr in entries:
        a = np.ascontiguousarray(arr)
        off += (-off) % BLOB_ALIGN
        tensors[name] = {"off": off, "nbytes": a.nbytes, "dtype": dtype, "shape": [int(d) for d in a.shape]}
        blobs.append((off, a))
        off += a.nbytes
    hdr = json.dumps({"config": config, "tensors": tensors}, separators=(",", ":")).encode()
    if 16 + len(hdr) > header_slot:
        raise ValueError(f"header of {len(hdr)} bytes does not fit the {header_slot}-byte slot")
    with open(path, "wb") as f:
        f.write(MAGIC + struct.pack("<Q", len(hdr)) + hdr)
        f.write(b"\0" * (header_slot - 16 - len(hdr)))
        pos = header_slot
        for o, a in blobs:
            f.write(b"\0" * (o - pos))
            f.write(a.tobytes())
            pos = o + a.nbytes
    return path


def synth_pack(path, shape: MoeShape, layers, seed=0, std=0.02, shared_int8_group=None):
    """Writes a pack of `layers` seeded synthetic MoE layers (host numpy PCG64 draws, no GPU): bf16 N(0, std) router
    and shared expert, rms2 = 1, and experts quantised by the rule of the device generator (moe_synth_int4_rows):
    weights rounded to bf16, then per group of G inputs scale = fp16(absmax / 7) and q = clamp(rint(w / scale),
    -7, 7) + 8 with that fp16 scale. The way to get group-64 packs, which no GPTQ checkpoint can be repacked to."""
    s = shape
    rng = np.random.default_rng(seed)

    def bf16(*shp):
        f = (std * rng.standard_normal(shp)).astype(np.float32)
        u = f.view(np.uint32).astype(np.uint64)
        return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)  # round to nearest even

    def int4_rows(n, k):
        w = (bf16(n, k // s.G, s.G).astype(np.uint32) << 16).view(np.float32)
        sc = (np.abs(w).max(axis=2, keepdims=True) / 7).astype(np.float16)
        scf = sc.astype(np.float32)
        q = np.clip(np.rint(np.divide(w, scf, out=np.zeros_like(w), where=scf > 0)), -7, 7).astype(np.int32) + 8
        q = q.reshape(n, k).astype(np.uint8)
        return (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8), sc.reshape(n, k // s.G)

    ents = []
    for li in range(layers):
        gq, gs = int4_rows(s.E * 2 * s.I, s.H)
        dq, ds = int4_rows(s.E * s.H, s.I)
        t = {"rms2": np.full(s.H, 0x3F80, np.uint16), "router": bf16(s.E, s.H),
             "exp_gu_q": gq.reshape(s.E, 2 * s.I, s.H // 2), "exp_gu_s": gs.reshape(s.E, 2 * s.I, s.H // s.G),
             "exp_dn_q": dq.reshape(s.E, s.H, s.I // 2), "exp_dn_s": ds.reshape(s.E, s.H, s.I // s.G),
             "shared_gate_up": bf16(2 * s.Is, s.H), "shared_down": bf16(s.H, s.Is), "shared_gate": bf16(s.H)}
        ents += block_entries(li, t, shared_int8_group=shared_int8_group)
    extra = {"dense": "int8"} if shared_int8_group else {}
    return write_pack(path, pack_config(s, layers, **extra), ents)


def _main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(prog="python -m mvcc_b200.pack",
                                 description="Inspect a .mvccq pack, or write a synthetic one.")
    sub = ap.add_subparsers(dest="cmd", required=True)
    pi = sub.add_parser("info", help="geometry, tensor count and each layer's block bytes on the device")
    pi.add_argument("pack")
    ps = sub.add_parser("synth", help="write a pack of seeded synthetic MoE layers")
    ps.add_argument("out")
    ps.add_argument("--layers", type=int, default=1)
    ps.add_argument("--hidden", type=int, default=2048)
    ps.add_argument("--experts", type=int, default=256)
    ps.add_argument("--topk", type=int, default=8)
    ps.add_argument("--inter", type=int, default=512)
    ps.add_argument("--shared-inter", type=int, default=512)
    ps.add_argument("--group", type=int, default=64)
    ps.add_argument("--seed", type=int, default=0)
    ps.add_argument("--int8-shared", type=int, default=0, metavar="GROUP",
                    help="store the shared expert as int8 rows with this scale group (convert.py --dense int8)")
    a = ap.parse_args(argv)
    if a.cmd == "synth":
        s = MoeShape(H=a.hidden, E=a.experts, TOPK=a.topk, I=a.inter, Is=a.shared_inter, G=a.group)
        synth_pack(a.out, s, a.layers, seed=a.seed, shared_int8_group=a.int8_shared or None)
        print(f"wrote {a.out}: {a.layers} layer(s), {os.path.getsize(a.out)} bytes")
        return 0
    with MoePack(a.pack) as pk:
        s = pk.shape
        print(f"{a.pack}: H={s.H} E={s.E} topk={s.TOPK} I={s.I} Is={s.Is} group={s.G} eps={s.eps:g} "
              f"layers={pk.layers} tensors={len(pk.names())}")
        for li in range(pk.layers):
            try:
                print(f"  L{li}: block {pk.layer_bytes(li)} bytes on the device")
            except PackError as e:
                print(f"  L{li}: {e}")
    return 0


if __name__ == "__main__":
    raise SystemExit(_main())
