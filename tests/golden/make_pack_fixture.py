"""Writes the .mvccq pack fixtures in tests/golden/ with the reference's own pack writer.

    python tests/golden/make_pack_fixture.py --reference <reference checkout> --out tests/golden

The reference's converter (examples/qwen/convert.py: `Writer`, `pack_nibbles`, `quant_int8_rows`) writes two tiny
two-layer packs from the seeded arrays of `entries()` below:
  * ref_pack_tiny.mvccq.gz       -- bf16 shared expert (convert.py's default --dense bf16);
  * ref_pack_tiny_int8.mvccq.gz  -- shared expert stored as int8 rows + fp16 group scales (--dense int8).
Beside the MoE block tensors they hold the non-block tensors a converted checkpoint carries (embedding, final norm,
an attention and a GDN tensor) so the reader is shown to skip them. ref_pack_tiny.json records each tensor's
SHA-256 and the geometry. The arrays are regenerated from the seed by tests/test_pack.py, which checks that
mvcc_b200.pack.write_pack writes the same bytes as the reference's writer did.
"""
import argparse
import gzip
import hashlib
import json
import os
import sys
import tempfile

import numpy as np

SEED = 11
GEOM = dict(H=64, E=4, TOPK=2, I=32, Is=32, G=32, L=2, V=16, eps=1e-6)


def config():
    g = GEOM
    # The key set convert.py:327-333 writes (geometry of the tiny model; attention/GDN values are placeholders).
    return {"hidden": g["H"], "layers": g["L"], "experts": g["E"], "topk": g["TOPK"], "inter": g["I"],
            "shared_inter": g["Is"], "q_heads": 2, "kv_heads": 1, "head_dim": 32, "gdn_k_heads": 1,
            "gdn_v_heads": 2, "gdn_k_dim": 32, "gdn_v_dim": 32, "conv_k": 4, "vocab": g["V"], "eps": g["eps"],
            "rope_theta": 10000000.0, "rope_dim": 16, "layer_kinds": [1, 0], "group": g["G"], "eos": [1, 2],
            "dense": "bf16", "lm_head": "bf16", "attn_gate": False}


def arrays():
    """The seeded tensors, keyed by pack name (bf16 as uint16 bit patterns; INT4 as unpacked nibbles 0..15)."""
    g = GEOM
    H, E, I, Is, G, V = g["H"], g["E"], g["I"], g["Is"], g["G"], g["V"]
    rng = np.random.default_rng(SEED)

    def bf16(*shape):
        f = (0.02 * rng.standard_normal(shape)).astype(np.float32)
        return (f.view(np.uint32) >> 16).astype(np.uint16)  # truncation: any bit pattern serves a format test

    out = {"embed": bf16(V, H), "final_norm": bf16(H)}
    for li in range(g["L"]):
        p = f"L{li}."
        out[p + "rms1"] = bf16(H)
        out[p + "rms2"] = bf16(H)
        out[p + "router"] = bf16(E, H)
        out[p + "shared.gate_up"] = bf16(2 * Is, H)
        out[p + "shared.down"] = bf16(H, Is)
        out[p + "shared.gate"] = bf16(H)
        out[p + "exp.gate_up.q4"] = rng.integers(0, 16, (E, 2 * I, H), dtype=np.uint8)
        out[p + "exp.gate_up.s"] = (0.01 * rng.random((E, 2 * I, H // G)) + 1e-3).astype(np.float16)
        out[p + "exp.down.q4"] = rng.integers(0, 16, (E, H, I), dtype=np.uint8)
        out[p + "exp.down.s"] = (0.01 * rng.random((E, H, I // G)) + 1e-3).astype(np.float16)
        out[p + ("gdn.A_log" if li == 0 else "attn.o")] = (
            rng.standard_normal(2).astype(np.float32) if li == 0 else bf16(H, 64))
    return out


def nibbles(q):
    """[N..., K] values 0..15 -> [N..., K/2] bytes, k = 2j in the low nibble (convert.py:154-156)."""
    return (q[..., 0::2] | (q[..., 1::2] << 4)).astype(np.uint8)


def entries(int8_shared=False, quant_int8=None):
    """(name, dtype, array) in the order the reference's converter adds them (convert.py:360-415)."""
    a = arrays()
    out = [("embed", "bf16", a["embed"]), ("final_norm", "bf16", a["final_norm"])]
    for li in range(GEOM["L"]):
        p = f"L{li}."
        out += [(p + "rms1", "bf16", a[p + "rms1"]), (p + "rms2", "bf16", a[p + "rms2"]),
                (p + "router", "bf16", a[p + "router"])]
        for nm in ("shared.gate_up", "shared.down"):
            if int8_shared:
                q, s = quant_int8(a[p + nm])
                out += [(p + nm + ".q8", "i8", q), (p + nm + ".s8", "f16", s)]
            else:
                out.append((p + nm, "bf16", a[p + nm]))
        out.append((p + "shared.gate", "bf16", a[p + "shared.gate"]))
        out += [(p + "exp.gate_up.q", "u8", nibbles(a[p + "exp.gate_up.q4"])),
                (p + "exp.gate_up.s", "f16", a[p + "exp.gate_up.s"]),
                (p + "exp.down.q", "u8", nibbles(a[p + "exp.down.q4"])),
                (p + "exp.down.s", "f16", a[p + "exp.down.s"])]
        extra = "gdn.A_log" if li == 0 else "attn.o"
        out.append((p + extra, "f32" if li == 0 else "bf16", a[p + extra]))
    return out


def _reference_convert(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "examples", "qwen"))
    import convert  # the reference's converter module (numpy + stdlib at import)
    return convert


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.dirname(os.path.abspath(__file__)))
    ap.add_argument("--reference", required=True, help="path to the reference checkout (holds examples/qwen)")
    args = ap.parse_args()
    conv = _reference_convert(args.reference)
    manifest = {"seed": SEED, "geometry": GEOM, "files": {}}
    for fname, int8 in (("ref_pack_tiny.mvccq", False), ("ref_pack_tiny_int8.mvccq", True)):
        with tempfile.TemporaryDirectory() as d:
            path = os.path.join(d, fname)
            w = conv.Writer(path)
            ents = entries(int8, lambda x: conv.quant_int8_rows(x, group=32))  # 128 exceeds the tiny rows
            for name, dtype, arr in ents:
                w.add(name, arr, dtype)
            cfg = config()
            if int8:
                cfg["dense"] = "int8"
            w.close(cfg)
            raw = open(path, "rb").read()
        with gzip.open(os.path.join(args.out, fname + ".gz"), "wb", compresslevel=9) as f:
            f.write(raw)
        manifest["files"][fname] = {
            "bytes": len(raw), "sha256": hashlib.sha256(raw).hexdigest(), "config": cfg,
            "tensors": {n: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest() for n, _, a in ents}}
    with open(os.path.join(args.out, "ref_pack_tiny.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    print("wrote", sorted(manifest["files"]))


if __name__ == "__main__":
    main()
