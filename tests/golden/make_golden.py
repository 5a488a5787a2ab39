"""Generates the golden vectors in tests/golden/ by running the reference's own CUDA kernels.

    make -C oracle ref REF=<reference checkout>   # builds oracle/_ref/libqk_ref.so
    python tests/golden/make_golden.py --out tests/golden   # on a machine with a B200

The reference's MoE block (examples/qwen/kernels.cuh launched in the order of qwen.cu:429-448, through
oracle/ref/qk_ref_shim.cu) runs on seeded inputs from oracle.make_layer / oracle.make_activations at the
reference's own geometry limits (group size 128, H % 1024 == 0, I % 512 == 0). Each case stores the outputs and
intermediates plus a SHA-256 of the regenerated inputs, so tests/test_golden.py can detect generator drift.
Cases with T < 8 exercise the reference's decode kernels, T >= 8 its sort + tensor-core tile kernels
(qwen.cu:347).
"""
import argparse
import hashlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

SHAPE = dict(H=1024, E=32, TOPK=8, I=512, Is=512, G=128, eps=1e-6)
LAYER_SEED = 7
CASES = [  # (name, T, activation seed, with next-layer norm)
    ("t1", 1, 101, False),
    ("t4_next", 4, 104, True),
    ("t16_tile", 16, 116, False),
    ("t40_tile_next", 40, 140, True),
]
KEEP = ("logits", "idx", "wts", "inter", "routed", "sout", "hidden", "normed")


def case_inputs(shape, T, seed, with_next):
    hidden, attn = O.make_activations(shape, T, seed)
    nr = O.f32_to_bf16(1.0 + 0.1 * O.normal(seed, 7, shape.H)) if with_next else None
    return hidden, attn, nr


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        if a is not None:
            h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def layer_digest(layer):
    return digest(*[layer[k] for k in sorted(layer)])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.dirname(os.path.abspath(__file__)))
    args = ap.parse_args()
    from oracle import ref_kernels as R
    shape = O.Shape(**SHAPE)
    layer = O.make_layer(shape, LAYER_SEED)
    os.makedirs(args.out, exist_ok=True)
    meta = {"shape": SHAPE, "layer_seed": LAYER_SEED, "layer_sha256": layer_digest(layer), "cases": {}}
    for name, T, seed, with_next in CASES:
        hidden, attn, nr = case_inputs(shape, T, seed, with_next)
        out = R.block_forward(shape, layer, hidden, attn, next_rms1=nr)
        keep = {k: out[k] for k in KEEP}
        if T > 16:
            keep.pop("inter")
        np.savez_compressed(os.path.join(args.out, f"ref_block_{name}.npz"), **keep)
        meta["cases"][name] = {"T": T, "seed": seed, "next": with_next,
                               "inputs_sha256": digest(hidden, attn, nr)}
        print(name, "idx[0] =", out["idx"][0].tolist())
    with open(os.path.join(args.out, "ref_block_meta.json"), "w") as f:
        json.dump(meta, f, indent=1)


if __name__ == "__main__":
    main()
