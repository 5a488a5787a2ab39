"""Generates the decode-stack golden vectors in tests/golden/ by running the reference's own CUDA kernels.

    make -C oracle ref REF=<reference checkout>          # builds oracle/_ref/libqk_ref.so
    python tests/golden/make_golden_stack.py --out tests/golden   # on a machine with a B200

The reference's attention branch (examples/qwen/kernels.cuh: attn_qk_norm_rope_kernel, attn_partial_kernel,
attn_combine_kernel, sigmoid_gate_kernel and the GEMVs, launched in the order of qwen.cu:413-425 with attention()'s
split count, qwen.cu:52-64) and its LM head (rmsnorm_kernel, the GEMV, argmax_partial_kernel and
argmax_final_kernel, qwen.cu:451-456) run through oracle/ref/qk_ref_shim.cu on seeded numpy inputs at a small
geometry that keeps the fixtures a few KB (H 512; 16 q heads, 2 kv heads, head_dim 256 as in the model; a 160-token
cache). Each case stores the outputs plus a SHA-256 of the regenerated inputs, so tests/test_golden_stack.py can
detect generator drift before comparing the oracle (oracle/decode_stack.py) with the reference.
"""
import argparse
import hashlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import decode_stack as S  # noqa: E402

ATTN = dict(H=512, Hq=16, Hkv=2, D=256, rope_dim=64, theta=1.0e7, eps=1e-6, ctx=160, gate=True)
ATTN_CASES = [("a_t1_p0", 1, 0, 201), ("a_t1_p100", 1, 100, 202), ("a_t3_p57", 3, 57, 203), ("a_t1_p159", 1, 159, 204)]
LM = dict(V=3000, H=512, eps=1e-6)
LM_SEED = 301


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        if a is not None:
            h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def attn_inputs(T, seed):
    """Seeded inputs of one attention case: weights (bf16 bits), caches, normed rows."""
    a = ATTN
    rng = np.random.default_rng(seed)
    nq, nqkv = a["Hq"] * a["D"], (a["Hq"] + 2 * a["Hkv"]) * a["D"]
    layer = {"qkv": S.bf16_bits(0.02 * rng.standard_normal((nqkv, a["H"]))),
             "gate": S.bf16_bits(0.02 * rng.standard_normal((nq, a["H"]))),
             "o": S.bf16_bits(0.02 * rng.standard_normal((a["H"], nq))),
             "q_norm": S.bf16_bits(1.0 + 0.1 * rng.standard_normal(a["D"])),
             "k_norm": S.bf16_bits(1.0 + 0.1 * rng.standard_normal(a["D"]))}
    kc = S.bf16_bits(rng.standard_normal((a["Hkv"], a["ctx"], a["D"])))
    vc = S.bf16_bits(rng.standard_normal((a["Hkv"], a["ctx"], a["D"])))
    normed = S.bf16_bits(rng.standard_normal((T, a["H"])))
    return layer, kc, vc, normed


def lm_inputs():
    rng = np.random.default_rng(LM_SEED)
    hidden = rng.standard_normal(LM["H"]).astype(np.float32)
    final_norm = S.bf16_bits(1.0 + 0.1 * rng.standard_normal(LM["H"]))
    head = S.bf16_bits(0.02 * rng.standard_normal((LM["V"], LM["H"])))
    return hidden, final_norm, head


def ref_attention(layer, kc, vc, normed, T, pos0):
    """The reference's attention branch on a B200 (oracle/_ref/libqk_ref.so); returns attn_out, q, kc, vc."""
    import ctypes

    import torch
    from oracle import ref_kernels as R
    a = ATTN
    lib = R.lib()
    lib.qkref_attn_forward.restype = ctypes.c_int
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).cuda()  # noqa: E731
    vp = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    nq, nqkv = a["Hq"] * a["D"], (a["Hq"] + 2 * a["Hkv"]) * a["D"]
    d = {k: dev(v) for k, v in layer.items()}
    kcd, vcd, x = dev(kc), dev(vc), dev(normed)
    qkv = torch.zeros(T, nqkv, dtype=torch.int16, device="cuda")
    z = torch.zeros(T, nq, dtype=torch.int16, device="cuda")
    q = torch.zeros(T, nq, dtype=torch.int16, device="cuda")
    o = torch.zeros(T, nq, dtype=torch.int16, device="cuda")
    part = torch.zeros(T * a["Hq"] * 32, a["D"] + 2, device="cuda")
    out = torch.zeros(T, a["H"], dtype=torch.int16, device="cuda")
    rc = lib.qkref_attn_forward(vp(x), vp(d["qkv"]), vp(d["gate"]) if a["gate"] else None, vp(d["o"]),
                                vp(d["q_norm"]), vp(d["k_norm"]), vp(kcd), vp(vcd), vp(qkv), vp(z), vp(q), vp(o),
                                vp(part), vp(out), T, a["H"], a["Hq"], a["Hkv"], a["D"], a["rope_dim"],
                                ctypes.c_float(a["theta"]), pos0, a["ctx"], ctypes.c_float(a["eps"]), None)
    torch.cuda.synchronize()
    if rc != 0:
        raise RuntimeError(f"reference attention failed: cudaError {rc}")
    h = lambda t: t.cpu().numpy().view(np.uint16)  # noqa: E731
    return h(out), h(q).reshape(T, a["Hq"], a["D"]), h(kcd), h(vcd)


def ref_lm_head(hidden, final_norm, head):
    import ctypes

    import torch
    from oracle import ref_kernels as R
    lib = R.lib()
    lib.qkref_lm_head.restype = ctypes.c_int
    vp = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    hd = torch.from_numpy(hidden).cuda()
    fn = torch.from_numpy(final_norm.view(np.int16)).cuda()
    wd = torch.from_numpy(head.view(np.int16)).cuda()
    normed = torch.zeros(LM["H"], dtype=torch.int16, device="cuda")
    logits = torch.zeros(LM["V"], device="cuda")
    pmax = torch.zeros(1024, device="cuda")
    pidx = torch.zeros(1024, dtype=torch.int32, device="cuda")
    nxt = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.qkref_lm_head(vp(hd), vp(fn), vp(wd), vp(normed), vp(logits), vp(pmax), vp(pidx), vp(nxt), LM["V"],
                           LM["H"], ctypes.c_float(LM["eps"]), None)
    torch.cuda.synchronize()
    if rc != 0:
        raise RuntimeError(f"reference LM head failed: cudaError {rc}")
    return logits.cpu().numpy(), int(nxt.item()), normed.cpu().numpy().view(np.uint16)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.dirname(os.path.abspath(__file__)))
    args = ap.parse_args()
    os.makedirs(args.out, exist_ok=True)
    meta = {"attn": ATTN, "lm": LM, "lm_seed": LM_SEED, "cases": {}}
    for name, T, pos0, seed in ATTN_CASES:
        layer, kc, vc, normed = attn_inputs(T, seed)
        out, q, kc2, vc2 = ref_attention(layer, kc, vc, normed, T, pos0)
        np.savez_compressed(os.path.join(args.out, f"ref_stack_{name}.npz"), attn_out=out, q=q,
                            k_new=kc2[:, pos0:pos0 + T], v_new=vc2[:, pos0:pos0 + T])
        meta["cases"][name] = {"T": T, "pos0": pos0, "seed": seed,
                               "inputs_sha256": digest(*[layer[k] for k in sorted(layer)], kc, vc, normed)}
        print(name, "attn_out[0,:4] =", out[0, :4].tolist())
    hidden, fnorm, head = lm_inputs()
    logits, nxt, normed = ref_lm_head(hidden, fnorm, head)
    np.savez_compressed(os.path.join(args.out, "ref_stack_lm.npz"), logits=logits, next=np.int32(nxt), normed=normed)
    meta["lm_sha256"] = digest(hidden, fnorm, head)
    print("lm next =", nxt)
    with open(os.path.join(args.out, "ref_stack_meta.json"), "w") as f:
        json.dump(meta, f, indent=1)


if __name__ == "__main__":
    main()
