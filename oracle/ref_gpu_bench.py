"""Times the reference's own CUDA kernels (examples/qwen/kernels.cuh via oracle/_ref/libqk_ref.so) for the MoE block
on a B200, next to libmoe_b200 on the same device-generated weights.

    python oracle/ref_gpu_bench.py [--T 1 4 8 16] [--prefill 4096]

TEST INFRASTRUCTURE: a comparison harness, not the product benchmark (bench.py). The reference hard-codes INT4
group 128 (kernels.cuh:842), so both sides run group-128 weights here. Two timings per case:
  warm  the reference's own method (qwen.cu:486-498): one warm-up call, then `reps` calls on the same layer between
        two CUDA events; the ~21 MB a decode step touches stays in the 126 MB L2;
  cold  calls cycle over `layers` layer copies (as bench.py does), so weights come from HBM.
Both are captured in a CUDA graph per side, so host launch overhead is excluded for both.
"""
import argparse
import ctypes
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import mvcc_b200 as m  # noqa: E402
from oracle import ref_kernels as R  # noqa: E402


def ref_structs(layer, T):
    s = layer.shape
    Tp = (T + 127) // 128 * 128
    z = dict(device="cuda")
    buf = {
        "logits_r": torch.zeros(Tp, s.E, **z), "topk_i": torch.zeros(Tp, s.TOPK, dtype=torch.int32, **z),
        "topk_w": torch.zeros(Tp, s.TOPK, **z), "inter": torch.zeros(Tp, s.TOPK, s.I, dtype=torch.int16, **z),
        "routed": torch.zeros(Tp, s.H, **z), "moe_off": torch.zeros(s.E + 1, dtype=torch.int32, **z),
        "moe_sorted": torch.zeros(Tp * s.TOPK, dtype=torch.int32, **z),
        "slot_out": torch.zeros(Tp * s.TOPK, s.H, **z), "sgu": torch.zeros(Tp, 2 * s.Is, dtype=torch.int16, **z),
        "sinter": torch.zeros(Tp, s.Is, dtype=torch.int16, **z), "sout": torch.zeros(Tp, s.H, dtype=torch.int16, **z),
    }
    t = layer.t
    L = R._Layer(*[ctypes.c_void_p(t[n].data_ptr()) for n, _ in R._Layer._fields_[:9]], s.H, s.E, s.TOPK, s.I,
                 s.Is, s.eps)
    W = R._Work(*[ctypes.c_void_p(buf[n].data_ptr()) for n, _ in R._Work._fields_])
    return L, W, buf


def time_graph(fn, steps, stream, reps=5, min_seconds=0.25):
    """Mean us per step over graph replays; doubles the replay count until the timed region lasts min_seconds."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(steps):
            fn(i)
    with torch.cuda.stream(stream):
        for _ in range(3):
            g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    while True:
        with torch.cuda.stream(stream):
            e0.record()
            for _ in range(reps):
                g.replay()
            e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if ms >= min_seconds * 1e3 or reps >= 4096:
            return ms * 1e3 / (reps * steps)
        reps *= 2


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--T", type=int, nargs="+", default=[1, 4, 8, 16])
    ap.add_argument("--prefill", type=int, default=4096)
    ap.add_argument("--layers", type=int, default=16)
    args = ap.parse_args()
    lib = R.lib()
    lib.qkref_block_forward.restype = ctypes.c_int
    lib.qkref_moe.restype = ctypes.c_int
    shape = m.MoeShape(G=128)
    layers = [m.synth_layer(shape, seed=500 + i) for i in range(args.layers)]
    stream = torch.cuda.Stream()
    out = {"group": 128, "layers": args.layers, "decode": {}, "prefill": {}}
    for T in args.T:
        hid, attn = m.synth_activations(shape, T, 3)
        Tp = (T + 127) // 128 * 128
        h = torch.zeros(Tp, shape.H, device="cuda")
        h[:T] = hid
        a = torch.zeros(Tp, shape.H, dtype=torch.int16, device="cuda")
        a[:T] = attn
        normed = torch.zeros(Tp, shape.H, dtype=torch.int16, device="cuda")
        refs = [ref_structs(l, T) for l in layers]
        blocks = [m.MoeBlock(l, T) for l in layers]
        torch.cuda.synchronize()
        st = ctypes.c_void_p(stream.cuda_stream)

        def ref_step(i, cyc):
            L, W, _ = refs[i % args.layers if cyc else 0]
            rc = lib.qkref_block_forward(ctypes.byref(L), ctypes.byref(W), ctypes.c_void_p(h.data_ptr()),
                                         ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(normed.data_ptr()), None,
                                         T, st)
            assert rc == 0

        def our_step(i, cyc):
            blocks[i % args.layers if cyc else 0].forward(h[:T], a[:T], normed[:T], stream=stream)

        row = {}
        for name, fn in (("reference", ref_step), ("b200", our_step)):
            row[name] = {"warm_us": time_graph(lambda i: fn(i, False), 32, stream),
                         "cold_us": time_graph(lambda i: fn(i, True), 64, stream)}
        out["decode"][T] = row
        print(f"decode T={T}: " + json.dumps(row), flush=True)
        del refs, blocks
    if args.prefill:
        T = args.prefill
        x = torch.empty(T, shape.H, dtype=torch.int16, device="cuda")
        m._lib.moe_synth_normal_bf16(ctypes.c_void_p(x.data_ptr()), x.numel(), 9, 1, 0.0, 1.0,
                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        L, W, buf = ref_structs(layers[0], T)
        # routing from the reference's own router on these activations, as its bench does (qwen.cu:559-566)
        st = ctypes.c_void_p(stream.cuda_stream)
        with torch.cuda.stream(stream):
            lib.qkref_dense_f32(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(layers[0].t["router"].data_ptr()),
                                ctypes.c_void_p(buf["logits_r"].data_ptr()), T, shape.E, shape.H, st)
            lib.qkref_router_topk(ctypes.c_void_p(buf["logits_r"].data_ptr()), ctypes.c_void_p(buf["topk_i"].data_ptr()),
                                  ctypes.c_void_p(buf["topk_w"].data_ptr()), T, shape.E, shape.TOPK, st)
        torch.cuda.synchronize()
        us = time_graph(lambda i: lib.qkref_moe(ctypes.byref(L), ctypes.byref(W), ctypes.c_void_p(x.data_ptr()), T, st),
                        2, stream, reps=3)
        flops = 2.0 * T * shape.TOPK * 3 * shape.I * shape.H
        out["prefill"] = {"T": T, "reference_moe_us": us, "reference_moe_tflops": flops / (us * 1e-6) / 1e12}
        print(f"prefill T={T}: reference moe() {us:.1f} us, {flops / (us * 1e-6) / 1e12:.1f} TFLOP/s", flush=True)
    print(json.dumps(out))


if __name__ == "__main__":
    main()
