#!/usr/bin/env python3
"""bench.py -- throughput of the B200 MoE block on BASELINE config 2 (int4 MoE decode).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl b200|reference]

One step is one pass of the MoE block (qwen.cu:429-448: RMSNorm, router + top-8, routed int4 experts, shared
expert, gated combine) over one decode batch of B tokens (default 1) for one layer, through the C ABI
(libmoe_b200.so). Weights (H=2048, E=256, top-8, I=Is=512, INT4 group 64) are generated on the device from a
seeded generator; each step uses the next of 32 distinct layer copies (13.7 GB), so no step reads weights a recent
step left in the 126 MB L2 (no flush needed). Steps are captured in CUDA graphs and timed with CUDA events on the
launching stream, bracketed by barrier + synchronize, max over ranks. Under torchrun (N > 1) every rank runs its
own replica (the decode block does not shard; expert-parallel prefill is the multi-GPU path).

`value`: tokens/s with weights and activations resident in HBM. `e2e`: the same steps with each step's input
(hidden fp32, attn_out bf16) copied from pinned host memory and its outputs (hidden, normed) copied back inside
the timed region. `roofline`: the dominant kernel (routed + shared gate/up), algorithmic bytes per launch over
its mean duration from graph-captured events. `cpu_baseline`: the C oracle (test infrastructure) on the host
cores, N=1 rank 0 only. `--impl reference` times the reference arm: the reference has no CPU implementation of
the block, so it is the oracle's restatement of the reference kernels, with every host thread.
"""
import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "int4 MoE decode tok/s + expert-GEMV HBM GB/s vs peak; EP prefill tok/s 1/2/4/8"
LAYER_COPIES = 32
GRAPH_STEPS = 256


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------ distributed plumbing

def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ clocks during the timed region

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        props = torch.cuda.get_device_properties(device)
        self.gpu = f"GPU-{props.uuid}" if getattr(props, "uuid", None) else str(device)
        self.samples = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        threading.Thread(target=self._read, daemon=True).start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), [c.strip() for c in line.split(",")]))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0, t1):
        win = [s for t, s in self.samples if t0 <= t <= t1]
        where = "timed region"
        if not win:
            win = [s for t, s in self.samples if t0 - 0.5 <= t <= t1 + 0.5]
            where = "within 0.5 s of the timed region"
        if not win:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        sm, smax = [], []
        for s in win:
            try:
                sm.append(float(s[1]))
                smax.append(float(s[2]))
            except (ValueError, IndexError):
                pass
            for i, n in enumerate(names):
                if len(s) > 5 + i and s[5 + i].lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(win), "window": where}


# ------------------------------------------------------------------ B200 arm

def algorithmic_bytes(shape, U, B):
    """Bytes the block must move per step (the reference's decode_weight_bytes terms, qwen.cu:463-477):
    router, U unique experts (gate/up + down weights and fp16 group scales), shared expert, norms, activations."""
    s = shape
    gu_exp = 2 * s.I * s.H // 2 + 2 * 2 * s.I * (s.H // s.G)
    dn_exp = s.H * s.I // 2 + 2 * s.H * (s.I // s.G)
    shared_gu = 2 * s.Is * s.H * 2
    shared_dn = s.H * s.Is * 2
    act = B * s.H * (4 + 2) + B * s.H * (4 + 2)  # hidden + attn_out in, hidden + normed out
    return {
        "route": s.E * s.H * 2 + 2 * s.H * 2 + B * s.H * 6,
        "gate_up": U * gu_exp + shared_gu,
        "down": U * dn_exp + shared_dn + B * s.H * 4 * 2,
        "experts": U * (gu_exp + dn_exp),
        "block": s.E * s.H * 2 + U * (gu_exp + dn_exp) + shared_gu + shared_dn + 2 * s.H * 2 + act,
    }


def capture(fn, steps, stream):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(steps):
            fn(i)
    return g


def run_graphs(graphs_counts, stream):
    """Replays on `stream` (CUDAGraph.replay launches on the current stream)."""
    with torch.cuda.stream(stream):
        for g, n in graphs_counts:
            for _ in range(n):
                g.replay()


def b200_arm(args, rank, world, local):
    import mvcc_b200 as m
    dev = torch.device("cuda", local)
    shape = m.MoeShape()
    B = args.batch
    K, W = args.steps, args.warmup
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        layers = [m.synth_layer(shape, seed=1000 + 97 * rank + i, stream=stream) for i in range(LAYER_COPIES)]
        blocks = [m.MoeBlock(l, B) for l in layers]
        hidden, attn = m.synth_activations(shape, B, seed=7 + rank, stream=stream)
        hidden0 = hidden.clone()
        normed = torch.zeros(B, shape.H, dtype=torch.int16, device=dev)
    torch.cuda.synchronize()

    def step(i):
        blocks[i % LAYER_COPIES].forward(hidden, attn, normed, stream=stream)

    # warm-up: W eager steps
    with torch.cuda.stream(stream):
        for i in range(W):
            step(i)
    torch.cuda.synchronize()
    # unique experts per step (B = 1: always TOPK), from the routing of one pass over the layer copies
    uniq = []
    for i in range(LAYER_COPIES):
        step(i)
        torch.cuda.synchronize()
        uniq.append(len(np.unique(blocks[i].trace(B)["idx"].cpu().numpy())))
    U = float(np.mean(uniq))
    hidden.copy_(hidden0)

    S = min(K, GRAPH_STEPS)
    g_main = capture(step, S, stream)
    rem = K % S
    g_rem = capture(step, rem, stream) if rem else None
    plan = [(g_main, K // S)] + ([(g_rem, 1)] if g_rem else [])
    run_graphs([(g_main, 1)], stream)  # graph upload, untimed
    torch.cuda.synchronize()

    clocks = ClockSampler(dev)
    clocks.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.time()
    e0.record(stream)
    run_graphs(plan, stream)
    e1.record(stream)
    torch.cuda.synchronize()
    t1 = time.time()
    barrier(world)
    clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    value = world * B * K / (ms / 1e3)

    # per-kernel durations from graph-captured events over the same steps
    evs = [[m.Event() for _ in range(4)] for _ in range(S)]
    g_ev = capture(lambda i: blocks[i % LAYER_COPIES].forward_events(hidden, attn, normed, evs[i], stream=stream),
                   S, stream)
    run_graphs([(g_ev, 1)], stream)
    torch.cuda.synchronize()
    reps = max(1, min(K // S, 8))
    acc = np.zeros(3)
    for _ in range(reps):
        run_graphs([(g_ev, 1)], stream)
        torch.cuda.synchronize()
        for e in evs:
            acc += [e[0].elapsed_ms(e[1]), e[1].elapsed_ms(e[2]), e[2].elapsed_ms(e[3])]
    stage_us = acc * 1e3 / (reps * S)

    # e2e: host-resident inputs and outputs copied inside the timed region
    h_in = hidden0.cpu().pin_memory()
    a_in = attn.cpu().pin_memory()
    h_out = torch.empty_like(h_in).pin_memory()
    n_out = torch.empty(normed.shape, dtype=normed.dtype).pin_memory()

    def e2e_step(i):
        hidden.copy_(h_in, non_blocking=True)
        attn.copy_(a_in, non_blocking=True)
        blocks[i % LAYER_COPIES].forward(hidden, attn, normed, stream=stream)
        h_out.copy_(hidden, non_blocking=True)
        n_out.copy_(normed, non_blocking=True)

    ge = capture(e2e_step, S, stream)
    ge_rem = capture(e2e_step, rem, stream) if rem else None
    plan_e = [(ge, K // S)] + ([(ge_rem, 1)] if ge_rem else [])
    run_graphs([(ge, 1)], stream)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0.record(stream)
    run_graphs(plan_e, stream)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms_e2e = max_over_ranks(e0.elapsed_time(e1), world)

    peak, peak_kind = load_peaks()
    ab = algorithmic_bytes(shape, U, B)
    gu_gbs = ab["gate_up"] / (stage_us[1] * 1e-6) / 1e9
    exp_gbs = (ab["gate_up"] + ab["down"]) / ((stage_us[1] + stage_us[2]) * 1e-6) / 1e9
    blk_gbs = ab["block"] / (ms / K * 1e-3) / 1e9
    result = {
        "metric": METRIC,
        "value": value,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": ms / K,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp32",
        "data": "synthetic (seeded device generator; bf16 N(0,0.02) weights, INT4 absmax/7 group-64 experts)",
        "config": {
            "workload": f"BASELINE config 2: one MoE layer, int4 G=64 experts, decode batch {B}",
            "H": shape.H, "E": shape.E, "topk": shape.TOPK, "I": shape.I, "Is": shape.Is, "G": shape.G,
            "batch": B, "layer_copies": LAYER_COPIES,
            "l2": f"inputs larger than L2: consecutive steps cycle over {LAYER_COPIES} layer copies "
                  f"({LAYER_COPIES * 428 / 1000:.1f} GB of weights); no flush",
            "parallelism": "replicas" if world > 1 else "single",
            "graph_steps": S,
        },
        "roofline": {
            "kernel": "gate_up_kernel (routed int4 gate/up + SiLU for the unique experts, shared gate/up)",
            "bound": "hbm", "achieved": gu_gbs, "peak": peak, "unit": "GB/s", "frac": gu_gbs / peak,
            "peak_kind": peak_kind, "bytes_per_launch": ab["gate_up"], "us_per_launch": stage_us[1],
            "traffic": None,
        },
        "expert_gemv": {"bytes_per_step": ab["gate_up"] + ab["down"], "us": stage_us[1] + stage_us[2],
                        "gbs": exp_gbs, "frac": exp_gbs / peak, "unique_experts": U},
        "block": {"bytes_per_step": ab["block"], "gbs": blk_gbs, "frac": blk_gbs / peak},
        "kernels_us": {"route": stage_us[0], "gate_up": stage_us[1], "down_combine": stage_us[2]},
        "e2e": {"value": world * B * K / (ms_e2e / 1e3), "unit": "tok/s",
                "h2d_bytes_per_step": B * shape.H * (4 + 2), "d2h_bytes_per_step": B * shape.H * (4 + 2)},
        "gpu_launches": 3 * K,
        "clocks": clocks.summary(t0, t1),
    }
    if world == 1 and rank == 0 and not args.no_cpu:
        result["cpu_baseline"] = cpu_baseline(layers[0], shape, B, args.cpu_seconds)
    return result


# ------------------------------------------------------------------ CPU oracle (baseline / reference arm)

def host_layer(layer):
    return {n: (v.cpu().numpy() if v.dtype == torch.uint8 else v.cpu().numpy().view(np.uint16))
            for n, v in layer.t.items()}


def time_oracle(L, shape, B, seconds, max_steps=None):
    from oracle import oracle as O
    orc = O.Oracle()
    n = orc.max_threads()
    orc.set_threads(n)
    s = O.Shape(H=shape.H, E=shape.E, TOPK=shape.TOPK, I=shape.I, Is=shape.Is, G=shape.G, eps=shape.eps)
    hidden, attn = O.make_activations(s, B, 3)
    orc.block_forward(s, L, hidden, attn, mode=0)  # warm
    steps = 0
    t0 = time.perf_counter()
    while True:
        orc.block_forward(s, L, hidden, attn, mode=0)
        steps += 1
        el = time.perf_counter() - t0
        if el >= seconds or (max_steps and steps >= max_steps):
            break
    return steps, el, n


def cpu_baseline(layer, shape, B, seconds):
    L = host_layer(layer)
    steps, el, n = time_oracle(L, shape, B, seconds)
    return {"value": steps * B / el, "unit": "tok/s", "cores": n, "kind": "port",
            "sample": f"{steps} decode steps of batch {B} through the C oracle of the block (decode numerics) on one "
                      f"layer, {el:.1f} s, {n} threads ({os.cpu_count()} logical CPUs)"}


def reference_arm(args, rank, world, local):
    if rank != 0:
        return None
    import mvcc_b200 as m
    shape = m.MoeShape()
    B = args.batch
    layer = m.synth_layer(shape, seed=1000)
    torch.cuda.synchronize()
    L = host_layer(layer)
    del layer
    from oracle import oracle as O
    orc = O.Oracle()
    orc.set_threads(orc.max_threads())
    s = O.Shape()
    hidden, attn = O.make_activations(s, B, 3)
    for _ in range(min(args.warmup, 3)):
        orc.block_forward(s, L, hidden, attn, mode=0)
    steps, el, n = time_oracle(L, shape, B, seconds=args.ref_seconds, max_steps=args.steps)
    value = steps * B / el
    sample = (f"{steps} of the {args.steps} requested decode steps (batch {B}) through the C oracle of the block "
              f"on the host cores, bounded to {args.ref_seconds:.0f} s; {n} threads")
    return {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": el / steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": f"BASELINE config 2: one MoE layer, int4 G=64 experts, decode batch {B}",
                   "H": shape.H, "E": shape.E, "topk": shape.TOPK, "I": shape.I, "Is": shape.Is, "G": shape.G,
                   "batch": B},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": n, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference implements the block only as CUDA kernels (examples/qwen/kernels.cuh); its CPU "
                "arm is the oracle's scalar restatement of those kernels",
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=64)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-seconds", type=float, default=60.0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank, world, local = dist_init()
    try:
        if args.impl == "reference":
            res = reference_arm(args, rank, world, local)
        else:
            res = b200_arm(args, rank, world, local)
        if rank == 0 and res is not None:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
