#!/usr/bin/env python3
"""bench.py -- throughput of the B200 MoE block on BASELINE configs 2 (int4 decode), 3 (the 40-layer decode stack),
4 (Zipf-skewed prefill) and 5 (expert-parallel prefill).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl b200|reference] [--quick]

Headline (`value`): one step is one pass of the MoE block (qwen.cu:429-448: residual RMSNorm,
router + top-8, routed int4 experts, shared expert, gated combine) over one decode batch of B tokens (default 1)
for one layer, through the C ABI (libmoe_b200.so). Weights (H=2048, E=256, top-8, I=Is=512, INT4 group 64, scales
absmax/7 of N(0, 0.02) weights) come from a seeded device generator; step i uses layer copy i mod 32 (13.7 GB in
all), so no step finds its weights in the 126 MB L2 (inputs larger than L2; no flush). Steps are captured in CUDA
graphs and timed with CUDA events on the launching stream, bracketed by barrier + synchronize, max over ranks.

Further objects on the same line:
  roofline        the dominant kernel of the headline step (the fused decode kernel: the whole block is one launch
                  for B < 8), algorithmic block bytes per launch over its mean duration from graph-captured events;
  expert_gemv, block
                  the headline step's expert-weight bytes and whole-block bytes over its time, as fractions of the
                  measured HBM peak;
  decode_batches  the other batch sizes of config 2 (1, 4, 16) on the default path selection, and batches 8 and 16
                  on the decode kernels (decode numerics) beside the default's tile path;
  g128            the library on group-128 layers (the group the reference's kernels hard-code), timed as the
                  reference arm's `ref_gpu` object times the reference's own kernels: decode batches 1-16 and the
                  routed experts of a 4096-token prefill (N = 1);
  decode_stack    BASELINE config 3: one token through 40 x (attention over a 4096-token cache, MoE block) and the
                  LM head with argmax, one CUDA graph per token, with the attention / MoE / LM-head split;
  prefill         BASELINE config 4: 4096 tokens through one layer with the per-expert Zipf(1.1) router bias:
                  tok/s, the tensor-pipe roofline of its dominant kernel (the routed gate/up grouped GEMM) and of
                  the whole block, its own e2e and clocks, and the C oracle on a bounded token sample;
  e2e             the headline steps with each step's input (hidden fp32, attn_out bf16) copied from pinned host
                  memory and its outputs (hidden, normed) copied back inside the timed region, one copy each way
                  (the tensors sit back to back in one device buffer), the copies on their own streams over two
                  buffer sets so that they overlap the neighbouring steps' kernels;
  ep_prefill      BASELINE config 5: 16384 tokens per step through one int4 MoE layer, the 256 experts sharded over
                  the N ranks (N = 1: the single-GPU prefill block; N > 1: mvcc_b200.ep, records and partial rows
                  moved by the kernels' peer-memory stores (or NCCL all-to-all with --ep-exchange nccl), each
                  rank holding 16384 / N of the tokens), tokens/s of the whole job from the max-over-ranks time
                  (`scaling` strong: the total work is fixed);
  pack_load       one full-geometry layer loaded from a .mvccq weight pack into HBM (the library's pack loader),
                  N = 1 only, skipped with --quick;
  cpu_baseline    the C oracle (test infrastructure) of the decode block on the host cores, N=1 rank 0 only.
Under torchrun (N > 1) every rank runs its own replica of the single-GPU workloads (`value`, decode_batches,
prefill; `scaling` weak: the decode block does not shard); ep_prefill is the sharded one.

`--impl reference` times the reference arm: the reference implements the block only as GPU kernels
(examples/qwen/kernels.cuh) and has no CPU code for it, so the arm is the oracle's restatement of those kernels on
every host thread; under torchrun only rank 0 runs it.
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
PREFILL_T = 4096
PREFILL_COPIES = 2
EP_TOKENS = 16384
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch from one ncu capture of the same kernel on the
# same workload: the fused decode kernel at batch 1, the routed gate/up GEMM at prefill T=4096 with the Zipf bias.
NCU_TRAFFIC = {"fused_b1": 20834304 + 0, "gate_up_t4096": 160367360 + 22692352}
DTYPE = "int4/bf16 weights, bf16 activations, fp32 accumulate"
DATA = ("synthetic (seeded device generator: bf16 N(0,0.02) weights, INT4 absmax/7 group-64 experts, "
        "activations N(0,1))")


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm": float(d["hbm_gbs"]), "tf_burst": float(d["bf16_tflops"]),
                "tf_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "kind": "measured"}
    return {"hbm": 6650.0, "tf_burst": 1590.0, "tf_sustained": 1400.0, "kind": "fallback"}


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
        time.sleep(0.3)

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


# ------------------------------------------------------------------ algorithmic work

def decode_bytes(s, U, B):
    """Bytes the block must move per decode step (the reference's decode_weight_bytes terms, qwen.cu:463-477):
    router, U unique experts (gate/up + down INT4 weights and fp16 group scales), shared expert, norm vectors,
    activations (hidden fp32 + attn_out bf16 in, hidden fp32 + normed bf16 out)."""
    gu_exp = 2 * s.I * s.H // 2 + 2 * 2 * s.I * (s.H // s.G)
    dn_exp = s.H * s.I // 2 + 2 * s.H * (s.I // s.G)
    shared = 2 * s.Is * s.H * 2 + s.H * s.Is * 2
    act = B * s.H * (4 + 2) * 2
    return {"experts": U * (gu_exp + dn_exp),
            "block": s.E * s.H * 2 + U * (gu_exp + dn_exp) + shared + 2 * s.H * 2 + act}


def prefill_flops(s, T):
    """Multiply-add FLOPs of the block for T tokens: router, TOPK routed experts (gate/up, down) and the shared
    expert per token."""
    router = 2 * T * s.H * s.E
    gate_up = 2 * T * s.TOPK * s.H * 2 * s.I
    down = 2 * T * s.TOPK * s.I * s.H
    shared = 2 * T * s.H * 2 * s.Is + 2 * T * s.Is * s.H
    return {"router": router, "gate_up": gate_up, "down": down, "shared": shared,
            "block": router + gate_up + down + shared}


# ------------------------------------------------------------------ graph timing helpers

def capture(fn, steps, stream):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(steps):
            fn(i)
    return g


def run_graphs(plan, stream):
    """Replays on `stream` (CUDAGraph.replay launches on the current stream)."""
    with torch.cuda.stream(stream):
        for g, n in plan:
            for _ in range(n):
                g.replay()


def graph_plan(step, K, stream):
    S = min(K, GRAPH_STEPS)
    g = capture(step, S, stream)
    rem = K % S
    plan = [(g, K // S)] + ([(capture(step, rem, stream), 1)] if rem else [])
    run_graphs([(g, 1)], stream)  # upload, untimed
    torch.cuda.synchronize()
    return plan


def timed(plan, stream, world, clocks=None):
    """Device time (ms) of the plan, barrier + synchronize on both sides, max over ranks; clocks sampled inside."""
    if clocks is not None:
        clocks.start()
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
    clk = None
    if clocks is not None:
        clocks.stop()
        clk = clocks.summary(t0, t1)
    return max_over_ranks(e0.elapsed_time(e1), world), clk


def stage_times(m, fwd_events, S, reps, stream):
    """Mean per-stage durations (us) over S graph-captured steps replayed `reps` times: the four events the library
    records around one block (start, after routing, after gate/up, end)."""
    evs = [[m.Event() for _ in range(4)] for _ in range(S)]
    g = capture(lambda i: fwd_events(i, evs[i]), S, stream)
    run_graphs([(g, 1)], stream)
    torch.cuda.synchronize()
    acc = np.zeros(3)
    for _ in range(reps):
        run_graphs([(g, 1)], stream)
        torch.cuda.synchronize()
        for e in evs:
            acc += [e[0].elapsed_ms(e[1]), e[1].elapsed_ms(e[2]), e[2].elapsed_ms(e[3])]
    return acc * 1e3 / (reps * S)


def packed_io(hidden, attn, normed):
    """One device buffer holding a step's inputs and outputs back to back -- attn_out (bf16), hidden (fp32, in and
    out), normed (bf16) -- so that the inputs are one contiguous range (attn_out + hidden) and the results another
    (hidden + normed): one host-to-device and one device-to-host copy per step. Returns the buffer, the three views
    (initialised from the given tensors) and the input and output ranges."""
    T, H = hidden.shape
    na, nh, nn = attn.numel() * 2, hidden.numel() * 4, normed.numel() * 2
    buf = torch.empty(na + nh + nn, dtype=torch.uint8, device=hidden.device)
    a_v = buf[:na].view(torch.int16).view(T, H)
    h_v = buf[na:na + nh].view(torch.float32).view(T, H)
    n_v = buf[na + nh:].view(torch.int16).view(T, H)
    a_v.copy_(attn)
    h_v.copy_(hidden)
    n_v.copy_(normed)
    return buf, a_v, h_v, n_v, buf[:na + nh], buf[na:]


def e2e_time(block_at, hidden, attn, normed, K, stream, world):
    """The same steps fed from pinned host memory: inside the timed region, every step copies its inputs (attn_out
    + hidden, one contiguous range) host-to-device and its results (hidden + normed) device-to-host. As a server
    would, the copies run on their own streams over two device buffer sets: step i + 1's inputs land while step i
    computes and step i's results leave while step i + 1 computes (a step's inputs do not depend on the previous
    step's results here). Every step's two copies are inside the timed region."""
    sets = [packed_io(hidden, attn, normed) for _ in range(2)]
    host_in = sets[0][4].cpu().pin_memory()
    host_out = [torch.empty(sets[0][5].numel(), dtype=torch.uint8).pin_memory() for _ in range(2)]
    dev = hidden.device
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    fork = torch.cuda.Event()
    ready = [torch.cuda.Event() for _ in range(2)]     # a set's inputs have landed
    computed = [torch.cuda.Event() for _ in range(2)]  # a set's step has run
    drained = [torch.cuda.Event() for _ in range(2)]   # a set's results have left

    def steps(n):
        fork.record(stream)
        s_in.wait_event(fork)
        s_out.wait_event(fork)
        for i in range(n):
            b = i % 2
            _, a_v, h_v, n_v, inp, out = sets[b]
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(drained[b])  # step i - 2's results have left this set
                inp.copy_(host_in, non_blocking=True)
                ready[b].record(s_in)
            stream.wait_event(ready[b])
            block_at(i).forward(h_v, a_v, n_v, stream=stream)
            computed[b].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(computed[b])
                host_out[b].copy_(out, non_blocking=True)
                drained[b].record(s_out)
        stream.wait_event(drained[(n - 1) % 2])  # join: the last results (s_out runs in order)
        stream.wait_event(ready[(n - 1) % 2])

    def cap(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            steps(n)
        return g

    S = min(K, GRAPH_STEPS)
    plan = [(cap(S), K // S)] + ([(cap(K % S), 1)] if K % S else [])
    run_graphs([(plan[0][0], 1)], stream)  # upload, untimed
    torch.cuda.synchronize()
    ms, _ = timed(plan, stream, world)
    return ms, host_in.numel(), host_out[0].numel()


def launches_per_step(T, fused_max=7, prefill_min=8, chunk=16):
    """Kernels of this library one block launches: the fused decode kernel (T < 8), three per decode chunk, or the
    prefill sequence (norm, router GEMM, top-k, sort scan, sort scatter, gate/up GEMM, down GEMM, two shared-expert
    GEMMs, combine)."""
    if T >= prefill_min:
        return 10
    if T <= fused_max:
        return 1
    return 3 * ((T + chunk - 1) // chunk)


def counted_launches(m, fn):
    """Kernel launches the library issued while fn() ran, read from its own counter (moe_stats_get); None if the
    counter cannot be read."""
    try:
        before = m.stats()["launches"]
        fn()
        torch.cuda.synchronize()
        return int(m.stats()["launches"] - before)
    except Exception:  # noqa: BLE001 -- the launch plan's formula stands in
        return None


def launches_claim(per_step_counted, T, K):
    """gpu_launches for K steps: the counted launches of one step when available, else the launch plan's count."""
    if per_step_counted is not None:
        return per_step_counted * K, "library counter (moe_stats_get) over one untimed step, times the timed steps"
    return launches_per_step(T) * K, "launch plan of the path (counter unavailable)"


# ------------------------------------------------------------------ B200 arm

def decode_case(m, shape, blocks, B, K, W, stream, world, dev, clocks=None):
    hidden, attn = m.synth_activations(shape, B, seed=7, stream=stream)
    normed = torch.zeros(B, shape.H, dtype=torch.int16, device=dev)
    torch.cuda.synchronize()
    blk = [m.MoeBlock(b.layer, B) for b in blocks] if blocks[0].max_T < B else blocks
    step = lambda i: blk[i % len(blk)].forward(hidden, attn, normed, stream=stream)  # noqa: E731
    with torch.cuda.stream(stream):
        for i in range(W):
            step(i)
    torch.cuda.synchronize()
    uniq = []
    for i in range(len(blk)):
        step(i)
        torch.cuda.synchronize()
        uniq.append(len(np.unique(blk[i].trace(B)["idx"].cpu().numpy())))
    U = float(np.mean(uniq))
    per = counted_launches(m, lambda: step(0))
    hidden0 = hidden.clone()
    ms, clk = timed(graph_plan(step, K, stream), stream, world, clocks)
    S = min(K, GRAPH_STEPS)
    st = stage_times(m, lambda i, ev: blk[i % len(blk)].forward_events(hidden, attn, normed, ev, stream=stream),
                     S, max(1, min(K // S, 8)), stream)
    hidden.copy_(hidden0)
    ms_e2e, hb, db = e2e_time(lambda i: blk[i % len(blk)], hidden, attn, normed, K, stream, world)
    return {"ms": ms, "U": U, "stage_us": st, "clocks": clk, "ms_e2e": ms_e2e, "h2d": hb, "d2h": db,
            "launches_per_step": per}


def prefill_case(m, shape, K, W, stream, world, dev, peaks, cpu_seconds, do_cpu):
    T = PREFILL_T
    bias = torch.from_numpy(m.zipf_bias(shape.E, seed=0)).to(dev)
    layers = []
    for c in range(PREFILL_COPIES):
        base = m.synth_layer(shape, seed=2000 + c, stream=stream)
        t = dict(base.t)
        t["router_bias"] = bias
        layers.append(m.MoeLayer(shape, t))
    blocks = [m.MoeBlock(l, T) for l in layers]
    hidden, attn = m.synth_activations(shape, T, seed=17, stream=stream)
    normed = torch.zeros(T, shape.H, dtype=torch.int16, device=dev)
    torch.cuda.synchronize()
    hidden0 = hidden.clone()
    step = lambda i: blocks[i % PREFILL_COPIES].forward(hidden, attn, normed, stream=stream)  # noqa: E731
    with torch.cuda.stream(stream):
        for i in range(W):
            step(i)
    torch.cuda.synchronize()
    tr = blocks[(W - 1) % PREFILL_COPIES].trace(T)
    idx = tr["idx"].cpu().numpy()
    per = counted_launches(m, lambda: step(W))
    load = np.bincount(idx.ravel(), minlength=shape.E)
    err = blocks[0].error_word() | blocks[1 % PREFILL_COPIES].error_word()
    ms, clk = timed(graph_plan(step, K, stream), stream, world, ClockSampler(dev))
    st = stage_times(m, lambda i, ev: blocks[i % PREFILL_COPIES].forward_events(hidden, attn, normed, ev,
                                                                                  stream=stream),
                     min(K, 16), 2, stream)
    hidden.copy_(hidden0)
    ms_e2e, hb, db = e2e_time(lambda i: blocks[i % PREFILL_COPIES], hidden, attn, normed, K, stream, world)
    fl = prefill_flops(shape, T)
    step_us = ms / K * 1e3
    gu_tf = fl["gate_up"] / (st[1] * 1e-6) / 1e12
    blk_tf = fl["block"] / (step_us * 1e-6) / 1e12
    out = {
        "workload": f"BASELINE config 4: prefill of {T} tokens through one int4 G=64 MoE layer, router logits + "
                    f"per-expert Zipf(1.1) bias b_e = -1.1 ln(1 + pi(e)), pi a seed-0 permutation",
        "tokens": T, "value": world * T * K / (ms / 1e3), "unit": "tok/s", "ms_per_step": ms / K, "steps": K,
        "layer_copies": PREFILL_COPIES,
        "l2": f"inputs larger than L2: steps alternate over {PREFILL_COPIES} layer copies (428 MB of weights each); "
              "no flush",
        "expert_load": {"max_pairs": int(load.max()), "mean_pairs": float(load.mean()),
                        "top8_share": float(np.sort(load)[::-1][:8].sum() / load.sum()),
                        "experts_used": int((load > 0).sum())},
        "stages_us": {"route_sort": st[0], "gate_up_gemm": st[1], "down_shared_combine": st[2]},
        "roofline": {"kernel": "moe_gemm_kernel<256, INT4, EPI_SILU_TILE> (routed gate/up grouped GEMM + SiLU)",
                     "bound": "tensor", "achieved": gu_tf, "peak": peaks["tf_sustained"], "unit": "TFLOP/s",
                     "frac": gu_tf / peaks["tf_sustained"],
                     "peak_kind": f"{peaks['kind']} bf16 sustained",
                     "flops_per_launch": fl["gate_up"], "us_per_launch": st[1],
                     "traffic": NCU_TRAFFIC["gate_up_t4096"]},
        "block_tflops": {"achieved": blk_tf, "frac": blk_tf / peaks["tf_sustained"], "flops_per_step": fl["block"]},
        "e2e": {"value": world * T * K / (ms_e2e / 1e3), "unit": "tok/s", "h2d_bytes_per_step": hb,
                "d2h_bytes_per_step": db},
        "gpu_launches": launches_claim(per, T, K)[0],
        "gpu_launches_source": launches_claim(per, T, K)[1],
        "error_word": err,
        "clocks": clk,
    }
    if do_cpu:
        out["cpu_baseline"] = cpu_prefill(layers[0], shape, bias.cpu().numpy(), cpu_seconds)
    return out


def ep_parity(m, shape, layer, hidden0, attn, hidden_out, normed_out, world, rank, rows=64):
    """Parity of one untimed expert-parallel step on this rank against the oracle's expert-parallel restatement
    (oracle.ep_block_forward: tile numerics, per-rank slot-order partials summed in rank order), on a seeded sample
    of this rank's tokens; each token's outputs depend on that token alone. The oracle is the checker here, outside
    the timed region. Tokens whose 8th/9th router logits lie within twice the GPU-vs-oracle logit difference can
    route differently and are left out of the value comparison (counted in `excluded`)."""
    from oracle import oracle as O
    T = hidden0.shape[0]
    sel = np.sort(np.random.default_rng(1000 + rank).choice(T, min(rows, T), replace=False))
    L = host_layer(layer)
    orc = O.Oracle()
    orc.set_threads(max(1, (os.cpu_count() or 1) // world))
    s = oracle_shape(shape)
    h_in = hidden0[sel].cpu().numpy()
    a_in = attn[sel].cpu().numpy().view(np.uint16)
    ref = orc.ep_block_forward(s, L, h_in, a_in, world)
    # the GPU's own logits for the sample: the router on the GPU's normed rows (the step's router input)
    n = len(sel)
    blk = m.MoeBlock(layer, n)
    lg = torch.zeros(n, shape.E, device=hidden0.device)
    blk.router_topk(normed_out[sel].contiguous(), lg, torch.zeros(n, shape.TOPK, dtype=torch.int32,
                                                                  device=hidden0.device),
                    torch.zeros(n, shape.TOPK, device=hidden0.device))
    torch.cuda.synchronize()
    gl = lg.cpu().numpy()
    srt = np.sort(ref["logits"], axis=1)[:, ::-1]
    margin = srt[:, shape.TOPK - 1] - srt[:, shape.TOPK]
    ok = margin > 2 * np.abs(gl - ref["logits"]).max(axis=1) + 1e-6
    gh = hidden_out[sel].cpu().numpy()
    gn = normed_out[sel].cpu().numpy().view(np.uint16)
    err_h = float(O.max_rel_err(gh[ok], ref["hidden"][ok])) if ok.any() else None
    err_n = float(O.max_rel_err(O.bf16_to_f32(gn[ok]), O.bf16_to_f32(ref["normed"][ok]))) if ok.any() else None
    return {"rows": int(n), "excluded": int((~ok).sum()), "min_topk_margin": float(margin.min()),
            "max_rel_err_hidden": err_h, "max_rel_err_normed": err_n,
            "pass": bool(ok.mean() >= 0.9 and err_h is not None and err_h < 1e-2 and err_n < 1e-2)}


def ep_case(m, shape, K, W, stream, world, rank, dev, peaks, exchange="peers", parity=True):
    """Config 5: EP_TOKENS tokens per step over `world` ranks, experts sharded evenly, device time max over ranks."""
    T = EP_TOKENS // world
    peer_note = None
    with torch.cuda.stream(stream):
        layer = m.synth_layer(shape, seed=3000, stream=stream)  # same weights on every rank; each keeps its shard
        hidden, attn = m.synth_activations(shape, T, seed=31 + rank, stream=stream)
    normed = torch.zeros(T, shape.H, dtype=torch.int16, device=dev)
    torch.cuda.synchronize()
    hidden0 = hidden.clone()
    if world == 1:
        blk = m.MoeBlock(layer, T)
        step = lambda i: blk.forward(hidden, attn, normed, stream=stream)  # noqa: E731
        with torch.cuda.stream(stream):
            for i in range(W):
                step(i)
        torch.cuda.synchronize()
        ms, clk = timed(graph_plan(step, K, stream), stream, world, ClockSampler(dev))
        how = "single GPU: moe_block_forward prefill path (CUDA graph)"
        recv = None
        stages = None
        hidden.copy_(hidden0)
        step(0)
        torch.cuda.synchronize()
        h_out, n_out = hidden.clone(), normed.clone()
    else:
        import mvcc_b200.ep as ep
        st = ep.EpRank(layer, rank, world, T)
        ex = ep.NcclExchange()
        sizes = []
        flag = torch.zeros(1, device=dev)
        if exchange == "peers":
            # every rank maps the peers' buffers; if any rank cannot, all fall back to the NCCL exchange together
            fail = ""
            try:
                st.open_peers()
            except Exception as e:  # noqa: BLE001 - reported in the JSON line
                fail = f"{type(e).__name__}: {e}"
            ok = torch.tensor([0.0 if fail else 1.0], device=dev)
            torch.distributed.all_reduce(ok, op=torch.distributed.ReduceOp.MIN)
            if ok.item() < 1.0:
                st.close_peers()
                exchange = "nccl"
                peer_note = f"peer mapping unavailable, NCCL exchange used ({fail or 'on another rank'})"
        if exchange == "peers":
            step = lambda i: ep.ep_step_peers(st, hidden, attn, normed, stream=stream, flag=flag)  # noqa: E731
        else:
            step = lambda i: sizes.append(ep.ep_step(st, ex, hidden, attn, normed, stream=stream))  # noqa: E731
        for i in range(W):
            step(i)
        torch.cuda.synchronize()
        sizes.clear()
        clocks = ClockSampler(dev)
        clocks.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize()
        t0 = time.time()
        e0.record(stream)
        for i in range(K):
            step(i)
        e1.record(stream)
        torch.cuda.synchronize()
        t1 = time.time()
        barrier(world)
        clocks.stop()
        clk = clocks.summary(t0, t1)
        ms = max_over_ranks(e0.elapsed_time(e1), world)
        if exchange == "peers":
            how = (f"mvcc_b200.ep: {shape.E // world} experts per rank; the dispatch kernel stores each record into the "
                   "destination rank's buffer and the expert stage stores each partial row into the source rank's "
                   "buffer over NVLink (CUDA IPC mappings), a one-element NCCL all-reduce after each as the barrier; "
                   "no host synchronisation; shared expert on a side stream")
            counts = st.send_count.cpu().numpy()
            recv = {"records_sent_last_step": int(counts.sum())}
        else:
            how = (f"mvcc_b200.ep: {shape.E // world} experts per rank; count matrix all-gathered (one host read per "
                   "step, checked on every rank), records and partial rows exchanged with NCCL all_to_all_single; "
                   "shared expert on a side stream")
            recv = {"records_sent_per_step": float(np.mean([s for s, _ in sizes])),
                    "records_received_per_step": float(np.mean([r for _, r in sizes]))}
        stages = None
        if exchange == "peers":  # one untimed step with events between its stages, max over ranks per stage
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
            hidden.copy_(hidden0)
            ep.ep_step_peers(st, hidden, attn, normed, stream=stream, flag=flag, events=evs)
            torch.cuda.synchronize()
            stages = {n: max_over_ranks(evs[i].elapsed_time(evs[i + 1]), world) for i, n in enumerate(ep.EP_STAGES)}
        hidden.copy_(hidden0)
        sizes.clear()
        step(0)  # the untimed step whose outputs the parity check reads
        torch.cuda.synchronize()
        h_out, n_out = hidden.clone(), normed.clone()
        assert st.error_word() == 0
        barrier(world)
        st.close_peers()
    hidden.copy_(hidden0)
    fl = prefill_flops(shape, EP_TOKENS)
    tf = fl["block"] / (ms / K * 1e-3) / 1e12
    out = {"workload": f"BASELINE config 5: {EP_TOKENS} tokens per step through one int4 G=64 MoE layer, experts "
                       f"sharded over {world} GPU(s), {T} tokens per rank",
           "value": EP_TOKENS * K / (ms / 1e3), "unit": "tok/s", "ms_per_step": ms / K, "steps": K,
           "n_gpus": world, "scaling": "strong", "how": how,
           "tflops": {"achieved_job": tf, "per_gpu": tf / world, "frac_per_gpu": tf / world / peaks["tf_sustained"],
                      "peak_kind": f"{peaks['kind']} bf16 sustained", "flops_per_step": fl["block"]},
           "exchange": "none (one GPU)" if world == 1 else exchange,
           "gpu_launches_per_step_per_rank": launches_per_step(T) if world == 1 else 14,
           "clocks": clk}
    if recv:
        out["exchange_stats"] = recv
    if stages:
        out["stages_ms"] = stages
        out["stages_note"] = ("one untimed step with CUDA events between its stages on the launching stream, each stage "
                              "the max over ranks; the barriers include waiting for the slowest rank")
    if peer_note:
        out["note"] = peer_note
    if parity:
        try:
            p = ep_parity(m, shape, layer, hidden0, attn, h_out, n_out, world, rank)
        except Exception as e:  # noqa: BLE001 -- reported in the JSON line
            p = {"error": f"{type(e).__name__}: {e}"}
        if world > 1:  # every rank's result, gathered to rank 0
            allp = [None] * world
            torch.distributed.all_gather_object(allp, p)
            out["parity"] = {"per_rank": allp,
                             "pass": all(isinstance(q, dict) and q.get("pass") for q in allp)}
        else:
            out["parity"] = {"per_rank": [p], "pass": bool(p.get("pass"))}
    return out


def pack_load_case(m, shape, reps=3):
    """One full-geometry layer loaded from a .mvccq pack into HBM through the library's loader
    (moe_pack_upload_layer; the reference's Model::load lines, qwen.cu:181-190): random bytes in the pack layout,
    written once to a temporary file, then read from the page cache and copied to the device `reps` times; best of
    the reps, host wall clock around the call and a device synchronize. Failures are reported, not raised."""
    import tempfile
    from mvcc_b200 import pack
    try:
        s = shape
        rng = np.random.default_rng(0)

        def u16(*shp):
            return rng.integers(0, 1 << 16, shp, dtype=np.uint16)

        def u8(*shp):
            return rng.integers(0, 256, shp, dtype=np.uint8)

        t = {"rms2": u16(s.H), "router": u16(s.E, s.H), "exp_gu_q": u8(s.E, 2 * s.I, s.H // 2),
             "exp_gu_s": u16(s.E, 2 * s.I, s.H // s.G), "exp_dn_q": u8(s.E, s.H, s.I // 2),
             "exp_dn_s": u16(s.E, s.H, s.I // s.G), "shared_gate_up": u16(2 * s.Is, s.H),
             "shared_down": u16(s.H, s.Is), "shared_gate": u16(s.H)}
        with tempfile.TemporaryDirectory() as d:
            path = pack.write_pack(os.path.join(d, "layer.mvccq"), pack.pack_config(s, 1), pack.block_entries(0, t))
            del t
            best = None
            with pack.MoePack(path) as pk:
                n = pk.layer_bytes(0)
                for _ in range(reps):
                    torch.cuda.synchronize()
                    t0 = time.perf_counter()
                    ml = pk.layer(0)
                    torch.cuda.synchronize()
                    dt = time.perf_counter() - t0
                    best = dt if best is None else min(best, dt)
                    del ml
        return {"bytes": n, "ms": best * 1e3, "gbs": n / best / 1e9, "reps": reps,
                "how": "moe_pack_upload_layer: page-cached file mapping -> one pageable host-to-device copy per "
                       "tensor, 256-byte aligned in one device region; best of reps"}
    except Exception as e:  # noqa: BLE001 -- reported in the JSON line
        return {"error": f"{type(e).__name__}: {e}"}


def decode_config(shape, B, world, K, layer_copies):
    """The `config` object of the headline line; the reference arm prints the identical dict."""
    return {
        "workload": f"BASELINE config 2: one MoE layer, int4 G=64 experts, decode batch {B}",
        "H": shape.H, "E": shape.E, "topk": shape.TOPK, "I": shape.I, "Is": shape.Is, "G": shape.G,
        "batch": B, "layer_copies": layer_copies,
        "l2": f"inputs larger than L2: consecutive steps cycle over {layer_copies} layer copies "
              f"({layer_copies * 0.428:.1f} GB of weights); no flush",
        "parallelism": f"replicas x{world}" if world > 1 else "single",
        "graph_steps": min(K, GRAPH_STEPS),
    }


def time_graph_us(fn, steps, stream, reps=5, min_seconds=0.25):
    """Mean us per step over replays of a graph of `steps` calls of fn(i); doubles the replay count until the timed
    region lasts min_seconds (CUDA events on the launching stream)."""
    g = capture(fn, steps, stream)
    run_graphs([(g, 3)], stream)
    torch.cuda.synchronize()
    while True:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        run_graphs([(g, reps)], stream)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if ms >= min_seconds * 1e3 or reps >= 4096:
            return ms * 1e3 / (reps * steps)
        reps *= 2


def g128_case(m, stream, copies=16, Ts=(1, 4, 8, 16), prefill_T=4096):
    """This library at INT4 group 128 -- the group the reference's kernels hard-code (kernels.cuh:842) -- timed the
    way the reference arm's `ref_gpu` object times the reference's own kernels: decode blocks warm (one layer, the
    reference's time_ms method, qwen.cu:486-498) and cold (layer copies cycled), and the routed experts of a
    4096-token prefill on its own router's routing of N(0,1) activations."""
    shape = m.MoeShape(G=128)
    with torch.cuda.stream(stream):
        layers = [m.synth_layer(shape, seed=500 + i, stream=stream) for i in range(copies)]
    torch.cuda.synchronize()
    out = {"group": 128, "layer_copies": copies, "decode_us": {}}
    for T in Ts:
        hid, attn = m.synth_activations(shape, T, 3, stream=stream)
        normed = torch.zeros(T, shape.H, dtype=torch.int16, device=hid.device)
        blocks = [m.MoeBlock(l, T) for l in layers]
        torch.cuda.synchronize()
        out["decode_us"][str(T)] = {
            "warm": time_graph_us(lambda i: blocks[0].forward(hid, attn, normed, stream=stream), 32, stream),
            "cold": time_graph_us(lambda i: blocks[i % copies].forward(hid, attn, normed, stream=stream), 64, stream)}
        del blocks
    T = prefill_T
    blk = m.MoeBlock(layers[0], T)
    x = torch.empty(T, shape.H, dtype=torch.int16, device="cuda")
    m._check(m._lib.moe_synth_normal_bf16(m._ptr(x), x.numel(), 9, 1, 0.0, 1.0, m._stream(stream)), "synth")
    logits = torch.zeros(T, shape.E, device="cuda")
    idx = torch.zeros(T, shape.TOPK, dtype=torch.int32, device="cuda")
    wts = torch.zeros(T, shape.TOPK, device="cuda")
    routed = torch.zeros(T, shape.H, device="cuda")
    blk.router_topk(x, logits, idx, wts, stream=stream)
    torch.cuda.synchronize()
    us = time_graph_us(lambda i: blk.routed_experts(x, idx, wts, routed, stream=stream), 2, stream, reps=3)
    flops = 2.0 * T * shape.TOPK * 3 * shape.I * shape.H
    out["prefill_routed"] = {"T": T, "us": us, "tflops": flops / (us * 1e-6) / 1e12}
    return out


def decode_stack_case(m, stream, world, peaks, tokens=16, W=3):
    """a 40-layer decode step at batch 1 -- per layer RMSNorm -> GQA attention (16 q heads, 2 kv
    heads, head_dim 256, bf16 caches of 4096 tokens ~N(0,1)) -> RMSNorm -> the int4 G=64 MoE block; final RMSNorm and
    the bf16 LM head of 2048 x 151936 with argmax. The caches hold 4096 positions and every step decodes position
    4095, so each step reads all 4096 keys. Steps captured in one CUDA graph, CUDA events on the launching stream;
    every step restores the residual input first (an 8 KB device copy)."""
    from mvcc_b200 import stack as st
    stk = st.DecodeStack(L=40, ctx=4096, vocab=151936, seed=5)
    hidden0, _ = m.synth_activations(stk.moe_shape, 1, seed=41, stream=stream)
    hidden = hidden0.clone()
    torch.cuda.synchronize()

    def step(i):
        hidden.copy_(hidden0)
        stk.step(hidden, 4095, stream=stream)

    with torch.cuda.stream(stream):
        for i in range(W):
            step(i)
    torch.cuda.synchronize()
    per = counted_launches(m, lambda: step(0))
    ms, clk = timed(graph_plan(step, tokens, stream), stream, world, ClockSampler(torch.device("cuda")))
    us = ms / tokens * 1e3
    nb = stk.weight_bytes()
    gbs = nb / (us * 1e-6) / 1e9
    next_token = int(stk.next.item())

    # the same pieces timed apart (each its own graph of `tokens` repetitions): the 40 attention layers, the 40 MoE
    # blocks, the LM head with argmax; their sum exceeds the step by the overlap programmatic launch gives across
    # the pieces' boundaries
    a_sh = stk.attn_shape
    normed, attn_out = stk.normed[:1], stk.attn_out[:1]

    def attn_only(i):
        for j in range(stk.L):
            stk.attn[j].forward_rms(hidden, stk.rms1[j], attn_out, 4095, T=1, stream=stream)

    def moe_only(i):
        hidden.copy_(hidden0)
        for j in range(stk.L):
            nxt = stk.final_norm if j + 1 == stk.L else None
            stk.moe[j].forward(hidden, attn_out, normed, next_rms1=nxt, T=1, stream=stream)

    def head_only(i):
        stk.head.argmax(stk.normed[0], stk.next, stream=stream)

    split = {}
    for name, fn in (("attention", attn_only), ("moe", moe_only), ("lm_head", head_only)):
        sms, _ = timed(graph_plan(fn, tokens, stream), stream, world)
        split[name] = sms / tokens
    kv = 2 * a_sh.Hkv * stk.ctx * a_sh.D * 2
    attn_bytes = stk.L * (a_sh.weight_bytes() + kv)
    head_bytes = stk.V * a_sh.H * 2
    stage_frac = {"attention": attn_bytes / (split["attention"] * 1e-3) / 1e9 / peaks["hbm"],
                  "moe": (nb - attn_bytes - head_bytes) / (split["moe"] * 1e-3) / 1e9 / peaks["hbm"],
                  "lm_head": head_bytes / (split["lm_head"] * 1e-3) / 1e9 / peaks["hbm"]}
    hidden.copy_(hidden0)
    out = {"workload": "BASELINE config 3: 40 x (RMSNorm, GQA attention Hq 16 / Hkv 2 / D 256 over a 4096-token bf16 "
                       "cache, RMSNorm, int4 G=64 MoE block), final RMSNorm, bf16 LM head 2048 x 151936 + argmax; "
                       "batch 1",
           "value": world * 1e6 / us, "unit": "tok/s", "ms_per_token": us / 1e3, "tokens": tokens,
           "bytes_per_token": nb, "hbm_gbs": gbs, "frac": gbs / peaks["hbm"], "peak_kind": peaks["kind"],
           "roofline_ms_per_token": nb / (peaks["hbm"] * 1e9) * 1e3,
           "stage_ms_per_token": split, "stage_hbm_frac": stage_frac,
           "gpu_launches_per_token": per, "next_token": next_token, "clocks": clk,
           "how": "mvcc_b200.stack.DecodeStack.step: 40 x (moe_attn_forward_rms: the layer's input norm fused into "
                  "its qkv GEMV, moe_block_forward; the last one with the final norm), moe_lm_head_argmax; one CUDA "
                  "graph of the token steps"}
    del stk
    return out


def b200_arm(args, rank, world, local):
    import mvcc_b200 as m
    dev = torch.device("cuda", local)
    shape = m.MoeShape()
    B = args.batch
    K, W = args.steps, args.warmup
    peaks = load_peaks()
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        layers = [m.synth_layer(shape, seed=1000 + 97 * rank + i, stream=stream) for i in range(args.layer_copies)]
    blocks = [m.MoeBlock(l, max(B, 16)) for l in layers]
    torch.cuda.synchronize()

    head = decode_case(m, shape, blocks, B, K, W, stream, world, dev, ClockSampler(dev))
    ms = head["ms"]
    st = head["stage_us"]
    ab = decode_bytes(shape, head["U"], B)
    step_us = ms / K * 1e3
    fused = B < 8
    if fused:
        # the step is one launch of the fused kernel, so its duration is bounded by the plain graph's step time
        # (launch gaps included); events inside the graph would defeat the kernel's programmatic dependent launch
        achieved = ab["block"] / (step_us * 1e-6) / 1e9
        roof = {"kernel": "moe_fused_decode_kernel (the whole block in one cooperative launch)",
                "bound": "hbm", "achieved": achieved, "peak": peaks["hbm"], "unit": "GB/s",
                "frac": achieved / peaks["hbm"], "peak_kind": peaks["kind"], "bytes_per_launch": ab["block"],
                "us_per_launch": step_us, "us_source": "plain graph step time (one launch per step)",
                "expert_bytes_per_launch": ab["experts"],
                "expert_frac": ab["experts"] / (step_us * 1e-6) / 1e9 / peaks["hbm"],
                "traffic": NCU_TRAFFIC["fused_b1"] if B == 1 else None}
    else:
        fl = prefill_flops(shape, B)
        achieved = fl["gate_up"] / (st[1] * 1e-6) / 1e12
        roof = {"kernel": "moe_gemm_kernel (routed gate/up grouped GEMM)", "bound": "tensor", "achieved": achieved,
                "peak": peaks["tf_sustained"], "unit": "TFLOP/s", "frac": achieved / peaks["tf_sustained"],
                "peak_kind": peaks["kind"], "flops_per_launch": fl["gate_up"], "us_per_launch": st[1],
                "traffic": None}
    exp_gbs = ab["experts"] / (step_us * 1e-6) / 1e9
    blk_gbs = ab["block"] / (step_us * 1e-6) / 1e9
    result = {
        "metric": METRIC,
        "value": world * B * K / (ms / 1e3),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": ms / K,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": DTYPE,
        "data": DATA,
        "config": decode_config(shape, B, world, K, args.layer_copies),
        "roofline": roof,
        "expert_gemv": {"bytes_per_step": ab["experts"], "unique_experts": head["U"], "gbs_over_step": exp_gbs,
                        "frac_over_step": exp_gbs / peaks["hbm"],
                        "note": "expert weight + scale bytes over the whole step time (router, shared expert and "
                                "norms included in the time)"},
        "block": {"bytes_per_step": ab["block"], "gbs": blk_gbs, "frac": blk_gbs / peaks["hbm"], "us": step_us},
        "kernels_us": {"fused_block_events": st[0]} if fused else
                      {"route": st[0], "gate_up": st[1], "down_combine": st[2]},
        "e2e": {"value": world * B * K / (head["ms_e2e"] / 1e3), "unit": "tok/s",
                "h2d_bytes_per_step": head["h2d"], "d2h_bytes_per_step": head["d2h"]},
        "gpu_launches": launches_claim(head["launches_per_step"], B, K)[0],
        "gpu_launches_source": launches_claim(head["launches_per_step"], B, K)[1],
        "clocks": head["clocks"],
    }
    if not args.quick:
        extra = {}
        for b in (1, 4, 16):
            if b == B:
                continue
            kb = min(K, 4096)
            r = decode_case(m, shape, blocks, b, kb, W, stream, world, dev)
            u = r["ms"] / kb * 1e3
            bb = decode_bytes(shape, r["U"], b)
            extra[str(b)] = {"tok_s": world * b * kb / (r["ms"] / 1e3), "us_per_step": u, "steps": kb,
                             "unique_experts": r["U"], "block_gbs": bb["block"] / (u * 1e-6) / 1e9,
                             "block_frac": bb["block"] / (u * 1e-6) / 1e9 / peaks["hbm"],
                             "path": "fused decode kernel" if b < 8 else "prefill (tile GEMMs)",
                             "stages_us": list(r["stage_us"]),
                             "e2e_tok_s": world * b * kb / (r["ms_e2e"] / 1e3)}
        # batches 8 and 16 on the decode kernels (decode numerics), which the default sends to the prefill path (the
        # reference's T >= 8 switch, qwen.cu:347, whose tile numerics the default keeps)
        m.set_prefill_min_tokens(17)
        try:
            for b in (8, 16):
                kb = min(K, 4096)
                r = decode_case(m, shape, blocks, b, kb, W, stream, world, dev)
                u = r["ms"] / kb * 1e3
                bb = decode_bytes(shape, r["U"], b)
                extra[f"{b}_decode_kernels"] = {
                    "tok_s": world * b * kb / (r["ms"] / 1e3), "us_per_step": u, "steps": kb,
                    "unique_experts": r["U"], "block_gbs": bb["block"] / (u * 1e-6) / 1e9,
                    "block_frac": bb["block"] / (u * 1e-6) / 1e9 / peaks["hbm"],
                    "path": ("fused decode kernel" if b <= 8 else "three-kernel decode path") +
                            " (moe_set_prefill_min_tokens(17): decode numerics)",
                    "stages_us": list(r["stage_us"]), "e2e_tok_s": world * b * kb / (r["ms_e2e"] / 1e3)}
        finally:
            m.set_prefill_min_tokens(0)
        result["decode_batches"] = extra
    del blocks, layers
    torch.cuda.empty_cache()
    if world == 1 and not args.quick:
        result["pack_load"] = pack_load_case(m, shape)
        torch.cuda.empty_cache()
        result["g128"] = g128_case(m, stream)
        torch.cuda.empty_cache()
    if not args.quick and not args.no_stack:
        result["decode_stack"] = decode_stack_case(m, stream, world, peaks)
        torch.cuda.empty_cache()
    if not args.no_prefill:
        do_cpu = world == 1 and rank == 0 and not args.no_cpu
        result["prefill"] = prefill_case(m, shape, args.prefill_steps, W, stream, world, dev, peaks,
                                         args.cpu_seconds / 2, do_cpu)
    if not args.no_ep and world <= 8 and shape.E % world == 0:
        torch.cuda.empty_cache()
        result["ep_prefill"] = ep_case(m, shape, args.ep_steps, W, stream, world, rank, dev, peaks, args.ep_exchange,
                                       parity=not args.no_ep_parity)
    if world == 1 and rank == 0 and not args.no_cpu:
        with torch.cuda.stream(stream):
            l0 = m.synth_layer(shape, seed=1000, stream=stream)
        torch.cuda.synchronize()
        result["cpu_baseline"] = cpu_baseline(l0, shape, B, args.cpu_seconds)
    return result


# ------------------------------------------------------------------ CPU oracle (baseline / reference arm)

def host_layer(layer):
    out = {}
    for n, v in layer.t.items():
        a = v.cpu().numpy()
        out[n] = a.view(np.uint16) if v.dtype == torch.int16 else a
    return out


def oracle_shape(shape):
    from oracle import oracle as O
    return O.Shape(H=shape.H, E=shape.E, TOPK=shape.TOPK, I=shape.I, Is=shape.Is, G=shape.G, eps=shape.eps)


def time_oracle(L, shape, B, seconds, mode=0, max_steps=None, threads=None):
    """Steps of the C oracle's block on `threads` host threads (default: all) within `seconds`."""
    from oracle import oracle as O
    orc = O.Oracle()
    n = orc.max_threads() if threads is None else threads
    orc.set_threads(n)
    s = oracle_shape(shape)
    hidden, attn = O.make_activations(s, B, 3)
    orc.block_forward(s, L, hidden, attn, mode=mode)  # warm
    steps = 0
    t0 = time.perf_counter()
    while True:
        orc.block_forward(s, L, hidden, attn, mode=mode)
        steps += 1
        el = time.perf_counter() - t0
        if el >= seconds or (max_steps and steps >= max_steps):
            break
    return steps, el, n


def cpu_model():
    """The host CPU's model name (the first `model name` line of /proc/cpuinfo), or None where it cannot be read."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def cpu_baseline(layer, shape, B, seconds):
    """The oracle's block on every host thread, plus a shorter single-thread (scalar) timing beside it."""
    L = host_layer(layer)
    steps, el, n = time_oracle(L, shape, B, seconds)
    s1, el1, _ = time_oracle(L, shape, B, max(1.0, seconds / 4), threads=1)
    return {"value": steps * B / el, "unit": "tok/s", "cores": n, "kind": "port", "cpu": cpu_model(),
            "logical_cpus": os.cpu_count(),
            "sample": f"{steps} decode steps of batch {B} through the C oracle of the block (decode numerics) on one "
                      f"layer, {el:.1f} s, {n} threads ({os.cpu_count()} logical CPUs)",
            "single_thread": {"value": s1 * B / el1, "unit": "tok/s", "cores": 1,
                              "sample": f"{s1} decode steps of batch {B}, {el1:.1f} s, 1 thread"}}


def cpu_prefill(layer, shape, bias, seconds, tokens=64):
    L = host_layer(layer)
    L["router_bias"] = bias
    steps, el, n = time_oracle(L, shape, tokens, seconds, mode=1)
    return {"value": steps * tokens / el, "unit": "tok/s", "cores": n, "kind": "port",
            "sample": f"{steps} calls of {tokens} tokens through the C oracle of the block (tile numerics, Zipf "
                      f"bias) on one layer, {el:.1f} s, {n} threads ({os.cpu_count()} logical CPUs)"}


class _Shape:
    """The BASELINE config-2 geometry, for the reference arm (which loads nothing of this library)."""
    H, E, TOPK, I, Is, G, eps = 2048, 256, 8, 512, 512, 64, 1e-6

    def __init__(self, G=64):
        self.G = G


def fast_host_layer(shape, seed):
    """A layer in the pack layout from numpy's generator: bf16 N(0, 0.02) dense weights and router (so routing is
    spread as usual), one expert's uniform INT4 nibbles and fp16 group scales near absmax/7 of N(0, 0.02), repeated
    for every expert. The oracle's cost does not depend on the weight values, so this stands in for the seeded
    quantised layer, which takes a minute to build on the host."""
    s = shape
    rng = np.random.default_rng(seed)

    def bf16(*shp):
        a = (0.02 * rng.standard_normal(shp, dtype=np.float32)).view(np.uint32)
        return ((a + 0x7FFF + ((a >> 16) & 1)) >> 16).astype(np.uint16)

    def scales(*shp):
        return (0.0083 * (1.0 + 0.1 * rng.standard_normal(shp, dtype=np.float32))).astype(np.float16).view(np.uint16)

    def per_expert(a):
        return np.ascontiguousarray(np.broadcast_to(a, (s.E,) + a.shape))

    return {"rms2": np.full(s.H, 0x3F80, np.uint16), "router": bf16(s.E, s.H),
            "exp_gu_q": per_expert(rng.integers(0, 256, (2 * s.I, s.H // 2), dtype=np.uint8)),
            "exp_gu_s": per_expert(scales(2 * s.I, s.H // s.G)),
            "exp_dn_q": per_expert(rng.integers(0, 256, (s.H, s.I // 2), dtype=np.uint8)),
            "exp_dn_s": per_expert(scales(s.H, s.I // s.G)),
            "shared_gate_up": bf16(2 * s.Is, s.H), "shared_down": bf16(s.H, s.Is), "shared_gate": bf16(s.H)}


def ref_gpu_case(stream, copies=16, Ts=(1, 4, 8, 16), prefill_T=4096):
    """The reference's own CUDA kernels on this GPU: examples/qwen/kernels.cuh compiled unchanged for sm_100a into
    oracle/_ref/libqk_ref.so and launched in qwen.cu's order (oracle/ref/qk_ref_shim.cu). INT4 group 128, the
    group it hard-codes (kernels.cuh:842). Decode blocks warm -- one layer, the reference's own time_ms method
    (qwen.cu:486-498) -- and cold (layer copies cycled, weights from HBM); and its moe() (sort + tile GEMMs + slot
    reduce) for a 4096-token prefill on its own router's routing of N(0,1) activations (qwen.cu:559-566). Weights
    are random tensors of the pack layout made with torch; the library's `g128` object times the same cases."""
    import ctypes
    from oracle import ref_kernels as R
    if not R.available():
        return {"unavailable": "oracle/_ref/libqk_ref.so is not built (the reference tree was absent at build time)"}
    lib = R.lib()
    lib.qkref_block_forward.restype = ctypes.c_int
    lib.qkref_moe.restype = ctypes.c_int
    s = _Shape(G=128)
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(500)

    def bf16(*shp):
        return (0.02 * torch.randn(*shp, device=dev, generator=gen)).to(torch.bfloat16).view(torch.int16)

    def q(*shp):
        return torch.randint(0, 256, shp, device=dev, dtype=torch.uint8, generator=gen)

    def sc(*shp):
        return (0.0083 * (1 + 0.1 * torch.randn(*shp, device=dev, generator=gen))).to(torch.float16).view(torch.int16)

    layers = []
    for _ in range(copies):
        layers.append({"rms2": torch.full((s.H,), 0x3F80, dtype=torch.int16, device=dev), "router": bf16(s.E, s.H),
                       "exp_gu_q": q(s.E, 2 * s.I, s.H // 2), "exp_gu_s": sc(s.E, 2 * s.I, s.H // s.G),
                       "exp_dn_q": q(s.E, s.H, s.I // 2), "exp_dn_s": sc(s.E, s.H, s.I // s.G),
                       "shared_gate_up": bf16(2 * s.Is, s.H), "shared_down": bf16(s.H, s.Is),
                       "shared_gate": bf16(s.H)})

    def vp(t):
        return ctypes.c_void_p(t.data_ptr())

    def structs(t, T):
        Tp = (T + 127) // 128 * 128
        z = {"device": dev}
        buf = {"logits_r": torch.zeros(Tp, s.E, **z), "topk_i": torch.zeros(Tp, s.TOPK, dtype=torch.int32, **z),
               "topk_w": torch.zeros(Tp, s.TOPK, **z), "inter": torch.zeros(Tp, s.TOPK, s.I, dtype=torch.int16, **z),
               "routed": torch.zeros(Tp, s.H, **z), "moe_off": torch.zeros(s.E + 1, dtype=torch.int32, **z),
               "moe_sorted": torch.zeros(Tp * s.TOPK, dtype=torch.int32, **z),
               "slot_out": torch.zeros(Tp * s.TOPK, s.H, **z),
               "sgu": torch.zeros(Tp, 2 * s.Is, dtype=torch.int16, **z),
               "sinter": torch.zeros(Tp, s.Is, dtype=torch.int16, **z),
               "sout": torch.zeros(Tp, s.H, dtype=torch.int16, **z)}
        L = R._Layer(*[vp(t[n]) for n, _ in R._Layer._fields_[:9]], s.H, s.E, s.TOPK, s.I, s.Is, s.eps)
        W = R._Work(*[vp(buf[n]) for n, _ in R._Work._fields_])
        return L, W, buf

    st = ctypes.c_void_p(stream.cuda_stream)
    out = {"group": 128, "layer_copies": copies, "decode_us": {},
           "how": "reference kernels (kernels.cuh) built unchanged for sm_100a; CUDA graphs of calls, CUDA events"}
    for T in Ts:
        Tp = (T + 127) // 128 * 128
        h = torch.randn(Tp, s.H, device=dev, generator=gen)
        a = torch.randn(Tp, s.H, device=dev, generator=gen).to(torch.bfloat16).view(torch.int16)
        normed = torch.zeros(Tp, s.H, dtype=torch.int16, device=dev)
        refs = [structs(t, T) for t in layers]
        torch.cuda.synchronize()

        def step(i, cyc):
            L, W, _ = refs[i % copies if cyc else 0]
            rc = lib.qkref_block_forward(ctypes.byref(L), ctypes.byref(W), vp(h), vp(a), vp(normed), None, T, st)
            if rc != 0:
                raise RuntimeError(f"reference block: cudaError {rc}")

        out["decode_us"][str(T)] = {"warm": time_graph_us(lambda i: step(i, False), 32, stream),
                                    "cold": time_graph_us(lambda i: step(i, True), 64, stream)}
        del refs
    T = prefill_T
    x = torch.randn(T, s.H, device=dev, generator=gen).to(torch.bfloat16).view(torch.int16)
    L, W, buf = structs(layers[0], T)
    with torch.cuda.stream(stream):
        lib.qkref_dense_f32(vp(x), vp(layers[0]["router"]), vp(buf["logits_r"]), T, s.E, s.H, st)
        lib.qkref_router_topk(vp(buf["logits_r"]), vp(buf["topk_i"]), vp(buf["topk_w"]), T, s.E, s.TOPK, st)
    torch.cuda.synchronize()
    us = time_graph_us(lambda i: lib.qkref_moe(ctypes.byref(L), ctypes.byref(W), vp(x), T, st), 2, stream, reps=3)
    flops = 2.0 * T * s.TOPK * 3 * s.I * s.H
    out["prefill_routed"] = {"T": T, "us": us, "tflops": flops / (us * 1e-6) / 1e12}
    return out


def reference_arm(args, rank, world, local):
    if rank != 0:
        return None
    shape = _Shape()
    B = args.batch
    L = fast_host_layer(shape, 1000)
    from oracle import oracle as O
    orc = O.Oracle()
    orc.set_threads(orc.max_threads())
    s = oracle_shape(shape)
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
        "scaling": "weak", "vs_baseline": None, "dtype": DTYPE, "data": DATA,
        "config": decode_config(shape, B, world, args.steps, args.layer_copies),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": n, "kind": "port", "sample": sample,
                         "cpu": cpu_model(), "logical_cpus": os.cpu_count()},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference implements the block only as GPU kernels (examples/qwen/kernels.cuh); its CPU "
                "arm is the oracle's scalar restatement of those kernels; `ref_gpu` times those kernels themselves",
        "ref_gpu": ref_gpu_case(torch.cuda.Stream()) if torch.cuda.is_available() and not args.no_ref_gpu else None,
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=64)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--layer-copies", type=int, default=LAYER_COPIES,
                    help="decode layer copies cycled over (each 428 MB; the default keeps steps out of L2)")
    ap.add_argument("--prefill-steps", type=int, default=40)
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-4 prefill measurement")
    ap.add_argument("--ep-steps", type=int, default=20)
    ap.add_argument("--no-ep", action="store_true", help="skip the config-5 expert-parallel measurement")
    ap.add_argument("--no-ep-parity", action="store_true", help="skip the expert-parallel parity check")
    ap.add_argument("--no-stack", action="store_true", help="skip the config-3 40-layer decode-stack measurement")
    ap.add_argument("--ep-exchange", choices=["peers", "nccl"], default="peers",
                    help="expert-parallel exchange: kernels' peer-memory stores (default) or NCCL all-to-all")
    ap.add_argument("--quick", action="store_true", help="headline batch only (no decode_batches sweep)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-seconds", type=float, default=60.0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline legs")
    ap.add_argument("--no-ref-gpu", action="store_true", help="reference arm: skip timing the reference's GPU kernels")
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
