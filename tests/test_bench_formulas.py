"""CPU checks of bench.py's algorithmic work formulas against the figures the benchmark is quoted on: the decode
block's bytes per step (the reference's decode_weight_bytes terms, qwen.cu:463-477) and the prefill FLOPs per
4096-token step, and of the launch counts it reports."""
import importlib.util
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def load_bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class Shape:
    H, E, TOPK, I, Is, G = 2048, 256, 8, 512, 512, 64


def test_decode_bytes_match_the_quoted_figures():
    b = load_bench()
    ab = b.decode_bytes(Shape, 8, 1)
    # 8 experts x (gate_up q 1,048,576 + s 65,536 + down q 524,288 + s 32,768)
    assert ab["experts"] == 8 * 1_671_168 == 13_369_344
    # weights of the block (router, experts, shared expert, norm vectors) + activations in and out
    assert ab["block"] - 1 * Shape.H * (4 + 2) * 2 == 20_717_568
    # unique experts scale the expert term only
    assert b.decode_bytes(Shape, 30.5, 4)["experts"] == 30.5 * 1_671_168


def test_prefill_flops_match_the_quoted_figures():
    b = load_bench()
    fl = b.prefill_flops(Shape, 4096)
    assert abs(fl["gate_up"] + fl["down"] - 206.16e9) < 0.01e9
    assert abs(fl["shared"] - 25.77e9) < 0.01e9
    assert abs(fl["router"] - 4.29e9) < 0.01e9
    assert abs(fl["block"] - 236.2e9) < 0.1e9
    assert abs(b.prefill_flops(Shape, 16384)["block"] - 944.9e9) < 0.1e9


def test_launch_counts():
    b = load_bench()
    assert b.launches_per_step(1) == 1        # the fused decode kernel
    assert b.launches_per_step(7) == 1
    assert b.launches_per_step(8) == 10       # the prefill sequence
    assert b.launches_per_step(4096) == 10


def test_launch_claim_prefers_the_library_counter():
    """gpu_launches comes from the library's launch counter over one step when it can be read, else from the plan."""
    b = load_bench()

    class FakeLib:
        n = 0

        def stats(self):
            return {"launches": self.n}

    fake = FakeLib()

    def step():
        fake.n += 10

    import torch
    sync = torch.cuda.synchronize
    torch.cuda.synchronize = lambda *a: None  # no device here
    try:
        per = b.counted_launches(fake, step)
    finally:
        torch.cuda.synchronize = sync
    assert per == 10
    assert b.launches_claim(per, 4096, 7) == (70, b.launches_claim(per, 4096, 7)[1])
    assert "counter" in b.launches_claim(per, 1, 7)[1]
    assert b.launches_claim(None, 1, 7)[0] == 7 and "plan" in b.launches_claim(None, 1, 7)[1]
    assert b.counted_launches(object(), step) is None  # no counter: the plan stands in


def test_clock_summary_reads_reasons_and_window():
    """The clocks object of the bench line: median SM clock, max clock and the throttle reasons active in the timed
    region (the samples nvidia-smi prints as 'index, clocks.sm, clocks.max.sm, power, active, hw, hw_thermal,
    sw_thermal, sw_power_cap')."""
    b = load_bench()
    cs = b.ClockSampler.__new__(b.ClockSampler)
    cs.samples = [
        (0.5, ["0", "1965", "1965", "500", "0x0", "Not Active", "Not Active", "Not Active", "Not Active"]),
        (1.0, ["0", "1965", "1965", "700", "0x4", "Not Active", "Not Active", "Not Active", "Active"]),
        (1.5, ["0", "1900", "1965", "900", "0x4", "Not Active", "Not Active", "Not Active", "Active"]),
        (9.0, ["0", "1000", "1965", "900", "0x40", "Not Active", "Active", "Not Active", "Not Active"]),
    ]
    s = cs.summary(0.9, 2.0)
    assert s["sm_mhz"] == 1932.5 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"] and s["samples"] == 2 and s["window"] == "timed region"
    # a short timed region between samples falls back to the samples within 0.5 s of it
    s = cs.summary(1.6, 1.7)
    assert s["samples"] == 1 and s["sm_mhz"] == 1900.0 and s["window"] == "within 0.5 s of the timed region"
    assert cs.summary(20.0, 21.0)["sm_mhz"] is None


def test_oracle_timing_thread_counts():
    """The CPU baseline's timing loop runs the oracle's block on the requested host threads (1 = the scalar
    timing beside the all-threads one)."""
    b = load_bench()
    import mvcc_b200 as m
    from oracle import oracle as O
    s = m.MoeShape(H=256, E=8, TOPK=2, I=128, Is=128, G=64)
    L = O.make_layer(b.oracle_shape(s), 1)
    steps, el, n = b.time_oracle(L, s, 1, 0.05, threads=1)
    assert n == 1 and steps >= 1 and el >= 0.05
    steps, el, n = b.time_oracle(L, s, 2, 0.05, max_steps=3)
    assert n == O.Oracle().max_threads() and steps == 3 or el >= 0.05


def test_packed_io_layout():
    """e2e steps move their inputs in one copy (attn_out + hidden) and their results in one copy (hidden + normed):
    the views alias one buffer in that order, 16-byte aligned, with the byte counts of the separate tensors."""
    b = load_bench()
    import torch
    T, H = 3, 2048
    h = torch.randn(T, H)
    a = torch.randint(-30000, 30000, (T, H), dtype=torch.int16)
    n = torch.zeros(T, H, dtype=torch.int16)
    buf, av, hv, nv, inp, out = b.packed_io(h, a, n)
    assert torch.equal(av, a) and torch.equal(hv, h) and torch.equal(nv, n)
    assert inp.numel() == a.numel() * 2 + h.numel() * 4 and out.numel() == h.numel() * 4 + n.numel() * 2
    hv.add_(1)
    nv.fill_(7)
    o = out.clone()
    assert torch.equal(o[:T * H * 4].view(torch.float32).view(T, H), h + 1)
    assert bool((o[T * H * 4:].view(torch.int16) == 7).all())
    assert all(t.data_ptr() % 16 == 0 for t in (av, hv, nv))


def test_cpu_model_is_read_from_the_host():
    b = load_bench()
    name = b.cpu_model()
    assert name is None or (isinstance(name, str) and name)
