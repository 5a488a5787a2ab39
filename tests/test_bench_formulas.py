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
