"""GPU tests of the library's counters (moe_stats_get): the launches one block issues on each path, their
accounting under CUDA graph capture (counted once, at capture; replays add nothing), block calls, and the bytes the
pack loader copies. The per-path counts are the launch plans: one fused decode kernel for a batch-1 step, and the
ten-kernel prefill sequence (norm, router GEMM, top-k, sort scan, sort scatter, gate/up GEMM, down GEMM, two
shared-expert GEMMs, combine)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _block(T, shape=None, seed=31):
    import mvcc_b200 as m
    s = shape or m.MoeShape()
    layer = m.synth_layer(s, seed)
    hidden, attn = m.synth_activations(s, T, seed=seed + 1)
    normed = torch.zeros(T, s.H, dtype=torch.int16, device="cuda")
    torch.cuda.synchronize()
    return m.MoeBlock(layer, T), hidden, attn, normed


def _delta(fn):
    import mvcc_b200 as m
    torch.cuda.synchronize()
    a = m.stats()
    fn()
    torch.cuda.synchronize()
    b = m.stats()
    return {k: b[k] - a[k] for k in a}


def test_decode_batch1_is_one_launch():
    blk, h, a, n = _block(1)
    blk.forward(h, a, n)  # first call: one-time setup outside the count
    d = _delta(lambda: blk.forward(h, a, n))
    assert d == {"launches": 1, "block_calls": 1, "pack_bytes": 0}


def test_prefill_is_ten_launches():
    blk, h, a, n = _block(64)
    blk.forward(h, a, n)
    d = _delta(lambda: blk.forward(h, a, n))
    assert d == {"launches": 10, "block_calls": 1, "pack_bytes": 0}


def test_graph_capture_counts_once_and_replays_add_nothing():
    blk, h, a, n = _block(1)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        blk.forward(h, a, n, stream=s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()

    def capture():
        with torch.cuda.graph(g, stream=s):
            for _ in range(3):
                blk.forward(h, a, n, stream=s)

    assert _delta(capture)["launches"] == 3
    assert _delta(lambda: [g.replay() for _ in range(5)])["launches"] == 0
    del g


def test_pack_upload_bytes(tmp_path):
    import mvcc_b200 as m
    from mvcc_b200 import pack
    s = O.Shape(H=1024, E=32, TOPK=8, I=512, Is=512, G=64)
    L = O.make_layer(s, 5)
    ms = m.MoeShape(H=s.H, E=s.E, TOPK=s.TOPK, I=s.I, Is=s.Is, G=s.G)
    p = pack.write_pack(str(tmp_path / "s.mvccq"), pack.pack_config(ms, 1), pack.block_entries(0, L))
    with pack.MoePack(p) as pk:
        d = _delta(lambda: pk.layer(0))
    assert d["pack_bytes"] == sum(np.ascontiguousarray(a).nbytes for a in L.values())
    assert d["launches"] == 0
