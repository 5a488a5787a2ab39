"""The C++ integration driver (tests/cpp/qwen_block_host.cpp) on a B200: the sequence a maintainer adds to qwen.cu --
a .mvccq pack loaded into HBM through moe_pack.h, one workspace, moe_block_forward, the error word -- run as a
separate C++ process on a seeded two-layer pack, its outputs checked against the CPU oracle (decode numerics below
the prefill threshold, tile numerics above it)."""
import os
import subprocess

import numpy as np
import pytest

from oracle import oracle as O
from tests import parity
from tests.test_abi import build_block_host

pytestmark = pytest.mark.gpu
TOL_BF16 = 1e-2


@pytest.mark.parametrize("T", [2, 16])
def test_cpp_driver_runs_a_pack_against_the_oracle(tmp_path, orc, T):
    from mvcc_b200 import pack
    import mvcc_b200 as m
    s = O.Shape(H=1024, E=32, TOPK=8, I=512, Is=512, G=64)
    layers = [O.make_layer(s, 60 + i) for i in range(2)]
    path = str(tmp_path / "two_layers.mvccq")
    entries = pack.block_entries(0, layers[0]) + pack.block_entries(1, layers[1])
    pack.write_pack(path, pack.pack_config(m.MoeShape(H=s.H, E=s.E, TOPK=s.TOPK, I=s.I, Is=s.Is, G=s.G), 2), entries)
    hidden, attn = O.make_activations(s, T, 70 + T)
    fin, fout = str(tmp_path / "in.bin"), str(tmp_path / "out.bin")
    with open(fin, "wb") as f:
        f.write(np.ascontiguousarray(hidden, np.float32).tobytes())
        f.write(np.ascontiguousarray(attn, np.uint16).tobytes())
    exe = build_block_host(tmp_path)
    run = subprocess.run([exe, path, "1", str(T), fin, fout], capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stderr
    assert run.stdout.startswith(f"ok T={T}")
    raw = open(fout, "rb").read()
    n = T * s.H
    gh = np.frombuffer(raw[:4 * n], np.float32).reshape(T, s.H)
    gn = np.frombuffer(raw[4 * n:6 * n], np.uint16).reshape(T, s.H)
    gl = np.frombuffer(raw[6 * n:], np.float32).reshape(T, s.E)
    ref = orc.block_forward(s, layers[1], hidden, attn, mode=0 if T < 8 else 1)
    assert O.max_rel_err(gl, ref["logits"]) < 2e-3
    margin = parity.topk_margin(ref["logits"], s.TOPK)
    ok = parity.keep_stable(margin > 2 * np.abs(gl - ref["logits"]).max(axis=1) + 1e-6, margin)
    assert O.max_rel_err(gh[ok], ref["hidden"][ok]) < TOL_BF16
    assert O.max_rel_err(O.bf16_to_f32(gn[ok]), O.bf16_to_f32(ref["normed"][ok])) < TOL_BF16
