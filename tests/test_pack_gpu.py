"""GPU tests of loading a layer from a .mvccq pack into HBM (moe_pack_upload_layer) and running the block on it.

A pack of two seeded layers is written with mvcc_b200.pack.write_pack (whose output the CPU tests pin, byte for
byte, to the reference's converter); layer 1 is copied to the device through the C ABI; the device bytes must equal
the file's, and the block on those weights must match the CPU oracle on the same host arrays (int4 bar 2e-2, bf16
bar 1e-2, max relative error)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import parity

pytestmark = pytest.mark.gpu

TOL_BF16 = 1e-2


def _write(tmp_path, s, seeds, int8_group=None):
    """A pack of seeded layers; with int8_group the shared expert is stored as int8 rows (convert.py --dense int8)
    and the returned host layers carry the bf16 values the loader dequantises them to."""
    from mvcc_b200 import MoeShape, pack
    ms = MoeShape(H=s.H, E=s.E, TOPK=s.TOPK, I=s.I, Is=s.Is, G=s.G, eps=s.eps)
    layers = [O.make_layer(s, sd) for sd in seeds]
    ents = []
    for li, L in enumerate(layers):
        ents += pack.block_entries(li, L, shared_int8_group=int8_group)
    path = pack.write_pack(str(tmp_path / "m.mvccq"), pack.pack_config(ms, len(layers)), ents)
    if int8_group:
        with pack.MoePack(path) as pk:
            layers = [dict(L, **{f: pk.layer_host(li)[f] for f in ("shared_gate_up", "shared_down")})
                      for li, L in enumerate(layers)]
    return path, layers


@pytest.mark.parametrize("G,int8", [(64, None), (128, None), (64, 128)])
@pytest.mark.parametrize("T", [2, 16])
def test_block_on_uploaded_layer_matches_oracle(tmp_path, G, int8, T):
    """int8 = 128: the shared expert stored as int8 rows with group-128 scales, dequantised to bf16 by the loader."""
    import mvcc_b200 as m
    from mvcc_b200 import pack
    s = O.Shape(H=1024, E=32, TOPK=8, I=512, Is=512, G=G)
    path, layers = _write(tmp_path, s, (21, 22), int8)
    with pack.MoePack(path) as pk:
        layer = pk.layer(1)
    torch.cuda.synchronize()  # pack closed: the copies must not depend on the mapping any more
    for field in m.MoeLayer.NAMES:
        host = np.ascontiguousarray(layers[1][field])
        dev = layer.t[field].cpu().numpy()
        assert dev.tobytes() == host.tobytes(), field
    hidden, attn = O.make_activations(s, T, 5)
    blk = m.MoeBlock(layer, T)
    h = torch.from_numpy(hidden.copy()).cuda()
    a = torch.from_numpy(attn.view(np.int16)).cuda()
    n = torch.zeros(T, s.H, dtype=torch.int16, device="cuda")
    blk.forward(h, a, n)
    torch.cuda.synchronize()
    ref = O.Oracle().block_forward(s, layers[1], hidden, attn, mode=0 if T < 8 else 1)
    # tokens whose 8th/9th logit margin exceeds twice the GPU-vs-oracle logit error cannot route differently
    gl = blk.trace(T)["logits"].cpu().numpy()
    margin = parity.topk_margin(ref["logits"], s.TOPK)
    ok = parity.keep_stable(margin > 2 * np.abs(gl - ref["logits"]).max(axis=1) + 1e-6, margin)
    assert O.max_rel_err(h.cpu().numpy()[ok], ref["hidden"][ok]) < TOL_BF16
    nb = O.bf16_to_f32(n.cpu().numpy().view(np.uint16))
    assert O.max_rel_err(nb[ok], O.bf16_to_f32(ref["normed"])[ok]) < TOL_BF16
    assert blk.error_word() == 0


def test_upload_into_a_short_region_fails_cleanly(tmp_path):
    import ctypes

    import mvcc_b200 as m
    from mvcc_b200 import pack
    s = O.Shape(H=1024, E=32, TOPK=8, I=512, Is=512, G=64)
    path, _ = _write(tmp_path, s, (21,))
    with pack.MoePack(path) as pk:
        n = pk.layer_bytes(0)
        buf = torch.empty(n, dtype=torch.uint8, device="cuda")
        w = m.MoeLayerWeights()
        rc = m._lib.moe_pack_upload_layer(pk._h, 0, ctypes.c_void_p(buf.data_ptr()), n - 256, ctypes.byref(w),
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 1
        assert w.router is None  # nothing filled in


@pytest.mark.parametrize("T", [1, 3])
def test_decode_reads_the_int8_shared_expert(tmp_path, orc, T):
    """An int8 pack (group 128, the reference converter's --dense int8) on the single-launch decode kernel: its shared
    expert comes from the int8 rows with gemv_i8_kernel's numerics, half the bytes of the bf16 copy. To show which copy
    is read, the bf16 copy on the device is zeroed first: sout must still match the oracle's int8 GEMV numerics
    (bf16 bar 1e-2) and the block's output the oracle block on the dequantised weights."""
    import mvcc_b200 as m
    from mvcc_b200 import pack
    s = O.Shape(H=1024, E=32, TOPK=8, I=512, Is=512, G=64)
    path, layers = _write(tmp_path, s, (31, 32), 128)
    with pack.MoePack(path) as pk:
        layer = pk.layer(1)
        q8g, s8g = pk.tensor("L1.shared.gate_up.q8"), pk.tensor("L1.shared.gate_up.s8")
        q8d, s8d = pk.tensor("L1.shared.down.q8"), pk.tensor("L1.shared.down.s8")
    assert layer.c.shared_gate_up_q8 and layer.c.shared_group == 128
    layer.t["shared_gate_up"].zero_()
    layer.t["shared_down"].zero_()
    hidden, attn = O.make_activations(s, T, 90 + T)
    blk = m.MoeBlock(layer, T)
    h = torch.from_numpy(hidden.copy()).cuda()
    n = torch.zeros(T, s.H, dtype=torch.int16, device="cuda")
    blk.forward(h, torch.from_numpy(attn.view(np.int16)).cuda(), n)
    torch.cuda.synchronize()
    tr = blk.trace(T)
    ref = orc.block_forward(s, layers[1], hidden, attn, mode=0)
    _, sout8 = O.shared_i8(s, q8g, s8g, q8d, s8d, ref["normed"])
    gs = tr["sout"].cpu().numpy().view(np.uint16)
    assert O.max_rel_err(O.bf16_to_f32(gs), O.bf16_to_f32(sout8)) < TOL_BF16
    gl = tr["logits"].cpu().numpy()
    margin = parity.topk_margin(ref["logits"], s.TOPK)
    ok = parity.keep_stable(margin > 2 * np.abs(gl - ref["logits"]).max(axis=1) + 1e-6, margin)
    assert O.max_rel_err(h.cpu().numpy()[ok], ref["hidden"][ok]) < TOL_BF16
    assert blk.error_word() == 0
