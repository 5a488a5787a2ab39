"""CPU tests of the .mvccq pack reader (include/moe_pack.h) and writer (mvcc_b200.pack).

Pinned to packs written by the reference's own converter (tests/golden/make_pack_fixture.py runs convert.py's
Writer): the reader must return every tensor byte for byte and the layer geometry; our writer must reproduce the
reference writer's file byte for byte from the same arrays. Damaged packs must be refused with a reason, and the
device copy must check its destination before any CUDA call (nothing here touches a GPU)."""
import ctypes
import gzip
import hashlib
import importlib.util
import json
import os
import struct

import numpy as np
import pytest

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
MANIFEST = json.load(open(os.path.join(HERE, "ref_pack_tiny.json")))


def _fixture_module():
    spec = importlib.util.spec_from_file_location("make_pack_fixture", os.path.join(HERE, "make_pack_fixture.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


FIX = _fixture_module()


def _unpack(tmp_path, fname):
    raw = gzip.open(os.path.join(HERE, fname + ".gz"), "rb").read()
    assert hashlib.sha256(raw).hexdigest() == MANIFEST["files"][fname]["sha256"]
    p = tmp_path / fname
    p.write_bytes(raw)
    return str(p), raw


def P():
    from mvcc_b200 import pack
    return pack


def test_reads_reference_written_pack(tmp_path):
    path, _ = _unpack(tmp_path, "ref_pack_tiny.mvccq")
    man = MANIFEST["files"]["ref_pack_tiny.mvccq"]
    g = MANIFEST["geometry"]
    with P().MoePack(path) as pk:
        s = pk.shape
        assert (s.H, s.E, s.TOPK, s.I, s.Is, s.G, pk.layers) == (g["H"], g["E"], g["TOPK"], g["I"], g["Is"], g["G"],
                                                                 g["L"])
        assert abs(s.eps - g["eps"]) < 1e-12
        assert pk.names() == sorted(man["tensors"])
        for name, digest in man["tensors"].items():
            assert hashlib.sha256(pk.tensor(name).tobytes()).hexdigest() == digest, name
        ents = {n: a for n, _, a in FIX.entries()}
        for li in range(g["L"]):
            host = pk.layer_host(li)
            for field, sub, _ in P().BLOCK_TENSORS:
                want = ents[f"L{li}.{sub}"]
                assert host[field].shape == want.shape
                assert host[field].tobytes() == np.ascontiguousarray(want).tobytes(), (li, field)


def test_layer_weights_point_into_the_mapping(tmp_path):
    """moe_pack_layer_host: the geometry plus host pointers at each tensor's file offset."""
    import mvcc_b200 as m
    path, raw = _unpack(tmp_path, "ref_pack_tiny.mvccq")
    with P().MoePack(path) as pk:
        w = m.MoeLayerWeights()
        assert m._lib.moe_pack_layer_host(pk._h, 1, ctypes.byref(w)) == 0
        assert (w.H, w.E, w.TOPK, w.I, w.Is, w.G) == (64, 4, 2, 32, 32, 32) and w.router_bias is None
        for field, sub, _ in P().BLOCK_TENSORS:
            inf = pk.info(f"L1.{sub}")
            assert getattr(w, field) == inf.host
            assert ctypes.string_at(inf.host, inf.nbytes) == raw[inf.off:inf.off + inf.nbytes]
            assert inf.off % 64 == 0


def test_writer_matches_reference_writer(tmp_path):
    _, raw = _unpack(tmp_path, "ref_pack_tiny.mvccq")
    out = tmp_path / "ours.mvccq"
    P().write_pack(str(out), FIX.config(), FIX.entries())
    assert out.read_bytes() == raw


def test_layer_bytes_are_256_aligned_sums(tmp_path):
    path, _ = _unpack(tmp_path, "ref_pack_tiny.mvccq")
    with P().MoePack(path) as pk:
        want = sum((pk.info(f"L0.{sub}").nbytes + 255) // 256 * 256 for _, sub, _ in P().BLOCK_TENSORS)
        assert pk.layer_bytes(0) == want


def test_int8_shared_expert_is_dequantised_to_bf16(tmp_path):
    """A --dense int8 pack (written by the reference's converter): the shared expert's int8 rows come back as
    bf16(q * scale), bit for bit what numpy computes, within the int8 quantisation error of the original weights."""
    path, _ = _unpack(tmp_path, "ref_pack_tiny_int8.mvccq")
    bf_path, _ = _unpack(tmp_path, "ref_pack_tiny.mvccq")
    orig = FIX.arrays()
    with P().MoePack(path) as pk, P().MoePack(bf_path) as bf:
        assert "L0.shared.gate_up.q8" in pk.names() and "L0.shared.gate_up" not in pk.names()
        for li in range(2):
            host = pk.layer_host(li)
            for field, sub in (("shared_gate_up", "shared.gate_up"), ("shared_down", "shared.down")):
                q = pk.tensor(f"L{li}.{sub}.q8")
                sc = pk.tensor(f"L{li}.{sub}.s8")
                want = P().dequantize_int8_rows(q, sc)
                assert host[field].dtype == np.uint16 and np.array_equal(host[field], want), (li, field)
                w = (orig[f"L{li}.{sub}"].astype(np.uint32) << 16).view(np.float32)
                got = (host[field].astype(np.uint32) << 16).view(np.float32)
                grp = w.reshape(w.shape[0], -1, 32)
                bound = np.abs(grp).max(axis=2, keepdims=True) / 127 * 0.51 + np.abs(grp) * 2 ** -8
                assert (np.abs(got.reshape(grp.shape) - grp) <= bound + 1e-12).all()
            # every other block tensor is the same as in the bf16 pack
            hb = bf.layer_host(li)
            for field in ("rms2", "router", "exp_gu_q", "exp_gu_s", "exp_dn_q", "exp_dn_s", "shared_gate"):
                assert np.array_equal(host[field], hb[field])
        # the int8 rows and scales are uploaded as well, after the nine block tensors (256-byte aligned each)
        extra = sum(-(-pk.tensor(f"L0.{sub}.{k}").nbytes // 256) * 256
                    for sub in ("shared.gate_up", "shared.down") for k in ("q8", "s8"))
        assert pk.layer_bytes(0) == bf.layer_bytes(0) + extra


def test_int8_quantizer_and_writer_match_the_reference(tmp_path):
    """quantize_int8_rows reproduces the reference converter's int8 rows and scales, and write_pack its int8 pack,
    byte for byte."""
    _, raw = _unpack(tmp_path, "ref_pack_tiny_int8.mvccq")
    cfg = FIX.config()
    cfg["dense"] = "int8"
    out = tmp_path / "ours_int8.mvccq"
    P().write_pack(str(out), cfg, FIX.entries(True, lambda a: P().quantize_int8_rows(a, 32)))
    assert out.read_bytes() == raw


def test_int8_dequant_edge_values(tmp_path):
    """The loader's fp16 decoding and bf16 rounding on subnormal, large, zero and signed scales, q = -128..127 and
    many round-to-nearest-even ties, against numpy."""
    pk_mod = P()
    s, ents = _small_entries()
    rng = np.random.default_rng(9)
    q_gu = rng.integers(-128, 128, (2 * s.Is, s.H), dtype=np.int16).astype(np.int8)
    q_dn = rng.integers(-128, 128, (s.H, s.Is), dtype=np.int16).astype(np.int8)
    special = np.array([2.0 ** -24, 2.0 ** -20, 6.1e-5, 0.0, -0.0, 60000.0, -3.0, 1.0 / 3], np.float16)
    s_gu = rng.choice(special, (2 * s.Is, s.H // 8)).astype(np.float16)
    s_dn = (rng.standard_normal((s.H, s.Is // 8)) * 4).astype(np.float16)
    ents = [e for e in ents if e[0] not in ("L0.shared.gate_up", "L0.shared.down")]
    ents += [("L0.shared.gate_up.q8", "i8", q_gu), ("L0.shared.gate_up.s8", "f16", s_gu),
             ("L0.shared.down.q8", "i8", q_dn), ("L0.shared.down.s8", "f16", s_dn)]
    p = pk_mod.write_pack(str(tmp_path / "e.mvccq"), pk_mod.pack_config(s, 1), ents, header_slot=8192)
    with pk_mod.MoePack(p) as pk:
        h = pk.layer_host(0)
    assert np.array_equal(h["shared_gate_up"], pk_mod.dequantize_int8_rows(q_gu, s_gu))
    assert np.array_equal(h["shared_down"], pk_mod.dequantize_int8_rows(q_dn, s_dn))
    f = q_dn.astype(np.float32) * np.repeat(s_dn.astype(np.float32), 8, axis=1)
    assert ((f.view(np.uint32) & 0xFFFF) == 0x8000).sum() > 0  # ties exercised
    # the numpy rounding is round-to-nearest-even: check it against float64 on the ties' neighbours
    ref = (f.astype(np.float64))
    got = (h["shared_down"].astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    assert np.all(np.abs(got - ref) <= np.abs(ref) * 2.0 ** -8 + 1e-45)


def test_int8_scale_shape_is_checked(tmp_path):
    pk_mod = P()
    s, ents = _small_entries()
    ents = [e for e in ents if e[0] != "L0.shared.down"]
    ents += [("L0.shared.down.q8", "i8", np.zeros((s.H, s.Is), np.int8)),
             ("L0.shared.down.s8", "f16", np.zeros((s.H, 5), np.float16))]  # 5 does not divide Is = 32
    p = pk_mod.write_pack(str(tmp_path / "bad8.mvccq"), pk_mod.pack_config(s, 1), ents, header_slot=8192)
    with pk_mod.MoePack(p) as pk:
        with pytest.raises(pk_mod.PackError, match=r"shared\.down\.s8"):
            pk.layer_host(0)


def test_layer_out_of_range(tmp_path):
    path, _ = _unpack(tmp_path, "ref_pack_tiny.mvccq")
    with P().MoePack(path) as pk:
        for li in (-1, 2):
            with pytest.raises(P().PackError, match="outside"):
                pk.layer_host(li)


def test_upload_checks_destination_before_any_copy(tmp_path):
    import mvcc_b200 as m
    path, _ = _unpack(tmp_path, "ref_pack_tiny.mvccq")
    with P().MoePack(path) as pk:
        w = m.MoeLayerWeights()
        n = pk.layer_bytes(0)
        lib = m._lib
        assert lib.moe_pack_upload_layer(pk._h, 0, ctypes.c_void_p(8), n, ctypes.byref(w), None) == 1
        assert "aligned" in lib.moe_pack_last_error(pk._h).decode()
        assert lib.moe_pack_upload_layer(pk._h, 0, ctypes.c_void_p(4096), n - 1, ctypes.byref(w), None) == 1
        assert "needs" in lib.moe_pack_last_error(pk._h).decode()
        assert lib.moe_pack_upload_layer(pk._h, 0, None, n, ctypes.byref(w), None) == 1


def _small_entries(router_rows=None, drop=None):
    from mvcc_b200 import MoeShape
    s = MoeShape(H=64, E=4, TOPK=2, I=32, Is=32, G=32)
    rng = np.random.default_rng(3)
    t = {"rms2": np.zeros(s.H, np.uint16), "router": np.zeros((router_rows or s.E, s.H), np.uint16),
         "exp_gu_q": rng.integers(0, 255, (s.E, 2 * s.I, s.H // 2), dtype=np.uint8),
         "exp_gu_s": np.zeros((s.E, 2 * s.I, s.H // s.G), np.uint16),
         "exp_dn_q": rng.integers(0, 255, (s.E, s.H, s.I // 2), dtype=np.uint8),
         "exp_dn_s": np.zeros((s.E, s.H, s.I // s.G), np.uint16),
         "shared_gate_up": np.zeros((2 * s.Is, s.H), np.uint16), "shared_down": np.zeros((s.H, s.Is), np.uint16),
         "shared_gate": np.zeros(s.H, np.uint16)}
    ents = [e for e in P().block_entries(0, t) if e[0] != drop]
    return s, ents


def test_block_tensor_checks(tmp_path):
    pk_mod = P()
    s, ents = _small_entries(router_rows=5)
    p = pk_mod.write_pack(str(tmp_path / "a.mvccq"), pk_mod.pack_config(s, 1), ents, header_slot=4096)
    with pk_mod.MoePack(p) as pk:
        with pytest.raises(pk_mod.PackError, match=r"L0\.router is bf16 \[5,64\], expected bf16 \[4,64\]"):
            pk.layer_host(0)
    s, ents = _small_entries(drop="L0.exp.down.s")
    p = pk_mod.write_pack(str(tmp_path / "b.mvccq"), pk_mod.pack_config(s, 1), ents, header_slot=4096)
    with pk_mod.MoePack(p) as pk:
        with pytest.raises(pk_mod.PackError, match=r"no tensor L0\.exp\.down\.s"):
            pk.layer_bytes(0)
    # a wrong dtype on an otherwise well-formed entry
    s, ents = _small_entries()
    ents = [(n, "f16" if n == "L0.rms2" else d, a) for n, d, a in ents]
    p = pk_mod.write_pack(str(tmp_path / "c.mvccq"), pk_mod.pack_config(s, 1), ents, header_slot=4096)
    with pk_mod.MoePack(p) as pk:
        with pytest.raises(pk_mod.PackError, match="rms2 is f16"):
            pk.layer_host(0)


def test_config_without_group_means_128(tmp_path):
    """Packs written before the "group" key existed carry the converter's default group size (convert.py:311)."""
    pk_mod = P()
    from mvcc_b200 import MoeShape
    s = MoeShape(H=256, E=2, TOPK=1, I=128, Is=128, G=128)
    cfg = pk_mod.pack_config(s, 1)
    del cfg["group"]
    p = pk_mod.write_pack(str(tmp_path / "g.mvccq"), cfg, [("x", "u8", np.zeros(4, np.uint8))], header_slot=1024)
    with pk_mod.MoePack(p) as pk:
        assert pk.shape.G == 128


def test_unicode_names_round_trip(tmp_path):
    pk_mod = P()
    s, ents = _small_entries()
    name = "L0.xé中\U0001F600"
    ents.append((name, "f32", np.arange(3, dtype=np.float32)))
    p = pk_mod.write_pack(str(tmp_path / "u.mvccq"), pk_mod.pack_config(s, 1), ents, header_slot=8192)
    with pk_mod.MoePack(p) as pk:
        assert name in pk.names()
        assert np.array_equal(pk.tensor(name), np.arange(3, dtype=np.float32))


def _raw_pack(header: bytes, body: bytes = b"", hlen=None):
    n = len(header) if hlen is None else hlen
    return b"MVCCQ001" + struct.pack("<Q", n) + header + body


CFG = {"hidden": 64, "layers": 1, "experts": 4, "topk": 2, "inter": 32, "shared_inter": 32, "eps": 1e-6,
       "group": 32}


def _hdr(tensors, cfg=CFG):
    return json.dumps({"config": cfg, "tensors": tensors}).encode()


@pytest.mark.parametrize("case,expect", [
    ("magic", "bad magic"),
    ("short", "too short"),
    ("hlen", "header length"),
    ("json", "header JSON"),
    ("trailing", "trailing"),
    ("nested", "nested too deeply"),
    ("no_config", "no \"config\""),
    ("bad_geometry", "config.experts"),
    ("indivisible", "multiples of group"),
    ("outside", "outside the file"),
    ("in_header", "outside the file"),
    ("nbytes", "nbytes disagrees"),
    ("fraction", "shape holds a non-integer"),
    ("escape", "escape"),
])
def test_damaged_packs_are_refused(tmp_path, case, expect):
    body = b"\0" * 256
    ok_t = {"x": {"off": 0, "nbytes": 16, "dtype": "u8", "shape": [16]}}

    if case == "magic":
        raw = b"MVCCQ002" + _raw_pack(_hdr({}))[8:]
    elif case == "short":
        raw = b"MVCCQ001"
    elif case == "hlen":
        raw = _raw_pack(_hdr({}), hlen=1 << 40)
    elif case == "json":
        raw = _raw_pack(b'{"config": {"hidden": 64,}}')
    elif case == "trailing":
        raw = _raw_pack(_hdr({}) + b" x")
    elif case == "nested":
        raw = _raw_pack(b'{"config": ' + b"[" * 100 + b"]" * 100 + b"}")
    elif case == "no_config":
        raw = _raw_pack(b'{"tensors": {}}')
    elif case == "bad_geometry":
        raw = _raw_pack(_hdr({}, dict(CFG, experts=0)))
    elif case == "indivisible":
        raw = _raw_pack(_hdr({}, dict(CFG, hidden=48)))
    elif case in ("outside", "in_header", "nbytes", "fraction"):
        h0 = _hdr(ok_t)
        start = 16 + len(h0) + 64
        t = {"x": {"off": start, "nbytes": 16, "dtype": "u8", "shape": [16]}}
        if case == "outside":
            t["x"]["nbytes"] = 1 << 20
            t["x"]["shape"] = [1 << 20]
        elif case == "in_header":
            t["x"]["off"] = 8
        elif case == "nbytes":
            t["x"]["dtype"] = "bf16"
        else:
            t["x"]["shape"] = [15.5]
        h = _hdr(t)
        h += b" " * (len(h0) + 64 - len(h))  # keep the data start where the offsets assume it
        raw = _raw_pack(h, body)
    elif case == "escape":
        raw = _raw_pack(b'{"config": {"a\\q": 1}, "tensors": {}}')
    p = tmp_path / f"{case}.mvccq"
    p.write_bytes(raw)
    with pytest.raises(P().PackError, match=expect):
        P().MoePack(str(p))


def test_missing_file(tmp_path):
    with pytest.raises(P().PackError, match="cannot open"):
        P().MoePack(str(tmp_path / "nope.mvccq"))


def test_int8_shared_expert_within_the_bf16_bar_of_int8_gemv_numerics(orc):
    """The block on the loader's bf16 copy of an int8 shared expert (the oracle on those weights) against the
    reference's int8 GEMV numerics (kernels.cuh:215-274: fp32 products of the int8 values and their scales, no
    weight rounding), restated here in float64 with the block's bf16 rounding points (sgu, sinter, sout): within the
    bf16 bar, max relative error 1e-2."""
    from oracle import oracle as O
    pk_mod = P()
    s = O.Shape(H=256, E=8, TOPK=2, I=128, Is=128, G=64)
    L = O.make_layer(s, 4)
    T = 3
    hidden, attn = O.make_activations(s, T, 6)
    qgu, sgu = pk_mod.quantize_int8_rows(L["shared_gate_up"], 128)
    qdn, sdn = pk_mod.quantize_int8_rows(L["shared_down"], 128)
    L8 = dict(L, shared_gate_up=pk_mod.dequantize_int8_rows(qgu, sgu),
              shared_down=pk_mod.dequantize_int8_rows(qdn, sdn))
    ref = orc.block_forward(s, L8, hidden, attn, mode=0)
    x = O.bf16_to_f32(ref["normed"]).astype(np.float64)  # the post-attention norm feeds the shared expert

    def deq(q, sc):
        return q.astype(np.float64) * np.repeat(sc.astype(np.float64), q.shape[1] // sc.shape[1], axis=1)

    def bf(v):
        return O.bf16_to_f32(O.f32_to_bf16(v.astype(np.float32))).astype(np.float64)

    gu = bf(x @ deq(qgu, sgu).T)
    g, u = gu[:, :s.Is], gu[:, s.Is:]
    inter = bf(g / (1.0 + np.exp(-g)) * u)
    sout = bf(inter @ deq(qdn, sdn).T)
    assert O.max_rel_err(O.bf16_to_f32(ref["sout"]), sout) < 1e-2


def test_synth_pack_and_command_line(tmp_path, capsys):
    """`python -m mvcc_b200.pack synth` writes a loadable pack whose INT4 experts follow the generator's rule, and
    `info` reports its geometry and each layer's device bytes."""
    pk_mod = P()
    out = tmp_path / "syn.mvccq"
    assert pk_mod._main(["synth", str(out), "--layers", "2", "--hidden", "256", "--experts", "8", "--topk", "2",
                         "--inter", "128", "--shared-inter", "128", "--group", "64", "--int8-shared", "128"]) == 0
    with pk_mod.MoePack(str(out)) as pk:
        assert (pk.shape.H, pk.shape.E, pk.shape.G, pk.layers) == (256, 8, 64, 2)
        h = pk.layer_host(1)
        q = h["exp_gu_q"]
        nib = np.stack([q & 15, q >> 4], axis=-1).reshape(q.shape[0], q.shape[1], -1)
        assert nib.min() >= 1 and nib.max() <= 15  # q - 8 in [-7, 7]
        sc = h["exp_gu_s"].astype(np.float32)
        assert (sc > 0).all() and sc.max() < 0.02 * 6 / 7
        assert "L0.shared.down.q8" in pk.names()
    assert pk_mod._main(["info", str(out)]) == 0
    text = capsys.readouterr().out
    assert "H=256 E=8 topk=2 I=128 Is=128 group=64" in text and "L1: block" in text
