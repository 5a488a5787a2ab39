"""CPU tests of the C-ABI library: it loads, exports every entry point include/*.h declares, and its host-side
shape and workspace checks behave. No kernel is launched here."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", f) for f in sorted(os.listdir(os.path.join(ROOT, "include")))
           if f.endswith(".h")]


def _declared():
    names = set()
    for h in HEADERS:
        names |= set(re.findall(r"^MOE_API\s+[\w\s\*]+?\b(moe_\w+)\s*\(", open(h).read(), flags=re.M))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    import mvcc_b200
    names = _declared()
    assert len(names) >= 10
    lib = ctypes.CDLL(mvcc_b200.LIB_PATH)
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) <= set(mvcc_b200.EXPORTED)


def test_stats_counters_read_and_reset():
    """moe_stats_get / moe_stats_reset; a call refused before launch counts neither a launch nor a block call."""
    import mvcc_b200
    mvcc_b200.reset_stats()
    assert mvcc_b200.stats() == {"launches": 0, "block_calls": 0, "pack_bytes": 0}
    w = _w()
    assert mvcc_b200._lib.moe_block_forward(ctypes.byref(w), None, 0, None, None, None, None, 1, None) == 1
    assert mvcc_b200.stats() == {"launches": 0, "block_calls": 0, "pack_bytes": 0}


def test_version():
    import mvcc_b200
    assert "sm_100a" in mvcc_b200.version()


def _w(**kw):
    import mvcc_b200
    d = dict(H=2048, E=256, TOPK=8, I=512, Is=512, G=64, eps=1e-6)
    d.update(kw)
    return mvcc_b200.MoeLayerWeights(*([None] * 9), d["H"], d["E"], d["TOPK"], d["I"], d["Is"], d["G"], d["eps"])


@pytest.mark.parametrize("kw,ok", [
    ({}, True), ({"G": 128}, True), ({"G": 32}, True), ({"H": 1024, "E": 32}, True),
    ({"G": 48}, False), ({"H": 2000}, False), ({"TOPK": 9}, False), ({"E": 512}, False), ({"I": 500}, False),
    ({"TOPK": 0}, False), ({"E": 4, "TOPK": 8}, False),
])
def test_shape_check(kw, ok):
    import mvcc_b200
    rc = mvcc_b200._lib.moe_check_shape(ctypes.byref(_w(**kw)))
    assert (rc == 0) == ok


def test_workspace_bytes_monotone_and_aligned():
    import mvcc_b200
    w = _w()
    prev = 0
    for T in (1, 2, 16, 128, 4096):
        b = mvcc_b200._lib.moe_workspace_bytes(ctypes.byref(w), T)
        assert b > prev and b % 256 == 0
        prev = b
    assert mvcc_b200._lib.moe_workspace_bytes(ctypes.byref(_w(G=48)), 1) == 0


def test_entry_points_reject_bad_arguments_before_launch():
    """Invalid shapes, null workspaces and T < 1 return cudaErrorInvalidValue without touching the GPU."""
    import mvcc_b200
    lib = mvcc_b200._lib
    w = _w()
    assert lib.moe_block_forward(ctypes.byref(w), None, 0, None, None, None, None, 1, None) == 1
    assert lib.moe_block_forward(ctypes.byref(_w(G=48)), ctypes.c_void_p(256), 1 << 30, None, None, None, None, 1,
                                 None) == 1
    assert lib.moe_router_topk(ctypes.byref(w), ctypes.c_void_p(256), 1 << 30, None, None, None, None, 0, None) == 1
    # misaligned workspace
    assert lib.moe_shared_expert(ctypes.byref(w), ctypes.c_void_p(8), 1 << 30, None, None, 1, None) == 1
    # the attention workspace's error-word reader: null, too small or misaligned workspaces
    assert lib.moe_attn_workspace_error(None, 1 << 20, None) == -1
    assert lib.moe_attn_workspace_error(ctypes.c_void_p(256), 2, None) == -1
    assert lib.moe_attn_workspace_error(ctypes.c_void_p(8), 1 << 20, None) == -1


def test_expert_bytes_match_reference_formula():
    """decode_weight_bytes (qwen.cu:463-477) at G=64: 1,671,168 bytes per routed expert."""
    import mvcc_b200
    assert mvcc_b200.MoeShape().expert_bytes() == 1_671_168


def test_expert_parallel_entry_points_check_before_launch():
    """The expert-parallel stages reject unsupported splits and missing buffers with cudaErrorInvalidValue before any
    launch, size their exchange buffers by formula, and launch nothing for an empty receive set."""
    import mvcc_b200
    import mvcc_b200.ep as ep
    lib = mvcc_b200._lib
    w = _w()
    wp = ctypes.byref(w)
    rec = lib.moe_ep_record_bytes(wp)
    assert rec == 2 * 2048 + 8 * 8 == 4160
    # world must divide E into shards of a multiple of 16 experts, at least TOPK, at most 8 ranks
    for world, ok in ((1, True), (2, True), (8, True), (3, False), (16, False), (32, False)):
        nb = lib.moe_ep_recv_bytes(wp, world, 64)
        assert (nb > 0) == ok
        if ok:
            off = lib.moe_ep_rcount_offset(wp, world, 64)
            assert off % 256 == 0 and off >= world * 64 * rec and nb >= off + 4 * world
            assert lib.moe_ep_ret_bytes(wp, world, 64) == world * 64 * 2048 * 2  # bf16 rows
    ws = ctypes.c_void_p(1 << 20)  # never dereferenced: every call below fails its checks first
    assert lib.moe_ep_dispatch(wp, ws, 1 << 30, None, None, None, 4, 3, None, None, None, None) == 1
    assert lib.moe_ep_dispatch(wp, None, 1 << 30, None, None, None, 4, 2, None, None, None, None) == 1
    assert lib.moe_ep_combine(wp, ws, 1 << 30, None, None, None, None, None, 4, 2, None, None, None) == 1
    # empty receive set: nothing to do, nothing launched
    wl = _w(E=128)
    for n in ("exp_gu_q", "exp_gu_s", "exp_dn_q", "exp_dn_s"):
        setattr(wl, n, 1 << 20)  # present but never read: no record arrived
    assert lib.moe_ep_experts(ctypes.byref(wl), ws, 1 << 30, None, 0, None, None) == 0
    # peer mode: missing buffers or a rank outside the world
    peers = ep.MoeEpPeers()
    peers.rank, peers.cap = 0, 4
    assert lib.moe_ep_dispatch_peers(wp, ws, 1 << 30, None, None, None, 4, 2, ctypes.byref(peers), None, None,
                                     None) == 1
    for d in range(2):
        peers.recv[d] = peers.rcount[d] = peers.ret[d] = 1 << 20
    peers.rank = 2
    assert lib.moe_ep_experts_peers(ctypes.byref(wl), ws, 1 << 30, 2, ctypes.byref(peers), None) == 1
    assert ctypes.sizeof(ep.MoeEpPeers) == 3 * 8 * 8 + 8


def _abi_program(names):
    """A program that includes every header and references every declared entry point (its address), so that
    compiling it checks the headers and linking it checks the library's exports, from C and from C++."""
    incs = "".join(f'#include "{os.path.basename(h)}"\n' for h in HEADERS)
    refs = "".join(f"  (void *)&{n},\n" for n in names)
    return (incs + "#include <stdio.h>\n"
            "int main(void) {\n"
            f"  void *fns[] = {{\n{refs}  0}};\n"
            "  int n = 0;\n"
            "  for (unsigned i = 0; i + 1 < sizeof fns / sizeof fns[0]; ++i) n += fns[i] != 0;\n"
            "  moe_stats st;\n"
            "  moe_stats_get(&st);\n"
            "  printf(\"%d %llu\\n\", n, (unsigned long long)st.launches);\n"
            "  return 0;\n}\n")


@pytest.mark.parametrize("lang", ["c", "c++"])
def test_headers_compile_and_link_from_c_and_cpp(tmp_path, lang):
    """The boundary is a C ABI: the headers compile as C11 and C++17 with warnings as errors, and a program that
    references every declared entry point links against libmoe_b200.so and runs on a host without a GPU."""
    import subprocess

    import mvcc_b200
    names = _declared()
    src = tmp_path / ("abi.c" if lang == "c" else "abi.cpp")
    src.write_text(_abi_program(names))
    exe = tmp_path / "abi"
    cc = ["gcc", "-std=c11"] if lang == "c" else ["g++", "-std=c++17"]
    libdir = os.path.dirname(mvcc_b200.LIB_PATH)
    cmd = cc + ["-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe),
                "-L", libdir, "-lmoe_b200", f"-Wl,-rpath,{libdir}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stderr
    n, launches = run.stdout.split()
    assert int(n) == len(names) and int(launches) == 0


def build_block_host(out_dir):
    """Compiles tests/cpp/qwen_block_host.cpp (the block driven from C++ as qwen.cu would: pack -> HBM, workspace,
    forward, error word) against include/ and libmoe_b200.so; returns the executable's path."""
    import subprocess

    import mvcc_b200
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    libdir = os.path.dirname(mvcc_b200.LIB_PATH)
    exe = os.path.join(str(out_dir), "qwen_block_host")
    cmd = ["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(cuda, "include"), os.path.join(ROOT, "tests", "cpp", "qwen_block_host.cpp"),
           "-o", exe, "-L", libdir, "-lmoe_b200", f"-Wl,-rpath,{libdir}", "-L", os.path.join(cuda, "lib64"),
           "-lcudart", f"-Wl,-rpath,{os.path.join(cuda, 'lib64')}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_cpp_block_host_builds(tmp_path):
    """The C++ driver of the integration sequence (pack -> HBM -> workspace -> forward -> error word) compiles and
    links; without arguments it prints its usage."""
    import subprocess
    exe = build_block_host(tmp_path)
    run = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert run.returncode == 2 and "usage" in run.stderr
    run = subprocess.run([exe, str(tmp_path / "missing.mvccq")], capture_output=True, text=True, timeout=60)
    assert run.returncode == 1 and "cannot open" in run.stderr  # refused before any CUDA call


def test_tensor_stats_follow_the_reference_debug_report():
    """tensor_stats (the reference's --debug statistics, qwen.cu:66-89) on host tensors: non-finite values are
    counted and left out of the sums, the mean and rms divide by every element, bf16 bits are decoded."""
    import torch
    import mvcc_b200
    x = torch.tensor([1.0, -3.0, float("nan"), float("inf"), 2.0], dtype=torch.float32)
    st = mvcc_b200.tensor_stats(x)
    assert st["n"] == 5 and st["nonfinite"] == 2
    assert st["mean"] == 0.0 and abs(st["rms"] - (14 / 5) ** 0.5) < 1e-12 and st["absmax"] == 3.0
    assert st["head"][:2] == [1.0, -3.0]
    b = torch.tensor([0.5, -0.25], dtype=torch.bfloat16).view(torch.int16)
    sb = mvcc_b200.tensor_stats(b)
    assert sb["absmax"] == 0.5 and sb["mean"] == 0.125 and sb["nonfinite"] == 0
