"""GPU parity tests of the expert-parallel stages (include/moe_ep.h, mvcc_b200/ep.py) on one GPU: every rank's
dispatch, experts and combine run in one process (`emulated_step`, the all-to-alls as device copies in the order
NCCL would deliver), so the multi-rank numerics are checked without a second GPU. Bars: routing as for the block;
outputs against the oracle's expert-parallel restatement (per-rank slot-order partials rounded to bf16 -- the rows
that cross the return exchange -- and summed in rank order) within 1e-2 (bf16) and 2e-2 (int4); world = 1 equals the
single-GPU prefill block up to that one bf16 rounding of the routed row; world = W equals world = 1 up to the
per-rank roundings and fp32 summation order."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.test_decode_gpu import TOL_BF16, TOL_INT4, check_routing, host16, mb, stable_rows, to_dev16, upload

pytestmark = pytest.mark.gpu

S128 = O.Shape(H=1024, E=128, TOPK=8, I=512, Is=512, G=64)
_cache = {}


def layer128():
    if "l" not in _cache:
        L = O.make_layer(S128, 41)
        _cache["l"] = (L, upload(S128, L))
    return _cache["l"]


def ep():
    import mvcc_b200.ep as E
    return E


def run_emulated(layer, world, Ts, seed, next_rms1=None, s=S128):
    E = ep()
    ranks = [E.EpRank(layer, r, world, max(Ts)) for r in range(world)]
    acts = [O.make_activations(s, T, seed + r) for r, T in enumerate(Ts)]
    hid = [torch.from_numpy(np.ascontiguousarray(h, np.float32)).cuda() for h, _ in acts]
    att = [to_dev16(a) for _, a in acts]
    nrm = [torch.zeros(T, s.H, dtype=torch.int16, device="cuda") for T in Ts]
    nr = None if next_rms1 is None else to_dev16(next_rms1)
    C = E.emulated_step(ranks, hid, att, nrm, next_rms1=nr)
    torch.cuda.synchronize()
    return ranks, acts, hid, nrm, C


def test_world1_equals_block_prefill_up_to_the_bf16_return_row():
    """One rank: the block's prefill path, except that the routed row is rounded to bf16 once (half a bf16 ulp of
    |routed|, below one ulp of the largest hidden value)."""
    m = mb()
    L, layer = layer128()
    T = 300
    ranks, acts, hid, nrm, _ = run_emulated(layer, 1, [T], 500)
    h0 = torch.from_numpy(np.ascontiguousarray(acts[0][0], np.float32)).cuda()
    n0 = torch.zeros(T, S128.H, dtype=torch.int16, device="cuda")
    m.MoeBlock(layer, T).forward(h0, to_dev16(acts[0][1]), n0)
    torch.cuda.synchronize()
    assert O.max_rel_err(hid[0].cpu().numpy(), h0.cpu().numpy()) < 2.0 ** -8
    assert O.max_rel_err(O.bf16_to_f32(host16(nrm[0])), O.bf16_to_f32(host16(n0))) < TOL_BF16
    assert ranks[0].error_word() == 0


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_emulated_ranks_against_oracle(orc, world):
    L, layer = layer128()
    Ts = [40 + 13 * r for r in range(world)]
    nr = O.f32_to_bf16(1.0 + 0.1 * O.normal(171, 1, S128.H)) if world == 4 else None
    ranks, acts, hid, nrm, C = run_emulated(layer, world, Ts, 600 + world, next_rms1=nr)
    C = np.array(C)
    for r in range(world):
        hidden, attn = acts[r]
        ref = orc.ep_block_forward(S128, L, hidden, attn, world, next_rms1=nr)
        tr = ranks[r].src.trace(Ts[r])
        gl = tr["logits"].cpu().numpy()
        check_routing(orc, S128, gl, tr["idx"].cpu().numpy(), tr["wts"].cpu().numpy(), ref["logits"], ref["idx"],
                      ref["wts"], logit_tol=2e-3)
        ok = stable_rows(S128, ref["logits"], gpu_logits=gl)
        assert O.max_rel_err(hid[r].cpu().numpy()[ok], ref["hidden"][ok]) < TOL_BF16
        assert O.max_rel_err(O.bf16_to_f32(host16(nrm[r])[ok]), O.bf16_to_f32(ref["normed"][ok])) < TOL_BF16
        # the plan: records per destination = tokens with >= 1 expert on it
        owner = tr["idx"].cpu().numpy() // (S128.E // world)
        want = [int((owner == d).any(axis=1).sum()) for d in range(world)]
        assert list(C[r]) == want
        pos = ranks[r].tok_pos[:Ts[r]].cpu().numpy()
        for d in range(world):
            sent = (owner == d).any(axis=1)
            base = C[r][:d].sum()
            assert np.array_equal(pos[sent, d], base + np.arange(sent.sum()))
            assert (pos[~sent, d] == -1).all()
        assert ranks[r].error_word() == 0


def test_emulated_routed_against_oracle_int4(orc):
    """The routed partials themselves (int4 bar) through the returned rows: hidden - residual - gated shared."""
    L, layer = layer128()
    world, Ts = 2, [64, 96]
    ranks, acts, hid, nrm, _ = run_emulated(layer, world, Ts, 700)
    for r in range(world):
        hidden, attn = acts[r]
        ref = orc.ep_block_forward(S128, L, hidden, attn, world)
        S = int(ranks[r].send_count.sum())
        pos = ranks[r].tok_pos[:Ts[r]].cpu().numpy()
        ret = O.bf16_to_f32(host16(ranks[r].ret[:S]))
        routed = np.zeros((Ts[r], S128.H), np.float32)
        for d in range(world):
            on = pos[:, d] >= 0
            routed[on] += ret[pos[on, d]]
        tr = ranks[r].src.trace(Ts[r])
        ok = stable_rows(S128, ref["logits"], gpu_logits=tr["logits"].cpu().numpy())
        assert O.max_rel_err(routed[ok], ref["routed"][ok]) < TOL_INT4


def test_world8_matches_world1_full_geometry():
    """BASELINE geometry (H=2048, E=256, top-8, I=Is=512, G=64) on the device generator: the same 1024 tokens on one
    rank and split over 8 ranks give the same block output up to the bf16 rounding of the returned partial rows (one
    per rank) and the fp32 summation order."""
    m = mb()
    E = ep()
    ms = m.MoeShape()
    layer = m.synth_layer(ms, seed=13)
    hid, att = m.synth_activations(ms, 1024, 17)
    torch.cuda.synchronize()
    outs = {}
    for world in (1, 8):
        T = 1024 // world
        ranks = [E.EpRank(layer, r, world, T) for r in range(world)]
        hs = [hid[r * T:(r + 1) * T].clone() for r in range(world)]
        at = [att[r * T:(r + 1) * T].contiguous() for r in range(world)]
        nm = [torch.zeros(T, ms.H, dtype=torch.int16, device="cuda") for _ in range(world)]
        E.emulated_step(ranks, hs, at, nm)
        torch.cuda.synchronize()
        outs[world] = (torch.cat(hs).cpu().numpy(), torch.cat(nm).cpu().numpy())
        assert all(r.error_word() == 0 for r in ranks)
        del ranks
    h1, n1 = outs[1]
    h8, n8 = outs[8]
    assert O.max_rel_err(h8, h1) < 2.0 ** -8
    assert O.max_rel_err(O.bf16_to_f32(n8.view(np.uint16)), O.bf16_to_f32(n1.view(np.uint16))) < TOL_BF16


def test_all_tokens_on_one_shard():
    """A router bias that sends every pick to rank 0's experts: rank 1 receives no record (R = 0) and sends its tokens
    only to rank 0; results still match the oracle."""
    m = mb()
    E = ep()
    L, layer = layer128()
    world = 2
    bias = np.where(np.arange(S128.E) < S128.E // world, 50.0, 0.0).astype(np.float32)
    t = dict(layer.t)
    t["router_bias"] = torch.from_numpy(bias).cuda()
    blayer = m.MoeLayer(layer.shape, t)
    Lb = dict(L)
    Lb["router_bias"] = bias
    ranks, acts, hid, nrm, C = run_emulated(blayer, world, [24, 40], 800)
    assert C[0][1] == 0 and C[1][1] == 0
    orc = O.Oracle()
    for r in range(world):
        ref = orc.ep_block_forward(S128, Lb, acts[r][0], acts[r][1], world)
        tr = ranks[r].src.trace(acts[r][0].shape[0])
        ok = stable_rows(S128, ref["logits"], gpu_logits=tr["logits"].cpu().numpy())
        assert O.max_rel_err(hid[r].cpu().numpy()[ok], ref["hidden"][ok]) < TOL_BF16
        assert ranks[r].error_word() == 0


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_peer_exchange_equals_packed_exchange(world):
    """The peer-memory exchange (records and partial rows stored by the kernels into the other ranks' buffers) gives
    the packed all-to-all exchange's results bit for bit: same records, same reductions, same rank order."""
    E = ep()
    L, layer = layer128()
    Ts = [30 + 11 * r for r in range(world)]
    a_ranks, acts, a_hid, a_nrm, _ = run_emulated(layer, world, Ts, 900 + world)
    b_ranks = [E.EpRank(layer, r, world, max(Ts)) for r in range(world)]
    hid = [torch.from_numpy(np.ascontiguousarray(h, np.float32)).cuda() for h, _ in acts]
    att = [to_dev16(a) for _, a in acts]
    nrm = [torch.zeros(T, S128.H, dtype=torch.int16, device="cuda") for T in Ts]
    E.emulated_step_peers(b_ranks, hid, att, nrm)
    torch.cuda.synchronize()
    for r in range(world):
        assert np.array_equal(hid[r].cpu().numpy(), a_hid[r].cpu().numpy())
        assert np.array_equal(host16(nrm[r]), host16(a_nrm[r]))
        assert b_ranks[r].error_word() == 0
    # a second step on the same buffers (stale counts and records of the first must not leak)
    E.emulated_step_peers(b_ranks, hid, att, nrm)
    E.emulated_step(a_ranks, a_hid, [to_dev16(a) for _, a in acts], a_nrm)
    torch.cuda.synchronize()
    for r in range(world):
        assert np.array_equal(hid[r].cpu().numpy(), a_hid[r].cpu().numpy())
