"""CPU tests of the expert-parallel host logic (mvcc_b200/ep.py): the step's exchanges over a real torch.distributed
process group (gloo, world sizes 2 and 3, uneven token counts per rank) with the three GPU stages replaced by numpy
doubles that restate their contracts (include/moe_ep.h): dispatch records grouped by destination with local expert
ids, one partial row per received record, partials summed per token in rank order. The result must equal a direct
single-process evaluation bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

H, E, K = 32, 12, 3


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def routing(rank, T):
    rng = np.random.default_rng(100 + rank)
    idx = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    if T > 2:  # one token whose experts all live on rank 0's shard (nothing sent to the others)
        idx[1] = np.arange(K)
    wts = rng.random((T, K)).astype(np.float32)
    return idx, wts


def expert_fn(e, x):
    return (x * np.float32(e + 1) + np.float32(0.25 * e)).astype(np.float32)


class HostRank:
    """numpy double of EpRank's kernels; buffers and counts in the EpRank layout."""

    device = torch.device("cpu")

    def __init__(self, rank, world, max_tokens):
        self.rank, self.world, self.El = rank, world, E // world
        cap = max_tokens * world
        self.rec = 4 * H + 8 * K  # fp32 activations in this double, then ids and weights
        self.send = torch.zeros(cap, self.rec, dtype=torch.uint8)
        self.recv = torch.zeros(cap, self.rec, dtype=torch.uint8)
        self.send_count = torch.zeros(world, dtype=torch.int32)
        self.recv_count = torch.zeros(world, dtype=torch.int32)
        self.part = torch.zeros(cap, H, dtype=torch.float32)
        self.ret = torch.zeros(cap, H, dtype=torch.float32)

    def dispatch(self, hidden, attn_out, normed, stream):
        T = hidden.shape[0]
        x = hidden.numpy()
        self.idx, self.wts = routing(self.rank, T)
        owner = self.idx // self.El
        self.tok_pos = -np.ones((T, self.world), np.int32)
        send = self.send.numpy()
        pos = 0
        for d in range(self.world):
            n = 0
            for t in range(T):
                if not (owner[t] == d).any():
                    continue
                rec = send[pos]
                rec[:4 * H] = x[t].view(np.uint8)
                ids = np.where(owner[t] == d, self.idx[t] - d * self.El, -1).astype(np.int32)
                rec[4 * H:4 * H + 4 * K] = ids.view(np.uint8)
                rec[4 * H + 4 * K:] = self.wts[t].view(np.uint8)
                self.tok_pos[t, d] = pos
                pos += 1
                n += 1
            self.send_count[d] = n

    def experts(self, R, stream):
        recv = self.recv.numpy()
        part = self.part.numpy()
        for r in range(R):
            x = recv[r, :4 * H].view(np.float32)
            ids = recv[r, 4 * H:4 * H + 4 * K].view(np.int32)
            w = recv[r, 4 * H + 4 * K:].view(np.float32)
            acc = np.zeros(H, np.float32)
            for k in range(K):
                if ids[k] >= 0:
                    acc = acc + w[k] * expert_fn(ids[k] + self.rank * self.El, x)
            part[r] = acc

    def combine(self, hidden, attn_out, normed, next_rms1, stream):
        h = hidden.numpy()
        ret = self.ret.numpy()
        for t in range(h.shape[0]):
            acc = np.zeros(H, np.float32)
            for d in range(self.world):
                if self.tok_pos[t, d] >= 0:
                    acc = acc + ret[self.tok_pos[t, d]]
            h[t] = h[t] + acc


def expected(rank, world, x):
    idx, wts = routing(rank, x.shape[0])
    El = E // world
    out = x.copy()
    for t in range(x.shape[0]):
        acc = np.zeros(H, np.float32)
        for d in range(world):
            if not (idx[t] // El == d).any():
                continue
            p = np.zeros(H, np.float32)
            for k in range(K):
                if idx[t, k] // El == d:
                    p = p + wts[t, k] * expert_fn(idx[t, k], x[t])
            acc = acc + p
        out[t] = out[t] + acc
    return out


def worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mvcc_b200.ep import NcclExchange, ep_step
        T = 5 + 4 * rank
        x = np.random.default_rng(rank).standard_normal((T, H)).astype(np.float32)
        hidden = torch.from_numpy(x.copy())
        st = HostRank(rank, world, max_tokens=16)
        S, R = ep_step(st, NcclExchange(), hidden, None, None)
        ok = np.array_equal(hidden.numpy(), expected(rank, world, x))
        q.put((rank, ok, S, R))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_ep_step_over_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    assert all(ok for _, ok, _, _ in res), res
    # every record sent is received somewhere
    assert sum(S for _, _, S, _ in res) == sum(R for _, _, _, R in res)


# ---------------------------------------------------------------------------------------------- failure detection
# Failures are made on the host among CPU ranks (no GPU is involved): a rank that reports an impossible record count,
# a rank that leaves before the step, a rank that stalls past the process group's timeout. Every surviving rank must
# end its step with EpError within a bound instead of hanging.

PG_TIMEOUT_S = 4


def failing_worker(rank, world, port, q, mode):
    import datetime
    import time
    # the rendezvous gets a long timeout of its own (spawned ranks may take seconds to import torch); the short
    # group timeout bounds the collectives of the step
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=120))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))
    from mvcc_b200.ep import EpError, NcclExchange, ep_step
    x = np.random.default_rng(rank).standard_normal((5 + rank, H)).astype(np.float32)
    st = HostRank(rank, world, max_tokens=16)
    faulty = rank == world - 1
    if mode == "bad_count" and faulty:
        dispatch = st.dispatch

        def bad_dispatch(*a):
            dispatch(*a)
            st.send_count[0] = 10 ** 6  # more records than any rank can receive from one source

        st.dispatch = bad_dispatch
    if mode in ("leaves", "stalls") and faulty:
        if mode == "stalls":
            time.sleep(4 * PG_TIMEOUT_S)
        q.put((rank, "left", 0.0))
        q.close()
        q.join_thread()
        os._exit(0)  # leaves without taking part in the step or tearing the group down
    t0 = time.monotonic()
    try:
        ep_step(st, NcclExchange(), torch.from_numpy(x), None, None)
        out = "completed"
    except EpError as e:
        out = f"EpError: {e}"
    q.put((rank, out, time.monotonic() - t0))
    q.close()
    q.join_thread()
    if mode == "bad_count":  # every rank abandoned the step at the same point: the group is still usable
        dist.barrier()
        dist.destroy_process_group()
    os._exit(0)


def run_failing(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=failing_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = sorted(q.get(timeout=120) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.exitcode is None:
                p.kill()
    return res


@pytest.mark.parametrize("world", [2, 3])
def test_bad_count_stops_every_rank_at_the_same_step(world):
    res = run_failing(world, "bad_count")
    msgs = {out for _, out, _ in res}
    assert len(msgs) == 1, res  # the same verdict on every rank
    (msg,) = msgs
    assert msg.startswith("EpError: ") and f"rank {world - 1} reports 1000000 records for rank 0" in msg


@pytest.mark.parametrize("mode", ["leaves", "stalls"])
def test_missing_rank_ends_the_step_with_an_error(mode):
    world = 3
    res = run_failing(world, mode)
    assert res[-1][:2] == (world - 1, "left")
    for rank, out, dt in res[:-1]:
        assert out.startswith("EpError: ") and "count exchange" in out, res
        assert dt < 3 * PG_TIMEOUT_S + 10, res  # bounded by the group's timeout, not a hang


def liveness_worker(rank, world, port, q):
    """ExpertParallelMoe's step-entry liveness check, alone (no device state): every rank passes step 0, the last rank
    then leaves; the others must raise EpError at step 1 within the check's bound."""
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from torch.distributed import distributed_c10d as c10d

    from mvcc_b200.ep import EpError, ExpertParallelMoe
    moe = object.__new__(ExpertParallelMoe)  # the check only: no layer, no device buffers
    moe.rank, moe.world, moe.liveness_s, moe._steps, moe._store = rank, world, 2, 0, c10d._get_default_store()
    moe._check_peers()  # step 0: everyone arrives
    if rank == world - 1:
        q.put((rank, "left", 0.0))
        q.close()
        q.join_thread()
        os._exit(0)
    t0 = time.monotonic()
    try:
        moe._check_peers()
        out = "passed"
    except EpError as e:
        out = f"EpError: {e}"
    q.put((rank, out, time.monotonic() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


def test_liveness_check_finds_a_rank_that_left_before_any_collective():
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=liveness_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = sorted(q.get(timeout=120) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.exitcode is None:
                p.kill()
    assert res[-1][:2] == (world - 1, "left"), res
    for rank, out, dt in res[:-1]:
        assert out.startswith("EpError: ") and "step 1 not reached" in out, res
        assert dt < 2 + 10, res
