"""Expert-parallel MoE layer: the block of `MoeBlock` with its routed experts sharded over the GPUs of one node.

Rank d of `world` holds experts [d * E / world, (d + 1) * E / world) and the replicated router, norm and shared
expert. One step on each rank (include/moe_ep.h):

  1. dispatch: residual RMSNorm, router + top-k, one record per (token, rank owning >= 1 of its experts);
  2. the shared expert of the rank's own tokens on a side stream, overlapping 3-4;
  3. the records reach their ranks, which run their experts over them -> one bf16 partial row per record (summed
     in fp32, rounded once);
  4. the partial rows return to their source ranks; combine: per token the partials in rank order + the gated shared
     expert into hidden.

Two exchanges. `ep_step_peers` (the default of ExpertParallelMoe): the dispatch kernel stores each record into the
destination rank's receive buffer and the expert stage stores each partial row into the source rank's return buffer,
over NVLink through CUDA IPC mappings, with a one-element all-reduce after each stage as the barrier that publishes
the stores; no host synchronisation. `ep_step`: packed buffers through all_to_all_single (the W x W count matrix
all-gathered and read back to the host for the split sizes and checked on every rank, then records and partial rows). `emulated_step` / `emulated_step_peers` run every
rank's stages in one process on one GPU, for single-GPU parity tests of the multi-rank numerics. The reference runs
the block on one GPU only (qwen.cu:429-448); the split has no counterpart there.
"""
import contextlib
import ctypes
import dataclasses

import torch

from . import (MoeBlock, MoeError, MoeLayer, MoeLayerWeights, MoeShape, _check, _lib, _ptr, _stream)


class MoeEpPeers(ctypes.Structure):
    """ctypes mirror of `moe_ep_peers` (include/moe_ep.h)."""

    _fields_ = [("recv", ctypes.c_void_p * 8), ("rcount", ctypes.c_void_p * 8), ("ret", ctypes.c_void_p * 8),
                ("rank", ctypes.c_int32), ("cap", ctypes.c_int32)]


class DeviceBuffer:
    """cudaMalloc'd device memory (shareable through CUDA IPC) owned by this object."""

    def __init__(self, nbytes):
        p = ctypes.c_void_p()
        _check(_lib.moe_device_alloc(nbytes, ctypes.byref(p)), "moe_device_alloc")
        self.ptr, self.nbytes = p.value, nbytes

    def ipc_handle(self):
        h = ctypes.create_string_buffer(64)
        _check(_lib.moe_ipc_handle(ctypes.c_void_p(self.ptr), h), "moe_ipc_handle")
        return h.raw

    def free(self):
        if self.ptr:
            _lib.moe_device_free(ctypes.c_void_p(self.ptr))
            self.ptr = None

    def __del__(self):
        if _lib is not None:  # not during interpreter teardown
            self.free()


def _ipc_open(handle):
    p = ctypes.c_void_p()
    _check(_lib.moe_ipc_open(ctypes.create_string_buffer(handle, 64), ctypes.byref(p)), "moe_ipc_open")
    return p.value


class ExpertShard:
    """Rank `rank`'s routed experts of `layer` (tensors of the shard only; E = E / world) as a moe_layer_weights
    whose router and shared-expert pointers are NULL: moe_ep_experts reads the expert tensors alone."""

    def __init__(self, layer: MoeLayer, rank: int, world: int, copy=True):
        s = layer.shape
        if world < 1 or s.E % world:
            raise ValueError(f"E={s.E} does not split over {world} ranks")
        El = s.E // world
        self.shape = dataclasses.replace(s, E=El)
        self.rank, self.world, self.first = rank, world, rank * El
        self.t = {}
        for n in ("exp_gu_q", "exp_gu_s", "exp_dn_q", "exp_dn_s"):
            v = layer.t[n][rank * El:(rank + 1) * El]
            self.t[n] = v.clone() if copy else v
        null = ctypes.c_void_p()
        self.c = MoeLayerWeights(null, null, *[ctypes.c_void_p(self.t[n].data_ptr()) for n in
                                               ("exp_gu_q", "exp_gu_s", "exp_dn_q", "exp_dn_s")],
                                 null, null, null, s.H, El, s.TOPK, s.I, s.Is, s.G, s.eps, None)


class EpRank:
    """One rank's state and stages: buffers sized for up to `max_tokens` tokens on every rank."""

    def __init__(self, layer: MoeLayer, rank: int, world: int, max_tokens: int, device=None, copy_shard=True):
        s = layer.shape
        self.layer, self.shape = layer, s
        self.rank, self.world, self.max_tokens = rank, world, max_tokens
        self.device = layer.t["router"].device if device is None else torch.device(device)
        self.shard = ExpertShard(layer, rank, world, copy=copy_shard)
        self.src = MoeBlock(layer, max_tokens)      # dispatch + combine workspace
        self.sh = MoeBlock(layer, max_tokens)       # shared-expert workspace (side stream)
        cap = max_tokens * world                    # records a rank can send or receive
        self.rec_bytes = _lib.moe_ep_record_bytes(ctypes.byref(layer.c))
        xb = _lib.moe_workspace_bytes(ctypes.byref(self.shard.c), max(8, cap))
        if self.rec_bytes == 0 or xb == 0:
            raise ValueError("moe_ep: unsupported geometry")
        dev = self.device
        self.xws_bytes = xb
        self.xws = torch.empty(xb, dtype=torch.uint8, device=dev)
        _check(_lib.moe_workspace_init(_ptr(self.xws), xb, _stream(None)), "moe_workspace_init")
        self.send = torch.empty(cap, self.rec_bytes, dtype=torch.uint8, device=dev)
        self.recv = torch.empty(cap, self.rec_bytes, dtype=torch.uint8, device=dev)
        self.send_count = torch.zeros(world, dtype=torch.int32, device=dev)
        self.recv_count = torch.zeros(world, dtype=torch.int32, device=dev)
        self.tok_pos = torch.empty(max_tokens, world, dtype=torch.int32, device=dev)
        self.part = torch.empty(cap, s.H, dtype=torch.int16, device=dev)  # bf16 partial rows
        self.ret = torch.empty(cap, s.H, dtype=torch.int16, device=dev)
        self.sout = torch.empty(max_tokens, s.H, dtype=torch.int16, device=dev)
        self.side = torch.cuda.Stream(device=dev)
        self._shared_done = None
        # peer-mode exchange buffers: records in ([world][cap][record] + counts), bf16 partial rows back
        # ([world][cap][H])
        lc = ctypes.byref(layer.c)
        self.recv_bytes = _lib.moe_ep_recv_bytes(lc, world, max_tokens)
        self.ret_bytes = _lib.moe_ep_ret_bytes(lc, world, max_tokens)
        self.rcount_off = _lib.moe_ep_rcount_offset(lc, world, max_tokens)
        self.precv = DeviceBuffer(self.recv_bytes)
        self.pret = DeviceBuffer(self.ret_bytes)
        self.peers = None
        self._opened = []
        torch.cuda.current_stream(dev).synchronize()

    def set_peers(self, recv_ptrs, ret_ptrs):
        """Every rank's receive and return buffers as addresses valid on this device (rank order)."""
        pe = MoeEpPeers()
        for d in range(self.world):
            pe.recv[d] = recv_ptrs[d]
            pe.rcount[d] = recv_ptrs[d] + self.rcount_off
            pe.ret[d] = ret_ptrs[d]
        pe.rank, pe.cap = self.rank, self.max_tokens
        self.peers = pe

    def open_peers(self, group=None):
        """Exchange CUDA IPC handles of the exchange buffers over the process group and map the peers' buffers."""
        import torch.distributed as dist
        mine = (self.precv.ipc_handle(), self.pret.ipc_handle())
        allh = [None] * self.world
        dist.all_gather_object(allh, mine, group=group)
        recv, ret = [], []
        for d in range(self.world):
            if d == self.rank:
                recv.append(self.precv.ptr)
                ret.append(self.pret.ptr)
            else:
                pr, pt = _ipc_open(allh[d][0]), _ipc_open(allh[d][1])
                self._opened += [pr, pt]
                recv.append(pr)
                ret.append(pt)
        self.set_peers(recv, ret)

    def close_peers(self):
        for p in self._opened:
            _lib.moe_ipc_close(ctypes.c_void_p(p))
        self._opened = []
        self.peers = None

    # -- peer-mode stages
    def _need_peers(self):
        if self.peers is None:
            raise MoeError("peer exchange buffers are not mapped: call open_peers() (or set_peers()) first")

    def dispatch_peers(self, hidden, attn_out, normed, stream):
        self._need_peers()
        T = hidden.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens > max_tokens {self.max_tokens}")
        _check(_lib.moe_ep_dispatch_peers(ctypes.byref(self.layer.c), _ptr(self.src.ws), self.src.ws_bytes,
                                          _ptr(hidden), _ptr(attn_out), _ptr(normed), T, self.world,
                                          ctypes.byref(self.peers), _ptr(self.send_count), _ptr(self.tok_pos),
                                          _stream(stream)), "moe_ep_dispatch_peers")
        self.side.wait_stream(stream)
        _check(_lib.moe_shared_expert(ctypes.byref(self.layer.c), _ptr(self.sh.ws), self.sh.ws_bytes, _ptr(normed),
                                      _ptr(self.sout), T, _stream(self.side)), "moe_shared_expert")
        self._shared_done = torch.cuda.Event()
        self._shared_done.record(self.side)

    def experts_peers(self, stream):
        self._need_peers()
        _check(_lib.moe_ep_experts_peers(ctypes.byref(self.shard.c), _ptr(self.xws), self.xws_bytes, self.world,
                                         ctypes.byref(self.peers), _stream(stream)), "moe_ep_experts_peers")

    def combine_peers(self, hidden, attn_out, normed, next_rms1, stream):
        T = hidden.shape[0]
        stream.wait_event(self._shared_done)
        _check(_lib.moe_ep_combine(ctypes.byref(self.layer.c), _ptr(self.src.ws), self.src.ws_bytes, _ptr(hidden),
                                   _ptr(attn_out), _ptr(self.sout), _ptr(normed), _ptr(next_rms1), T, self.world,
                                   _ptr(self.tok_pos), ctypes.c_void_p(self.pret.ptr), _stream(stream)),
               "moe_ep_combine")

    # -- stages (all asynchronous on `stream`)
    def dispatch(self, hidden, attn_out, normed, stream):
        T = hidden.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens > max_tokens {self.max_tokens}")
        _check(_lib.moe_ep_dispatch(ctypes.byref(self.layer.c), _ptr(self.src.ws), self.src.ws_bytes, _ptr(hidden),
                                    _ptr(attn_out), _ptr(normed), T, self.world, _ptr(self.send),
                                    _ptr(self.send_count), _ptr(self.tok_pos), _stream(stream)), "moe_ep_dispatch")
        # the shared expert needs normed only: run it beside the exchange
        self.side.wait_stream(stream)
        _check(_lib.moe_shared_expert(ctypes.byref(self.layer.c), _ptr(self.sh.ws), self.sh.ws_bytes, _ptr(normed),
                                      _ptr(self.sout), T, _stream(self.side)), "moe_shared_expert")
        self._shared_done = torch.cuda.Event()
        self._shared_done.record(self.side)

    def experts(self, R, stream):
        _check(_lib.moe_ep_experts(ctypes.byref(self.shard.c), _ptr(self.xws), self.xws_bytes, _ptr(self.recv), R,
                                   _ptr(self.part), _stream(stream)), "moe_ep_experts")

    def combine(self, hidden, attn_out, normed, next_rms1, stream):
        T = hidden.shape[0]
        stream.wait_event(self._shared_done)
        _check(_lib.moe_ep_combine(ctypes.byref(self.layer.c), _ptr(self.src.ws), self.src.ws_bytes, _ptr(hidden),
                                   _ptr(attn_out), _ptr(self.sout), _ptr(normed), _ptr(next_rms1), T, self.world,
                                   _ptr(self.tok_pos), _ptr(self.ret), _stream(stream)), "moe_ep_combine")

    def error_word(self):
        """Error bits recorded by this rank's kernels since the last read (the three workspaces)."""
        w = self.src.error_word() | self.sh.error_word()
        rc = _lib.moe_workspace_error(_ptr(self.xws), self.xws_bytes, _stream(None))
        if rc < 0:
            raise RuntimeError(f"moe_workspace_error failed: cudaError {-rc}")
        return w | rc


class EpError(MoeError):
    """An expert-parallel step that cannot complete: a bad record count, or an exchange that failed (a rank that
    left, stalled past the process group's timeout, or whose collective errored)."""


def check_count_matrix(counts, per_source):
    """counts[s][d] = records rank s sends to rank d. A token goes at most once to each rank, so every entry lies in
    [0, per_source] (the receive buffer holds per_source records from each source). Raises EpError on the first
    entry outside that range, naming the source and destination ranks."""
    for s, row in enumerate(counts):
        for d, v in enumerate(row):
            if not 0 <= v <= per_source:
                raise EpError(f"rank {s} reports {v} records for rank {d} (valid: 0..{per_source}); "
                              "step abandoned on every rank before the record exchange")


class NcclExchange:
    """The exchanges of one rank over a torch.distributed process group (NCCL on GPUs, gloo in the CPU tests)."""

    def __init__(self, group=None):
        self.group = group

    def counts(self, rank_state):
        """Per-destination record counts out, per-source counts in, as host lists. The whole W x W count matrix is
        all-gathered (read back to the host once) and every rank checks all of it, so a bad count stops every rank
        at the same point with the same EpError: no rank enters the record exchange with sizes its peers disagree
        with."""
        import torch.distributed as dist
        W, r = rank_state.world, rank_state.rank
        flat = torch.empty(W * W, dtype=torch.int32, device=rank_state.send_count.device)
        dist.all_gather_into_tensor(flat, rank_state.send_count, group=self.group)
        mat = flat.view(W, W)
        host = mat.cpu().tolist()
        check_count_matrix(host, rank_state.recv.shape[0] // W)
        rank_state.recv_count.copy_(mat[:, r])
        return host[r], [row[r] for row in host]

    def a2a(self, out, inp, out_splits, in_splits):
        import torch.distributed as dist
        if out.dtype == torch.int16:  # bf16 bit patterns (the partial rows): NCCL has no 16-bit integer type
            out, inp = out.view(torch.bfloat16), inp.view(torch.bfloat16)
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)


def ep_step(rank_state, exchange, hidden, attn_out, normed, next_rms1=None, stream=None):
    """One expert-parallel step of one rank (every rank of the group calls it with its own tokens):
    hidden (fp32 [T,H], in/out), attn_out (bf16 bits [T,H]), normed (out), as MoeBlock.forward."""
    if rank_state.device.type == "cuda":
        st = torch.cuda.current_stream(rank_state.device) if stream is None else stream
        ctx = torch.cuda.stream(st)
    else:  # host-side doubles of the stages (CPU tests over gloo)
        st, ctx = None, contextlib.nullcontext()
    stage = "dispatch"
    try:
        with ctx:
            rank_state.dispatch(hidden, attn_out, normed, st)
            stage = "count exchange"
            sc, rc = exchange.counts(rank_state)
            S, R = sum(sc), sum(rc)
            stage = "record exchange"
            exchange.a2a(rank_state.recv[:R], rank_state.send[:S], rc, sc)
            stage = "experts"
            rank_state.experts(R, st)
            stage = "partial-row exchange"
            exchange.a2a(rank_state.ret[:S], rank_state.part[:R], sc, rc)
            stage = "combine"
            rank_state.combine(hidden, attn_out, normed, next_rms1, st)
    except EpError:
        raise
    except RuntimeError as e:  # collective errors and timeouts (torch.distributed raises RuntimeError subclasses)
        raise EpError(f"rank {rank_state.rank}: expert-parallel step failed in the {stage}: {e}") from e
    return S, R


EP_STAGES = ("dispatch", "barrier_1", "experts", "barrier_2", "combine")


def ep_step_peers(rank_state, hidden, attn_out, normed, next_rms1=None, stream=None, group=None, flag=None,
                  events=None):
    """One expert-parallel step of one rank with the peer-memory exchange: the dispatch kernel stores the records
    into the destination ranks' buffers and the expert stage stores the partial rows into the source ranks' buffers
    (NVLink); a one-element all-reduce after each publishes the stores to every rank. No host synchronisation.
    `events` (optional, 6 CUDA events) are recorded on the stream before the step and after each of its stages
    (EP_STAGES) for a per-stage time split."""
    import torch.distributed as dist
    st = torch.cuda.current_stream(rank_state.device) if stream is None else stream
    if flag is None:
        flag = torch.zeros(1, device=rank_state.device)

    def mark(i):
        if events is not None:
            events[i].record(st)

    with torch.cuda.stream(st):
        mark(0)
        rank_state.dispatch_peers(hidden, attn_out, normed, st)
        mark(1)
        dist.all_reduce(flag, group=group)
        mark(2)
        rank_state.experts_peers(st)
        mark(3)
        dist.all_reduce(flag, group=group)
        mark(4)
        rank_state.combine_peers(hidden, attn_out, normed, next_rms1, st)
        mark(5)


class ExpertParallelMoe:
    """The expert-parallel MoE layer of one rank: `forward` is MoeBlock.forward for this rank's tokens, with the
    routed experts sharded over the process group."""

    def __init__(self, layer: MoeLayer, max_tokens: int, group=None, rank=None, world=None, exchange="peers",
                 liveness_s=None):
        """exchange: "peers" (records and partial rows stored by the kernels into the peers' buffers over NVLink,
        CUDA IPC mappings set up here) or "nccl" (all_to_all_single of packed buffers, one host read per step)."""
        import torch.distributed as dist
        self.group = group
        self.rank = dist.get_rank(group) if rank is None else rank
        self.world = dist.get_world_size(group) if world is None else world
        self.state = EpRank(layer, self.rank, self.world, max_tokens)
        self.mode = exchange
        # liveness_s (optional): before every step each rank posts a key to the process group's store and waits at
        # most this long for every peer's: a rank that has left is found on the host, before any collective of the
        # step is launched (a collective waiting for a peer that is gone would hold its GPU until the group's
        # timeout, or for good where the timeout cannot end it)
        self.liveness_s = liveness_s
        self._steps = 0
        self._store = None
        if liveness_s is not None:
            from torch.distributed import distributed_c10d as c10d
            self._store = c10d._get_default_store()
        self.exchange = NcclExchange(group)
        self.flag = torch.zeros(1, device=self.state.device)
        if exchange == "peers":
            self.state.open_peers(group)
        elif exchange != "nccl":
            raise ValueError(f"unknown exchange {exchange!r}")

    def _check_peers(self):
        """Every rank reaches step k or this rank raises EpError (the store's wait runs out)."""
        import datetime
        k = self._steps
        self._steps += 1
        st = self._store
        st.set(f"mvcc_ep/{k}/{self.rank}", "1")
        try:
            st.wait([f"mvcc_ep/{k}/{d}" for d in range(self.world)], datetime.timedelta(seconds=self.liveness_s))
        except Exception as e:  # noqa: BLE001 -- the store raises its own timeout / connection errors
            raise EpError(f"rank {self.rank}: expert-parallel step {k} not reached by every rank within "
                          f"{self.liveness_s} s ({e})") from e
        if k >= 2:
            st.delete_key(f"mvcc_ep/{k - 2}/{self.rank}")

    def forward(self, hidden, attn_out, normed, next_rms1=None, stream=None):
        if self._store is not None:
            self._check_peers()
        if self.mode == "peers":
            return ep_step_peers(self.state, hidden, attn_out, normed, next_rms1, stream, self.group, self.flag)
        return ep_step(self.state, self.exchange, hidden, attn_out, normed, next_rms1, stream)

    def close(self):
        """Unmaps the peers' buffers (before the process group goes away)."""
        self.state.close_peers()

    def error_word(self):
        return self.state.error_word()


def emulated_step(ranks, hiddens, attn_outs, normeds, next_rms1=None, stream=None):
    """All ranks of an expert-parallel step in one process (every EpRank on one device, exchanges as device copies
    in the order the all-to-alls define): the multi-rank numerics on a single GPU."""
    W = len(ranks)
    st = torch.cuda.current_stream() if stream is None else stream
    with torch.cuda.stream(st):
        for r in range(W):
            ranks[r].dispatch(hiddens[r], attn_outs[r], normeds[r], st)
        C = torch.stack([r.send_count for r in ranks]).cpu().tolist()  # C[s][d]
        soff = [[sum(C[s][:d]) for d in range(W)] for s in range(W)]
        roff = [[sum(C[x][d] for x in range(s)) for s in range(W)] for d in range(W)]  # roff[d][s]
        R = [sum(C[s][d] for s in range(W)) for d in range(W)]
        for d in range(W):
            for s in range(W):
                n = C[s][d]
                if n:
                    ranks[d].recv[roff[d][s]:roff[d][s] + n].copy_(ranks[s].send[soff[s][d]:soff[s][d] + n])
        for d in range(W):
            ranks[d].experts(R[d], st)
        for s in range(W):
            for d in range(W):
                n = C[s][d]
                if n:
                    ranks[s].ret[soff[s][d]:soff[s][d] + n].copy_(ranks[d].part[roff[d][s]:roff[d][s] + n])
        for r in range(W):
            ranks[r].combine(hiddens[r], attn_outs[r], normeds[r], next_rms1, st)
    return C


def emulated_step_peers(ranks, hiddens, attn_outs, normeds, next_rms1=None, stream=None):
    """All ranks of a peer-mode step in one process on one GPU: every rank's buffers are local, each rank's kernels
    store into the others' buffers directly, and stream order stands in for the barriers."""
    W = len(ranks)
    recv = [r.precv.ptr for r in ranks]
    ret = [r.pret.ptr for r in ranks]
    for r in ranks:
        if r.peers is None:
            r.set_peers(recv, ret)
    st = torch.cuda.current_stream() if stream is None else stream
    with torch.cuda.stream(st):
        for r in range(W):
            ranks[r].dispatch_peers(hiddens[r], attn_outs[r], normeds[r], st)
        for r in range(W):
            ranks[r].experts_peers(st)
        for r in range(W):
            ranks[r].combine_peers(hiddens[r], attn_outs[r], normeds[r], next_rms1, st)


__all__ = ["ExpertShard", "EpRank", "NcclExchange", "ExpertParallelMoe", "ep_step", "ep_step_peers", "emulated_step",
           "emulated_step_peers", "MoeShape", "MoeEpPeers", "DeviceBuffer", "EpError", "check_count_matrix"]
