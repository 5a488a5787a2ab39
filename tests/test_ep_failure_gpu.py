"""Failure detection of the expert-parallel step on 2 GPUs (skipped with fewer), without a GPU fault: two ranks run
a complete step over NCCL (the packed all-to-all exchange, no peer mappings; NVLS off), then rank 1 leaves between
steps -- none of its kernels or collectives in flight -- without tearing the group down. Rank 0's next step must end
with mvcc_b200.ep.EpError on the host, before it launches any collective of that step: the layer's liveness check
(every rank posts a key to the process group's store before a step and waits a bounded time for its peers') runs
out instead of a collective waiting for the missing rank."""
import datetime
import os
import socket
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2
PG_TIMEOUT_S = 15
LIVENESS_S = 5


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    # NVLS off in NCCL; a timed-out collective raises in the calling thread instead of the watchdog ending the process
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["TORCH_NCCL_BLOCKING_WAIT"] = "1"
    os.environ["TORCH_NCCL_ASYNC_ERROR_HANDLING"] = "0"
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=PG_TIMEOUT_S),
                            device_id=torch.device("cuda", rank))
    try:
        from oracle import oracle as O
        from tests.test_decode_gpu import to_dev16, upload
        import mvcc_b200.ep as E
        s = O.Shape(H=1024, E=128, TOPK=8, I=512, Is=512, G=64)
        layer = upload(s, O.make_layer(s, 43))
        T = 40 + 9 * rank
        hidden, attn = O.make_activations(s, T, 950 + rank)
        h = torch.from_numpy(np.ascontiguousarray(hidden, np.float32)).cuda()
        a = to_dev16(attn)
        n = torch.zeros(T, s.H, dtype=torch.int16, device="cuda")
        moe = E.ExpertParallelMoe(layer, 64, exchange="nccl", liveness_s=LIVENESS_S)
        moe.forward(h, a, n)  # step 1: every rank takes part
        torch.cuda.synchronize()
        if rank == world - 1:  # leaves between steps, nothing in flight, without destroying the group
            q.put((rank, "left", 0.0, int(moe.error_word())))
            q.close()
            q.join_thread()
            os._exit(0)
        t0 = time.monotonic()
        try:
            moe.forward(h, a, n)
            torch.cuda.synchronize()
            out = "completed"
        except E.EpError as e:
            out = f"EpError: {e}"
        q.put((rank, out, time.monotonic() - t0, 0))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, f"unexpected: {e!r}", 0.0, -1))
    q.close()
    q.join_thread()
    os._exit(0)  # the group lost a member: exit without a collective teardown


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_rank_leaving_between_steps_ends_the_next_step_with_ep_error():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, WORLD, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    try:
        res = sorted(q.get(timeout=240) for _ in range(WORLD))
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.exitcode is None:
                p.kill()
    assert res[-1][:2] == (WORLD - 1, "left") and res[-1][3] == 0, res
    rank, out, dt, _ = res[0]
    assert rank == 0 and out.startswith("EpError: ") and "rank 0" in out and "not reached" in out, res
    assert dt < LIVENESS_S + 30, res  # ended by the liveness check, not a hang
