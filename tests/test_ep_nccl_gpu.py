"""Expert-parallel step on 2 GPUs (skipped with fewer), with either exchange: NCCL all-to-all of packed buffers, or
the kernels' own peer-memory stores over NVLink (CUDA IPC mappings) with all-reduce barriers. Every rank runs
mvcc_b200.ep.ExpertParallelMoe on its own tokens; its result must equal, bit for bit, the single-process emulation of
the same ranks (the exchange moves bytes, so both run the same kernels on the same data), and match the oracle's
expert-parallel restatement within the block's tolerances."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank, world, port, q, mode):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from oracle import oracle as O
        from tests.test_decode_gpu import TOL_BF16, host16, stable_rows, to_dev16, upload
        import mvcc_b200.ep as E
        s = O.Shape(H=1024, E=128, TOPK=8, I=512, Is=512, G=64)
        L = O.make_layer(s, 41)
        layer = upload(s, L)
        Ts = [48 + 17 * r for r in range(world)]
        acts = [O.make_activations(s, T, 900 + r) for r, T in enumerate(Ts)]

        def dev(r):
            h = torch.from_numpy(np.ascontiguousarray(acts[r][0], np.float32)).cuda()
            return h, to_dev16(acts[r][1]), torch.zeros(Ts[r], s.H, dtype=torch.int16, device="cuda")

        h, a, n = dev(rank)
        moe = E.ExpertParallelMoe(layer, max(Ts), exchange=mode)
        moe.forward(h, a, n)
        torch.cuda.synchronize()
        err = moe.error_word()
        moe.close()
        # the same ranks emulated in this process
        ranks = [E.EpRank(layer, r, world, max(Ts)) for r in range(world)]
        hs, as_, ns = zip(*[dev(r) for r in range(world)])
        E.emulated_step(ranks, list(hs), list(as_), list(ns))
        torch.cuda.synchronize()
        same = np.array_equal(h.cpu().numpy(), hs[rank].cpu().numpy()) and \
            np.array_equal(host16(n), host16(ns[rank]))
        ref = O.Oracle().ep_block_forward(s, L, acts[rank][0], acts[rank][1], world)
        tr = moe.state.src.trace(Ts[rank])
        ok = stable_rows(s, ref["logits"], gpu_logits=tr["logits"].cpu().numpy())
        close = O.max_rel_err(h.cpu().numpy()[ok], ref["hidden"][ok]) < TOL_BF16
        q.put((rank, bool(same), bool(close), int(err)))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, False, False, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["nccl", "peers"])
def test_ep_step_over_nccl_matches_emulation(mode):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, WORLD, port, q, mode)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), res
    assert all(same and close and err == 0 for _, same, close, err in res), res
