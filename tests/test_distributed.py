"""Multi-process host logic on CPU (gloo, world size 2): the DDP helpers of
subq_audio.engine (reference python/subq_audio/engine.py:202-238) and failure
detection by process-group timeout. No GPU is used and none is faulted: a
failing rank is a host process that exits before a collective.
"""
import multiprocessing as mp
import os
import socket
import time
import traceback


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _ddp_rank(rank, world, port, q):
    try:
        os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world),
                          MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch

        from subq_audio.engine import (cleanup_distributed, create_distributed_dataloader, setup_distributed,
                                       wrap_model_ddp)

        r, lr, ws = setup_distributed(backend="gloo", timeout_s=30)
        assert (r, lr, ws) == (rank, rank, world)
        torch.manual_seed(0)
        model = wrap_model_ddp(torch.nn.Linear(8, 4))
        data = torch.arange(40, dtype=torch.float32).view(10, 4)
        ds = torch.utils.data.TensorDataset(torch.arange(10))
        dl = create_distributed_dataloader(ds, batch_size=5, rank=rank, world_size=world, shuffle=False)
        seen = [int(i) for (b,) in dl for i in b]
        x = torch.full((3, 8), float(rank + 1))
        model(x).sum().backward()
        g = model.module.weight.grad.clone()
        q.put((rank, seen, g.tolist(), float(data.sum())))
        cleanup_distributed()
    except Exception:  # report to the parent instead of hanging it
        q.put((rank, "error", traceback.format_exc(), None))


def _run(target, world, extra=()):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + tuple(extra)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    deadline = time.time() + 120
    while len(out) < world and time.time() < deadline:
        try:
            r, *rest = q.get(timeout=5)
            out[r] = rest
        except Exception:
            if not any(p.is_alive() for p in procs):
                break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
            p.join()
    return out


def test_ddp_helpers_allreduce_gradients_and_shard_data():
    out = _run(_ddp_rank, 2)
    assert set(out) == {0, 1}, out
    for r in (0, 1):
        assert out[r][0] != "error", out[r][1]
    # the sampler gives the ranks disjoint halves of the dataset
    assert sorted(out[0][0] + out[1][0]) == list(range(10))
    assert not set(out[0][0]) & set(out[1][0])
    # DDP averaged the gradients: both ranks hold the same values, the mean of
    # the per-rank gradients (inputs 1 and 2 -> mean input 1.5, 3 rows)
    g0, g1 = out[0][1], out[1][1]
    assert g0 == g1
    assert abs(g0[0][0] - 1.5 * 3) < 1e-5


def _dropout_rank(rank, world, port, q):
    try:
        os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world),
                          MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch
        import torch.distributed as dist

        from subq_audio.engine import setup_distributed

        setup_distributed(backend="gloo", timeout_s=5)
        t = torch.ones(4)
        dist.all_reduce(t)  # step 1: every rank takes part
        if rank == 1:
            q.put((rank, "left", None, None))
            q.close()
            q.join_thread()  # flush the message before the abrupt exit
            os._exit(0)  # leaves between steps, with no collective in flight
        t0 = time.time()
        try:
            dist.all_reduce(t)  # step 2: the peer is gone
            q.put((rank, "no error", time.time() - t0, None))
        except Exception as e:  # noqa: BLE001
            q.put((rank, "detected", time.time() - t0, type(e).__name__))
    except Exception:
        q.put((rank, "error", traceback.format_exc(), None))


def test_lost_rank_is_detected_by_the_survivor():
    out = _run(_dropout_rank, 2)
    assert out.get(1, [None])[0] == "left", out
    status, waited, _ = out[0]
    assert status == "detected", out[0]
    assert waited < 60
