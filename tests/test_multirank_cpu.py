"""World-size-2 tests of the (batch*head) sharding path on CPU (gloo).

The attention itself is the C oracle here (a CPU stand-in for the kernel);
what is under test is the host-side partition, the output all-gather and
the failure behaviour of the collective, which are the same code the GPU
benchmark runs over NCCL.
"""
import multiprocessing as mp
import os
import socket
import traceback

import pytest
import torch


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port, timeout_s=20):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _worker_gather(rank, world, port, q):
    try:
        import oracle
        from rocm_attn_b200.sharding import sharded_forward
        from rocm_attn_b200.workloads import Shape, make_qkv

        dist = _init(rank, world, port)
        err = 0.0
        # 6 slices over 2 ranks (equal shards: gathered in place) and 5 slices
        # (3 + 2: padded for the collective, then reassembled)
        for shape in (Shape(2, 3, 20, 24, 64), Shape(1, 5, 17, 9, 64)):
            qq, kk, vv = make_qkv(shape, torch.float32, seed=5)
            full = sharded_forward(oracle.c_oracle_forward, qq, kk, vv, causal=True, world=world, rank=rank,
                                   gather=True)
            ref = oracle.c_oracle_forward(qq, kk, vv, causal=True)
            assert full.shape == ref.shape
            err = max(err, oracle.max_abs_err(full, ref))
        # max-over-ranks reduction used for timing
        t = torch.tensor([float(rank + 1)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        q.put((rank, err, float(t.item())))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


def _worker_fail(rank, world, port, q):
    try:
        dist = _init(rank, world, port, timeout_s=5)
        if rank == 1:
            raise RuntimeError("rank 1 fails before the collective")
        try:
            t = torch.zeros(4)
            dist.all_reduce(t)
            q.put((rank, "no-error"))
        except Exception as e:  # the surviving rank must see an error, not hang
            q.put((rank, "detected", type(e).__name__))
    except RuntimeError as e:
        q.put((rank, "raised", str(e)))


def _run(target, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = []
    for _ in range(world):
        out.append(q.get(timeout=timeout))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda x: x[0])


def test_sharded_forward_gathers_full_output():
    res = _run(_worker_gather)
    for rank, err, tmax in res:
        assert err != "error", tmax
        assert err < 1e-6
        assert tmax == 2.0


def test_failed_rank_is_detected_not_hung():
    res = _run(_worker_fail)
    assert res[1][1] == "raised"
    assert res[0][1] == "detected", res[0]
