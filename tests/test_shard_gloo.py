"""Host-side logic of the column-sharded quantized matmul, on CPU ranks.

world_size-2 gloo process groups stand in for the GPUs: each rank computes
its column block with the oracle, the blocks are all-gathered and laid out
by the same code the GPU path uses, and the result must equal the unsharded
oracle bit for bit.  A rank that leaves before the collective must make the
other rank's collective fail within the group timeout (no hang)."""
import datetime
import os
import socket
import sys

import numpy as np
import pytest

import shard


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_partition_math():
    plan = shard.ColumnShard(152064, 8)
    assert plan.cols == 19008 and plan.rows(7) == (133056, 152064)
    (b0, b1), (s0, s1) = plan.w4_slices(1, 3584, 32)
    assert (b0, b1) == (19008 * 1792, 2 * 19008 * 1792) and (s0, s1) == (19008 * 112, 2 * 19008 * 112)
    with pytest.raises(ValueError):
        shard.ColumnShard(10, 3)
    with pytest.raises(ValueError):
        plan.rows(8)
    assert shard.ColumnShard(3584, 1).rows(0) == (0, 3584)


def _worker(rank, world, port, mode, result_q):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        import oracle
        import synth

        m, k, n, g = 5, 256, 96, 32
        A, WT, bias = synth.qgemm_case(m, k, n, 1, 2, 3)
        t4 = oracle.quantize_int4(WT.ravel(), g)
        plan = shard.ColumnShard(n, world)
        (b0, b1), (s0, s1) = plan.w4_slices(rank, k, g)
        r0, r1 = plan.rows(rank)
        if mode == "dropout" and rank == 1:
            result_q.put((rank, "left"))
            return  # leaves without joining the collective
        local = oracle.qgemm_w4a8(m, k, plan.cols, g, A, t4.data[b0:b1], t4.scales[s0:s1], bias[r0:r1])
        try:
            full = shard.gather_columns(torch.from_numpy(local.reshape(m, plan.cols)), plan)
        except Exception as e:  # the collective fails instead of hanging
            result_q.put((rank, f"error:{type(e).__name__}"))
            return
        ref = oracle.qgemm_w4a8(m, k, n, g, A, t4.data, t4.scales, bias)
        ok = np.array_equal(full.numpy().ravel().view(np.uint32), ref.view(np.uint32))
        result_q.put((rank, "ok" if ok else "mismatch"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, mode):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    res = {}
    while not q.empty():
        r, v = q.get()
        res[r] = v
    return res


def test_gloo_two_ranks_gather_matches_unsharded():
    res = _run(2, "normal")
    assert res == {0: "ok", 1: "ok"}


def test_rank_dropout_fails_collective_instead_of_hanging():
    res = _run(2, "dropout")
    assert res.get(1) == "left"
    assert res.get(0, "").startswith("error:")
