"""Column-sharded INT4 GEMM (W4A8 and weight-only) on 2+ GPUs (one process per GPU, NCCL
all-gather): the gathered [M][N] result must equal, bit for bit, the
shards' products computed on one GPU and laid side by side (the exchange
and layout add nothing to the arithmetic).
Skipped when fewer than two GPUs are visible."""
import datetime
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, shape, q, weight_only=False):
    import torch
    import torch.distributed as dist

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        import opencuda_cuda as oc
        import shard
        import synth

        m, k, n, g = shape
        A, WT, bias = synth.qgemm_case(m, k, n, 4, 5, 6)
        Wd = torch.from_numpy(WT).to(dev)
        q4, s4 = oc.quantize_int4(Wd, g)
        Ad = torch.from_numpy(A).to(dev)
        bd = torch.from_numpy(bias).to(dev)
        plan = shard.ColumnShard(n, world)
        sharded = shard.sharded_qgemm_w4 if weight_only else shard.sharded_qgemm_w4a8
        single = (lambda a, w, sc, grp, b: oc.qgemm_w4(a, w, sc, grp, bias=b)) if weight_only else oc.qgemm_w4a8
        y = sharded(Ad, q4, s4, g, bd, plan, rank)
        # the gathered result must equal, bit for bit, each shard's product
        # computed on one GPU and laid side by side
        parts = []
        for r in range(world):
            (b0, b1), (s0, s1) = plan.w4_slices(r, k, g)
            r0, r1 = plan.rows(r)
            parts.append(single(Ad, q4[b0:b1], s4[s0:s1], g, bd[r0:r1]))
        full = torch.cat(parts, dim=1)
        torch.cuda.synchronize()
        ok = torch.equal(y.view(torch.int32), full.view(torch.int32))
        q.put((rank, "ok" if ok else "mismatch"))
    except Exception as e:
        q.put((rank, f"error:{e}"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("weight_only", [False, True])
@pytest.mark.parametrize("shape", [(64, 3584, 3584, 32), (512, 3584, 18944, 32), (1, 3584, 152064, 32)])
def test_sharded_w4a8_matches_single_gpu(shape, weight_only):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shape, q, weight_only)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
    res = {}
    while not q.empty():
        r, v = q.get()
        res[r] = v
    assert res == {0: "ok", 1: "ok"}, res
