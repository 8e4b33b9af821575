"""Expert-parallel MoE exchange logic on CPU ranks (gloo).

moe.moe_forward_ep runs unchanged with the oracle stand-ins of each step
(tests/moe_oracle_ops.py): every rank owns E/g experts and T/g tokens, rows
travel to the experts' owners in one all-to-all and come back in another.
Each rank's output must equal the single-process oracle on its tokens bit
for bit.  A rank that leaves before the exchange makes the others' collective
fail within the group timeout."""
import datetime
import os
import socket

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _case():
    import oracle
    import synth

    T, D, F, E, k = 24, 64, 48, 8, 3
    x, lg, W1, W2, SW1, SW2 = synth.moe_case(T, D, F, E, 21)
    # skew the router so one expert gets no tokens and one rank gets most rows
    lg[:, 5] = -50.0
    lg[:, 0] += 2.0
    q = [oracle.quantize_int8(W.ravel(), W.shape[-1]) for W in (W1, W2, SW1, SW2)]
    w = (q[0].data.reshape(E, F, D), q[0].scales, q[1].data.reshape(E, D, F), q[1].scales,
         q[2].data.reshape(F, D), q[2].scales, q[3].data.reshape(D, F), q[3].scales)
    return T, D, F, E, k, x, lg, w


def _worker(rank, world, port, mode, result_q):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        import moe
        import oracle
        from moe_oracle_ops import OracleOps

        T, D, F, E, k, x, lg, w = _case()
        full = moe.MoEWeights(*[torch.from_numpy(np.ascontiguousarray(a)) for a in w])
        local = moe.local_experts(full, rank, world)
        t0, t1 = rank * T // world, (rank + 1) * T // world
        if mode == "dropout" and rank == world - 1:
            result_q.put((rank, "left"))
            return
        try:
            y = moe.moe_forward_ep(torch.from_numpy(x[t0:t1]), torch.from_numpy(lg[t0:t1]), local, E, k,
                                   ops=OracleOps)
        except Exception as e:
            result_q.put((rank, f"error:{type(e).__name__}"))
            return
        ref = oracle.moe_forward(x, lg, *w, k)[t0:t1]
        ok = np.array_equal(y.numpy().view(np.uint32), ref.view(np.uint32))
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


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_matches_single_process(world):
    assert _run(world, "normal") == {r: "ok" for r in range(world)}


def test_single_process_ops_match_oracle():
    import torch

    import moe
    import oracle
    from moe_oracle_ops import OracleOps

    T, D, F, E, k, x, lg, w = _case()
    full = moe.MoEWeights(*[torch.from_numpy(np.ascontiguousarray(a)) for a in w])
    y = moe.moe_forward(torch.from_numpy(x), torch.from_numpy(lg), full, k, ops=OracleOps)
    ref = oracle.moe_forward(x, lg, *w, k)
    assert np.array_equal(y.numpy().view(np.uint32), ref.view(np.uint32))


def test_rank_dropout_fails_exchange_instead_of_hanging():
    res = _run(2, "dropout")
    assert res.get(1) == "left"
    assert res.get(0, "").startswith("error:")
