"""MoE block on the GPU against the oracle: routing bit-exact, dispatch
invariants, the grouped tcgen05 GEMM against per-expert W8A8 products, the
gelu + requantize step, and the whole block (small shapes against the
oracle block; the full DeepSeek-style shape -- 8192 tokens, 256 experts,
top-8, d_model 7168, d_ff 2048 -- on sampled tokens)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

import oracle  # noqa: E402
import synth  # noqa: E402


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda", 0)


@pytest.fixture(scope="module")
def moe():
    import moe as m
    return m


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("T,E,k", [(1, 4, 1), (333, 64, 6), (1000, 256, 8)])
def test_route_bit_exact(dev, moe, T, E, k):
    lg = synth.normal(30 + T, T * E).reshape(T, E)
    lg[::7, 3] = lg[::7, 1]  # ties
    lg[::11, 0] = np.nan
    idx, w = moe.route(torch.from_numpy(lg).to(dev), k)
    ridx, rw = oracle.moe_route(lg, T, E, k)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert np.array_equal(_bits(w.cpu().numpy()), _bits(rw))


def test_route_all_nan_row_uniform(dev, moe):
    lg = np.full((2, 8), np.nan, np.float32)
    lg[1] = np.arange(8)
    idx, w = moe.route(torch.from_numpy(lg).to(dev), 4)
    assert idx.cpu().tolist()[0] == [0, 1, 2, 3] and w.cpu().tolist()[0] == [0.25] * 4
    ridx, rw = oracle.moe_route(lg, 2, 8, 4)
    assert np.array_equal(idx.cpu().numpy(), ridx) and np.array_equal(_bits(w.cpu().numpy()), _bits(rw))


def test_dispatch_invariants(dev, moe):
    T, E, k, D = 777, 32, 4, 80
    lg = synth.normal(41, T * E).reshape(T, E)
    lg[:, 9] = -1e9  # expert 9 gets nothing
    idx, _ = moe.route(torch.from_numpy(lg).to(dev), k)
    qx = torch.randint(-127, 128, (T, D), dtype=torch.int8, device=dev)
    sx = torch.rand(T, device=dev)
    counts, offs, pos, src, xg, sg = moe.dispatch(idx, qx, sx, E)
    I = idx.cpu().numpy().ravel()
    c = counts.cpu().numpy()
    o = offs.cpu().numpy()
    p = pos.cpu().numpy()
    assert np.array_equal(c, np.bincount(I, minlength=E)) and c[9] == 0
    assert o[0] == 0 and np.array_equal(np.diff(o), c) and o[-1] == T * k
    assert np.array_equal(np.sort(p), np.arange(T * k))
    grp = np.searchsorted(o, p, side="right") - 1
    assert np.array_equal(grp, I)  # every pair lands in its expert's rows
    tok = np.repeat(np.arange(T), k)
    assert np.array_equal(src.cpu().numpy()[p], tok)
    assert torch.equal(xg[pos.long()], qx[torch.from_numpy(tok).to(dev)])
    assert torch.equal(sg[pos.long()], sx[torch.from_numpy(tok).to(dev)])


@pytest.mark.parametrize("sizes,N,K", [([0, 5, 128, 300, 1, 0, 129], 384, 256), ([2048] * 4, 2048, 7168),
                                       ([17], 256, 64)])
def test_grouped_gemm_matches_per_expert(dev, moe, sizes, N, K):
    import opencuda_cuda as oc

    G = len(sizes)
    R = sum(sizes)
    g = torch.Generator(device=dev)
    g.manual_seed(R + N)
    xg = torch.randint(-127, 128, (R, K), dtype=torch.int8, device=dev, generator=g)
    sg = torch.rand(R, device=dev, generator=g) * 0.01
    W = torch.randint(-127, 128, (G * N, K), dtype=torch.int8, device=dev, generator=g)
    sw = torch.rand(G * N, device=dev, generator=g) * 0.01
    offs = torch.tensor(np.concatenate([[0], np.cumsum(sizes)]), dtype=torch.int32, device=dev)
    Y = moe.grouped_gemm(xg, sg, W, sw, offs, G)
    for e in range(G):
        a, b = int(offs[e]), int(offs[e + 1])
        if a == b:
            continue
        ref = oc.igemm_w8a8(xg[a:b].contiguous(), sg[a:b].contiguous(), W[e * N:(e + 1) * N].contiguous(),
                            sw[e * N:(e + 1) * N].contiguous())
        assert torch.equal(Y[a:b].view(torch.int32), ref.view(torch.int32)), e


def test_gelu_quantize_rows(dev, moe):
    R, F = 300, 2048
    H = torch.from_numpy(synth.uniform(51, R * F, -4.0, 4.0).reshape(R, F)).to(dev)
    q, s = moe.gelu_quantize_rows(H)
    g = oracle.gelu(H.cpu().numpy())
    rq, rs = oracle.quantize_rows_int8(g, R, F)
    assert np.array_equal(_bits(s.cpu().numpy()), _bits(rs))
    assert np.array_equal(q.cpu().numpy().ravel(), rq)


def _device_weights(w, dev, moe):
    return moe.MoEWeights(*[torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in w])


def _quantized_case(T, D, F, E, seed):
    x, lg, W1, W2, SW1, SW2 = synth.moe_case(T, D, F, E, seed)
    q = [oracle.quantize_int8(W.ravel(), W.shape[-1]) for W in (W1, W2, SW1, SW2)]
    w = (q[0].data.reshape(E, F, D), q[0].scales, q[1].data.reshape(E, D, F), q[1].scales,
         q[2].data.reshape(F, D), q[2].scales, q[3].data.reshape(D, F), q[3].scales)
    return x, lg, w


@pytest.mark.parametrize("T,D,F,E,k", [(1, 64, 64, 4, 2), (96, 256, 384, 16, 4), (500, 512, 256, 64, 6)])
def test_moe_block_matches_oracle(dev, moe, T, D, F, E, k):
    x, lg, w = _quantized_case(T, D, F, E, 60 + T)
    y = moe.moe_forward(torch.from_numpy(x).to(dev), torch.from_numpy(lg).to(dev), _device_weights(w, dev, moe), k)
    ref = oracle.moe_forward(x, lg, *w, k)
    assert np.array_equal(_bits(y.cpu().numpy()), _bits(ref))


def test_moe_full_shape_sampled_tokens(dev, moe):
    """8192 tokens, 256 experts (d_ff 2048), top-8, d_model 7168 + shared."""
    T, D, F, E, k = 8192, 7168, 2048, 256, 8
    w = moe.random_weights(E, D, F, 5, dev)
    x = torch.from_numpy(synth.uniform(70, T * D).reshape(T, D)).to(dev)
    lg = torch.from_numpy(synth.normal(71, T * E).reshape(T, E)).to(dev)
    y = moe.moe_forward(x, lg, w, k)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
    rows = [0, 1, 4095, 8191, 1234, 7777]
    lgs = lg[rows].cpu().numpy()
    idx, tw = oracle.moe_route(lgs, len(rows), E, k)
    cpu = lambda t: t.cpu().numpy()

    def mlp(xr, w1, s1, w2, s2):
        h = oracle.gelu(oracle.qgemm_w8a8(1, D, F, xr, cpu(w1), cpu(s1), None))
        return oracle.qgemm_w8a8(1, F, D, h, cpu(w2), cpu(s2), None)

    for j, t in enumerate(rows):
        xr = x[t].cpu().numpy()
        ref = mlp(xr, w.sw1, w.ss1, w.sw2, w.ss2)
        for i in range(k):
            e = int(idx[j, i])
            ref = ref + tw[j, i] * mlp(xr, w.w1[e], w.s1[e * F:(e + 1) * F], w.w2[e], w.s2[e * D:(e + 1) * D])
        assert np.array_equal(_bits(y[t].cpu().numpy()), _bits(ref)), t


def _ep_worker(rank, world, port, q):
    import datetime
    import os

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
        import moe
        import synth

        T, D, F, E, k = 2048, 1024, 512, 32, 4
        full = moe.random_weights(E, D, F, 9, dev)
        x = torch.from_numpy(synth.uniform(80, T * D).reshape(T, D)).to(dev)
        lg = torch.from_numpy(synth.normal(81, T * E).reshape(T, E)).to(dev)
        lg[: T // 2, 0] += 3.0  # rank 0's tokens prefer rank 0's experts
        t0, t1 = rank * T // world, (rank + 1) * T // world
        y = moe.moe_forward_ep(x[t0:t1], lg[t0:t1], moe.local_experts(full, rank, world), E, k)
        ref = moe.moe_forward(x[t0:t1], lg[t0:t1], full, k)
        torch.cuda.synchronize()
        q.put((rank, "ok" if torch.equal(y.view(torch.int32), ref.view(torch.int32)) else "mismatch"))
    except Exception as e:
        q.put((rank, f"error:{e}"))
    finally:
        dist.destroy_process_group()


def test_expert_parallel_two_gpus_matches_single_gpu():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import socket

    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_ep_worker, args=(r, 2, port, q)) for r in range(2)]
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
