"""Mixture-of-experts block on the CUDA library (one process per GPU).

The reference has no MoE; the semantics are the library's (see
include/opencuda_cuda.h and oracle/oracle_moe.c).  Every expert is the
reference's GPT MLP shape (fc -> gelu_new -> proj) with INT8 per-channel
weights, evaluated as W8A8 grouped GEMMs on the tcgen05 tensor cores.

moe_forward: one GPU, all experts local; routing, dispatch, both grouped
GEMMs, the shared expert and the combine all run as library kernels.

moe_forward_ep: expert parallelism over a torch.distributed group -- rank r
holds experts [r*E/g, (r+1)*E/g) and its own tokens.  Tokens travel to the
owners of their chosen experts as int8 rows (+ row scale + local expert id)
in one NCCL all-to-all, the owners run their grouped GEMMs, and the expert
outputs travel back in a second all-to-all; the combine happens at the
token's home rank.  Both exchanges use the same split sizes (exchanged
first as counts).  The per-(token, choice) arithmetic is identical to the
single-GPU path, so results are bit-identical.
"""
from __future__ import annotations

from dataclasses import dataclass

import opencuda_cuda as oc


@dataclass
class MoEWeights:
    """INT8 expert weights on one device: w1 [E][F][D] (scales s1 [E*F]),
    w2 [E][D][F] (s2 [E*D]); the shared expert sw1 [F][D], sw2 [D][F]."""

    w1: object
    s1: object
    w2: object
    s2: object
    sw1: object
    ss1: object
    sw2: object
    ss2: object

    @property
    def num_experts(self):
        return self.w1.shape[0]

    @property
    def d_model(self):
        return self.w1.shape[2]

    @property
    def d_ff(self):
        return self.w1.shape[1]


def _t():
    import torch
    return torch


def quantize_expert_weights(W1, W2, SW1, SW2):
    """Per-output-channel INT8 quantization (quantize_int8 with group = in)
    of f32 device weights W1 [E][F][D], W2 [E][D][F] and the shared pair."""
    E, F, D = W1.shape
    q1, s1 = oc.quantize_int8(W1.reshape(-1), D)
    q2, s2 = oc.quantize_int8(W2.reshape(-1), F)
    qs1, ss1 = oc.quantize_int8(SW1.reshape(-1), D)
    qs2, ss2 = oc.quantize_int8(SW2.reshape(-1), F)
    return MoEWeights(q1.view(E, F, D), s1, q2.view(E, D, F), s2, qs1.view(F, D), ss1, qs2.view(D, F), ss2)


def _stream():
    return _t().cuda.current_stream().cuda_stream


def route(logits, k: int):
    torch = _t()
    T, E = logits.shape
    idx = torch.empty(T, k, dtype=torch.int32, device=logits.device)
    w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    oc.check(oc.lib().oc_moe_route(logits.data_ptr(), T, E, k, idx.data_ptr(), w.data_ptr(), _stream()))
    return idx, w


def dispatch(idx, qx, sx, num_groups: int):
    """Groups the (token, choice) rows by idx value (expert or rank)."""
    torch = _t()
    T, k = idx.shape
    D = qx.shape[1]
    dev = qx.device
    counts = torch.empty(num_groups, dtype=torch.int32, device=dev)
    offs = torch.empty(num_groups + 1, dtype=torch.int32, device=dev)
    cursor = torch.empty(num_groups, dtype=torch.int32, device=dev)
    pos = torch.empty(T * k, dtype=torch.int32, device=dev)
    src = torch.empty(max(T * k, 1), dtype=torch.int32, device=dev)
    xg = torch.empty(max(T * k, 1), D, dtype=torch.int8, device=dev)
    sg = torch.empty(max(T * k, 1), dtype=torch.float32, device=dev)
    oc.check(oc.lib().oc_moe_dispatch(idx.data_ptr(), T, k, num_groups, qx.data_ptr(), sx.data_ptr(), D,
                                      counts.data_ptr(), offs.data_ptr(), pos.data_ptr(), src.data_ptr(),
                                      xg.data_ptr(), sg.data_ptr(), cursor.data_ptr(), _stream()))
    return counts, offs, pos, src, xg[: T * k], sg[: T * k]


def grouped_gemm(xg, sg, W, sw, offs, groups: int):
    torch = _t()
    R, K = xg.shape
    N = W.shape[0] // groups if W.dim() == 2 else W.shape[1]
    Y = torch.empty(max(R, 1), N, dtype=torch.float32, device=xg.device)
    oc.check(oc.lib().oc_grouped_igemm_w8a8(R, N, K, xg.data_ptr(), sg.data_ptr(), W.data_ptr(), sw.data_ptr(),
                                            None, offs.data_ptr(), groups, Y.data_ptr(), _stream()))
    return Y[:R]


def gelu_quantize_rows(H):
    torch = _t()
    R, F = H.shape
    q = torch.empty(max(R, 1), F, dtype=torch.int8, device=H.device)
    s = torch.empty(max(R, 1), dtype=torch.float32, device=H.device)
    oc.check(oc.lib().oc_gelu_quantize_rows(H.data_ptr(), R, F, q.data_ptr(), s.data_ptr(), _stream()))
    return q[:R], s[:R]


def experts(xg, sg, offs, w: MoEWeights, first: int, count: int):
    """Expert MLPs on grouped int8 rows (groups = experts first..first+count)."""
    E, F, D = w.w1.shape
    W1 = w.w1[first:first + count].reshape(count * F, D)
    S1 = w.s1[first * F:(first + count) * F]
    W2 = w.w2[first:first + count].reshape(count * D, F)
    S2 = w.s2[first * D:(first + count) * D]
    H = grouped_gemm(xg, sg, W1, S1, offs, count)
    qh, sh = gelu_quantize_rows(H)
    return grouped_gemm(qh, sh, W2, S2, offs, count)


def shared_expert(qx, sx, w: MoEWeights):
    H = oc.igemm_w8a8(qx, sx, w.sw1, w.ss1)
    qh, sh = gelu_quantize_rows(H)
    return oc.igemm_w8a8(qh, sh, w.sw2, w.ss2)


def combine(S, O, pos, topk_w):
    torch = _t()
    T, k = topk_w.shape
    D = O.shape[1] if O.numel() else S.shape[1]
    y = torch.empty(T, D, dtype=torch.float32, device=topk_w.device)
    oc.check(oc.lib().oc_moe_combine(S.data_ptr() if S is not None else None, O.data_ptr(), pos.data_ptr(),
                                     topk_w.data_ptr(), T, k, D, y.data_ptr(), _stream()))
    return y


class CudaOps:
    """The library kernels behind each MoE step (the product path)."""

    quantize_rows = staticmethod(oc.quantize_rows_int8)
    route = staticmethod(route)
    dispatch = staticmethod(dispatch)
    experts = staticmethod(experts)
    shared = staticmethod(shared_expert)
    combine = staticmethod(combine)


def moe_forward(x, logits, w: MoEWeights, k: int, ops=CudaOps):
    """y [T][D] for tokens x [T][D] (f32) with router logits [T][E]."""
    qx, sx = ops.quantize_rows(x)
    idx, tw = ops.route(logits, k)
    E = w.num_experts
    counts, offs, pos, src, xg, sg = ops.dispatch(idx, qx, sx, E)
    O = ops.experts(xg, sg, offs, w, 0, E)
    S = ops.shared(qx, sx, w)
    return ops.combine(S, O, pos, tw)


def _pack_rows(xs, ss, eid):
    """[n][row bytes | scale f32 | local expert int32] as one uint8 message."""
    torch = _t()
    n = xs.shape[0]
    xb = xs.contiguous().view(torch.uint8).view(n, -1)
    buf = torch.empty(n, xb.shape[1] + 8, dtype=torch.uint8, device=xs.device)
    buf[:, : xb.shape[1]] = xb
    buf[:, xb.shape[1]: xb.shape[1] + 4] = ss.contiguous().view(torch.uint8).view(n, 4)
    buf[:, xb.shape[1] + 4:] = eid.contiguous().view(torch.uint8).view(n, 4)
    return buf


def _unpack_rows(buf, row_dtype, D):
    torch = _t()
    n = buf.shape[0]
    rb = buf.shape[1] - 8
    xr = buf[:, :rb].contiguous().view(row_dtype).view(n, D)
    sr = buf[:, rb: rb + 4].contiguous().view(torch.float32).view(n)
    er = buf[:, rb + 4:].contiguous().view(torch.int32).view(n)
    return xr, sr, er


def moe_forward_ep(x, logits, w_local: MoEWeights, num_experts: int, k: int, group=None, ops=CudaOps):
    """Expert-parallel MoE on this rank's tokens x [T][D] with logits [T][E].

    w_local holds this rank's E/g experts ([E/g][F][D] etc.) and the
    replicated shared expert.  Exchanges (NCCL on GPUs, gloo on CPU): the
    per-rank row counts, the packed token rows (one all-to-all) and the
    expert outputs (one all-to-all back)."""
    torch = _t()
    import torch.distributed as dist

    g = dist.get_world_size(group)
    e_loc = num_experts // g
    if e_loc * g != num_experts or w_local.num_experts != e_loc:
        raise ValueError(f"{num_experts} experts do not split into {g} ranks of {w_local.num_experts}")
    T, D = x.shape
    qx, sx = ops.quantize_rows(x)
    idx, tw = ops.route(logits, k)
    dest = torch.div(idx, e_loc, rounding_mode="floor").to(torch.int32)
    # rows grouped by destination rank: dispatch with one group per rank
    cnt_send, _, pos_send, _, xs, ss = ops.dispatch(dest, qx, sx, g)
    eid = torch.empty(T * k, dtype=torch.int32, device=x.device)
    eid[pos_send.long()] = (idx - dest * e_loc).reshape(-1).to(torch.int32)
    cnt_recv = torch.empty_like(cnt_send)
    dist.all_to_all_single(cnt_recv, cnt_send, group=group)
    send_splits = [int(v) for v in cnt_send.tolist()]
    recv_splits = [int(v) for v in cnt_recv.tolist()]
    n_recv = sum(recv_splits)
    sendbuf = _pack_rows(xs, ss, eid)
    recvbuf = torch.empty(n_recv, sendbuf.shape[1], dtype=torch.uint8, device=x.device)
    dist.all_to_all_single(recvbuf, sendbuf, recv_splits, send_splits, group=group)
    if n_recv:
        xr, sr, er = _unpack_rows(recvbuf, qx.dtype, D)
        # rows grouped by local expert, computed, then put back in received order
        _, offs_e, pos_e, _, xe, se = ops.dispatch(er.view(-1, 1), xr, sr, e_loc)
        Oe = ops.experts(xe, se, offs_e, w_local, 0, e_loc)
        Or = Oe.index_select(0, pos_e.long())
    else:
        Or = torch.empty(0, D, dtype=torch.float32, device=x.device)
    Ob = torch.empty(T * k, D, dtype=torch.float32, device=x.device)
    dist.all_to_all_single(Ob, Or.contiguous(), send_splits, recv_splits, group=group)
    S = ops.shared(qx, sx, w_local)
    return ops.combine(S, Ob, pos_send, tw)


def local_experts(w: MoEWeights, rank: int, world: int) -> MoEWeights:
    """The slice of a full MoEWeights that rank `rank` of `world` owns."""
    E, F, D = w.w1.shape
    e = E // world
    a, b = rank * e, (rank + 1) * e
    return MoEWeights(w.w1[a:b], w.s1[a * F:b * F], w.w2[a:b], w.s2[a * D:b * D], w.sw1, w.ss1, w.sw2, w.ss2)


def random_weights(E: int, D: int, F: int, seed: int, device, chunk: int = 16) -> MoEWeights:
    """Seeded random-init expert weights ~ N(0, 0.02) drawn on the device
    (torch's generator, in chunks of experts so the f32 draw stays small)
    and quantized per output channel by the library's quantize_int8."""
    torch = _t()
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    w1 = torch.empty(E, F, D, dtype=torch.int8, device=device)
    w2 = torch.empty(E, D, F, dtype=torch.int8, device=device)
    s1 = torch.empty(E * F, dtype=torch.float32, device=device)
    s2 = torch.empty(E * D, dtype=torch.float32, device=device)
    for a in range(0, E, chunk):
        b = min(E, a + chunk)
        for W, S, shape, inner in ((w1, s1, (b - a, F, D), D), (w2, s2, (b - a, D, F), F)):
            f = torch.randn(*shape, generator=gen, device=device, dtype=torch.float32).mul_(0.02)
            q, s = oc.quantize_int8(f, inner)
            W[a:b].view(-1).copy_(q)
            S[a * shape[1]:b * shape[1]].copy_(s)
            del f
    f1 = torch.randn(F, D, generator=gen, device=device).mul_(0.02)
    f2 = torch.randn(D, F, generator=gen, device=device).mul_(0.02)
    q1, t1 = oc.quantize_int8(f1, D)
    q2, t2 = oc.quantize_int8(f2, F)
    return MoEWeights(w1, s1, w2, s2, q1.view(F, D), t1, q2.view(D, F), t2)
