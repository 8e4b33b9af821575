"""CPU stand-ins for the MoE steps, built on the oracle (test helper only).

They let the expert-parallel exchange logic of moe.moe_forward_ep run on
gloo CPU ranks: token rows travel as f32 (each expert re-quantizes its rows
per row, exactly as the oracle's W8A8 product does), dispatch is a stable
sort by key, and every expert MLP is the oracle's W8A8 -> gelu_new -> W8A8."""
import numpy as np
import torch

import oracle


class OracleOps:
    @staticmethod
    def quantize_rows(x):
        return x.contiguous(), torch.zeros(x.shape[0], dtype=torch.float32)

    @staticmethod
    def route(logits, k):
        T, E = logits.shape
        idx, w = oracle.moe_route(logits.numpy(), T, E, k)
        return torch.from_numpy(idx), torch.from_numpy(w)

    @staticmethod
    def dispatch(keys, rows, scales, groups):
        n, k = keys.shape
        flat = keys.reshape(-1).numpy().astype(np.int64)
        order = np.argsort(flat, kind="stable")
        counts = np.bincount(flat, minlength=groups).astype(np.int32)
        offs = np.zeros(groups + 1, np.int32)
        offs[1:] = np.cumsum(counts)
        pos = np.empty(n * k, np.int32)
        pos[order] = np.arange(n * k, dtype=np.int32)
        src = (order // k).astype(np.int32)
        s = torch.from_numpy(src).long()
        return (torch.from_numpy(counts), torch.from_numpy(offs), torch.from_numpy(pos), torch.from_numpy(src),
                rows[s], scales[s])

    @staticmethod
    def _mlp(x, w1, s1, w2, s2):
        R, D = x.shape
        F = w1.shape[0]
        if R == 0:
            return np.zeros((0, D), np.float32)
        h = oracle.qgemm_w8a8(R, D, F, x, w1.numpy(), s1.numpy(), None)
        h = oracle.gelu(h)
        return oracle.qgemm_w8a8(R, F, D, h, w2.numpy(), s2.numpy(), None).reshape(R, D)

    @staticmethod
    def experts(xg, sg, offs, w, first, count):
        E, F, D = w.w1.shape
        out = np.zeros((xg.shape[0], D), np.float32)
        o = offs.numpy()
        for e in range(first, first + count):
            a, b = int(o[e - first]), int(o[e - first + 1])
            out[a:b] = OracleOps._mlp(xg[a:b].numpy(), w.w1[e], w.s1[e * F:(e + 1) * F], w.w2[e],
                                      w.s2[e * D:(e + 1) * D])
        return torch.from_numpy(out)

    @staticmethod
    def shared(x, s, w):
        return torch.from_numpy(OracleOps._mlp(x.numpy(), w.sw1, w.ss1, w.sw2, w.ss2))

    @staticmethod
    def combine(S, O, pos, tw):
        T, k = tw.shape
        y = S.numpy().copy()
        Pn, On, Wn = pos.numpy().reshape(T, k), O.numpy(), tw.numpy()
        for i in range(k):
            y = y + Wn[:, i:i + 1] * On[Pn[:, i]]
        return torch.from_numpy(y)
