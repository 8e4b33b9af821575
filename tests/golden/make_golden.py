"""Generates the golden input/output fixtures in this folder from the CPU
oracle (run once; the .npz files are committed).  The oracle is pinned to
the reference's own known-answer tests (tests/test_oracle_kat.py); these
fixtures freeze its outputs on small seeded inputs so the CUDA parity tests
and the oracle's regression test compare against fixed vectors.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "open-cuda_b200"), os.path.join(ROOT, "tests")):
    sys.path.insert(0, p)

import oracle  # noqa: E402
import synth  # noqa: E402


def sgemm():
    m, k, n = 17, 33, 29
    v = synth.normal(0, m * k + k * n + m * n, 0.0, 0.02)
    A, B, C0 = v[: m * k], v[m * k: m * k + k * n], v[m * k + k * n:]
    C = oracle.sgemm(m, k, n, 1.5, A, B, 0.5, C0.copy())
    np.savez_compressed(os.path.join(HERE, "sgemm_17x33x29.npz"), m=m, k=k, n=n, alpha=1.5, beta=0.5, A=A, B=B,
                        C0=C0, C=C)


def qgemm():
    m, k, n, g = 9, 256, 96, 32
    A, WT, bias = synth.qgemm_case(m, k, n, 1, 2, 3)
    t8 = oracle.quantize_int8(WT.ravel(), k)
    t4 = oracle.quantize_int4(WT.ravel(), g)
    y8, acc8 = oracle.qgemm_w8a8(m, k, n, A, t8.data, t8.scales, bias, want_acc=True)
    y4, acc4 = oracle.qgemm_w4a8(m, k, n, g, A, t4.data, t4.scales, bias, want_acc=True)
    np.savez_compressed(os.path.join(HERE, "qgemm_9x256x96.npz"), m=m, k=k, n=n, group=g, A=A, WT=WT, bias=bias,
                        q8=t8.data, s8=t8.scales, q4=t4.data, s4=t4.scales, y8=y8, acc8=acc8, y4=y4, acc4=acc4)


def attention():
    seq, d, block = 17, 8, 5
    q = synth.uniform(11, seq * d)
    k = synth.uniform(12, seq * d)
    v = synth.uniform(13, seq * d)
    flash = oracle.flash_attention(q, k, v, seq, d, block)
    sdpa = oracle.scaled_dot_product_attention(q, k, v, seq, d)
    np.savez_compressed(os.path.join(HERE, "attention_17x8.npz"), seq=seq, d=d, block=block, q=q, k=k, v=v,
                        flash=flash, sdpa=sdpa)


def mla():
    seq, dh, dc = 12, 64, 16
    kv = synth.normal(21, seq * dh, 0.0, 0.02)
    down = synth.normal(22, dh * dc, 0.0, 0.02)
    up = synth.normal(23, dc * dh, 0.0, 0.02)
    lat = oracle.mla_compress_kv(seq, dh, dc, kv, down)
    rec = oracle.mla_decompress_kv(seq, dc, dh, lat, up)
    np.savez_compressed(os.path.join(HERE, "mla_12x64x16.npz"), seq=seq, dh=dh, dc=dc, kv=kv, down=down, up=up,
                        latent=lat, recon=rec)


def gpt():
    vocab, seed, new = 97, 42, 6
    cfg = oracle.GptConfig(vocab, 64, 2, 4, 256, 64, 1e-5)
    prompt = np.array([104, 105], np.uint32) % vocab
    m = oracle.GptModel(cfg, seed)
    m.set_attention(flash=True, block=4)
    toks, logits = m.generate(prompt, new, want_logits=True)
    np.savez_compressed(os.path.join(HERE, "gpt_tiny_seed42.npz"), vocab=vocab, hidden=64, layers=2, heads=4,
                        inter=256, ctx=64, eps=1e-5, seed=seed, prompt=prompt, tokens=toks, logits=logits)


def moe():
    T, D, F, E, k = 10, 64, 48, 6, 2
    x, lg, W1, W2, SW1, SW2 = synth.moe_case(T, D, F, E, 31)
    q = [oracle.quantize_int8(W.ravel(), W.shape[-1]) for W in (W1, W2, SW1, SW2)]
    w = (q[0].data.reshape(E, F, D), q[0].scales, q[1].data.reshape(E, D, F), q[1].scales,
         q[2].data.reshape(F, D), q[2].scales, q[3].data.reshape(D, F), q[3].scales)
    y = oracle.moe_forward(x, lg, *w, k)
    idx, tw = oracle.moe_route(lg, T, E, k)
    np.savez_compressed(os.path.join(HERE, "moe_10x64.npz"), T=T, D=D, F=F, E=E, k=k, x=x, logits=lg,
                        w1=w[0], s1=w[1], w2=w[2], s2=w[3], sw1=w[4], ss1=w[5], sw2=w[6], ss2=w[7], idx=idx, tw=tw,
                        y=y)


if __name__ == "__main__":
    oracle.build()
    for f in (sgemm, qgemm, attention, mla, gpt, moe):
        f()
    print("golden fixtures written to", HERE)
