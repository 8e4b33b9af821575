"""The oracle reproduces the committed golden fixtures (tests/golden/,
written by tests/golden/make_golden.py) bit for bit, and every fixture is
self-consistent with the reference semantics it was drawn from (CPU)."""
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLD, name))


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_sgemm_golden(oracle):
    g = load("sgemm_17x33x29.npz")
    m, k, n = int(g["m"]), int(g["k"]), int(g["n"])
    for faithful in (False, True):
        C = oracle.sgemm(m, k, n, float(g["alpha"]), g["A"], g["B"], float(g["beta"]), g["C0"].copy(),
                         faithful=faithful)
        assert np.array_equal(bits(C), bits(g["C"]))


def test_qgemm_golden(oracle):
    g = load("qgemm_9x256x96.npz")
    m, k, n, grp = (int(g[x]) for x in ("m", "k", "n", "group"))
    t8 = oracle.quantize_int8(g["WT"].ravel(), k)
    t4 = oracle.quantize_int4(g["WT"].ravel(), grp)
    assert np.array_equal(t8.data, g["q8"]) and np.array_equal(t4.data, g["q4"])
    y8, acc8 = oracle.qgemm_w8a8(m, k, n, g["A"], g["q8"], g["s8"], g["bias"], want_acc=True)
    y4, acc4 = oracle.qgemm_w4a8(m, k, n, grp, g["A"], g["q4"], g["s4"], g["bias"], want_acc=True)
    assert np.array_equal(bits(y8), bits(g["y8"])) and np.array_equal(acc8, g["acc8"])
    assert np.array_equal(bits(y4), bits(g["y4"])) and np.array_equal(acc4, g["acc4"])
    # exact accumulators equal the integer products of the quantized operands
    qa, sa = oracle.quantize_rows_int8(g["A"], m, k)
    ref = qa.reshape(m, k).astype(np.int64) @ g["q8"].reshape(n, k).astype(np.int64).T
    assert np.array_equal(acc8.reshape(m, n), ref)


def test_attention_golden(oracle):
    g = load("attention_17x8.npz")
    seq, d, blk = int(g["seq"]), int(g["d"]), int(g["block"])
    assert np.array_equal(bits(oracle.flash_attention(g["q"], g["k"], g["v"], seq, d, blk)), bits(g["flash"]))
    assert np.array_equal(bits(oracle.scaled_dot_product_attention(g["q"], g["k"], g["v"], seq, d)),
                          bits(g["sdpa"]))
    np.testing.assert_allclose(g["flash"], g["sdpa"], atol=1e-5)


def test_mla_golden(oracle):
    g = load("mla_12x64x16.npz")
    seq, dh, dc = int(g["seq"]), int(g["dh"]), int(g["dc"])
    lat = oracle.mla_compress_kv(seq, dh, dc, g["kv"], g["down"])
    assert np.array_equal(bits(lat), bits(g["latent"]))
    assert np.array_equal(bits(oracle.mla_decompress_kv(seq, dc, dh, lat, g["up"])), bits(g["recon"]))


def test_gpt_golden(oracle):
    g = load("gpt_tiny_seed42.npz")
    cfg = oracle.GptConfig(int(g["vocab"]), int(g["hidden"]), int(g["layers"]), int(g["heads"]), int(g["inter"]),
                           int(g["ctx"]), float(g["eps"]))
    m = oracle.GptModel(cfg, int(g["seed"]))
    m.set_attention(flash=True, block=4)
    toks, logits = m.generate(g["prompt"], len(g["tokens"]), want_logits=True)
    assert toks.tolist() == g["tokens"].tolist()
    assert np.array_equal(bits(logits), bits(g["logits"]))
    assert [int(np.argmax(r)) for r in g["logits"]] == g["tokens"].tolist()


def test_moe_golden(oracle):
    g = load("moe_10x64.npz")
    k = int(g["k"])
    idx, tw = oracle.moe_route(g["logits"], int(g["T"]), int(g["E"]), k)
    assert np.array_equal(idx, g["idx"]) and np.array_equal(bits(tw), bits(g["tw"]))
    y = oracle.moe_forward(g["x"], g["logits"], g["w1"], g["s1"], g["w2"], g["s2"], g["sw1"], g["ss1"], g["sw2"],
                           g["ss2"], k)
    assert np.array_equal(bits(y), bits(g["y"]))


def test_gpt2_124m_golden_prefix(oracle):
    """The GPT-2 124M decode fixture (tests/golden/make_gpt2_golden.py): the
    oracle reproduces the first 12 tokens of sequence 0 and their logits at
    the stored vocabulary ids bit for bit; the fixture's prompts are the
    workload's prompts."""
    import synth
    g = load("gpt2_124m_seed3_128tok.npz")
    assert np.array_equal(g["prompts"], synth.gpt_prompts(32, 32))
    model = oracle.GptModel(oracle.GptConfig.gpt2_124m(), int(g["seed"]))
    model.set_attention(flash=True, block=int(g["block"]))
    toks, lg = model.generate(g["prompts"][0], 12, want_logits=True)
    assert toks.tolist() == g["tokens"][0][:12].tolist()
    assert np.array_equal(bits(lg[:, g["sub_idx"]]), bits(g["sub_seq0"][:12]))
    assert np.all(g["margin"] > 0) and np.array_equal(g["tokens"][:, :12][0], toks)
