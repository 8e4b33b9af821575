"""The CUDA library against the committed golden fixtures (tests/golden/),
through the C ABI: integer and quantized results bit-exact, f32 results
within the stated relative Frobenius tolerance, GPT tokens identical."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
REL_FRO = 1e-5  # f32 outputs: relative Frobenius error
LOGITS_ATOL = 1e-4


def load(name):
    return np.load(os.path.join(GOLD, name))


def rel_fro(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


@pytest.fixture(scope="module")
def oc():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import opencuda_cuda
    return opencuda_cuda


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.cuda() if dtype is None else t.to(dtype).cuda()


def test_sgemm(oc):
    g = load("sgemm_17x33x29.npz")
    m, k, n = int(g["m"]), int(g["k"]), int(g["n"])
    C = dev(g["C0"].reshape(m, n))
    oc.sgemm(dev(g["A"].reshape(m, k)), dev(g["B"].reshape(k, n)), float(g["alpha"]), float(g["beta"]), C=C)
    assert rel_fro(C.cpu().numpy(), g["C"]) <= REL_FRO


def test_quantize_and_qgemm(oc):
    g = load("qgemm_9x256x96.npz")
    m, k, n, grp = (int(g[x]) for x in ("m", "k", "n", "group"))
    W = dev(g["WT"])
    q8, s8 = oc.quantize_int8(W, k)
    q4, s4 = oc.quantize_int4(W, grp)
    assert np.array_equal(q8.cpu().numpy(), g["q8"]) and np.array_equal(q4.cpu().numpy(), g["q4"])
    assert np.array_equal(s8.cpu().numpy(), g["s8"]) and np.array_equal(s4.cpu().numpy(), g["s4"])
    A, b = dev(g["A"].reshape(m, k)), dev(g["bias"])
    y8, acc8 = oc.qgemm_w8a8(A, q8.view(n, k), s8, b, want_acc=True)
    y4, acc4 = oc.qgemm_w4a8(A, q4, s4, grp, b, want_acc=True)
    assert np.array_equal(acc8.cpu().numpy().ravel(), g["acc8"])
    assert np.array_equal(acc4.cpu().numpy().ravel(), g["acc4"])
    assert np.array_equal(y8.cpu().numpy().ravel().view(np.uint32), g["y8"].view(np.uint32))
    assert np.array_equal(y4.cpu().numpy().ravel().view(np.uint32), g["y4"].view(np.uint32))


def test_attention(oc):
    g = load("attention_17x8.npz")
    seq, d, blk = int(g["seq"]), int(g["d"]), int(g["block"])
    q, k, v = (dev(g[x].reshape(seq, d)) for x in ("q", "k", "v"))
    assert rel_fro(oc.flash_attention(q, k, v, blk).cpu().numpy(), g["flash"]) <= REL_FRO
    assert rel_fro(oc.scaled_dot_product_attention(q, k, v).cpu().numpy(), g["sdpa"]) <= REL_FRO


def test_mla(oc):
    g = load("mla_12x64x16.npz")
    seq, dh, dc = int(g["seq"]), int(g["dh"]), int(g["dc"])
    lat = oc.mla_compress_kv(dev(g["kv"].reshape(seq, dh)), dev(g["down"].reshape(dh, dc)))
    assert rel_fro(lat.cpu().numpy(), g["latent"]) <= REL_FRO
    rec = oc.mla_decompress_kv(dev(g["latent"].reshape(seq, dc)), dev(g["up"].reshape(dc, dh)))
    assert rel_fro(rec.cpu().numpy(), g["recon"]) <= REL_FRO


def test_gpt_tokens_and_logits(oc):
    import gpt

    g = load("gpt_tiny_seed42.npz")
    cfg = gpt.GptConfig(int(g["vocab"]), int(g["hidden"]), int(g["layers"]), int(g["heads"]), int(g["inter"]),
                        int(g["ctx"]), float(g["eps"]))
    m = gpt.GptModel.load_random(cfg, int(g["seed"]))
    toks, logits = m.generate(g["prompt"], len(g["tokens"]), want_logits=True)
    m.close()
    assert toks.tolist() == g["tokens"].tolist()
    assert np.abs(logits - g["logits"]).max() <= LOGITS_ATOL


def test_moe(oc):
    import moe

    g = load("moe_10x64.npz")
    w = moe.MoEWeights(*[dev(g[x]) for x in ("w1", "s1", "w2", "s2", "sw1", "ss1", "sw2", "ss2")])
    idx, tw = moe.route(dev(g["logits"]), int(g["k"]))
    assert np.array_equal(idx.cpu().numpy(), g["idx"])
    assert np.array_equal(tw.cpu().numpy().view(np.uint32), g["tw"].view(np.uint32))
    y = moe.moe_forward(dev(g["x"]), dev(g["logits"]), w, int(g["k"]))
    assert np.array_equal(y.cpu().numpy().view(np.uint32), g["y"].view(np.uint32))
