"""GPT-2 checkpoint loading (crates/open-cuda-llm/src/lib.rs:661-731) on the
host: the safetensors reader against the reference implementation of the
format (the `safetensors` package), config.json parsing (llm:76-110), the
tensor plan for both naming conventions (with and without the
`transformer.` prefix, llm:681-687), the tied lm_head (llm:722-728) and the
reference's errors.  No GPU: the plan is what the loader uploads."""
import json
import shutil
from pathlib import Path

import numpy as np
import pytest

import gpt

st = pytest.importorskip("safetensors.numpy")

TMP = Path(__file__).parent / "_tmp"


@pytest.fixture
def tmpdir_repo(request):
    d = TMP / request.node.name.replace("[", "_").replace("]", "_")
    if d.exists():
        shutil.rmtree(d)
    d.mkdir(parents=True)
    yield d
    shutil.rmtree(d)


def tiny_checkpoint(rng, V=50, H=32, L=2, heads=4, ctx=64, prefix=""):
    I = 4 * H
    t = {prefix + "wte.weight": rng.standard_normal((V, H)), prefix + "wpe.weight": rng.standard_normal((ctx, H)),
         prefix + "ln_f.weight": rng.standard_normal(H), prefix + "ln_f.bias": rng.standard_normal(H)}
    for i in range(L):
        p = f"{prefix}h.{i}."
        for name, shape in (("attn.c_attn", (H, 3 * H)), ("attn.c_proj", (H, H)), ("mlp.c_fc", (H, I)),
                            ("mlp.c_proj", (I, H))):
            t[p + name + ".weight"] = rng.standard_normal(shape)
            t[p + name + ".bias"] = rng.standard_normal(shape[1])
        for ln in ("ln_1", "ln_2"):
            t[p + ln + ".weight"] = rng.standard_normal(H)
            t[p + ln + ".bias"] = rng.standard_normal(H)
    t = {k: v.astype(np.float32) for k, v in t.items()}
    cfg = {"vocab_size": V, "n_embd": H, "n_layer": L, "n_head": heads, "n_positions": ctx}
    return cfg, t


def write(d, cfg, tensors):
    (d / "config.json").write_text(json.dumps(cfg))
    st.save_file(tensors, str(d / "model.safetensors"), metadata={"format": "pt"})


def test_reader_matches_reference_format(tmpdir_repo):
    rng = np.random.default_rng(1)
    tensors = {"a": rng.standard_normal((3, 5)).astype(np.float32), "b": np.arange(7, dtype=np.int32),
               "c": rng.standard_normal(4).astype(np.float16), "empty": np.zeros((0, 3), np.float32)}
    st.save_file(tensors, str(tmpdir_repo / "x.safetensors"), metadata={"k": "v"})
    got = gpt.read_safetensors((tmpdir_repo / "x.safetensors").read_bytes())
    assert sorted(got) == sorted(tensors)
    for name, arr in tensors.items():
        dtype, shape, raw = got[name]
        assert shape == arr.shape
        assert dtype == {"float32": "F32", "int32": "I32", "float16": "F16"}[str(arr.dtype)]
        assert bytes(raw) == arr.tobytes()
    with pytest.raises(ValueError):
        gpt.read_safetensors(b"\x01\x00")
    with pytest.raises(ValueError):
        gpt.read_safetensors((1 << 40).to_bytes(8, "little") + b"{}")


def test_config_parsing():
    c = gpt.gpt2_config_from_json(json.dumps({"vocab_size": 50257, "n_embd": 768, "n_layer": 12, "n_head": 12,
                                              "n_ctx": 1024}))
    assert (c.vocab_size, c.hidden_size, c.num_layers, c.num_heads, c.intermediate_size, c.max_seq_len) == \
        (50257, 768, 12, 12, 3072, 1024)
    assert c.layer_norm_eps == pytest.approx(1e-5)
    # n_positions wins over n_ctx; an explicit epsilon is kept
    c = gpt.gpt2_config_from_json(json.dumps({"vocab_size": 10, "n_embd": 8, "n_layer": 1, "n_head": 2,
                                              "n_ctx": 16, "n_positions": 32, "layer_norm_epsilon": 1e-6}))
    assert c.max_seq_len == 32 and c.layer_norm_eps == pytest.approx(1e-6)
    with pytest.raises(ValueError, match="n_positions or n_ctx"):
        gpt.gpt2_config_from_json(json.dumps({"vocab_size": 10, "n_embd": 8, "n_layer": 1, "n_head": 2}))
    with pytest.raises(ValueError, match="not divisible"):
        gpt.gpt2_config_from_json(json.dumps({"vocab_size": 10, "n_embd": 9, "n_layer": 1, "n_head": 2,
                                              "n_ctx": 4}))


@pytest.mark.parametrize("prefix", ["", "transformer."])
def test_plan_both_naming_conventions(tmpdir_repo, prefix):
    cfg, t = tiny_checkpoint(np.random.default_rng(2), prefix=prefix)
    write(tmpdir_repo, cfg, t)
    c, plan = gpt.gpt2_checkpoint_plan(tmpdir_repo)
    assert (c.vocab_size, c.hidden_size, c.num_layers, c.max_seq_len) == (50, 32, 2, 64)
    got = {(name, layer): v for name, layer, v in plan}
    assert len(got) == 2 + 12 * 2 + 4
    src = {"qkv": "attn.c_attn", "attn_out": "attn.c_proj", "fc": "mlp.c_fc", "proj": "mlp.c_proj",
           "ln1": "ln_1", "ln2": "ln_2"}
    for i in range(2):
        for key, name in src.items():
            for wb, suffix in (("_w", ".weight"), ("_b", ".bias")):
                assert np.array_equal(got[(key + wb, i)], t[f"{prefix}h.{i}.{name}{suffix}"].ravel())
    assert np.array_equal(got[("wte", 0)], t[prefix + "wte.weight"].ravel())
    assert np.array_equal(got[("wpe", 0)], t[prefix + "wpe.weight"].ravel())
    # lm_head tied to wte: [hidden][vocab], no bias
    assert np.array_equal(got[("lm_head_w", 0)].reshape(32, 50), t[prefix + "wte.weight"].T)
    assert not got[("lm_head_b", 0)].any()


def test_plan_errors(tmpdir_repo):
    cfg, t = tiny_checkpoint(np.random.default_rng(3))
    with pytest.raises(ValueError, match="config.json"):
        gpt.gpt2_checkpoint_plan(tmpdir_repo)
    bad = dict(t)
    del bad["h.1.mlp.c_fc.bias"]
    write(tmpdir_repo, cfg, bad)
    with pytest.raises(ValueError, match="missing tensor 'h.1.mlp.c_fc.bias'"):
        gpt.gpt2_checkpoint_plan(tmpdir_repo)
    bad = dict(t)
    bad["h.0.ln_1.weight"] = bad["h.0.ln_1.weight"].astype(np.float16)
    write(tmpdir_repo, cfg, bad)
    with pytest.raises(ValueError, match="unexpected dtype F16"):
        gpt.gpt2_checkpoint_plan(tmpdir_repo)
    bad = dict(t)
    bad["h.0.attn.c_proj.weight"] = bad["h.0.attn.c_proj.weight"][:, :31].copy()
    write(tmpdir_repo, cfg, bad)
    with pytest.raises(ValueError, match="expected 32x32"):
        gpt.gpt2_checkpoint_plan(tmpdir_repo)
