"""GptModel on the CUDA backend (crates/open-cuda-llm/src/lib.rs:600-942).

A thin Python face of the C ABI's oc_gpt_*: the same constructor
(load_random with a seed), the same generate contract (greedy, prompt
excluded from the output, ValueError for an empty prompt or an out-of-range
token), executed entirely on the device (weights, KV cache, argmax)."""
from __future__ import annotations

import ctypes as C

import numpy as np

import opencuda_cuda as oc


class GptConfig(C.Structure):
    """GptConfig (llm:45-69)."""

    _fields_ = [
        ("vocab_size", C.c_size_t), ("hidden_size", C.c_size_t), ("num_layers", C.c_size_t),
        ("num_heads", C.c_size_t), ("intermediate_size", C.c_size_t), ("max_seq_len", C.c_size_t),
        ("layer_norm_eps", C.c_float),
    ]

    @staticmethod
    def tiny(vocab_size: int) -> "GptConfig":
        """GptConfig::tiny (llm:57-68)."""
        return GptConfig(vocab_size, 32, 2, 4, 64, 256, 1e-5)

    @staticmethod
    def gpt2_124m() -> "GptConfig":
        return GptConfig(50257, 768, 12, 12, 3072, 1024, 1e-5)


_SIGS = {
    "oc_gpt_create": (C.c_int, [C.c_int, C.POINTER(GptConfig), C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "oc_gpt_destroy": (C.c_int, [C.c_void_p]),
    "oc_gpt_load_random": (C.c_int, [C.c_void_p, C.c_uint64]),
    "oc_gpt_set_weight": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t]),
    "oc_gpt_get_weight": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t]),
    "oc_gpt_generate": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                  C.POINTER(C.c_int)]),
    "oc_gpt_stream": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "oc_gpt_kernel_launches": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint64)]),
    "oc_gpt_enable_mla": (C.c_int, [C.c_void_p, C.c_size_t, C.c_uint64]),
}

WEIGHT_IDS = {
    "wte": 0, "wpe": 1, "qkv_w": 2, "qkv_b": 3, "attn_out_w": 4, "attn_out_b": 5,
    "fc_w": 6, "fc_b": 7, "proj_w": 8, "proj_b": 9, "ln1_w": 10, "ln1_b": 11,
    "ln2_w": 12, "ln2_b": 13, "lnf_w": 14, "lnf_b": 15, "lm_head_w": 16, "lm_head_b": 17,
    "mla_down": 18, "mla_up": 19,
}


def _lib():
    L = oc.lib()
    if not getattr(L, "_gpt_sigs", False):
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        L._gpt_sigs = True
    return L


class GptModel:
    """Device-resident GptModel: load_random(config, seed) + generate."""

    def __init__(self, config: GptConfig, seed: int | None = None, device: int = 0, max_batch: int = 1,
                 max_prompt_len: int = 64):
        self.config = config
        self.max_batch = max_batch
        h = C.c_void_p()
        oc.check(_lib().oc_gpt_create(device, C.byref(config), max_batch, max_prompt_len, C.byref(h)))
        self._h = h
        if seed is not None:
            oc.check(_lib().oc_gpt_load_random(self._h, seed))

    @classmethod
    def load_random(cls, config: GptConfig, seed: int, **kw) -> "GptModel":
        return cls(config, seed, **kw)

    def close(self):
        if getattr(self, "_h", None):
            _lib().oc_gpt_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _shape(self, name):
        c = self.config
        H, V, I, ctx = c.hidden_size, c.vocab_size, c.intermediate_size, c.max_seq_len
        return {"wte": V * H, "wpe": ctx * H, "qkv_w": H * 3 * H, "qkv_b": 3 * H, "attn_out_w": H * H,
                "attn_out_b": H, "fc_w": H * I, "fc_b": I, "proj_w": I * H, "proj_b": H, "ln1_w": H, "ln1_b": H,
                "ln2_w": H, "ln2_b": H, "lnf_w": H, "lnf_b": H, "lm_head_w": H * V, "lm_head_b": V,
                "mla_down": H * getattr(self, "mla_dc", 0), "mla_up": H * getattr(self, "mla_dc", 0)}[name]

    def set_weight(self, name: str, values, layer: int = 0):
        v = np.ascontiguousarray(values, np.float32).ravel()
        oc.check(_lib().oc_gpt_set_weight(self._h, WEIGHT_IDS[name], layer, v.ctypes.data_as(C.c_void_p), v.size))

    def weight(self, name: str, layer: int = 0) -> np.ndarray:
        out = np.zeros(self._shape(name), np.float32)
        oc.check(_lib().oc_gpt_get_weight(self._h, WEIGHT_IDS[name], layer, out.ctypes.data_as(C.c_void_p),
                                          out.size))
        return out

    def enable_mla_kv_compression(self, d_c: int, seed: int):
        """enable_mla_kv_compression (llm:822-838): K/V kept as d_c-dim latents
        per head, attention over their reconstruction; 0 < d_c < head_dim."""
        oc.check(_lib().oc_gpt_enable_mla(self._h, d_c, seed))
        self.mla_dc = d_c

    def kernel_launches(self) -> int:
        """Kernels launched by generate on this model so far."""
        n = C.c_uint64(0)
        oc.check(_lib().oc_gpt_kernel_launches(self._h, C.byref(n)))
        return n.value

    def stream(self) -> int:
        s = C.c_void_p()
        oc.check(_lib().oc_gpt_stream(self._h, C.byref(s)))
        return s.value or 0

    def generate(self, prompt_ids, max_new_tokens: int, want_logits: bool = False):
        """generate (llm:910-929).  prompt_ids: [len] or [batch, len]."""
        p = np.ascontiguousarray(prompt_ids, np.uint32)
        single = p.ndim == 1
        if single:
            p = p[None, :]
        if p.shape[1] == 0:
            raise ValueError("open-cuda-llm: prompt_ids must not be empty")
        b, L = p.shape
        out = np.zeros((b, max_new_tokens), np.uint32)
        lg = np.zeros((b, max_new_tokens, self.config.vocab_size), np.float32) if want_logits else None
        produced = C.c_int(0)
        oc.check(_lib().oc_gpt_generate(self._h, b, p.ctypes.data_as(C.c_void_p), L, max_new_tokens,
                                        out.ctypes.data_as(C.c_void_p),
                                        None if lg is None else lg.ctypes.data_as(C.c_void_p), C.byref(produced)))
        n = produced.value
        toks = out[:, :n]
        if want_logits:
            lg = lg[:, :n]
            return (toks[0], lg[0]) if single else (toks, lg)
        return toks[0] if single else toks


# ---- checkpoint loading (llm:661-731) -------------------------------------

def read_safetensors(data: bytes) -> dict:
    """Tensors of a safetensors file: {name: (dtype, shape, bytes)}.

    The format: an 8-byte little-endian header length N, N bytes of JSON
    ({name: {"dtype", "shape", "data_offsets": [begin, end]}}, plus an
    optional "__metadata__" entry), then the tensor bytes, offsets relative
    to the end of the header."""
    import json
    import struct

    if len(data) < 8:
        raise ValueError("open-cuda-llm: failed to parse model.safetensors (truncated header)")
    (n,) = struct.unpack("<Q", data[:8])
    if 8 + n > len(data):
        raise ValueError("open-cuda-llm: failed to parse model.safetensors (header length past the end)")
    header = json.loads(data[8:8 + n].decode("utf-8"))
    base = 8 + n
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        b, e = info["data_offsets"]
        if not (0 <= b <= e <= len(data) - base):
            raise ValueError(f"open-cuda-llm: failed to parse model.safetensors (tensor '{name}' out of range)")
        out[name] = (info["dtype"], tuple(info["shape"]), memoryview(data)[base + b:base + e])
    return out


def _tensor_f32(tensors: dict, name: str) -> np.ndarray:
    """tensor_f32 (llm:112-126): an F32 tensor's values, little-endian."""
    if name not in tensors:
        raise ValueError(f"open-cuda-llm: missing tensor '{name}'")
    dtype, _, raw = tensors[name]
    if dtype != "F32":
        raise ValueError(f"open-cuda-llm: tensor '{name}' has unexpected dtype {dtype} (expected F32)")
    if len(raw) % 4:
        raise ValueError(f"open-cuda-llm: tensor '{name}' byte length not a multiple of 4")
    return np.frombuffer(raw, dtype="<f4").astype(np.float32)


def gpt2_config_from_json(text: str) -> GptConfig:
    """GPT2Config::into_gpt_config (llm:76-110): n_positions (else n_ctx) is
    the context length, intermediate size 4 * n_embd, eps 1e-5 by default."""
    import json

    raw = json.loads(text)
    ctx = raw.get("n_positions") if raw.get("n_positions") is not None else raw.get("n_ctx")
    if ctx is None:
        raise ValueError("open-cuda-llm: config.json must have n_positions or n_ctx")
    h, heads = int(raw["n_embd"]), int(raw["n_head"])
    if h % heads:
        raise ValueError(f"open-cuda-llm: n_embd {h} not divisible by n_head {heads}")
    eps = raw.get("layer_norm_epsilon")
    return GptConfig(int(raw["vocab_size"]), h, int(raw["n_layer"]), heads, 4 * h, int(ctx),
                     1e-5 if eps is None else float(eps))


def gpt2_checkpoint_plan(directory) -> tuple[GptConfig, list]:
    """GptModel::load (llm:661-731) up to the weights: the config and the
    list of (weight name, layer, values) to upload.  Tensor names may carry
    the `transformer.` prefix (detected from wte.weight, llm:681-687); the
    Conv1D weights are already [in][out]; lm_head is tied to wte, transposed
    to [hidden][vocab] with a zero bias (llm:722-728)."""
    from pathlib import Path

    d = Path(directory)
    try:
        cfg_text = (d / "config.json").read_text()
    except OSError as e:
        raise ValueError(f"open-cuda-llm: failed to read config.json in {d}: {e}") from e
    cfg = gpt2_config_from_json(cfg_text)
    try:
        data = (d / "model.safetensors").read_bytes()
    except OSError as e:
        raise ValueError(f"open-cuda-llm: failed to read model.safetensors in {d}: {e}") from e
    t = read_safetensors(data)
    prefix = "" if "wte.weight" in t else ("transformer." if "transformer.wte.weight" in t else "")
    H, V, I, ctx = cfg.hidden_size, cfg.vocab_size, cfg.intermediate_size, cfg.max_seq_len
    plan = []

    def sized(name, count, what):
        v = _tensor_f32(t, prefix + name)
        if v.size != count:
            raise ValueError(f"open-cuda-llm: '{prefix}{name}' has {v.size} elements, expected {what}")
        return v

    wte = sized("wte.weight", V * H, f"{V}x{H}")
    plan.append(("wte", 0, wte))
    plan.append(("wpe", 0, sized("wpe.weight", ctx * H, f"{ctx}x{H}")))
    for i in range(cfg.num_layers):
        p = f"h.{i}."
        for key, (tensor, n_in, n_out) in {"qkv": ("attn.c_attn", H, 3 * H), "attn_out": ("attn.c_proj", H, H),
                                           "fc": ("mlp.c_fc", H, I), "proj": ("mlp.c_proj", I, H)}.items():
            plan.append((key + "_w", i, sized(p + tensor + ".weight", n_in * n_out, f"{n_in}x{n_out}")))
            plan.append((key + "_b", i, _tensor_f32(t, prefix + p + tensor + ".bias")))
        for key, ln in (("ln1", "ln_1"), ("ln2", "ln_2")):
            plan.append((key + "_w", i, _tensor_f32(t, prefix + p + ln + ".weight")))
            plan.append((key + "_b", i, _tensor_f32(t, prefix + p + ln + ".bias")))
    plan.append(("lnf_w", 0, _tensor_f32(t, prefix + "ln_f.weight")))
    plan.append(("lnf_b", 0, _tensor_f32(t, prefix + "ln_f.bias")))
    plan.append(("lm_head_w", 0, np.ascontiguousarray(wte.reshape(V, H).T).ravel()))
    plan.append(("lm_head_b", 0, np.zeros(V, np.float32)))
    return cfg, plan


def load_gpt2(directory, device: int = 0, max_batch: int = 1, max_prompt_len: int = 64) -> GptModel:
    """GptModel::load (llm:661-731) onto the device: config.json and
    model.safetensors of a Hugging Face GPT-2 checkpoint in `directory`."""
    cfg, plan = gpt2_checkpoint_plan(directory)
    m = GptModel(cfg, None, device=device, max_batch=max_batch, max_prompt_len=max_prompt_len)
    for name, layer, values in plan:
        m.set_weight(name, values, layer)
    return m


GptModel.load = staticmethod(load_gpt2)
