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
}

WEIGHT_IDS = {
    "wte": 0, "wpe": 1, "qkv_w": 2, "qkv_b": 3, "attn_out_w": 4, "attn_out_b": 5,
    "fc_w": 6, "fc_b": 7, "proj_w": 8, "proj_b": 9, "ln1_w": 10, "ln1_b": 11,
    "ln2_w": 12, "ln2_b": 13, "lnf_w": 14, "lnf_b": 15, "lm_head_w": 16, "lm_head_b": 17,
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
                "ln2_w": H, "ln2_b": H, "lnf_w": H, "lnf_b": H, "lm_head_w": H * V, "lm_head_b": V}[name]

    def set_weight(self, name: str, values, layer: int = 0):
        v = np.ascontiguousarray(values, np.float32).ravel()
        oc.check(_lib().oc_gpt_set_weight(self._h, WEIGHT_IDS[name], layer, v.ctypes.data_as(C.c_void_p), v.size))

    def weight(self, name: str, layer: int = 0) -> np.ndarray:
        out = np.zeros(self._shape(name), np.float32)
        oc.check(_lib().oc_gpt_get_weight(self._h, WEIGHT_IDS[name], layer, out.ctypes.data_as(C.c_void_p),
                                          out.size))
        return out

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
