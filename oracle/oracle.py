"""ctypes binding of the CPU oracle (oracle/liboc_oracle.so).

TEST INFRASTRUCTURE ONLY.  This is the checker for the CUDA library and the
timed CPU baseline.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline legs import it; the product path never does.

The oracle restates the open-cuda reference's CPU loops (Rust crates
opencuda-blas and open-cuda-llm) in C; see oracle.c for the per-function
citations.  Functions here mirror the reference's names and argument
meanings and raise ValueError where the reference `bail!`s.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboc_oracle.so")
_lib = None

f32p = C.POINTER(C.c_float)
i8p = C.POINTER(C.c_int8)
u8p = C.POINTER(C.c_uint8)
i32p = C.POINTER(C.c_int32)
u32p = C.POINTER(C.c_uint32)
sz = C.c_size_t


def build() -> str:
    """Compiles the oracle with its Makefile (gcc only, seconds)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


class GptConfig(C.Structure):
    """GptConfig (llm:45-69)."""

    _fields_ = [
        ("vocab_size", sz), ("hidden_size", sz), ("num_layers", sz),
        ("num_heads", sz), ("intermediate_size", sz), ("max_seq_len", sz),
        ("layer_norm_eps", C.c_float),
    ]

    @staticmethod
    def tiny(vocab_size: int) -> "GptConfig":
        """GptConfig::tiny (llm:57-68)."""
        return GptConfig(vocab_size, 32, 2, 4, 64, 256, 1e-5)

    @staticmethod
    def gpt2_124m() -> "GptConfig":
        return GptConfig(50257, 768, 12, 12, 3072, 1024, 1e-5)


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH) or (
        os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "oracle.c"))
        and os.access(_HERE, os.W_OK)
    ):
        build()
    L = C.CDLL(_LIB_PATH)
    sig = {
        "ocr_set_threads": (None, [C.c_int]),
        "ocr_get_threads": (C.c_int, []),
        "ocr_sgemm": (C.c_int, [sz, sz, sz, C.c_float, f32p, f32p, C.c_int, C.c_float, f32p, C.c_int]),
        "ocr_group_scales": (None, [f32p, sz, sz, C.c_float, f32p]),
        "ocr_quantize_int8": (C.c_int, [f32p, sz, sz, i8p, f32p]),
        "ocr_quantize_int4": (C.c_int, [f32p, sz, sz, u8p, f32p]),
        "ocr_dequantize_int8": (None, [i8p, f32p, sz, sz, f32p]),
        "ocr_dequantize_int4": (None, [u8p, f32p, sz, sz, f32p]),
        "ocr_quantize_int4_awq": (C.c_int, [f32p, sz, sz, f32p, sz, C.c_float, u8p, f32p, f32p]),
        "ocr_dequantize_int4_awq": (None, [u8p, f32p, sz, sz, sz, f32p, f32p]),
        "ocr_row_softmax": (None, [f32p, sz, sz, f32p]),
        "ocr_sdpa": (C.c_int, [f32p, f32p, f32p, sz, sz, f32p]),
        "ocr_flash_attention": (C.c_int, [f32p, f32p, f32p, sz, sz, sz, f32p]),
        "ocr_attend_one": (None, [f32p, f32p, f32p, sz, sz, C.c_int, sz, f32p]),
        "ocr_mla_compress_kv": (C.c_int, [sz, sz, sz, f32p, f32p, f32p]),
        "ocr_mla_decompress_kv": (C.c_int, [sz, sz, sz, f32p, f32p, f32p]),
        "ocr_mla_memory_reduction_percent": (C.c_double, [sz, sz]),
        "ocr_quantize_rows_int8": (C.c_int, [f32p, sz, sz, i8p, f32p]),
        "ocr_qgemm_w8a8": (C.c_int, [sz, sz, sz, f32p, i8p, f32p, f32p, f32p, i32p]),
        "ocr_qgemm_w4a8": (C.c_int, [sz, sz, sz, sz, f32p, u8p, f32p, f32p, f32p, i32p]),
        "ocr_qgemm_weight_only": (C.c_int, [C.c_int, sz, sz, sz, sz, f32p, C.c_void_p, f32p, f32p, f32p, C.c_int]),
        "ocr_splitmix64_fill": (None, [C.c_uint64, C.c_float, sz, f32p]),
        "ocr_moe_route": (C.c_int, [f32p, sz, sz, sz, i32p, f32p]),
        "ocr_moe_forward": (C.c_int, [sz, sz, sz, sz, sz, f32p, f32p, i8p, f32p, i8p, f32p, i8p, f32p, i8p, f32p,
                                      f32p]),
        "ocr_gpt_load_random": (C.c_void_p, [C.POINTER(GptConfig), C.c_uint64]),
        "ocr_gpt_free": (None, [C.c_void_p]),
        "ocr_gpt_set_attention": (None, [C.c_void_p, C.c_int, sz, C.c_int]),
        "ocr_gpt_enable_mla": (C.c_int, [C.c_void_p, sz, C.c_uint64]),
        "ocr_gpt_weight": (f32p, [C.c_void_p, C.c_int, sz, sz, C.POINTER(sz)]),
        "ocr_gpt_state_new": (C.c_void_p, [C.c_void_p]),
        "ocr_gpt_state_free": (None, [C.c_void_p]),
        "ocr_gpt_forward_step": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, sz, f32p]),
        "ocr_gpt_forward_prefill": (C.c_int, [C.c_void_p, C.c_void_p, u32p, sz, f32p]),
        "ocr_gpt_generate": (C.c_long, [C.c_void_p, u32p, sz, sz, u32p, f32p]),
        "ocr_argmax": (C.c_uint32, [f32p, sz]),
        "ocr_layer_norm": (None, [f32p, sz, sz, f32p, f32p, C.c_float]),
        "ocr_gelu": (None, [f32p, sz]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32)


def _p(a: np.ndarray, t=f32p):
    return a.ctypes.data_as(t)


def set_threads(n: int) -> None:
    lib().ocr_set_threads(int(n))


def threads() -> int:
    return int(lib().ocr_get_threads())


# ---- blas ------------------------------------------------------------------

def sgemm(m, k, n, alpha, a, b, beta, c, transpose_b=False, faithful=False) -> np.ndarray:
    """opencuda_blas::sgemm (blas:260-295) on the CpuNaive path.  Returns C."""
    a, b = _f32(a).ravel(), _f32(b).ravel()
    c = _f32(c).ravel().copy()
    if a.size != m * k:
        raise ValueError(f"sgemm: a.len()={a.size} != m*k={m * k}")
    if b.size != k * n:
        raise ValueError(f"sgemm: b.len()={b.size} != k*n={k * n}")
    if c.size != m * n:
        raise ValueError(f"sgemm: c.len()={c.size} != m*n={m * n}")
    rc = lib().ocr_sgemm(m, k, n, alpha, _p(a), _p(b), int(transpose_b), beta, _p(c), int(faithful))
    if rc:
        raise RuntimeError(f"ocr_sgemm rc={rc}")
    return c


class QuantizedInt8Tensor:
    """QuantizedInt8Tensor (blas:787-792)."""

    def __init__(self, data, scales, group_size, length):
        self.data, self.scales, self.group_size, self.len = data, scales, group_size, length


class QuantizedInt4Tensor:
    """QuantizedInt4Tensor (blas:777-782)."""

    def __init__(self, data, scales, group_size, length):
        self.data, self.scales, self.group_size, self.len = data, scales, group_size, length


def _validate_quant(x: np.ndarray, group_size: int) -> None:
    if x.size == 0:
        raise ValueError("quantize: input must not be empty")
    if group_size == 0:
        raise ValueError("quantize: group_size must be > 0")


def quantize_int8(x, group_size: int) -> QuantizedInt8Tensor:
    x = _f32(x).ravel()
    _validate_quant(x, group_size)
    ng = -(-x.size // group_size)
    data = np.zeros(x.size, np.int8)
    scales = np.zeros(ng, np.float32)
    lib().ocr_quantize_int8(_p(x), x.size, group_size, _p(data, i8p), _p(scales))
    return QuantizedInt8Tensor(data, scales, group_size, x.size)


def quantize_int4(x, group_size: int) -> QuantizedInt4Tensor:
    x = _f32(x).ravel()
    _validate_quant(x, group_size)
    ng = -(-x.size // group_size)
    data = np.zeros((x.size + 1) // 2, np.uint8)
    scales = np.zeros(ng, np.float32)
    lib().ocr_quantize_int4(_p(x), x.size, group_size, _p(data, u8p), _p(scales))
    return QuantizedInt4Tensor(data, scales, group_size, x.size)


def dequantize_int8(t: QuantizedInt8Tensor) -> np.ndarray:
    out = np.zeros(t.len, np.float32)
    lib().ocr_dequantize_int8(_p(t.data, i8p), _p(t.scales), t.len, t.group_size, _p(out))
    return out


def dequantize_int4(t: QuantizedInt4Tensor) -> np.ndarray:
    out = np.zeros(t.len, np.float32)
    lib().ocr_dequantize_int4(_p(t.data, u8p), _p(t.scales), t.len, t.group_size, _p(out))
    return out


class QuantizedInt4AwqTensor:
    """QuantizedInt4AwqTensor (blas:963-970)."""

    def __init__(self, inner, awq_scale, rows, cols):
        self.inner, self.awq_scale, self.rows, self.cols = inner, awq_scale, rows, cols


def quantize_int4_awq(weight, rows, cols, activation_scale, group_size, alpha) -> QuantizedInt4AwqTensor:
    w, s = _f32(weight).ravel(), _f32(activation_scale).ravel()
    if rows == 0 or cols == 0:
        raise ValueError("quantize_int4_awq: rows and cols must be > 0")
    if w.size != rows * cols:
        raise ValueError("quantize_int4_awq: weight.len() must equal rows*cols")
    if s.size != cols:
        raise ValueError("quantize_int4_awq: activation_scale.len() must equal cols")
    _validate_quant(w, group_size)
    data = np.zeros((w.size + 1) // 2, np.uint8)
    scales = np.zeros(-(-w.size // group_size), np.float32)
    awq = np.zeros(cols, np.float32)
    lib().ocr_quantize_int4_awq(_p(w), rows, cols, _p(s), group_size, alpha, _p(data, u8p), _p(scales), _p(awq))
    return QuantizedInt4AwqTensor(QuantizedInt4Tensor(data, scales, group_size, w.size), awq, rows, cols)


def dequantize_int4_awq(t: QuantizedInt4AwqTensor) -> np.ndarray:
    out = np.zeros(t.rows * t.cols, np.float32)
    lib().ocr_dequantize_int4_awq(_p(t.inner.data, u8p), _p(t.inner.scales), t.rows, t.cols,
                                  t.inner.group_size, _p(t.awq_scale), _p(out))
    return out


def _check_qkv(name, q, k, v, seq, d):
    for nm, x in (("q", q), ("k", k), ("v", v)):
        if x.size != seq * d:
            raise ValueError(f"{name}: {nm}.len()={x.size} != seq_len*head_dim={seq * d}")


def scaled_dot_product_attention(q, k, v, seq_len, head_dim) -> np.ndarray:
    """blas:411-540 on the CpuNaive path (GEMM, CPU softmax, GEMM)."""
    q, k, v = _f32(q).ravel(), _f32(k).ravel(), _f32(v).ravel()
    _check_qkv("attention", q, k, v, seq_len, head_dim)
    out = np.zeros(seq_len * head_dim, np.float32)
    lib().ocr_sdpa(_p(q), _p(k), _p(v), seq_len, head_dim, _p(out))
    return out


def flash_attention(q, k, v, seq_len, head_dim, block_size) -> np.ndarray:
    """blas:589-678."""
    q, k, v = _f32(q).ravel(), _f32(k).ravel(), _f32(v).ravel()
    _check_qkv("flash_attention", q, k, v, seq_len, head_dim)
    if block_size == 0:
        raise ValueError("flash_attention: block_size must be > 0")
    out = np.zeros(seq_len * head_dim, np.float32)
    lib().ocr_flash_attention(_p(q), _p(k), _p(v), seq_len, head_dim, block_size, _p(out))
    return out


def attend_one(q, k, v, n, d, flash=True, block=64) -> np.ndarray:
    q, k, v = _f32(q).ravel(), _f32(k).ravel(), _f32(v).ravel()
    out = np.zeros(d, np.float32)
    lib().ocr_attend_one(_p(q), _p(k), _p(v), n, d, int(flash), block, _p(out))
    return out


def row_softmax(scores, rows, cols) -> np.ndarray:
    s = _f32(scores).ravel()
    out = np.zeros(rows * cols, np.float32)
    lib().ocr_row_softmax(_p(s), rows, cols, _p(out))
    return out


def mla_compress_kv(seq_len, d_h, d_c, kv, down_proj) -> np.ndarray:
    kv, dp = _f32(kv).ravel(), _f32(down_proj).ravel()
    if kv.size != seq_len * d_h:
        raise ValueError(f"mla_compress_kv: kv.len()={kv.size} != seq_len*d_h={seq_len * d_h}")
    if dp.size != d_h * d_c:
        raise ValueError(f"mla_compress_kv: down_proj.len()={dp.size} != d_h*d_c={d_h * d_c}")
    out = np.zeros(seq_len * d_c, np.float32)
    lib().ocr_mla_compress_kv(seq_len, d_h, d_c, _p(kv), _p(dp), _p(out))
    return out


def mla_decompress_kv(seq_len, d_c, d_h, latent, up_proj) -> np.ndarray:
    lt, up = _f32(latent).ravel(), _f32(up_proj).ravel()
    if lt.size != seq_len * d_c:
        raise ValueError(f"mla_decompress_kv: latent.len()={lt.size} != seq_len*d_c={seq_len * d_c}")
    if up.size != d_c * d_h:
        raise ValueError(f"mla_decompress_kv: up_proj.len()={up.size} != d_c*d_h={d_c * d_h}")
    out = np.zeros(seq_len * d_h, np.float32)
    lib().ocr_mla_decompress_kv(seq_len, d_c, d_h, _p(lt), _p(up), _p(out))
    return out


def mla_memory_reduction_percent(d_h, d_c) -> float:
    return float(lib().ocr_mla_memory_reduction_percent(d_h, d_c))


# ---- quantized matmul oracles ---------------------------------------------

def quantize_rows_int8(a, m, k):
    a = _f32(a).ravel()
    qa = np.zeros(m * k, np.int8)
    sa = np.zeros(m, np.float32)
    lib().ocr_quantize_rows_int8(_p(a), m, k, _p(qa, i8p), _p(sa))
    return qa, sa


def qgemm_w8a8(m, k, n, a, wq, wscale, bias, want_acc=False):
    a, ws = _f32(a).ravel(), _f32(wscale).ravel()
    wq = np.ascontiguousarray(wq, np.int8).ravel()
    b = None if bias is None else _f32(bias).ravel()
    y = np.zeros(m * n, np.float32)
    acc = np.zeros(m * n, np.int32) if want_acc else None
    rc = lib().ocr_qgemm_w8a8(m, k, n, _p(a), _p(wq, i8p), _p(ws), None if b is None else _p(b),
                              _p(y), None if acc is None else _p(acc, i32p))
    if rc:
        raise ValueError(f"qgemm_w8a8 rc={rc}")
    return (y, acc) if want_acc else y


def qgemm_w4a8(m, k, n, group, a, wq, wscale, bias, want_acc=False):
    a, ws = _f32(a).ravel(), _f32(wscale).ravel()
    wq = np.ascontiguousarray(wq, np.uint8).ravel()
    b = None if bias is None else _f32(bias).ravel()
    y = np.zeros(m * n, np.float32)
    acc = np.zeros(m * n * (k // group), np.int32) if want_acc else None
    rc = lib().ocr_qgemm_w4a8(m, k, n, group, _p(a), _p(wq, u8p), _p(ws), None if b is None else _p(b),
                              _p(y), None if acc is None else _p(acc, i32p))
    if rc:
        raise ValueError(f"qgemm_w4a8 rc={rc}")
    return (y, acc) if want_acc else y


def qgemm_weight_only(bits, m, k, n, group, a, wq, wscale, bias, faithful=False):
    a, ws = _f32(a).ravel(), _f32(wscale).ravel()
    wq = np.ascontiguousarray(wq).ravel()
    b = None if bias is None else _f32(bias).ravel()
    y = np.zeros(m * n, np.float32)
    rc = lib().ocr_qgemm_weight_only(bits, m, k, n, group, _p(a), wq.ctypes.data_as(C.c_void_p), _p(ws),
                                     None if b is None else _p(b), _p(y), int(faithful))
    if rc:
        raise ValueError(f"qgemm_weight_only rc={rc}")
    return y


# ---- mixture of experts -------------------------------------------------------

def moe_route(logits, T, E, k):
    lg = _f32(logits).ravel()
    idx = np.zeros(T * k, np.int32)
    w = np.zeros(T * k, np.float32)
    if lib().ocr_moe_route(_p(lg), T, E, k, _p(idx, i32p), _p(w)):
        raise ValueError("moe_route: bad arguments")
    return idx.reshape(T, k), w.reshape(T, k)


def moe_forward(x, logits, w1, s1, w2, s2, sw1, ss1, sw2, ss2, k):
    """x [T][D]; w1 [E][F][D] int8 + s1 [E][F]; w2 [E][D][F] + s2 [E][D]; shared sw1 [F][D], sw2 [D][F]."""
    x = _f32(x)
    T, D = x.shape
    E, F, _ = w1.shape
    y = np.zeros((T, D), np.float32)
    args = [np.ascontiguousarray(a) for a in (w1, s1, w2, s2, sw1, ss1, sw2, ss2)]
    rc = lib().ocr_moe_forward(T, D, F, E, k, _p(x), _p(_f32(logits)), _p(args[0], i8p), _p(_f32(args[1])),
                               _p(args[2], i8p), _p(_f32(args[3])), _p(args[4], i8p), _p(_f32(args[5])),
                               _p(args[6], i8p), _p(_f32(args[7])), _p(y))
    if rc:
        raise RuntimeError(f"ocr_moe_forward rc={rc}")
    return y


# ---- GPT -------------------------------------------------------------------

def splitmix64_fill(seed: int, scale: float, n: int) -> np.ndarray:
    out = np.zeros(n, np.float32)
    lib().ocr_splitmix64_fill(seed, scale, n, _p(out))
    return out


def layer_norm(x, rows, dim, w, b, eps) -> np.ndarray:
    x = _f32(x).ravel().copy()
    lib().ocr_layer_norm(_p(x), rows, dim, _p(_f32(w)), _p(_f32(b)), eps)
    return x


def gelu(x) -> np.ndarray:
    x = _f32(x).ravel().copy()
    lib().ocr_gelu(_p(x), x.size)
    return x


def argmax(x) -> int:
    x = _f32(x).ravel()
    return int(lib().ocr_argmax(_p(x), x.size))


WEIGHT_IDS = {
    "wte": 0, "wpe": 1, "qkv_w": 2, "qkv_b": 3, "attn_out_w": 4, "attn_out_b": 5,
    "fc_w": 6, "fc_b": 7, "proj_w": 8, "proj_b": 9, "ln1_w": 10, "ln1_b": 11,
    "ln2_w": 12, "ln2_b": 13, "lnf_w": 14, "lnf_b": 15, "lm_head_w": 16, "lm_head_b": 17,
    "mla_down": 18, "mla_up": 19,
}


class GptModel:
    """GptModel (llm:600-929) on the oracle: load_random + generate."""

    def __init__(self, config: GptConfig, seed: int):
        self.config = config
        self._h = lib().ocr_gpt_load_random(C.byref(config), seed)
        if not self._h:
            raise MemoryError("ocr_gpt_load_random failed")

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and _lib is not None:
            _lib.ocr_gpt_free(h)
            self._h = None

    def set_attention(self, flash=True, block=64, faithful=False):
        lib().ocr_gpt_set_attention(self._h, int(flash), block, int(faithful))

    def enable_mla_kv_compression(self, d_c: int, seed: int):
        if lib().ocr_gpt_enable_mla(self._h, d_c, seed):
            hd = self.config.hidden_size // self.config.num_heads
            raise ValueError(f"enable_mla_kv_compression: d_c={d_c} must satisfy 0 < d_c < head_dim={hd}")

    def weight(self, name: str, layer: int = 0, head: int = 0) -> np.ndarray:
        n = sz(0)
        p = lib().ocr_gpt_weight(self._h, WEIGHT_IDS[name], layer, head, C.byref(n))
        if not p:
            raise KeyError(name)
        return np.ctypeslib.as_array(p, shape=(n.value,))

    def new_state(self):
        return _State(self)

    def generate(self, prompt_ids, max_new_tokens, want_logits=False):
        p = np.ascontiguousarray(prompt_ids, np.uint32)
        if p.size == 0:
            raise ValueError("open-cuda-llm: prompt_ids must not be empty")
        out = np.zeros(max_new_tokens, np.uint32)
        lg = np.zeros(max_new_tokens * self.config.vocab_size, np.float32) if want_logits else None
        n = lib().ocr_gpt_generate(self._h, _p(p, u32p), p.size, max_new_tokens, _p(out, u32p),
                                   None if lg is None else _p(lg))
        if n < 0:
            raise RuntimeError("ocr_gpt_generate failed")
        toks = out[:n].copy()
        if want_logits:
            return toks, lg.reshape(max_new_tokens, -1)[:n].copy()
        return toks


class _State:
    def __init__(self, model: GptModel):
        self.model = model
        self._s = lib().ocr_gpt_state_new(model._h)

    def __del__(self):
        if getattr(self, "_s", None) and _lib is not None:
            _lib.ocr_gpt_state_free(self._s)
            self._s = None

    def forward_step(self, token: int, pos: int) -> np.ndarray:
        out = np.zeros(self.model.config.vocab_size, np.float32)
        if lib().ocr_gpt_forward_step(self.model._h, self._s, token, pos, _p(out)):
            raise ValueError("forward_step failed")
        return out

    def forward_prefill(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.uint32)
        out = np.zeros(self.model.config.vocab_size, np.float32)
        if lib().ocr_gpt_forward_prefill(self.model._h, self._s, _p(ids, u32p), ids.size, _p(out)):
            raise ValueError("forward_prefill failed")
        return out


def byte_encode(text: str) -> list[int]:
    """ByteTokenizer::encode (llm:953-955)."""
    return list(text.encode("utf-8"))


BYTE_VOCAB_SIZE = 256 + 4  # ByteTokenizer::VOCAB_SIZE (llm:949)
