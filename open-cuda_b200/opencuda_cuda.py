"""ctypes binding of libopencuda_cuda.so (the B200 backend's C ABI).

This is the Python face of the reference's `opencuda-blas` API for the
CUDA backend: the same function names, argument meanings and error
behaviour (ValueError where the reference `bail!`s), executed by the
sm_100a kernels of libopencuda_cuda.so.  There is no CPU fallback: if the
library or a CUDA device is missing, calls raise.

Two flavours:
  * device tensors (torch CUDA tensors, asynchronous on the current
    stream): quantize_int8, qgemm_w8a8, ...
  * host slices (numpy arrays, synchronous, like the reference's blas
    functions that copy to the device and back): Device.quantize_int8, ...
torch only provides device memory and streams here.
"""
from __future__ import annotations

import ctypes as C
import os
import re
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "libopencuda_cuda.so")
HEADER = os.path.join(ROOT, "include", "opencuda_cuda.h")

OC_OK = 0
OC_ERR_INVALID_VALUE = 1
OC_ERR_OUT_OF_MEMORY = 2
OC_ERR_LAUNCH_FAILED = 8
OC_ERR_NO_DEVICE = 100
OC_ERR_NOT_SUPPORTED = 801
OC_ERR_TIMEOUT = 702

_lib = None
vp = C.c_void_p
sz = C.c_size_t
ci = C.c_int
cf = C.c_float


class OcError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


def build(jobs: int = 8) -> str:
    """Compiles libopencuda_cuda.so for sm_100a with the package Makefile."""
    subprocess.run(["make", "-s", "-j", str(jobs), "-C", HERE], check=True)
    return LIB_PATH


def declared_functions() -> list[str]:
    """Names of the functions include/opencuda_cuda.h declares."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*\b(oc_[a-z0-9_]+)\s*\(", text, flags=re.M)
    return sorted(set(names))


class DeviceInfo(C.Structure):
    _fields_ = [("ordinal", ci), ("cc_major", ci), ("cc_minor", ci), ("total_memory", C.c_uint64),
                ("compute_units", C.c_uint32), ("name", C.c_char * 256)]


_SIGS = {
    "oc_get_last_error": (C.c_char_p, []),
    "oc_get_device_count": (ci, [C.POINTER(ci)]),
    "oc_device_open": (ci, [ci, C.POINTER(vp)]),
    "oc_device_close": (ci, [vp]),
    "oc_device_get_info": (ci, [vp, C.POINTER(DeviceInfo)]),
    "oc_device_alloc": (ci, [vp, sz, C.POINTER(C.c_uint64)]),
    "oc_device_free": (ci, [vp, C.c_uint64]),
    "oc_device_memcpy_h2d": (ci, [vp, C.c_uint64, vp, sz]),
    "oc_device_memcpy_d2h": (ci, [vp, vp, C.c_uint64, sz]),
    "oc_device_memcpy_d2d": (ci, [vp, C.c_uint64, C.c_uint64, sz]),
    "oc_device_synchronize": (ci, [vp]),
    "oc_partition_layers_by_memory": (ci, [C.POINTER(C.c_uint64), sz, sz, vp]),
    "oc_partition_layers": (ci, [C.POINTER(vp), sz, sz, vp]),
    "oc_transfer_between_devices": (ci, [vp, C.c_uint64, vp, C.c_uint64, sz]),
    "oc_device_stream": (vp, [vp]),
    "oc_get_device_status": (ci, [C.POINTER(ci)]),
    "oc_sgemm": (ci, [ci, ci, ci, cf, vp, ci, vp, ci, ci, cf, vp, ci, vp, vp]),
    "oc_sgemm_prepared_b_size": (ci, [ci, ci, C.POINTER(sz)]),
    "oc_sgemm_prepare_b": (ci, [ci, ci, vp, ci, ci, vp, vp]),
    "oc_sgemm_prepared": (ci, [ci, ci, ci, cf, vp, ci, vp, cf, vp, ci, vp, vp]),
    "oc_softmax_rows": (ci, [vp, ci, ci, vp]),
    "oc_flash_attention": (ci, [vp, vp, vp, vp, ci, ci, ci, vp]),
    "oc_flash_attention_fwd": (ci, [vp, vp, vp, vp, ci, ci, ci, ci, cf, ci, vp]),
    "oc_sdpa_workspace_size": (ci, [ci, C.POINTER(sz)]),
    "oc_sdpa": (ci, [vp, vp, vp, vp, ci, ci, vp, sz, vp]),
    "oc_mla_compress_kv": (ci, [ci, ci, ci, vp, vp, vp, vp]),
    "oc_mla_decompress_kv": (ci, [ci, ci, ci, vp, vp, vp, vp]),
    "oc_device_launch": (ci, [vp, C.c_char_p, vp, vp, sz]),
    "oc_blas_sgemm": (ci, [vp, sz, sz, sz, cf, vp, vp, cf, vp]),
    "oc_blas_softmax_rows": (ci, [vp, sz, sz, vp, vp]),
    "oc_blas_flash_attention": (ci, [vp, vp, vp, vp, sz, sz, sz, vp]),
    "oc_blas_sdpa": (ci, [vp, vp, vp, vp, sz, sz, vp]),
    "oc_blas_mla_compress_kv": (ci, [vp, sz, sz, sz, vp, vp, vp]),
    "oc_blas_mla_decompress_kv": (ci, [vp, sz, sz, sz, vp, vp, vp]),
    "oc_gather_columns": (ci, [vp, vp, ci, ci, ci, vp]),
    "oc_moe_route": (ci, [vp, ci, ci, ci, vp, vp, vp]),
    "oc_moe_dispatch": (ci, [vp, ci, ci, ci, vp, vp, ci, vp, vp, vp, vp, vp, vp, vp, vp]),
    "oc_grouped_igemm_w8a8": (ci, [ci, ci, ci, vp, vp, vp, vp, vp, vp, ci, vp, vp]),
    "oc_gelu_quantize_rows": (ci, [vp, ci, ci, vp, vp, vp]),
    "oc_moe_combine": (ci, [vp, vp, vp, vp, ci, ci, ci, vp, vp]),
    "oc_awq_scales": (ci, [vp, sz, cf, vp]),
    "oc_quantize_int4_awq": (ci, [vp, sz, sz, vp, sz, vp, vp, vp]),
    "oc_dequantize_int4_awq": (ci, [vp, vp, sz, sz, sz, vp, vp, vp]),
    "oc_quantize_int8": (ci, [vp, sz, sz, vp, vp, vp]),
    "oc_quantize_int4": (ci, [vp, sz, sz, vp, vp, vp]),
    "oc_dequantize_int8": (ci, [vp, vp, sz, sz, vp, vp]),
    "oc_dequantize_int4": (ci, [vp, vp, sz, sz, vp, vp]),
    "oc_qgemm_workspace_size": (ci, [ci, ci, C.POINTER(sz)]),
    "oc_qgemm_w8a8": (ci, [ci, ci, ci, vp, vp, vp, vp, vp, vp, sz, vp, vp]),
    "oc_qgemm_w4a8": (ci, [ci, ci, ci, ci, vp, vp, vp, vp, vp, vp, sz, vp, vp]),
    "oc_igemm_w8a8": (ci, [ci, ci, ci, vp, vp, vp, vp, vp, vp, vp, vp]),
    "oc_igemm_w4a8": (ci, [ci, ci, ci, ci, vp, vp, vp, vp, vp, vp, vp, vp]),
    "oc_quantize_rows_int8": (ci, [vp, ci, ci, vp, vp, vp]),
    "oc_qgemm_w8": (ci, [ci, ci, ci, vp, vp, vp, vp, vp, vp]),
    "oc_qgemm_w4": (ci, [ci, ci, ci, ci, vp, vp, vp, vp, vp, vp]),
    "oc_qgemm_w8a8_noalloc": (ci, [ci, ci, ci, vp, vp, vp, vp, vp, vp]),
    "oc_qgemm_w8a8_noalloc_max_bytes": (ci, [C.POINTER(sz)]),
    "oc_blas_quantize_int8": (ci, [vp, vp, sz, sz, vp, vp]),
    "oc_blas_quantize_int4": (ci, [vp, vp, sz, sz, vp, vp]),
    "oc_blas_qgemm_w8a8": (ci, [vp, sz, sz, sz, vp, vp, vp, vp, vp]),
    "oc_blas_qgemm_w4a8": (ci, [vp, sz, sz, sz, sz, vp, vp, vp, vp, vp]),
    "oc_blas_qgemm_w8": (ci, [vp, sz, sz, sz, vp, vp, vp, vp, vp]),
    "oc_blas_qgemm_w4": (ci, [vp, sz, sz, sz, sz, vp, vp, vp, vp, vp]),
}


def lib():
    """Loads libopencuda_cuda.so (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C {HERE}` (nvcc, sm_100a)")
    L = C.CDLL(LIB_PATH)
    for name, (res, args) in _SIGS.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    return lib().oc_get_last_error().decode(errors="replace")


def check(rc: int) -> None:
    if rc != OC_OK:
        msg = last_error()
        if rc == OC_ERR_INVALID_VALUE:
            raise ValueError(msg)
        raise OcError(rc, msg)


def device_count() -> int:
    n = ci(0)
    rc = lib().oc_get_device_count(C.byref(n))
    return n.value if rc == OC_OK else 0


# ---- device tensors (torch CUDA tensors) -------------------------------------

def _torch():
    import torch
    return torch


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return _torch().cuda.current_stream().cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("expected CUDA tensors")


def sgemm(A, B, alpha: float = 1.0, beta: float = 0.0, C=None, transpose_b: bool = False, bias=None):
    """sgemm (blas:260-295): C = alpha*A.B + beta*C on the device.

    A [m, k]; B [k, n] (or [n, k] with transpose_b, the launch_naive_gemm
    form); returns C [m, n] (allocated when C is None)."""
    torch = _torch()
    _need_cuda(A, B, C, bias)
    m, k = A.shape
    n = B.shape[0] if transpose_b else B.shape[1]
    if (B.shape[1] if transpose_b else B.shape[0]) != k:
        raise ValueError(f"sgemm: B shape {tuple(B.shape)} does not match k={k}")
    if C is None:
        C = torch.zeros(m, n, dtype=torch.float32, device=A.device)
    check(lib().oc_sgemm(m, n, k, alpha, _ptr(A), A.stride(0), _ptr(B), B.stride(0), int(transpose_b), beta,
                         _ptr(C), C.stride(0), _ptr(bias), _stream()))
    return C


def softmax_rows(x):
    """In-place row softmax of a [rows, cols] CUDA tensor (cpu_row_softmax semantics)."""
    _need_cuda(x)
    rows, cols = x.shape
    check(lib().oc_softmax_rows(_ptr(x), rows, cols, _stream()))
    return x


def flash_attention(q, k, v, block_size: int):
    """flash_attention_with_spirv (blas:707-766): q, k, v [seq, d] -> [seq, d]."""
    torch = _torch()
    _need_cuda(q, k, v)
    seq, d = q.shape
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError(f"flash_attention_with_spirv: q/k/v shapes differ: {q.shape} {k.shape} {v.shape}")
    o = torch.empty_like(q)
    check(lib().oc_flash_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(o), seq, d, block_size, _stream()))
    return o


def flash_attention_fwd(q, k, v, scale=None, causal=False):
    """Multi-head attention: q [bh, sq, d], k/v [bh, skv, d] -> [bh, sq, d]."""
    torch = _torch()
    _need_cuda(q, k, v)
    bh, sq, d = q.shape
    skv = k.shape[1]
    o = torch.empty_like(q)
    s = (1.0 / d ** 0.5) if scale is None else scale
    check(lib().oc_flash_attention_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(o), bh, sq, skv, d, s, int(causal),
                                       _stream()))
    return o


def scaled_dot_product_attention(q, k, v):
    """scaled_dot_product_attention (blas:411-540), unfused, on the device."""
    torch = _torch()
    _need_cuda(q, k, v)
    seq, d = q.shape
    need = sz(0)
    check(lib().oc_sdpa_workspace_size(seq, C.byref(need)))
    ws = torch.empty(max(need.value, 4), dtype=torch.uint8, device=q.device)
    o = torch.empty_like(q)
    check(lib().oc_sdpa(_ptr(q), _ptr(k), _ptr(v), _ptr(o), seq, d, _ptr(ws), ws.numel(), _stream()))
    return o


def mla_compress_kv(kv, down_proj):
    """mla_compress_kv (blas:1045-1052): kv [seq, d_h] . down [d_h, d_c]."""
    torch = _torch()
    seq, dh = kv.shape
    dc = down_proj.shape[1]
    out = torch.empty(seq, dc, dtype=torch.float32, device=kv.device)
    check(lib().oc_mla_compress_kv(seq, dh, dc, _ptr(kv), _ptr(down_proj), _ptr(out), _stream()))
    return out


def mla_decompress_kv(latent, up_proj):
    """mla_decompress_kv (blas:1060-1067): latent [seq, d_c] . up [d_c, d_h]."""
    torch = _torch()
    seq, dc = latent.shape
    dh = up_proj.shape[1]
    out = torch.empty(seq, dh, dtype=torch.float32, device=latent.device)
    check(lib().oc_mla_decompress_kv(seq, dc, dh, _ptr(latent), _ptr(up_proj), _ptr(out), _stream()))
    return out


def quantize_int8(x, group_size: int):
    """quantize_int8 (blas:935-940) on the device: returns (data int8, scales f32)."""
    torch = _torch()
    _need_cuda(x)
    x = x.contiguous().view(-1)
    n = x.numel()
    q = torch.empty(n, dtype=torch.int8, device=x.device)
    s = torch.empty(max(1, -(-n // max(group_size, 1))), dtype=torch.float32, device=x.device)
    check(lib().oc_quantize_int8(_ptr(x), n, group_size, _ptr(q), _ptr(s), _stream()))
    return q, s


def quantize_int4(x, group_size: int):
    """quantize_int4 (blas:901-919) on the device: returns (packed uint8, scales f32)."""
    torch = _torch()
    _need_cuda(x)
    x = x.contiguous().view(-1)
    n = x.numel()
    q = torch.empty((n + 1) // 2, dtype=torch.uint8, device=x.device)
    s = torch.empty(max(1, -(-n // max(group_size, 1))), dtype=torch.float32, device=x.device)
    check(lib().oc_quantize_int4(_ptr(x), n, group_size, _ptr(q), _ptr(s), _stream()))
    return q, s


def quantize_int4_awq(weight, activation_scale, group_size: int, alpha: float):
    """quantize_int4_awq (blas:958-989): weight [rows, cols] CUDA tensor,
    activation_scale [cols] host values.  Returns (packed, scales, awq_scale)."""
    torch = _torch()
    _need_cuda(weight)
    rows, cols = weight.shape
    act = np.ascontiguousarray(activation_scale, np.float32).ravel()
    if rows == 0 or cols == 0:
        raise ValueError("quantize_int4_awq: rows and cols must be > 0")
    if act.size != cols:
        raise ValueError("quantize_int4_awq: activation_scale.len() must equal cols")
    awq = np.zeros(cols, np.float32)
    check(lib().oc_awq_scales(act.ctypes.data_as(vp), cols, alpha, awq.ctypes.data_as(vp)))
    awq_d = torch.from_numpy(awq).to(weight.device)
    n = rows * cols
    q = torch.empty((n + 1) // 2, dtype=torch.uint8, device=weight.device)
    s = torch.empty(-(-n // max(group_size, 1)), dtype=torch.float32, device=weight.device)
    check(lib().oc_quantize_int4_awq(_ptr(weight.contiguous()), rows, cols, _ptr(awq_d), group_size, _ptr(q),
                                     _ptr(s), _stream()))
    return q, s, awq_d


def dequantize_int4_awq(q, scales, rows: int, cols: int, group_size: int, awq_scale):
    torch = _torch()
    out = torch.empty(rows * cols, dtype=torch.float32, device=q.device)
    check(lib().oc_dequantize_int4_awq(_ptr(q), _ptr(scales), rows, cols, group_size, _ptr(awq_scale), _ptr(out),
                                       _stream()))
    return out


def dequantize_int8(q, scales, length: int, group_size: int):
    torch = _torch()
    out = torch.empty(length, dtype=torch.float32, device=q.device)
    check(lib().oc_dequantize_int8(_ptr(q), _ptr(scales), length, group_size, _ptr(out), _stream()))
    return out


def dequantize_int4(q, scales, length: int, group_size: int):
    torch = _torch()
    out = torch.empty(length, dtype=torch.float32, device=q.device)
    check(lib().oc_dequantize_int4(_ptr(q), _ptr(scales), length, group_size, _ptr(out), _stream()))
    return out


_workspaces: dict = {}


def workspace(m: int, k: int, device):
    """Grow-only scratch for the quantized matmuls, one per device."""
    torch = _torch()
    need = sz(0)
    check(lib().oc_qgemm_workspace_size(m, k, C.byref(need)))
    key = str(device)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < need.value:
        ws = torch.empty(max(need.value, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def qgemm_w8a8(A, Wq, w_scales, bias=None, out=None, want_acc=False):
    """Y = A . dequant(W8)^T + bias with exact int32 accumulation (W8A8).

    A [m, k] f32, Wq [n, k] int8 (quantize_int8 of W^T, group = k),
    w_scales [n] f32.  Returns Y [m, n] (and the int32 accumulators)."""
    torch = _torch()
    _need_cuda(A, Wq, w_scales, bias)
    m, k = A.shape
    n = Wq.shape[0] if Wq.dim() == 2 else Wq.numel() // k
    Y = out if out is not None else torch.empty(m, n, dtype=torch.float32, device=A.device)
    acc = torch.empty(m, n, dtype=torch.int32, device=A.device) if want_acc else None
    ws = workspace(m, k, A.device)
    check(lib().oc_qgemm_w8a8(m, n, k, _ptr(A), _ptr(Wq), _ptr(w_scales), _ptr(bias), _ptr(Y), _ptr(ws),
                              ws.numel(), _ptr(acc), _stream()))
    return (Y, acc) if want_acc else Y


def qgemm_w4a8(A, Wq, w_scales, group: int, bias=None, out=None, want_acc=False):
    """Y = A . dequant(W4)^T + bias with exact per-group int32 partials (W4A8).

    Wq [n, k/2] uint8 packed as quantize_int4 packs W^T, w_scales [n*k/group]."""
    torch = _torch()
    _need_cuda(A, Wq, w_scales, bias)
    m, k = A.shape
    n = Wq.numel() * 2 // k
    Y = out if out is not None else torch.empty(m, n, dtype=torch.float32, device=A.device)
    acc = torch.empty(m, n, k // group, dtype=torch.int32, device=A.device) if want_acc else None
    ws = workspace(m, k, A.device)
    check(lib().oc_qgemm_w4a8(m, n, k, group, _ptr(A), _ptr(Wq), _ptr(w_scales), _ptr(bias), _ptr(Y), _ptr(ws),
                              ws.numel(), _ptr(acc), _stream()))
    return (Y, acc) if want_acc else Y


def qgemm_w8(A, Wq, w_scales, bias=None, out=None):
    """Weight-only INT8: Y = A . dequantize_int8(Wq)^T + bias in f32.

    A [m, k] f32, Wq [n, k] int8 (quantize_int8 of W^T, group = k),
    w_scales [n] f32.  Linear::forward over the dequantized weights
    (crates/open-cuda-llm/src/lib.rs:227-238)."""
    torch = _torch()
    _need_cuda(A, Wq, w_scales, bias)
    m, k = A.shape
    n = Wq.numel() // k
    Y = out if out is not None else torch.empty(m, n, dtype=torch.float32, device=A.device)
    check(lib().oc_qgemm_w8(m, n, k, _ptr(A), _ptr(Wq), _ptr(w_scales), _ptr(bias), _ptr(Y), _stream()))
    return Y


def qgemm_w4(A, Wq, w_scales, group: int, bias=None, out=None):
    """Weight-only INT4: Y = A . dequantize_int4(Wq)^T + bias in f32.

    Wq packed as quantize_int4 packs W^T ([n*k/2] bytes), w_scales
    [ceil(n*k/group)] f32."""
    torch = _torch()
    _need_cuda(A, Wq, w_scales, bias)
    m, k = A.shape
    n = Wq.numel() * 2 // k
    Y = out if out is not None else torch.empty(m, n, dtype=torch.float32, device=A.device)
    check(lib().oc_qgemm_w4(m, n, k, group, _ptr(A), _ptr(Wq), _ptr(w_scales), _ptr(bias), _ptr(Y), _stream()))
    return Y


def quantize_rows_int8(A):
    """quantize_int8(A, group = k) of a [m, k] f32 matrix: (qa [m, k] int8, sa [m] f32)."""
    torch = _torch()
    _need_cuda(A)
    A = A.contiguous()
    m, k = A.shape
    qa = torch.empty(m, k, dtype=torch.int8, device=A.device)
    sa = torch.empty(m, dtype=torch.float32, device=A.device)
    check(lib().oc_quantize_rows_int8(_ptr(A), m, k, _ptr(qa), _ptr(sa), _stream()))
    return qa, sa


def igemm_w8a8(qa, sa, Wq, w_scales, bias=None, out=None):
    """W8A8 product on pre-quantized activations (qa [m, k] int8, sa [m])."""
    torch = _torch()
    m, k = qa.shape
    n = Wq.numel() // k
    Y = out if out is not None else torch.empty(m, n, dtype=torch.float32, device=qa.device)
    check(lib().oc_igemm_w8a8(m, n, k, _ptr(qa), _ptr(sa), _ptr(Wq), _ptr(w_scales), _ptr(bias), _ptr(Y), None,
                              _stream()))
    return Y


def igemm_w4a8(qa, sa, Wq, w_scales, group: int, bias=None, out=None):
    """W4A8 product on pre-quantized activations."""
    torch = _torch()
    m, k = qa.shape
    n = Wq.numel() * 2 // k
    Y = out if out is not None else torch.empty(m, n, dtype=torch.float32, device=qa.device)
    check(lib().oc_igemm_w4a8(m, n, k, group, _ptr(qa), _ptr(sa), _ptr(Wq), _ptr(w_scales), _ptr(bias), _ptr(Y),
                              None, _stream()))
    return Y


# ---- host slices: the GpuDevice object ---------------------------------------

def _np_ptr(a):
    return None if a is None else a.ctypes.data_as(vp)


class Device:
    """A GpuDevice (crates/opencuda-core/src/device.rs:88-132) on CUDA."""

    def __init__(self, ordinal: int = 0):
        h = vp()
        check(lib().oc_device_open(ordinal, C.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            lib().oc_device_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def info(self) -> DeviceInfo:
        d = DeviceInfo()
        check(lib().oc_device_get_info(self._h, C.byref(d)))
        return d

    def stream(self) -> int:
        return lib().oc_device_stream(self._h)

    def alloc(self, nbytes: int) -> int:
        a = C.c_uint64(0)
        rc = lib().oc_device_alloc(self._h, nbytes, C.byref(a))
        if rc == OC_ERR_OUT_OF_MEMORY:
            raise MemoryError(last_error())
        check(rc)
        return a.value

    def free(self, addr: int) -> None:
        check(lib().oc_device_free(self._h, addr))

    def memcpy_h2d(self, dst: int, src: np.ndarray) -> None:
        src = np.ascontiguousarray(src)
        rc = lib().oc_device_memcpy_h2d(self._h, dst, _np_ptr(src), src.nbytes)
        if rc == OC_ERR_OUT_OF_MEMORY:
            raise MemoryError(last_error())
        check(rc)

    def memcpy_d2h(self, dst: np.ndarray, src: int) -> None:
        check(lib().oc_device_memcpy_d2h(self._h, _np_ptr(dst), src, dst.nbytes))

    def memcpy_d2d(self, dst: int, src: int, nbytes: int) -> None:
        check(lib().oc_device_memcpy_d2d(self._h, dst, src, nbytes))

    def synchronize(self) -> None:
        check(lib().oc_device_synchronize(self._h))

    # -- blas on host slices --
    def quantize_int8(self, x, group_size: int):
        x = np.ascontiguousarray(x, np.float32).ravel()
        if x.size == 0:
            raise ValueError("quantize: input must not be empty")
        if group_size == 0:
            raise ValueError("quantize: group_size must be > 0")
        q = np.zeros(x.size, np.int8)
        s = np.zeros(-(-x.size // group_size), np.float32)
        check(lib().oc_blas_quantize_int8(self._h, _np_ptr(x), x.size, group_size, _np_ptr(q), _np_ptr(s)))
        return q, s

    def quantize_int4(self, x, group_size: int):
        x = np.ascontiguousarray(x, np.float32).ravel()
        if x.size == 0:
            raise ValueError("quantize: input must not be empty")
        if group_size == 0:
            raise ValueError("quantize: group_size must be > 0")
        q = np.zeros((x.size + 1) // 2, np.uint8)
        s = np.zeros(-(-x.size // group_size), np.float32)
        check(lib().oc_blas_quantize_int4(self._h, _np_ptr(x), x.size, group_size, _np_ptr(q), _np_ptr(s)))
        return q, s

    def qgemm_w8a8(self, m, n, k, a, wq, w_scales, bias=None, out=None):
        a = np.ascontiguousarray(a, np.float32)
        y = out if out is not None else np.zeros(m * n, np.float32)
        check(lib().oc_blas_qgemm_w8a8(self._h, m, n, k, _np_ptr(a), _np_ptr(np.ascontiguousarray(wq)),
                                       _np_ptr(np.ascontiguousarray(w_scales, np.float32)),
                                       _np_ptr(None if bias is None else np.ascontiguousarray(bias, np.float32)),
                                       _np_ptr(y)))
        return y

    def qgemm_w4a8(self, m, n, k, group, a, wq, w_scales, bias=None, out=None):
        a = np.ascontiguousarray(a, np.float32)
        y = out if out is not None else np.zeros(m * n, np.float32)
        check(lib().oc_blas_qgemm_w4a8(self._h, m, n, k, group, _np_ptr(a), _np_ptr(np.ascontiguousarray(wq)),
                                       _np_ptr(np.ascontiguousarray(w_scales, np.float32)),
                                       _np_ptr(None if bias is None else np.ascontiguousarray(bias, np.float32)),
                                       _np_ptr(y)))
        return y

    def qgemm_w8(self, m, n, k, a, wq, w_scales, bias=None, out=None):
        """Weight-only INT8 on host slices (oc_blas_qgemm_w8)."""
        a = np.ascontiguousarray(a, np.float32)
        y = out if out is not None else np.zeros(m * n, np.float32)
        check(lib().oc_blas_qgemm_w8(self._h, m, n, k, _np_ptr(a), _np_ptr(np.ascontiguousarray(wq)),
                                     _np_ptr(np.ascontiguousarray(w_scales, np.float32)),
                                     _np_ptr(None if bias is None else np.ascontiguousarray(bias, np.float32)),
                                     _np_ptr(y)))
        return y

    def qgemm_w4(self, m, n, k, group, a, wq, w_scales, bias=None, out=None):
        """Weight-only INT4 on host slices (oc_blas_qgemm_w4)."""
        a = np.ascontiguousarray(a, np.float32)
        y = out if out is not None else np.zeros(m * n, np.float32)
        check(lib().oc_blas_qgemm_w4(self._h, m, n, k, group, _np_ptr(a), _np_ptr(np.ascontiguousarray(wq)),
                                     _np_ptr(np.ascontiguousarray(w_scales, np.float32)),
                                     _np_ptr(None if bias is None else np.ascontiguousarray(bias, np.float32)),
                                     _np_ptr(y)))
        return y


class DevicePartition(C.Structure):
    """DevicePartition (crates/opencuda-multidev/src/lib.rs:17-22)."""

    _fields_ = [("device_id", sz), ("layer_start", sz), ("layer_end", sz)]


def partition_layers_by_memory(total_memory, total_layers: int) -> list[tuple[int, int, int]]:
    """partition_layers (multidev:28-74) on a list of device memory sizes:
    [(device_id, layer_start, layer_end)]."""
    n = len(total_memory)
    mem = (C.c_uint64 * max(n, 1))(*[int(x) for x in total_memory])
    out = (DevicePartition * max(n, 1))()
    check(lib().oc_partition_layers_by_memory(mem, n, total_layers, out))
    return [(p.device_id, p.layer_start, p.layer_end) for p in out[:n]]


def partition_layers(devices, total_layers: int) -> list[tuple[int, int, int]]:
    """partition_layers (multidev:28-74) over Device objects."""
    n = len(devices)
    hs = (vp * max(n, 1))(*[d.handle for d in devices])
    out = (DevicePartition * max(n, 1))()
    check(lib().oc_partition_layers(hs, n, total_layers, out))
    return [(p.device_id, p.layer_start, p.layer_end) for p in out[:n]]


def transfer_between_devices(src: "Device", src_addr: int, dst: "Device", dst_addr: int, nbytes: int) -> None:
    """transfer_between_devices (multidev:78-83): allocation to allocation,
    NVLink peer copy or staged through host memory; synchronous."""
    check(lib().oc_transfer_between_devices(src.handle, src_addr, dst.handle, dst_addr, nbytes))


class LaunchConfig(C.Structure):
    """LaunchConfig (crates/opencuda-core/src/device.rs:45-85)."""

    _fields_ = [("grid", C.c_uint32 * 3), ("block", C.c_uint32 * 3), ("shared_mem", C.c_uint32)]


class _ArgV(C.Union):
    _fields_ = [("ptr", C.c_uint64), ("u32", C.c_uint32), ("i32", C.c_int32), ("f32", C.c_float),
                ("usize", C.c_uint64)]


class KernelArg(C.Structure):
    """KernelArg (crates/opencuda-core/src/kernel.rs:88-100)."""

    _fields_ = [("kind", ci), ("v", _ArgV)]

    @staticmethod
    def ptr(addr):
        a = KernelArg(0)
        a.v.ptr = addr
        return a

    @staticmethod
    def usize(x):
        a = KernelArg(4)
        a.v.usize = x
        return a

    @staticmethod
    def u32(x):
        a = KernelArg(1)
        a.v.u32 = x
        return a

    @staticmethod
    def f32(x):
        a = KernelArg(3)
        a.v.f32 = x
        return a


def _f32c(x):
    return np.ascontiguousarray(x, np.float32).ravel()


def _device_blas_methods():
    """Host-slice blas methods of Device (the reference's signatures)."""

    def launch_kernel(self, name: str, args, grid=(1, 1, 1), block=(1, 1, 1)):
        cfg = LaunchConfig((C.c_uint32 * 3)(*grid), (C.c_uint32 * 3)(*block), 0)
        arr = (KernelArg * len(args))(*args)
        check(lib().oc_device_launch(self._h, name.encode(), C.byref(cfg), arr, len(args)))

    def sgemm(self, m, k, n, alpha, a, b, beta, c):
        a, b = _f32c(a), _f32c(b)
        c = np.ascontiguousarray(c, np.float32).ravel().copy()
        if a.size != m * k:
            raise ValueError(f"sgemm: a.len()={a.size} != m*k={m * k}")
        if b.size != k * n:
            raise ValueError(f"sgemm: b.len()={b.size} != k*n={k * n}")
        if c.size != m * n:
            raise ValueError(f"sgemm: c.len()={c.size} != m*n={m * n}")
        check(lib().oc_blas_sgemm(self._h, m, k, n, alpha, _np_ptr(a), _np_ptr(b), beta, _np_ptr(c)))
        return c

    def softmax_rows(self, rows, cols, data):
        d = _f32c(data)
        if d.size != rows * cols:
            raise ValueError(f"softmax_vulkan_generic: data.len()={d.size} != rows*cols={rows * cols}")
        out = np.zeros(rows * cols, np.float32)
        check(lib().oc_blas_softmax_rows(self._h, rows, cols, _np_ptr(d), _np_ptr(out)))
        return out

    def _qkv(self, name, q, k, v, seq, d):
        q, k, v = _f32c(q), _f32c(k), _f32c(v)
        for nm, x in (("q", q), ("k", k), ("v", v)):
            if x.size != seq * d:
                raise ValueError(f"{name}: {nm}.len()={x.size} != seq_len*head_dim={seq * d}")
        return q, k, v

    def flash_attention(self, q, k, v, seq_len, head_dim, block_size):
        q, k, v = self._qkv("flash_attention_with_spirv", q, k, v, seq_len, head_dim)
        if block_size == 0:
            raise ValueError("flash_attention_with_spirv: block_size must be > 0")
        out = np.zeros(seq_len * head_dim, np.float32)
        check(lib().oc_blas_flash_attention(self._h, _np_ptr(q), _np_ptr(k), _np_ptr(v), seq_len, head_dim,
                                            block_size, _np_ptr(out)))
        return out

    def scaled_dot_product_attention(self, q, k, v, seq_len, head_dim):
        q, k, v = self._qkv("attention", q, k, v, seq_len, head_dim)
        out = np.zeros(seq_len * head_dim, np.float32)
        check(lib().oc_blas_sdpa(self._h, _np_ptr(q), _np_ptr(k), _np_ptr(v), seq_len, head_dim, _np_ptr(out)))
        return out

    def mla_compress_kv(self, seq_len, d_h, d_c, kv, down_proj):
        kv, dp = _f32c(kv), _f32c(down_proj)
        if kv.size != seq_len * d_h:
            raise ValueError(f"mla_compress_kv: kv.len()={kv.size} != seq_len*d_h={seq_len * d_h}")
        if dp.size != d_h * d_c:
            raise ValueError(f"mla_compress_kv: down_proj.len()={dp.size} != d_h*d_c={d_h * d_c}")
        out = np.zeros(seq_len * d_c, np.float32)
        check(lib().oc_blas_mla_compress_kv(self._h, seq_len, d_h, d_c, _np_ptr(kv), _np_ptr(dp), _np_ptr(out)))
        return out

    def mla_decompress_kv(self, seq_len, d_c, d_h, latent, up_proj):
        lt, up = _f32c(latent), _f32c(up_proj)
        if lt.size != seq_len * d_c:
            raise ValueError(f"mla_decompress_kv: latent.len()={lt.size} != seq_len*d_c={seq_len * d_c}")
        if up.size != d_c * d_h:
            raise ValueError(f"mla_decompress_kv: up_proj.len()={up.size} != d_c*d_h={d_c * d_h}")
        out = np.zeros(seq_len * d_h, np.float32)
        check(lib().oc_blas_mla_decompress_kv(self._h, seq_len, d_c, d_h, _np_ptr(lt), _np_ptr(up), _np_ptr(out)))
        return out

    for f in (launch_kernel, sgemm, softmax_rows, _qkv, flash_attention, scaled_dot_product_attention,
              mla_compress_kv, mla_decompress_kv):
        setattr(Device, f.__name__, f)


_device_blas_methods()
