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
    "oc_device_stream": (vp, [vp]),
    "oc_get_device_status": (ci, [C.POINTER(ci)]),
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
    "oc_qgemm_w8a8_noalloc": (ci, [ci, ci, ci, vp, vp, vp, vp, vp, vp]),
    "oc_qgemm_w8a8_noalloc_max_bytes": (ci, [C.POINTER(sz)]),
    "oc_blas_quantize_int8": (ci, [vp, vp, sz, sz, vp, vp]),
    "oc_blas_quantize_int4": (ci, [vp, vp, sz, sz, vp, vp]),
    "oc_blas_qgemm_w8a8": (ci, [vp, sz, sz, sz, vp, vp, vp, vp, vp]),
    "oc_blas_qgemm_w4a8": (ci, [vp, sz, sz, sz, sz, vp, vp, vp, vp, vp]),
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
