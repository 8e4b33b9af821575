"""GPU test of oc_qgemm_w8a8_noalloc, the allocation-free W8A8 matmul.

That entry point exists for callers that cannot call cudaMalloc (stream
callbacks, embedders whose device memory is owned by another allocator,
bindings that only get input and output buffers): its activation scratch is
a fixed 16 MiB device array inside the library.  This test calls it through
the C ABI twice in a row, on different inputs, and checks each result
against oc_qgemm_w8a8 (which uses a caller workspace); both compute the
same exact-int32 product, so the tolerance is zero (bit-identical).

The file is named to be collected last, so a run that stops at the first
failure has already run every other test.  It passes alone in a fresh
process and after the other tests.
"""
import ctypes as C

import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def oc():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import opencuda_cuda
    return opencuda_cuda


def _case(oc, m, k, n, seed):
    A, WT, bias = synth.qgemm_case(m, k, n, seed, seed + 1, seed + 2)
    Wd = torch.from_numpy(WT).cuda()
    q8, s8 = oc.quantize_int8(Wd, k)
    return torch.from_numpy(A).cuda(), q8.view(n, k), s8, torch.from_numpy(bias).cuda()


def _noalloc(oc, A, Wq, ws, bias):
    m, k = A.shape
    n = Wq.shape[0]
    Y = torch.empty(m, n, dtype=torch.float32, device=A.device)
    rc = oc.lib().oc_qgemm_w8a8_noalloc(m, n, k, A.data_ptr(), Wq.data_ptr(), ws.data_ptr(),
                                        None if bias is None else bias.data_ptr(), Y.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream)
    oc.check(rc)
    return Y


@pytest.mark.parametrize("m,k,n", [(2048, 768, 3072), (5, 768, 1000), (20, 100, 96)])
def test_noalloc_matches_workspace_entry_point_twice(oc, m, k, n):
    # two calls in a row on different inputs: the shared scratch keeps the
    # previous call's contents, which must not leak into the next result
    # (tensor-core GEMM, skinny kernel, and the scalar kernel for k % 16 != 0)
    for seed in (21, 42):
        A, Wq, ws, bias = _case(oc, m, k, n, seed)
        y_ref = oc.qgemm_w8a8(A, Wq, ws, bias)
        y = _noalloc(oc, A, Wq, ws, bias)
        torch.cuda.synchronize()
        a = y.cpu().numpy().view(np.uint32)
        b = y_ref.cpu().numpy().view(np.uint32)
        assert np.array_equal(a, b), f"seed {seed}: {(a != b).sum()} mismatches"


def test_noalloc_rejects_oversize(oc):
    cap = C.c_size_t(0)
    oc.check(oc.lib().oc_qgemm_w8a8_noalloc_max_bytes(C.byref(cap)))
    assert cap.value == 16 << 20
    m, k = 8192, 4096  # 32 MiB of quantized activations: over the limit
    rc = oc.lib().oc_qgemm_w8a8_noalloc(m, 64, k, 16, 16, 16, None, 16, None)
    assert rc == oc.OC_ERR_INVALID_VALUE
    assert "16 MiB" in oc.last_error()


@pytest.mark.parametrize("m,k,n", [(1500, 768, 2048), (7, 512, 300), (24, 100, 96)])
def test_noalloc_allocates_no_device_memory(oc, m, k, n):
    # The entry point's claim: no device allocation, even on the first call at
    # a size it has not seen.  The workspace entry point runs first at the same
    # size, so the kernels on this path are already loaded; then the device's
    # free memory must be the same before and after the allocation-free call.
    A, Wq, ws, bias = _case(oc, m, k, n, 7)
    y_ref = oc.qgemm_w8a8(A, Wq, ws, bias)
    Y = torch.empty(m, n, dtype=torch.float32, device=A.device)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    rc = oc.lib().oc_qgemm_w8a8_noalloc(m, n, k, A.data_ptr(), Wq.data_ptr(), ws.data_ptr(), bias.data_ptr(),
                                        Y.data_ptr(), torch.cuda.current_stream().cuda_stream)
    oc.check(rc)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"free device memory changed by {free0 - free1} bytes"
    assert np.array_equal(Y.cpu().numpy().view(np.uint32), y_ref.cpu().numpy().view(np.uint32))
