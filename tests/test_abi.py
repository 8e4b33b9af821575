"""CPU-side checks of the C ABI: the library loads, exports every function
include/opencuda_cuda.h declares, and rejects bad arguments before touching
a device.  No kernel runs here."""
import ctypes as C
import os

import numpy as np
import pytest

import opencuda_cuda as oc


def test_library_exports_every_declared_function():
    L = oc.lib()
    names = oc.declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert missing == []


def test_binding_covers_header():
    # every declared function has a ctypes signature in the bindings
    import gpt
    assert sorted(set(oc._SIGS) | set(gpt._SIGS)) == oc.declared_functions()


def test_no_device_reports_status_instead_of_crashing():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    rc = oc.lib().oc_device_open(0, C.byref(h))
    assert rc in (oc.OC_ERR_NO_DEVICE, oc.OC_ERR_LAUNCH_FAILED)
    assert oc.last_error() != ""
    assert oc.device_count() == 0


def test_quantize_rejects_empty_and_zero_group_before_launch():
    L = oc.lib()
    assert L.oc_quantize_int8(None, 0, 4, None, None, None) == oc.OC_ERR_INVALID_VALUE
    assert "empty" in oc.last_error()
    assert L.oc_quantize_int4(None, 8, 0, None, None, None) == oc.OC_ERR_INVALID_VALUE
    assert "group_size" in oc.last_error()


def test_qgemm_argument_checks():
    L = oc.lib()
    n = C.c_size_t(0)
    assert L.oc_qgemm_workspace_size(0, 768, C.byref(n)) == oc.OC_ERR_INVALID_VALUE
    assert L.oc_qgemm_workspace_size(16, 768, C.byref(n)) == 0 and n.value >= 16 * 768 + 64
    # group must be a multiple of 32 dividing k
    assert L.oc_qgemm_w4a8(4, 8, 96, 48, None, None, None, None, None, None, 0, None, None) == 1
    assert L.oc_qgemm_w8a8(0, 8, 96, None, None, None, None, None, None, 0, None, None) == 1
    # workspace too small
    buf = (C.c_uint8 * 64)()
    rc = L.oc_qgemm_w8a8(4, 8, 96, C.addressof(buf), C.addressof(buf), C.addressof(buf), None,
                         C.addressof(buf), C.addressof(buf), 8, None, None)
    assert rc == 1 and "workspace" in oc.last_error()


def test_synth_splitmix_matches_oracle(oracle):
    import synth
    x = synth.next_f32(77, 1000, 0.02)
    y = oracle.splitmix64_fill(77, 0.02, 1000)
    assert np.array_equal(x.view(np.uint32), y.view(np.uint32))
    n = synth.normal(5, 10001, 0.0, 0.02)
    assert abs(float(n.mean())) < 1e-3 and abs(float(n.std()) - 0.02) < 1e-3
    u = synth.uniform(1, 10000)
    assert u.min() >= -1.0 and u.max() < 1.0
