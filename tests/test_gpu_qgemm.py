"""GPU parity: quantization and the quantized matmuls through the C ABI,
bit-exact against the oracle (integer work and the defined f32 epilogue
order are reproducible exactly)."""
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


def bits_equal(a, b):
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    assert a.shape == b.shape, (a.shape, b.shape)
    if a.dtype == np.float32:
        bad = np.nonzero(a.view(np.uint32) != b.view(np.uint32))[0]
    else:
        bad = np.nonzero(a != b)[0]
    assert bad.size == 0, f"{bad.size} mismatches, first at {bad[:5]}: {a.ravel()[bad[:5]]} vs {b.ravel()[bad[:5]]}"


QUANT_CASES = [
    (5, 5, [7.0, -7.0, 0.0, 3.5, 1.0]),
    (8, 4, [0.0] * 8),
    (4, 2, [700.0, -350.0, 0.007, -0.0035]),
    (1001, 7, None),
    (3072 * 768, 768, None),
    (3072 * 768, 32, None),
    (100003, 33, None),
]


@pytest.mark.parametrize("n,group,vals", QUANT_CASES)
def test_quantize_matches_oracle(oc, oracle, n, group, vals):
    x = np.array(vals, np.float32) if vals is not None else synth.normal(11, n, 0.0, 3.0)
    if vals is None:
        x[::97] = 0.0
        x[5] = 2.5 * 3.0 / 127  # a tie near half a step
    xd = torch.from_numpy(x).cuda()
    q8, s8 = oc.quantize_int8(xd, group)
    q4, s4 = oc.quantize_int4(xd, group)
    torch.cuda.synchronize()
    r8 = oracle.quantize_int8(x, group)
    r4 = oracle.quantize_int4(x, group)
    bits_equal(s8.cpu().numpy(), r8.scales)
    bits_equal(q8.cpu().numpy(), r8.data)
    bits_equal(s4.cpu().numpy(), r4.scales)
    bits_equal(q4.cpu().numpy(), r4.data)
    d8 = oc.dequantize_int8(q8, s8, n, group)
    d4 = oc.dequantize_int4(q4, s4, n, group)
    bits_equal(d8.cpu().numpy(), oracle.dequantize_int8(r8))
    bits_equal(d4.cpu().numpy(), oracle.dequantize_int4(r4))


def test_host_slice_quantize_and_errors(oc, oracle):
    dev = oc.Device(0)
    x = synth.normal(3, 4099, 0.0, 1.0)
    q, s = dev.quantize_int8(x, 64)
    r = oracle.quantize_int8(x, 64)
    bits_equal(q, r.data)
    bits_equal(s, r.scales)
    q4, s4 = dev.quantize_int4(x, 32)
    r4 = oracle.quantize_int4(x, 32)
    bits_equal(q4, r4.data)
    bits_equal(s4, r4.scales)
    with pytest.raises(ValueError):
        dev.quantize_int8(np.zeros(0, np.float32), 4)
    with pytest.raises(ValueError):
        dev.quantize_int4(np.ones(3, np.float32), 0)
    dev.close()


def _weights(oracle, wt, bits, group):
    n, k = wt.shape
    if bits == 8:
        t = oracle.quantize_int8(wt.ravel(), k)
    else:
        t = oracle.quantize_int4(wt.ravel(), group)
    return t.data, t.scales


QGEMM_SHAPES = [
    # config-2 sweep (K=768, N=3072)
    (1, 768, 3072), (16, 768, 3072), (128, 768, 3072), (2048, 768, 3072),
    # ragged / small shapes through every path
    (3, 64, 40), (17, 96, 72), (37, 256, 200), (129, 384, 130), (300, 512, 264),
    # 7B-class K
    (8, 3584, 512), (64, 3584, 384),
]


@pytest.mark.parametrize("m,k,n", QGEMM_SHAPES)
def test_qgemm_w8a8_bit_exact(oc, oracle, m, k, n):
    A, WT, bias = synth.qgemm_case(m, k, n, 1, 2, 3)
    wq, ws = _weights(oracle, WT, 8, k)
    y_ref, acc_ref = oracle.qgemm_w8a8(m, k, n, A, wq, ws, bias, want_acc=True)
    Ad = torch.from_numpy(A).cuda()
    y, acc = oc.qgemm_w8a8(Ad, torch.from_numpy(wq).cuda().view(n, k), torch.from_numpy(ws).cuda(),
                           torch.from_numpy(bias).cuda(), want_acc=True)
    torch.cuda.synchronize()
    bits_equal(acc.cpu().numpy().ravel(), acc_ref)
    bits_equal(y.cpu().numpy().ravel(), y_ref)


@pytest.mark.parametrize("m,k,n", QGEMM_SHAPES)
def test_qgemm_w4a8_bit_exact(oc, oracle, m, k, n):
    if k % 32:
        pytest.skip("group 32 needs k % 32 == 0")
    A, WT, bias = synth.qgemm_case(m, k, n, 1, 2, 3)
    wq, ws = _weights(oracle, WT, 4, 32)
    y_ref, acc_ref = oracle.qgemm_w4a8(m, k, n, 32, A, wq, ws, bias, want_acc=True)
    y, acc = oc.qgemm_w4a8(torch.from_numpy(A).cuda(), torch.from_numpy(wq).cuda(), torch.from_numpy(ws).cuda(),
                           32, torch.from_numpy(bias).cuda(), want_acc=True)
    torch.cuda.synchronize()
    bits_equal(acc.cpu().numpy().ravel(), acc_ref)
    bits_equal(y.cpu().numpy().ravel(), y_ref)


def test_qgemm_no_bias_and_host_slices(oc, oracle):
    m, k, n = 40, 256, 96
    A, WT, _ = synth.qgemm_case(m, k, n, 7, 8, 9)
    wq, ws = _weights(oracle, WT, 8, k)
    y_ref = oracle.qgemm_w8a8(m, k, n, A, wq, ws, None)
    dev = oc.Device(0)
    bits_equal(dev.qgemm_w8a8(m, n, k, A, wq, ws, None), y_ref)
    wq4, ws4 = _weights(oracle, WT, 4, 32)
    y4_ref = oracle.qgemm_w4a8(m, k, n, 32, A, wq4, ws4, None)
    bits_equal(dev.qgemm_w4a8(m, n, k, 32, A, wq4, ws4, None), y4_ref)
    dev.close()


def test_qgemm_matches_weight_only_reference_loosely(oc, oracle):
    # The W8A8 result approximates the reference-composed weight-only
    # product sgemm(A, dequantize(W)^T) + bias; int8 activations add a
    # relative error of order 1/127.
    m, k, n = 64, 768, 256
    A, WT, bias = synth.qgemm_case(m, k, n)
    wq, ws = _weights(oracle, WT, 8, k)
    y_wo = oracle.qgemm_weight_only(8, m, k, n, k, A, wq, ws, bias)
    y = oc.qgemm_w8a8(torch.from_numpy(A).cuda(), torch.from_numpy(wq).cuda().view(n, k),
                      torch.from_numpy(ws).cuda(), torch.from_numpy(bias).cuda()).cpu().numpy().ravel()
    rel = np.linalg.norm(y - y_wo) / np.linalg.norm(y_wo)
    assert rel < 2e-2


@pytest.mark.parametrize("rows,cols,group,alpha", [(1, 4, 4, 1.0), (96, 768, 32, 0.5), (7, 33, 5, 0.8)])
def test_awq_bit_exact(oc, oracle, rows, cols, group, alpha):
    if rows == 1:  # blas:1274-1305 known answer: the salient channel survives
        w = np.array([10.0, 10.0, 10.0, 0.1], np.float32)
        act = np.array([1.0, 1.0, 1.0, 100.0], np.float32)
    else:
        w = synth.normal(rows + cols, rows * cols, 0.0, 0.02)
        act = np.abs(synth.normal(cols, cols, 0.0, 2.0))
        act[::7] = 0.0  # non-positive scales map to 1
    ref = oracle.quantize_int4_awq(w, rows, cols, act, group, alpha)
    q, s, awq = oc.quantize_int4_awq(torch.from_numpy(w).cuda().view(rows, cols), act, group, alpha)
    torch.cuda.synchronize()
    bits_equal(awq.cpu().numpy(), ref.awq_scale)
    bits_equal(s.cpu().numpy(), ref.inner.scales)
    bits_equal(q.cpu().numpy(), ref.inner.data)
    d = oc.dequantize_int4_awq(q, s, rows, cols, group, awq)
    bits_equal(d.cpu().numpy(), oracle.dequantize_int4_awq(ref))
    if rows == 1:
        assert abs(w[3] - d.cpu().numpy()[3]) < abs(w[3] - 0.0)


def test_device_alloc_copy_contract(oc):
    dev = oc.Device(0)
    with pytest.raises(MemoryError):
        dev.alloc(0)
    a = dev.alloc(64)
    x = np.arange(16, dtype=np.float32)
    dev.memcpy_h2d(a, x)
    with pytest.raises(MemoryError):
        dev.memcpy_h2d(a, np.zeros(17, np.float32))
    b = dev.alloc(64)
    dev.memcpy_d2d(b, a, 64)
    y = np.zeros(16, np.float32)
    dev.memcpy_d2h(y, b)
    assert np.array_equal(x, y)
    dev.free(a)
    with pytest.raises(ValueError):
        dev.free(a)
    with pytest.raises(ValueError):
        dev.memcpy_d2h(y, a)
    dev.synchronize()
    info = dev.info()
    assert info.cc_major == 10 and info.compute_units > 100
    dev.close()
