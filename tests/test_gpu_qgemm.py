"""GPU parity: quantization and the quantized matmuls through the C ABI
against the oracle.  Bit-exact: quantization, every int32 accumulator, the
W8A8 output, and the W4A8 output whenever the exact group partials are
requested (the per-group kernel).  The W4A8 output of the dequantizing
kernel (no partials requested, M > 16, k % 128 == 0) is f32 work and is held
to the dequantized-output tolerance: relative Frobenius error <= 1e-5."""
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


W4_REL_FRO = 1e-5  # dequantized f32 output of the W4A8 dequantizing kernel


def rel_fro(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


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
    # enough 128 x 256 tiles to fill the GPU, ragged N
    (1200, 384, 4100),
    # skinny rows whose activations exceed shared memory: split into launches
    (16, 16384, 40),
    # more tiles than SMs with a ragged last round (its tiles split in K) and
    # rows that are not 16-byte multiples (no TMA stores)
    (300, 256, 11522),
    # many rows (W4A8 through the expanded weight terms): long K, every tile
    # split in K and finished in the GEMM, ragged rows and columns; the same
    # with rows that are not 16-byte multiples; more tiles than SMs, ragged
    # columns
    (1800, 2048, 200), (1850, 2048, 202), (1900, 384, 4100),
    # short K, tiles filling half the GPU: not split
    (600, 256, 3000),
    # many rows on 192-row tiles (fewer MMA cycles on the busiest SM than
    # 256-row tiles): ragged rows and columns; columns not 16-byte multiples
    (2000, 256, 3000), (2050, 384, 3070),
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
    args = (torch.from_numpy(A).cuda(), torch.from_numpy(wq).cuda(), torch.from_numpy(ws).cuda(), 32,
            torch.from_numpy(bias).cuda())
    y, acc = oc.qgemm_w4a8(*args, want_acc=True)
    torch.cuda.synchronize()
    bits_equal(acc.cpu().numpy().ravel(), acc_ref)
    bits_equal(y.cpu().numpy().ravel(), y_ref)
    # without the partials: the dequantizing kernel (M > 16, k % 128 == 0) or
    # the same exact kernels
    y2 = oc.qgemm_w4a8(*args).cpu().numpy().ravel()
    qa, sa = oc.quantize_rows_int8(args[0])
    y3 = oc.igemm_w4a8(qa, sa, args[1], args[2], 32, args[4]).cpu().numpy().ravel()
    if m <= 16 or k % 128:
        bits_equal(y2, y_ref)
        bits_equal(y3, y_ref)
    else:
        assert rel_fro(y2, y_ref) <= W4_REL_FRO, rel_fro(y2, y_ref)
        bits_equal(y3, y2)  # int8 entry point: the same kernel on the same integers


def test_qgemm_no_bias_and_host_slices(oc, oracle):
    m, k, n = 40, 256, 96
    A, WT, _ = synth.qgemm_case(m, k, n, 7, 8, 9)
    wq, ws = _weights(oracle, WT, 8, k)
    y_ref = oracle.qgemm_w8a8(m, k, n, A, wq, ws, None)
    dev = oc.Device(0)
    bits_equal(dev.qgemm_w8a8(m, n, k, A, wq, ws, None), y_ref)
    wq4, ws4 = _weights(oracle, WT, 4, 32)
    y4_ref = oracle.qgemm_w4a8(m, k, n, 32, A, wq4, ws4, None)
    assert rel_fro(dev.qgemm_w4a8(m, n, k, 32, A, wq4, ws4, None), y4_ref) <= W4_REL_FRO
    dev.close()


@pytest.mark.parametrize("pinned", [False, True])
def test_host_slice_qgemm_row_chunks(oc, oracle, pinned):
    # outputs of >= 8 MB and >= 1024 rows go through row chunks whose copies
    # and matmuls overlap on three streams (3 chunks here: 128, 512, 460 rows);
    # pinned host buffers let the copies run asynchronously.  Opening and
    # closing the device object again releases and rebuilds its scratch.
    m, k, n = 1100, 256, 2048
    A, WT, bias = synth.qgemm_case(m, k, n, 21, 22, 23)
    wq, ws = _weights(oracle, WT, 8, k)
    wq4, ws4 = _weights(oracle, WT, 4, 32)
    y_ref = oracle.qgemm_w8a8(m, k, n, A, wq, ws, bias)
    y4_ref = oracle.qgemm_w4a8(m, k, n, 32, A, wq4, ws4, bias)
    if pinned:
        Ah = torch.from_numpy(A).pin_memory().numpy()
        y8 = torch.zeros(m * n).pin_memory().numpy()
        y4 = torch.zeros(m * n).pin_memory().numpy()
    else:
        Ah, y8, y4 = A, np.zeros(m * n, np.float32), np.zeros(m * n, np.float32)
    for _ in range(2):
        dev = oc.Device(0)
        dev.qgemm_w8a8(m, n, k, Ah, wq, ws, bias, out=y8)
        bits_equal(y8, y_ref)
        dev.qgemm_w4a8(m, n, k, 32, Ah, wq4, ws4, bias, out=y4)
        assert rel_fro(y4, y4_ref) <= W4_REL_FRO
        dev.close()


@pytest.mark.parametrize("m", [64, 1800])
@pytest.mark.parametrize("scale", [1e-30, 1e-6, 1.0, 1e6])
def test_w4a8_dequantizing_kernel_range(oc, oracle, scale, m):
    # per-column range factors keep the f16 terms in range for any scale
    # magnitude, in the dequantizing kernel (64 rows) and in the expanded
    # weight terms (1800 rows)
    k, n = 256, 160
    A, WT, bias = synth.qgemm_case(m, k, n, 11, 12, 13)
    WT = (WT * np.float32(scale)).astype(np.float32)
    WT[7] *= np.float32(1e-3)  # one column far smaller than the rest
    wq, ws = _weights(oracle, WT, 4, 32)
    y_ref = oracle.qgemm_w4a8(m, k, n, 32, A, wq, ws, None)
    y = oc.qgemm_w4a8(torch.from_numpy(A).cuda(), torch.from_numpy(wq).cuda(), torch.from_numpy(ws).cuda(),
                      32).cpu().numpy()
    assert rel_fro(y, y_ref) <= W4_REL_FRO
    assert rel_fro(y.reshape(m, n)[:, 7], y_ref.reshape(m, n)[:, 7]) <= W4_REL_FRO


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
