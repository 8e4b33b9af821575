"""GPU parity of the weight-only quantized matmuls (oc_qgemm_w8 / oc_qgemm_w4
and their host-slice twins) against the oracle's composition of the
reference: Y = sgemm(A, dequantize(Wq)^T) + bias (Linear::forward,
crates/open-cuda-llm/src/lib.rs:227-238, over dequantize_int8 / int4,
crates/opencuda-blas/src/lib.rs:922-945), f32 activations.  f32 work: the
tolerance is 1e-5 relative Frobenius error (the dequantized-output
tolerance of the f32 path)."""
import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

REL_FRO = 1e-5


@pytest.fixture(scope="module")
def oc():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import opencuda_cuda
    return opencuda_cuda


def rel_fro(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _quant(oracle, wt, bits, group):
    t = oracle.quantize_int8(wt.ravel(), wt.shape[1]) if bits == 8 else oracle.quantize_int4(wt.ravel(), group)
    return t.data, t.scales


def _run(oc, bits, A, wq, ws, group, bias):
    args = (torch.from_numpy(A).cuda(), torch.from_numpy(wq).cuda(), torch.from_numpy(ws).cuda())
    b = None if bias is None else torch.from_numpy(bias).cuda()
    y = oc.qgemm_w8(*args, bias=b) if bits == 8 else oc.qgemm_w4(*args, group, bias=b)
    return y.cpu().numpy().ravel()


WO_SHAPES = [
    # config-2 sweep (K=768, N=3072): skinny (1, 16) and tensor-core (128 split in K, 2048 on 192-row tiles)
    (1, 768, 3072), (16, 768, 3072), (128, 768, 3072), (2048, 768, 3072),
    # ragged / small shapes through every path
    (3, 64, 40), (17, 96, 72), (37, 256, 200), (129, 384, 130), (300, 512, 264),
    # 7B-class K: skinny with 8 rows, tensor-core split in K
    (8, 3584, 512), (64, 3584, 384),
    # enough tiles to fill the GPU, ragged N; columns not 16-byte multiples (no TMA stores)
    (1200, 384, 4100), (300, 256, 11522), (2050, 384, 3070),
    # skinny rows whose activations exceed shared memory: split into launches
    (16, 16384, 40),
    # long K, every tile split; 192-row tiles, ragged rows and columns
    (1800, 2048, 200), (2000, 256, 3000),
    # K % 64 != 0: skinny kernel over 16-row chunks (INT8 k % 16 == 0, INT4 k % 32 == 0)
    (40, 96, 72), (20, 160, 96),
    # K % 16 != 0: the scalar kernel
    (5, 100, 33), (20, 100, 96),
    # skinny GEMV: columns not a multiple of 16, one 32-k chunk, long K; INT8 with K % 32 == 16
    (12, 256, 130), (9, 32, 17), (2, 3584, 18944), (6, 48, 80),
]


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("m,k,n", WO_SHAPES)
def test_weight_only_matches_oracle(oc, oracle, bits, m, k, n):
    group = 32 if k % 32 == 0 else 20  # group 20 (k = 100): the scalar kernel
    A, WT, bias = synth.qgemm_case(m, k, n, 1, 2, 3)
    A[min(2, m - 1)] = 0.0  # an all-zero activation row
    wq, ws = _quant(oracle, WT, bits, group)
    y_ref = oracle.qgemm_weight_only(bits, m, k, n, k if bits == 8 else group, A, wq, ws, bias)
    y = _run(oc, bits, A, wq, ws, group, bias)
    assert rel_fro(y, y_ref) <= REL_FRO, rel_fro(y, y_ref)
    # every column, not only the whole matrix, meets the tolerance
    yr, rr = y.reshape(m, n), y_ref.reshape(m, n)
    worst = max(rel_fro(yr[:, c], rr[:, c]) for c in range(0, n, max(1, n // 64)))
    assert worst <= 10 * REL_FRO, worst


@pytest.mark.parametrize("m,k,n,group", [(7, 96, 50, 40), (30, 128, 70, 48), (24, 256, 130, 64), (24, 256, 130, 128),
                                         (12, 256, 130, 64), (3, 512, 50, 128), (5, 96, 40, 48)])
def test_w4_group_sizes(oc, oracle, m, k, n, group):
    # groups that straddle weight rows (40, 48: the flat quantization of the
    # reference) and groups of 64 / 128 on the tensor-core path
    A, WT, bias = synth.qgemm_case(m, k, n, 4, 5, 6)
    wq, ws = _quant(oracle, WT, 4, group)
    y_ref = oracle.qgemm_weight_only(4, m, k, n, group, A, wq, ws, bias)
    assert rel_fro(_run(oc, 4, A, wq, ws, group, bias), y_ref) <= REL_FRO


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("a_scale,w_scale", [(1e-30, 1.0), (1e6, 1.0), (1.0, 1e-30), (1.0, 1e6), (1e-15, 1e-12),
                                             (1e-20, 1e-15)])
@pytest.mark.parametrize("m", [2, 3, 8, 300])
def test_weight_only_value_range(oc, oracle, bits, a_scale, w_scale, m):
    # per-row and per-column powers of two keep the f16 terms in range for
    # any magnitude of activations and weights; one row and one weight
    # column far smaller than the rest
    k, n = 256, 160
    A, WT, bias = synth.qgemm_case(m, k, n, 11, 12, 13)
    A = (A * np.float32(a_scale)).astype(np.float32)
    A[1] *= np.float32(1e-4)
    WT = (WT * np.float32(w_scale)).astype(np.float32)
    WT[7] *= np.float32(1e-3)
    bias = (bias * np.float32(a_scale * w_scale)).astype(np.float32)
    wq, ws = _quant(oracle, WT, bits, 32)
    y_ref = oracle.qgemm_weight_only(bits, m, k, n, k if bits == 8 else 32, A, wq, ws, bias)
    y = _run(oc, bits, A, wq, ws, 32, bias)
    assert np.all(np.isfinite(y))
    assert rel_fro(y, y_ref) <= REL_FRO, rel_fro(y, y_ref)
    if a_scale * w_scale >= 1e-30:  # below that the small row's products are subnormal in the reference itself
        assert rel_fro(y.reshape(m, n)[1], y_ref.reshape(m, n)[1]) <= 10 * REL_FRO


@pytest.mark.parametrize("m", [1, 8, 512])
def test_w4_7b_vocab_shape_sampled_columns(oc, oracle, m):
    # K=3584, N=152064, INT4 group 32 (the large-N 7B-class shape): the weights
    # are drawn and quantized on the device (quantize_int4 is bit-exact with
    # the oracle's), the GEMM runs in L2-sized column chunks; 1024 columns
    # (both ends, chunk boundaries, a stride) are checked against the oracle
    # run on those columns' weights.
    k, n, group = 3584, 152064, 32
    g = torch.Generator(device="cuda").manual_seed(5)
    WT = torch.randn(n, k, generator=g, device="cuda") * 0.02
    wq, ws = oc.quantize_int4(WT.view(-1), group)
    del WT
    A = torch.from_numpy(synth.uniform(4, m * k).reshape(m, k)).cuda()
    bias = torch.from_numpy(synth.normal(6, n, 0.0, 0.02)).cuda()
    y = oc.qgemm_w4(A, wq, ws, group, bias=bias)
    torch.cuda.synchronize()
    cols = np.unique(np.concatenate([np.arange(256), np.arange(n - 256, n), np.arange(2816 - 64, 2816 + 64),
                                     np.arange(300, n, n // 384)]))[:1024]
    ct = torch.from_numpy(cols).cuda()
    wq_s = wq.view(n, k // 2)[ct].cpu().numpy()
    ws_s = ws.view(n, k // group)[ct].cpu().numpy()
    y_ref = oracle.qgemm_weight_only(4, m, k, len(cols), group, A.cpu().numpy(), wq_s, ws_s,
                                     bias.cpu().numpy()[cols])
    y_s = y[:, ct].cpu().numpy()
    assert rel_fro(y_s, y_ref) <= REL_FRO, rel_fro(y_s, y_ref)


@pytest.mark.parametrize("pinned", [False, True])
def test_host_slice_weight_only(oc, oracle, pinned):
    # host slices: small call, then outputs of >= 8 MB and >= 1024 rows in
    # row chunks (128, 512, 460 rows) whose later chunks reuse the weight
    # terms the first chunk expanded; a second weight set on the same device
    # object must not reuse the first one's terms
    dev = oc.Device(0)
    m, k, n = 40, 256, 96
    A, WT, bias = synth.qgemm_case(m, k, n, 7, 8, 9)
    for bits in (8, 4):
        wq, ws = _quant(oracle, WT, bits, 32)
        y_ref = oracle.qgemm_weight_only(bits, m, k, n, k if bits == 8 else 32, A, wq, ws, None)
        y = dev.qgemm_w8(m, n, k, A, wq, ws) if bits == 8 else dev.qgemm_w4(m, n, k, 32, A, wq, ws)
        assert rel_fro(y, y_ref) <= REL_FRO
    m, k, n = 1100, 256, 2048
    A, WT, bias = synth.qgemm_case(m, k, n, 21, 22, 23)
    WT2 = synth.normal(24, n * k, 0.0, 0.05).reshape(n, k)
    Ah = torch.from_numpy(A).pin_memory().numpy() if pinned else A
    for bits in (8, 4):
        for W in (WT, WT2):
            wq, ws = _quant(oracle, W, bits, 32)
            y_ref = oracle.qgemm_weight_only(bits, m, k, n, k if bits == 8 else 32, A, wq, ws, bias)
            y = np.zeros(m * n, np.float32)
            if pinned:
                y = torch.zeros(m * n).pin_memory().numpy()
            if bits == 8:
                dev.qgemm_w8(m, n, k, Ah, wq, ws, bias, out=y)
            else:
                dev.qgemm_w4(m, n, k, 32, Ah, wq, ws, bias, out=y)
            assert rel_fro(y, y_ref) <= REL_FRO, (bits, rel_fro(y, y_ref))
    dev.close()


def test_weight_only_errors(oc):
    A = torch.zeros(4, 64, device="cuda")
    wq = torch.zeros(32 * 64 // 2, dtype=torch.uint8, device="cuda")
    ws = torch.ones(32 * 64 // 32, device="cuda")
    with pytest.raises(ValueError):
        oc.qgemm_w4(A, wq, ws, 0)
    with pytest.raises(ValueError):
        oc.check(oc.lib().oc_qgemm_w8(0, 4, 64, A.data_ptr(), wq.data_ptr(), ws.data_ptr(), None,
                                      A.data_ptr(), None))
    dev = oc.Device(0)
    with pytest.raises(ValueError):
        dev.qgemm_w4(1, 4, 64, 0, np.zeros(64, np.float32), np.zeros(128, np.uint8), np.ones(8, np.float32))
    dev.close()


@pytest.mark.parametrize("bits", [8, 4])
def test_weight_only_launched_by_name(oc, oracle, bits):
    # the kernels the opencuda-blas qgemm_w8 / qgemm_w4 functions launch through
    # GpuDevice::launch_kernel: [A, Wq, scales, bias, Y ptr; m, n, k (, group) usize]
    K = oc.KernelArg
    m, k, n, group = 24, 256, 130, 32
    A, WT, bias = synth.qgemm_case(m, k, n, 31, 32, 33)
    wq, ws = _quant(oracle, WT, bits, group)
    y_ref = oracle.qgemm_weight_only(bits, m, k, n, k if bits == 8 else group, A, wq, ws, bias)
    dev = oc.Device(0)
    bufs = [dev.alloc(x.nbytes) for x in (A, wq, ws, bias)] + [dev.alloc(m * n * 4)]
    for p, x in zip(bufs, (A, wq, ws, bias)):
        dev.memcpy_h2d(p, np.ascontiguousarray(x))
    args = [K.ptr(p) for p in bufs] + [K.usize(m), K.usize(n), K.usize(k)]
    if bits == 4:
        args.append(K.usize(group))
    dev.launch_kernel("qgemm_w8" if bits == 8 else "qgemm_w4", args)
    dev.synchronize()
    y = np.zeros(m * n, np.float32)
    dev.memcpy_d2h(y, bufs[4])
    assert rel_fro(y, y_ref) <= REL_FRO
    with pytest.raises(ValueError):  # a too-small output allocation is refused before any launch
        small = dev.alloc(16)
        dev.launch_kernel("qgemm_w8" if bits == 8 else "qgemm_w4", args[:4] + [K.ptr(small)] + args[5:])
    dev.close()


@pytest.mark.parametrize("a_scale", [1.0, 1e-30, 1e6])
@pytest.mark.parametrize("m,group", [(1, 32), (2, 64), (3, 128)])
def test_w4_skinny_chunk_outliers(oc, oracle, m, group, a_scale):
    # skinny INT4 rows with one element per 32-element chunk 1000x the
    # others, some 1e-6x, a chunk of zeros, and rows of any magnitude keep
    # the f32 tolerance, per row as well
    k, n = 1024, 96
    A, WT, bias = synth.qgemm_case(m, k, n, 21, 22, 23)
    A = (A * np.float32(a_scale)).astype(np.float32)
    bias = (bias * np.float32(a_scale)).astype(np.float32)
    A[:, 5::32] *= np.float32(1000.0)
    A[:, 9::32] *= np.float32(1e-6)
    A[:, 64:96] = 0.0
    A = A.astype(np.float32)
    wq, ws = _quant(oracle, WT, 4, group)
    y_ref = oracle.qgemm_weight_only(4, m, k, n, group, A, wq, ws, bias)
    y = _run(oc, 4, A, wq, ws, group, bias)
    assert rel_fro(y, y_ref) <= REL_FRO, rel_fro(y, y_ref)
    yr, rr = y.reshape(m, n), y_ref.reshape(m, n)
    for r in range(m):
        assert rel_fro(yr[r], rr[r]) <= REL_FRO, (r, rel_fro(yr[r], rr[r]))


@pytest.mark.parametrize("m", [1, 2, 3, 7, 10, 12, 16, 17, 33, 64])
def test_w4_few_rows_many_columns(oc, oracle, m):
    # 1-64 rows over enough 128-column weight tiles to fill the GPU (here
    # 19000 columns, the last tile ragged), groups of 32: the packed weights
    # are widened to int8 in tensor memory, the activations enter as three
    # int8 digits and each group's exact int32 sums are scaled on their way
    # out; every output against the oracle
    k, n = 1024, 19000
    A, WT, bias = synth.qgemm_case(m, k, n, 31, 32, 33)
    A[0, :] *= np.float32(1e-3)  # a row far smaller than the others
    wq, ws = _quant(oracle, WT, 4, 32)
    y_ref = oracle.qgemm_weight_only(4, m, k, n, 32, A, wq, ws, bias)
    y = _run(oc, 4, A, wq, ws, 32, bias)
    assert rel_fro(y, y_ref) <= REL_FRO, rel_fro(y, y_ref)
    yr, rr = y.reshape(m, n), y_ref.reshape(m, n)
    for r in range(m):
        assert rel_fro(yr[r], rr[r]) <= REL_FRO, (r, rel_fro(yr[r], rr[r]))
    assert rel_fro(yr[:, -37:], rr[:, -37:]) <= REL_FRO  # the ragged last tile


@pytest.mark.parametrize("a_scale", [1.0, 1e-30, 1e6])
@pytest.mark.parametrize("m", [1, 5, 40])
def test_w4_few_rows_many_columns_outliers(oc, oracle, m, a_scale):
    # the int8-digit path with one element per 32-element chunk 1000x the
    # others, some 1e-6x, a chunk of zeros and rows of any magnitude: the
    # digits round to 2^-23 of each row's largest |a|, inside the f32
    # tolerance per row
    k, n = 1024, 19000
    A, WT, bias = synth.qgemm_case(m, k, n, 41, 42, 43)
    A = (A * np.float32(a_scale)).astype(np.float32)
    bias = (bias * np.float32(a_scale)).astype(np.float32)
    A[:, 5::32] *= np.float32(1000.0)
    A[:, 9::32] *= np.float32(1e-6)
    A[:, 64:96] = 0.0
    A = A.astype(np.float32)
    wq, ws = _quant(oracle, WT, 4, 32)
    y_ref = oracle.qgemm_weight_only(4, m, k, n, 32, A, wq, ws, bias)
    y = _run(oc, 4, A, wq, ws, 32, bias)
    yr, rr = y.reshape(m, n), y_ref.reshape(m, n)
    for r in range(m):
        assert rel_fro(yr[r], rr[r]) <= REL_FRO, (r, rel_fro(yr[r], rr[r]))


def test_w4_few_rows_many_columns_nonfinite_row(oc, oracle):
    # a NaN or an infinity in an activation row of the int8-digit path makes
    # that row's outputs NaN; the other rows are unaffected
    m, k, n = 3, 1024, 19000
    A, WT, bias = synth.qgemm_case(m, k, n, 51, 52, 53)
    wq, ws = _quant(oracle, WT, 4, 32)
    A[0, 77] = np.nan
    A[2, 500] = np.inf
    y = _run(oc, 4, A, wq, ws, 32, bias).reshape(m, n)
    assert np.all(np.isnan(y[0])) and np.all(np.isnan(y[2]))
    y_ref = oracle.qgemm_weight_only(4, 1, k, n, 32, A[1:2].copy(), wq, ws, bias)
    assert rel_fro(y[1], y_ref) <= REL_FRO
