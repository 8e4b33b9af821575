"""GPU parity: softmax, fused flash attention, SDPA, MLA and the name-routed
launcher, against the oracle (restated reference, blas:373-1078).

Tolerance: 1e-5 relative Frobenius error for f32 outputs (exp and the
summation order differ from the reference's sequential CPU loops)."""
import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
TOL = 1e-5


@pytest.fixture(scope="module")
def oc():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import opencuda_cuda
    return opencuda_cuda


def rel(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def cu(x, shape=None):
    t = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    return t.view(*shape) if shape else t


def test_softmax_rows(oc, oracle):
    for rows, cols in [(1, 1), (7, 33), (160, 160), (3, 5000)]:
        x = synth.normal(rows + cols, rows * cols, 0.0, 3.0)
        ref = oracle.row_softmax(x, rows, cols)
        got = oc.softmax_rows(cu(x, (rows, cols))).cpu().numpy().ravel()
        assert rel(got, ref) < TOL
    # all -inf row: the sum is NaN-free only if max handling matches; the
    # reference leaves exp(x - max) values when sum <= 0
    dev = oc.Device(0)
    x = synth.normal(9, 4 * 6, 0.0, 1.0)
    assert rel(dev.softmax_rows(4, 6, x), oracle.row_softmax(x, 4, 6)) < TOL
    dev.close()


def test_flash_known_inputs(oc, oracle):
    # blas:1685-1709 inputs: sin/cos/linear ramps, seq 7, d 5
    seq, d = 7, 5
    i = np.arange(seq * d, dtype=np.float32)
    q = np.sin(i * np.float32(0.13)).astype(np.float32)
    k = np.cos(i * np.float32(0.29)).astype(np.float32)
    v = (i * np.float32(0.05) - np.float32(1.0)).astype(np.float32)
    naive = oracle.scaled_dot_product_attention(q, k, v, seq, d)
    for bs in [1, 2, 3, 4, 7, 14]:
        got = oc.flash_attention(cu(q, (seq, d)), cu(k, (seq, d)), cu(v, (seq, d)), bs).cpu().numpy().ravel()
        assert np.all(np.abs(got - naive) < 1e-4)
        assert rel(got, oracle.flash_attention(q, k, v, seq, d, bs)) < TOL
    # seq_len = 1 returns v (blas:1740-1747)
    one = oc.flash_attention(cu([0.5, -1, 2, 0.25], (1, 4)), cu([1, 1, 1, 1], (1, 4)), cu([10, 20, 30, 40], (1, 4)), 3)
    assert one.cpu().numpy().ravel().tolist() == [10.0, 20.0, 30.0, 40.0]


@pytest.mark.parametrize("seq,d", [(17, 8), (160, 64), (512, 64), (300, 128), (64, 256), (1000, 40)])
def test_flash_random(oc, oracle, seq, d):
    q = synth.uniform(seq, seq * d)
    k = synth.uniform(seq + 1, seq * d)
    v = synth.uniform(seq + 2, seq * d)
    ref = oracle.flash_attention(q, k, v, seq, d, 64)
    got = oc.flash_attention(cu(q, (seq, d)), cu(k, (seq, d)), cu(v, (seq, d)), 64).cpu().numpy().ravel()
    assert rel(got, ref) < TOL
    dev = oc.Device(0)
    assert rel(dev.flash_attention(q, k, v, seq, d, 64), ref) < TOL
    sd = oracle.scaled_dot_product_attention(q, k, v, seq, d)
    assert rel(oc.scaled_dot_product_attention(cu(q, (seq, d)), cu(k, (seq, d)), cu(v, (seq, d))).cpu().numpy(),
               sd) < TOL
    assert rel(dev.scaled_dot_product_attention(q, k, v, seq, d), sd) < TOL
    dev.close()


def test_flash_errors(oc):
    z = torch.zeros(2, 2, device="cuda")
    with pytest.raises(ValueError):
        oc.flash_attention(z, z, z, 0)
    big = torch.zeros(2, 300, device="cuda")
    with pytest.raises(ValueError):
        oc.flash_attention(big, big, big, 4)
    dev = oc.Device(0)
    with pytest.raises(ValueError):
        dev.flash_attention([1, 2], [1] * 4, [1] * 4, 2, 2, 1)
    dev.close()


@pytest.mark.parametrize("causal", [False, True])
def test_flash_multihead_and_cross(oc, oracle, causal):
    bh, sq, skv, d = 12, 9, 40, 64
    q = synth.normal(1, bh * sq * d, 0, 1).reshape(bh, sq, d)
    k = synth.normal(2, bh * skv * d, 0, 1).reshape(bh, skv, d)
    v = synth.normal(3, bh * skv * d, 0, 1).reshape(bh, skv, d)
    got = oc.flash_attention_fwd(cu(q), cu(k), cu(v), causal=causal).cpu().numpy()
    ref = np.zeros_like(got)
    for h in range(bh):
        for i in range(sq):
            n = i + (skv - sq) + 1 if causal else skv
            ref[h, i] = oracle.attend_one(q[h, i], k[h, :n].ravel(), v[h, :n].ravel(), n, d, flash=True, block=64)
    assert rel(got, ref) < TOL


def test_mla(oc, oracle):
    seq, dh, dc = 257, 7168 // 8, 512 // 8
    kv = synth.normal(5, seq * dh, 0, 0.02)
    down = synth.normal(6, dh * dc, 0, 0.02)
    up = synth.normal(7, dc * dh, 0, 0.02)
    lat_ref = oracle.mla_compress_kv(seq, dh, dc, kv, down)
    rec_ref = oracle.mla_decompress_kv(seq, dc, dh, lat_ref, up)
    lat = oc.mla_compress_kv(cu(kv, (seq, dh)), cu(down, (dh, dc)))
    rec = oc.mla_decompress_kv(lat, cu(up, (dc, dh)))
    assert rel(lat.cpu().numpy(), lat_ref) < TOL
    assert rel(rec.cpu().numpy(), rec_ref) < TOL
    dev = oc.Device(0)
    assert rel(dev.mla_compress_kv(seq, dh, dc, kv, down), lat_ref) < TOL
    assert rel(dev.mla_decompress_kv(seq, dc, dh, lat_ref, up), rec_ref) < TOL
    with pytest.raises(ValueError):
        dev.mla_compress_kv(seq, dh, dc, kv[:-1], down)
    dev.close()


def test_host_sgemm_known_answers(oc, oracle):
    dev = oc.Device(0)
    assert dev.sgemm(2, 2, 2, 2.0, [1, 2, 3, 4], [5, 6, 7, 8], 3.0, [1, 1, 1, 1]).tolist() == [41, 47, 89, 103]
    with pytest.raises(ValueError):
        dev.sgemm(2, 2, 2, 1.0, [1, 2], [1, 0, 0, 1], 0.0, [0] * 4)
    m, k, n = 512, 768, 2304
    a = synth.normal(0, m * k, 0, 0.02)
    b = synth.normal(1, k * n, 0, 0.02)
    assert rel(dev.sgemm(m, k, n, 1.0, a, b, 0.0, np.zeros(m * n)),
               oracle.sgemm(m, k, n, 1.0, a, b, 0.0, np.zeros(m * n))) < TOL
    dev.close()


def test_launch_kernel_by_name(oc, oracle):
    K = oc.KernelArg
    dev = oc.Device(0)
    m, k, n = 3, 4, 5
    a = synth.uniform(1, m * k)
    b = synth.uniform(2, k * n)
    pa, pb, pc = dev.alloc(a.nbytes), dev.alloc(b.nbytes), dev.alloc(m * n * 4)
    dev.memcpy_h2d(pa, a)
    dev.memcpy_h2d(pb, b)
    dev.memcpy_h2d(pc, np.zeros(m * n, np.float32))
    base = [K.ptr(pa), K.ptr(pb), K.ptr(pc), K.usize(m), K.usize(k), K.usize(n), K.f32(1.0), K.f32(0.0)]
    # the reference's own 8-argument launch (blas:222-232) leaves transpose_b
    # inside the closure; its SDPA caller needs B transposed (blas:517), so the
    # backend refuses it rather than guess, before touching C
    sentinel = np.full(m * n, 7.0, np.float32)
    dev.memcpy_h2d(pc, sentinel)
    with pytest.raises(oc.OcError) as e:
        dev.launch_kernel("sgemm_naive", base)
    assert e.value.code == oc.OC_ERR_LAUNCH_FAILED and "transpose_b" in str(e.value)
    with pytest.raises(oc.OcError):
        dev.launch_kernel("sgemm_naive", base + [K.u32(2)])
    dev.synchronize()
    c = np.zeros(m * n, np.float32)
    dev.memcpy_d2h(c, pc)
    assert np.array_equal(c, sentinel)
    for tb in (0, 1):
        dev.memcpy_h2d(pc, np.zeros(m * n, np.float32))
        dev.launch_kernel("sgemm_naive", base + [K.u32(tb)])
        dev.synchronize()
        dev.memcpy_d2h(c, pc)
        # with transpose_b, b holds B as n x k (the Q.K^T form of blas:517)
        assert rel(c, oracle.sgemm(m, k, n, 1.0, a, b, 0.0, np.zeros(m * n), transpose_b=bool(tb))) < TOL, tb
    # quantize_symmetric: bit-exact with scales from group_scales
    x = synth.normal(3, 100, 0, 1)
    t = oracle.quantize_int8(x, 25)
    px, ps, pq = dev.alloc(x.nbytes), dev.alloc(t.scales.nbytes), dev.alloc(100)
    dev.memcpy_h2d(px, x)
    dev.memcpy_h2d(ps, t.scales)
    dev.launch_kernel("quantize_symmetric", [K.ptr(px), K.ptr(ps), K.ptr(pq), K.usize(100), K.usize(25),
                                             K.f32(-127.0), K.f32(127.0)])
    dev.synchronize()
    q = np.zeros(100, np.int8)
    dev.memcpy_d2h(q, pq)
    assert np.array_equal(q, t.data)
    # unknown kernels and foreign pointers are rejected before any launch
    with pytest.raises(oc.OcError):
        dev.launch_kernel("vector_add", [K.ptr(pa)])
    with pytest.raises(ValueError):
        dev.launch_kernel("softmax", [K.ptr(12345), K.usize(1), K.usize(1)])
    dev.close()


def _ref_rows(oracle, q, k, v, causal):
    bh, sq, d = q.shape
    skv = k.shape[1]
    ref = np.zeros((bh, sq, d), np.float32)
    for h in range(bh):
        if not causal and sq == skv:
            ref[h] = oracle.flash_attention(q[h].ravel(), k[h].ravel(), v[h].ravel(), sq, d, 64).reshape(sq, d)
            continue
        for i in range(sq):
            n = i + (skv - sq) + 1 if causal else skv
            ref[h, i] = oracle.attend_one(q[h, i], k[h, :n].ravel(), v[h, :n].ravel(), n, d, flash=True, block=64)
    return ref


@pytest.mark.parametrize("bh,sq,skv,d,causal", [(4, 1024, 1024, 64, True), (3, 700, 1300, 128, False),
                                               (2, 257, 1000, 64, True), (5, 128, 128, 128, True),
                                               (2, 1, 300, 64, False), (1, 1000, 1000, 64, False)])
def test_flash_tensor_core_shapes(oc, oracle, bh, sq, skv, d, causal):
    """Head dims 64 and 128 run on the tcgen05 kernel (f16 hi / lo terms of
    Q, K, V and P, S and O in tensor memory): ragged query / key tiles,
    causal and cross lengths, 1e-5 relative Frobenius against the oracle's
    flash attention (blas:589-678)."""
    q = synth.normal(bh + sq, bh * sq * d, 0, 1).reshape(bh, sq, d)
    k = synth.normal(bh + skv + 1, bh * skv * d, 0, 1).reshape(bh, skv, d)
    v = synth.normal(bh + skv + 2, bh * skv * d, 0, 1).reshape(bh, skv, d)
    got = oc.flash_attention_fwd(cu(q), cu(k), cu(v), causal=causal).cpu().numpy()
    ref = _ref_rows(oracle, q, k, v, causal)
    assert rel(got, ref) < TOL, rel(got, ref)
    worst = max(rel(got[h, i], ref[h, i]) for h in range(bh) for i in range(0, sq, max(1, sq // 50)))
    assert worst < 10 * TOL, worst


@pytest.mark.parametrize("qs,ks,vs", [(1e-3, 1e-3, 1e-20), (30.0, 1.0, 1e6), (1e-6, 1e6, 1.0), (1.0, 1.0, 1e-30)])
def test_flash_tensor_core_value_range(oc, oracle, qs, ks, vs):
    # per-row powers of two for Q and K, per-tile for V: large and tiny
    # magnitudes keep their precision; a very peaked softmax (qs = 30)
    bh, sq, d = 2, 200, 64
    q = (synth.normal(5, bh * sq * d, 0, 1) * np.float32(qs)).reshape(bh, sq, d).astype(np.float32)
    k = (synth.normal(6, bh * sq * d, 0, 1) * np.float32(ks)).reshape(bh, sq, d).astype(np.float32)
    v = (synth.normal(7, bh * sq * d, 0, 1) * np.float32(vs)).reshape(bh, sq, d).astype(np.float32)
    got = oc.flash_attention_fwd(cu(q), cu(k), cu(v)).cpu().numpy()
    ref = _ref_rows(oracle, q, k, v, False)
    assert np.all(np.isfinite(got))
    assert rel(got, ref) < TOL, rel(got, ref)
