"""GPU parity of oc_sgemm (f16-term and 3xTF32 tcgen05 GEMMs, the small-m GEMV) against
the oracle's restatement of the reference's naive sgemm (blas:148-295).

Tolerance: 1e-5 relative Frobenius error (the bound the north star sets for
f32 outputs); the reference's integer-valued known answers are exact."""
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


def rel_fro(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def test_reference_known_answers(oc):
    # blas:1090-1133
    A = torch.tensor([[1.0, 2.0], [3.0, 4.0]], device="cuda")
    I = torch.eye(2, device="cuda")
    assert oc.sgemm(A, I).cpu().tolist() == [[1.0, 2.0], [3.0, 4.0]]
    B = torch.tensor([[5.0, 6.0], [7.0, 8.0]], device="cuda")
    C = torch.ones(2, 2, device="cuda")
    assert oc.sgemm(A, B, alpha=2.0, beta=3.0, C=C).cpu().tolist() == [[41.0, 47.0], [89.0, 103.0]]
    B3 = torch.arange(1, 10, dtype=torch.float32, device="cuda").view(3, 3)
    assert oc.sgemm(torch.eye(3, device="cuda"), B3).cpu().tolist() == B3.cpu().tolist()
    with pytest.raises(ValueError):
        oc.sgemm(torch.ones(2, 3, device="cuda"), torch.ones(2, 2, device="cuda"))


SHAPES = [
    (512, 768, 2304),  # GPT-2 c_attn (config 1)
    (1, 768, 2304), (4, 768, 768), (8, 3072, 768), (9, 768, 3072),  # GEMV range and its edge
    (32, 768, 50257),  # lm_head, ragged n
    (130, 100, 70), (257, 64, 40), (1000, 33, 129),  # ragged k (TMA zero fill), n < 128
    (16384 // 8, 7168, 512),  # MLA compress slice
]


@pytest.mark.parametrize("trans_b", [False, True])
@pytest.mark.parametrize("m,k,n", SHAPES)
def test_sgemm_matches_oracle(oc, oracle, m, k, n, trans_b):
    rng_seed = m * 7 + k * 3 + n
    A = synth.normal(rng_seed, m * k, 0.0, 0.02).reshape(m, k)
    B = synth.normal(rng_seed + 1, k * n, 0.0, 0.02).reshape((n, k) if trans_b else (k, n))
    bias = synth.normal(rng_seed + 2, n, 0.0, 0.02)
    ref = oracle.sgemm(m, k, n, 1.0, A, B, 0.0, np.zeros(m * n), transpose_b=trans_b) + np.tile(bias, m)
    got = oc.sgemm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), transpose_b=trans_b,
                   bias=torch.from_numpy(bias).cuda())
    torch.cuda.synchronize()
    err = rel_fro(got.cpu().numpy(), ref)
    assert err < TOL, err


@pytest.mark.parametrize("m,k,n", [(300, 256, 200), (3, 40, 50)])
def test_sgemm_alpha_beta(oc, oracle, m, k, n):
    A = synth.uniform(1, m * k).reshape(m, k)
    B = synth.uniform(2, k * n).reshape(k, n)
    C0 = synth.uniform(3, m * n).reshape(m, n)
    ref = oracle.sgemm(m, k, n, 0.5, A, B, -1.5, C0)
    got = oc.sgemm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), alpha=0.5, beta=-1.5,
                   C=torch.from_numpy(C0.copy()).cuda())
    assert rel_fro(got.cpu().numpy(), ref) < TOL


def test_sgemm_prepared_b_matches(oc, oracle):
    import ctypes as C
    m, k, n = 300, 3072, 768
    A = synth.normal(11, m * k, 0, 0.02).reshape(m, k)
    B = synth.normal(12, k * n, 0, 0.02).reshape(k, n)
    ref = oracle.sgemm(m, k, n, 1.0, A, B, 0.0, np.zeros(m * n))
    nbytes = C.c_size_t(0)
    oc.check(oc.lib().oc_sgemm_prepared_b_size(k, n, C.byref(nbytes)))
    prep = torch.empty(nbytes.value // 4, dtype=torch.float32, device="cuda")
    Bd = torch.from_numpy(B).cuda()
    s = torch.cuda.current_stream().cuda_stream
    oc.check(oc.lib().oc_sgemm_prepare_b(k, n, Bd.data_ptr(), n, 0, prep.data_ptr(), s))
    Ad = torch.from_numpy(A).cuda()
    out = torch.zeros(m, n, device="cuda")
    oc.check(oc.lib().oc_sgemm_prepared(m, n, k, 1.0, Ad.data_ptr(), k, prep.data_ptr(), 0.0, out.data_ptr(), n,
                                        None, s))
    assert rel_fro(out.cpu().numpy(), ref) < TOL


def test_sgemm_k_zero_scales_c(oc):
    C0 = torch.full((3, 5), 2.0, device="cuda")
    out = oc.sgemm(torch.empty(3, 0, device="cuda"), torch.empty(0, 5, device="cuda"), beta=0.5, C=C0)
    assert torch.all(out == 1.0)


@pytest.mark.parametrize("trans_b", [False, True])
@pytest.mark.parametrize("m,k,n", [(200, 640, 300), (64, 768, 20000), (40, 2048, 2304)])
def test_sgemm_value_ranges(oc, oracle, m, k, n, trans_b):
    """beta = 0 with k % 64 == 0 and m > 16 runs the f16-term GEMM: every row
    of A and column of op(B) is scaled by its own power of two before the
    split, so rows and columns far apart in magnitude (1e-25 .. 1e6), zero
    rows and columns, alpha != 1 and column chunks past the first (n = 20000)
    keep the f32 bound."""
    A = synth.uniform(21, m * k).reshape(m, k) * (10.0 ** np.linspace(-25, 6, m))[:, None]
    Bkn = synth.uniform(22, k * n).reshape(k, n) * (10.0 ** np.linspace(-20, 5, n))[None, :]
    A[3] = 0.0
    Bkn[:, 7] = 0.0
    A, Bkn = A.astype(np.float32), Bkn.astype(np.float32)
    B = np.ascontiguousarray(Bkn.T) if trans_b else Bkn
    alpha = 0.37
    ref = oracle.sgemm(m, k, n, alpha, A, B, 0.0, np.zeros(m * n), transpose_b=trans_b).reshape(m, n)
    got = oc.sgemm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), alpha=alpha, transpose_b=trans_b)
    got = got.cpu().numpy()
    assert rel_fro(got, ref) < TOL
    # per row as well: a row 1e-25 times the largest keeps its own relative error
    for r in (0, 1, m // 2, m - 1):
        assert rel_fro(got[r], ref[r]) < TOL, r
    assert np.all(got[3] == 0.0) and np.all(got[:, 7] == 0.0)
