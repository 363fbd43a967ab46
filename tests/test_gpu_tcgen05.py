"""The tcgen05/TMEM tensor-core GEMM (m >= 128, fp32 weights, TF32 multiplies).

Parity bound of the tensor-core path: max over rows of ||C - C_ref||_inf / ||C_ref row||_2 <=
5e-3 against matmul_naive on identical inputs. Tighter checks pin the arithmetic: the result
must sit within the fp32-accumulation noise of a float64 product of TF32-converted operands,
and repeats must be bit-identical.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import llme_b200 as L
from conftest import row_rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def uni(rng, *shape):
    return rng.uniform(-1, 1, shape).astype(np.float32)


def tf32_trunc(x):
    return (x.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)


def tf32_round(x):
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0xFFF + ((u >> 13) & 1)) & 0xFFFFE000).astype(np.uint32)
    return r.view(np.float32)


def run(A, B, C0=None, accumulate=False, rms=None):
    m, k = A.shape
    n = B.shape[1]
    assert L.plan(m, n, k, q8=False, kernel="tiled", rms_addr=256 if rms is not None else 0)[
        "path_name"] == "tcgen05"
    dC = torch.from_numpy(C0.copy()).cuda() if C0 is not None else torch.empty(m, n, device="cuda")
    L.matmul(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), C=dC, kernel="tiled",
             accumulate=accumulate,
             rms_weight=torch.from_numpy(rms).cuda() if rms is not None else None)
    torch.cuda.synchronize()
    return dC.cpu().numpy()


@pytest.fixture(scope="module", autouse=True)
def _tensor_math():
    L.load()
    prev = L.set_math(L.MATH_TENSOR)
    yield
    L.set_math(prev)
    L.device_status()


# B read as stored (MN-major) below 6144 rows; from 6144 rows through a B^T pass (K-major).
@pytest.mark.parametrize("m,k,n", [(128, 32, 256), (128, 256, 256), (256, 512, 512),
                                   (130, 72, 1028), (300, 1000, 260), (128, 4096, 4096),
                                   (6200, 264, 516), (6144, 96, 260), (4096, 96, 260)])
def test_tf32_gemm_matches_oracle(m, k, n):
    assert (L.plan(m, n, k, q8=False)["operand_bytes"] > 0) == (m >= 6144)
    rng = np.random.default_rng(m + 3 * k + 7 * n)
    A, B = uni(rng, m, k), uni(rng, k, n)
    got = run(A, B)
    want = oracle.matmul_naive(A, B)
    err = row_rel_err(got, want)
    assert err <= 5e-3, err
    # Against float64 products of TF32 operands the only error left is fp32 accumulation.
    ref_t = tf32_trunc(A).astype(np.float64) @ tf32_trunc(B).astype(np.float64)
    ref_r = tf32_round(A).astype(np.float64) @ tf32_round(B).astype(np.float64)
    e_t = np.abs(got - ref_t).max()
    e_r = np.abs(got - ref_r).max()
    print(f"tf32 m={m} k={k} n={n}: row-rel {err:.2e}; vs trunc {e_t:.2e}, vs round {e_r:.2e}")
    assert min(e_t, e_r) <= 1e-5 * k


def test_tf32_gemm_accumulate_and_rmsnorm():
    rng = np.random.default_rng(5)
    m, k, n = 200, 512, 768
    A, B, C0, w = uni(rng, m, k), uni(rng, k, n), uni(rng, m, n), uni(rng, k)
    got = run(A, B, C0=C0, accumulate=True, rms=w)
    want = C0 + oracle.matmul_naive(oracle.rmsnorm(A, w), B)
    assert row_rel_err(got, want) <= 5e-3


def test_tf32_gemm_repeats_bit_identical():
    rng = np.random.default_rng(6)
    A, B = uni(rng, 384, 1024), uni(rng, 1024, 1024)
    np.testing.assert_array_equal(run(A, B), run(A, B))


def test_config2_square_1024():
    # The square SGEMM at N = 1024 (A, B ~ U(-1, 1)), checked against the oracle.
    rng = np.random.default_rng(2)
    A, B = uni(rng, 1024, 1024), uni(rng, 1024, 1024)
    assert row_rel_err(run(A, B), oracle.matmul_naive(A, B)) <= 5e-3


@pytest.mark.parametrize("n", [2048, 4096, 8192])
def test_config2_square_sampled_rows(n):
    """configs[2] at the sizes its TF32 target is quoted on (A, B ~ U(-1, 1), seed 2): the
    whole N^3 product runs on the GPU; 64 rows of C (the first, the last, rows of the last
    128-row tile and random ones) are compared with matmul_naive of those rows of A against
    all of B, within the 5e-3 row bound, and with the float64 product of TF32 operands within
    the fp32 accumulation noise. (The naive oracle would need minutes for the whole 8192^3.)"""
    rng = np.random.default_rng(2)
    A = rng.random((n, n), dtype=np.float32) * 2 - 1
    B = rng.random((n, n), dtype=np.float32) * 2 - 1
    assert L.plan(n, n, n, q8=False)["path_name"] == "tcgen05"
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    dC = torch.full((n, n), float("nan"), device="cuda")
    L.matmul(dA, dB, C=dC)
    torch.cuda.synchronize()
    rows = np.unique(np.concatenate([[0, n - 1, n - 128, n - 65],
                                     rng.choice(n, 60, replace=False)]))
    got = dC[torch.from_numpy(rows).cuda()].cpu().numpy()
    assert np.isfinite(got).all()
    want = oracle.matmul_naive(A[rows], B)
    err = row_rel_err(got, want)
    ref_t = tf32_trunc(A[rows]).astype(np.float64) @ tf32_trunc(B).astype(np.float64)
    e_t = np.abs(got - ref_t).max()
    print(f"square {n}: row-rel {err:.2e} over {rows.size} rows; vs tf32 operands {e_t:.2e}")
    assert err <= 5e-3, err
    assert e_t <= 1e-5 * n
