"""fp32-weight products with 9..16 rows in fp32 arithmetic (LLME_MATH_FP32) on the TMA GEMV
(LLME_PATH_GEMV_TMA at 16 rows): exact fp32 FMA arithmetic with each output's accumulator
paired over even and odd k, the rows past m read as the TMA's zero fill and never stored, the k
slices of a column strip reduced in one thread-block cluster; RMSNorm by the library's row pass
before the GEMV.

The reference runs these shapes on sgemm_tiled<64,4,Split,float> (tiled_split,
src/cuda_matmul.cu:71-125, 352-363). Held to the decode path's accuracy bound, max over rows of
||C - C_ref||_inf / ||C_ref row||_2 <= 1e-5, against the oracle (matmul_naive, the reference's
src/matmul.cpp restated and pinned); MatmulFusion's accumulate and
RMSNorm (tests/test_cuda.cpp:190-212); bit-identical repeats; no write past row m; and the
decode sweep's fp32 m = 16 x 4096^2 at full size.
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


def weights(rng, k, n):
    return (rng.standard_normal((k, n)) * 0.02).astype(np.float32)


def run(A, W, C0=None, accumulate=False, rms=None, kernel="automatic", math=L.MATH_FP32,
        spare_rows=0):
    """C through the library; `spare_rows` NaN rows after C's m rows must stay NaN."""
    m, k = A.shape
    n = W.shape[1]
    p = L.plan(m, n, k, q8=False, kernel=kernel, math=math,
               rms_addr=256 if rms is not None else 0)
    assert p["path_name"] == "gemv_tma" and p["tile_m"] == 16, p
    full = torch.full((m + spare_rows, n), float("nan"), device="cuda")
    if C0 is not None:
        full[:m] = torch.from_numpy(C0).cuda()
    prev = L.set_math(math)
    try:
        L.matmul(torch.from_numpy(A).cuda(), torch.from_numpy(W).cuda(), C=full[:m],
                 kernel=kernel, accumulate=accumulate,
                 rms_weight=torch.from_numpy(rms).cuda() if rms is not None else None,
                 weights_static=True)
        torch.cuda.synchronize()
    finally:
        L.set_math(prev)
    out = full.cpu().numpy()
    assert np.isnan(out[m:]).all(), "a row past m was written"
    return out[:m]


@pytest.fixture(scope="module", autouse=True)
def _loaded():
    L.load()
    yield
    L.device_status()


# (m, k, n): 9..16 rows; the k slices as a cluster of 2 and as one CTA; k not a multiple of
# the 128-row box; n a multiple of 4 but not of the 32-column strip; tiny k.
SHAPES = [(9, 4096, 4096), (12, 4096, 4096), (16, 4096, 4096), (13, 11008, 4096),
          (16, 4096, 11008), (10, 1000, 276), (15, 300, 4100), (11, 4, 128), (16, 128, 32000)]


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_rows16_matches_oracle(m, k, n):
    rng = np.random.default_rng(m * 13 + k + 7 * n)
    A, W = uni(rng, m, k), weights(rng, k, n)
    got = run(A, W, spare_rows=3)
    err = row_rel_err(got, oracle.matmul_naive(A, W))
    print(f"gemv rows16 m={m} k={k} n={n}: row-rel {err:.2e}")
    assert err <= 1e-5
    # The reference's own bound for fp32 products (tests/test_cuda.cpp:38-47): 1e-5 * k.
    assert np.abs(got - oracle.matmul_naive(A, W)).max() <= 1e-5 * k


@pytest.mark.parametrize("m,k,n", [(12, 3000, 1536), (16, 4096, 4096), (9, 256, 260)])
def test_rows16_fusion(m, k, n):
    # MatmulFusion{accumulate, rms_weight} (tests/test_cuda.cpp:190-212): the RMSNorm row
    # pass, then the GEMV over one slice or a cluster of them.
    rng = np.random.default_rng(8 + m + k)
    A, C0, w, W = uni(rng, m, k), uni(rng, m, n), uni(rng, k), weights(rng, k, n)
    got = run(A, W, C0=C0, accumulate=True, spare_rows=2)
    assert row_rel_err(got, C0 + oracle.matmul_naive(A, W)) <= 1e-5
    got = run(A, W, C0=C0, accumulate=True, rms=w, spare_rows=2)
    assert row_rel_err(got, C0 + oracle.matmul_naive(oracle.rmsnorm(A, w), W)) <= 1e-5
    got = run(A, W, rms=w, spare_rows=2)
    assert row_rel_err(got, oracle.matmul_naive(oracle.rmsnorm(A, w), W)) <= 1e-5


def test_rows16_explicit_tiled_and_tiled_split():
    rng = np.random.default_rng(21)
    A, W = uni(rng, 14, 2048), weights(rng, 2048, 1024)
    want = oracle.matmul_naive(A, W)
    for kernel in ("tiled", "tiled_split"):
        assert row_rel_err(run(A, W, kernel=kernel), want) <= 1e-5


def test_rows16_repeats_bit_identical():
    rng = np.random.default_rng(9)
    A, W = uni(rng, 16, 4096), weights(rng, 4096, 4096)
    first = run(A, W)
    gen = L.scratch_generation()
    for _ in range(5):
        np.testing.assert_array_equal(run(A, W), first)
    assert L.scratch_generation() == gen


def test_config1_fp32_m16_decode_sweep_full_size():
    # The decode sweep's fp32 m = 16 case, 4096 x 4096, in fp32 arithmetic.
    rng = np.random.default_rng(1)
    W = weights(rng, 4096, 4096)
    A = uni(rng, 16, 4096)
    assert row_rel_err(run(A, W), oracle.matmul_naive(A, W)) <= 1e-5
