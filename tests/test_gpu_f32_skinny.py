"""Decode-shaped fp32-weight products on the tensor cores (LLME_PATH_TCGEN05_F32_SKINNY): three
TF32 terms (W_hi A_hi + W_hi A_lo + W_lo A_hi), k slices of a column tile added through
distributed shared memory of one thread-block cluster.

Held to the decode path's accuracy bound: max over rows of
||C - C_ref||_inf / ||C_ref row||_2 <= 1e-5 against the oracle (matmul_naive, the reference's
src/matmul.cpp restated and pinned); repeats bit-identical (the cluster adds its partials in
rank order); MatmulFusion's accumulate and RMSNorm (tests/test_cuda.cpp:190-212); and the
decode sweep's fp32 shapes (m = 16, 64 x 4096^2) at full size.
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


def run(A, W, C0=None, accumulate=False, rms=None, kernel="automatic"):
    m, k = A.shape
    n = W.shape[1]
    assert L.plan(m, n, k, q8=False, kernel=kernel, math=L.MATH_TENSOR,
                  rms_addr=256 if rms is not None else 0)["path_name"] == "tcgen05_f32_skinny"
    dC = torch.from_numpy(C0.copy()).cuda() if C0 is not None else \
        torch.full((m, n), float("nan"), device="cuda")
    L.matmul(torch.from_numpy(A).cuda(), torch.from_numpy(W).cuda(), C=dC, kernel=kernel,
             accumulate=accumulate,
             rms_weight=torch.from_numpy(rms).cuda() if rms is not None else None,
             weights_static=True)
    torch.cuda.synchronize()
    return dC.cpu().numpy()


@pytest.fixture(scope="module", autouse=True)
def _tensor_math():
    L.load()
    prev = L.set_math(L.MATH_TENSOR)
    yield
    L.set_math(prev)
    L.device_status()


# (m, k, n): every row tile (16 / 32 / 64, two 64-row tiles), ragged m, k not a multiple of 32,
# n a multiple of 4 but not of 128, one k slice and the full cluster of 8.
SHAPES = [(9, 4096, 4096), (16, 4096, 4096), (17, 1000, 276), (32, 512, 1040), (33, 4100, 52),
          (64, 4096, 4096), (65, 300, 4096), (100, 11008, 4096), (127, 72, 260), (12, 11008, 11008),
          (20, 4, 128)]


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_f32_skinny_matches_oracle(m, k, n):
    rng = np.random.default_rng(m * 11 + k + 5 * n)
    A, W = uni(rng, m, k), weights(rng, k, n)
    got = run(A, W)
    err = row_rel_err(got, oracle.matmul_naive(A, W))
    print(f"f32 skinny m={m} k={k} n={n}: row-rel {err:.2e}")
    assert err <= 1e-5


@pytest.mark.parametrize("m", [1, 4, 8])
def test_f32_skinny_small_m_through_tiled_split(m):
    rng = np.random.default_rng(50 + m)
    A, W = uni(rng, m, 2048), weights(rng, 2048, 1024)
    assert row_rel_err(run(A, W, kernel="tiled_split"), oracle.matmul_naive(A, W)) <= 1e-5


def test_f32_skinny_keeps_the_low_terms():
    # Operands whose low 13 mantissa bits matter: TF32 alone misses the bound by far.
    rng = np.random.default_rng(12)
    m, k, n = 16, 2048, 512
    A, W = uni(rng, m, k), weights(rng, k, n)
    trunc = lambda x: (x.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)
    tf32_only = trunc(A).astype(np.float64) @ trunc(W).astype(np.float64)
    exact = A.astype(np.float64) @ W.astype(np.float64)
    assert row_rel_err(tf32_only, exact) > 5e-5      # about 1.3e-4 for these operands
    assert row_rel_err(run(A, W), exact) <= 1e-6     # three terms: about 1e-7


def test_f32_skinny_fusion():
    # MatmulFusion{accumulate, rms_weight} (tests/test_cuda.cpp:190-212).
    rng = np.random.default_rng(8)
    m, k, n = 24, 3000, 1536
    A, C0, w, W = uni(rng, m, k), uni(rng, m, n), uni(rng, k), weights(rng, k, n)
    got = run(A, W, C0=C0, accumulate=True)
    assert row_rel_err(got, C0 + oracle.matmul_naive(A, W)) <= 1e-5
    got = run(A, W, C0=C0, accumulate=True, rms=w)
    assert row_rel_err(got, C0 + oracle.matmul_naive(oracle.rmsnorm(A, w), W)) <= 1e-5
    got = run(A, W, rms=w)
    assert row_rel_err(got, oracle.matmul_naive(oracle.rmsnorm(A, w), W)) <= 1e-5


def test_f32_skinny_accumulate_through_a_cluster():
    # k split over 8 CTAs: C += A W read and written once, by the CTA that owns the row.
    rng = np.random.default_rng(14)
    A, W, C0 = uni(rng, 16, 4096), weights(rng, 4096, 1024), uni(rng, 16, 1024)
    assert L.plan(16, 1024, 4096, q8=False)["slices"] == 8
    got = run(A, W, C0=C0, accumulate=True)
    assert row_rel_err(got, C0 + oracle.matmul_naive(A, W)) <= 1e-5


def test_f32_skinny_repeats_bit_identical():
    rng = np.random.default_rng(9)
    A, W = uni(rng, 48, 4096), weights(rng, 4096, 4096)
    first = run(A, W)
    gen = L.scratch_generation()
    for _ in range(5):
        np.testing.assert_array_equal(run(A, W), first)
    assert L.scratch_generation() == gen


def test_config1_fp32_decode_sweep_full_size():
    # The decode sweep, fp32 half: m in {16, 64} (the rows this path takes), 4096 x 4096.
    rng = np.random.default_rng(1)
    W = weights(rng, 4096, 4096)
    for m in (16, 64):
        A = uni(rng, m, 4096)
        assert row_rel_err(run(A, W), oracle.matmul_naive(A, W)) <= 1e-5
