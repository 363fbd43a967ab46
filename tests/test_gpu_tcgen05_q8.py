"""The int8-weight tcgen05 GEMM (m >= 128, LLME_MATH_TENSOR): activation rows split into two
int8 terms, kind::i8 MMAs with exact s32 sums in TMEM, fp32 epilogue.

Three checks per shape:
* against the oracle (matmul_naive on the dequantised weights, the reference's int8 parity
  reference, tests/test_quant.cpp:57-79) with the tensor-core path's bound: max over rows
  of ||C - C_ref||_inf / ||C_ref row||_2 <= 5e-3 -- and, since the split keeps 16 bits of each
  activation, a much tighter 1e-4 that pins the arithmetic as well;
* bit for bit against a numpy restatement of the kernel's own arithmetic (the split of each
  row, exact integer sums, the rounded epilogue), for rows without RMSNorm;
* repeats bit-identical.
Each test runs with single CTAs (the default) and with CTA pairs (cta_group::2), which must
give the same bits.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

import oracle
import llme_b200 as L
from conftest import int8_digits, row_rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def uni(rng, *shape):
    return rng.uniform(-1, 1, shape).astype(np.float32)


def weights(rng, k, n):
    return oracle.quantize_q8((rng.standard_normal((k, n)) * 0.02).astype(np.float32))


def split_rows(A):
    """The split pass for rows without RMSNorm, as the kernel computes it in fp32:
    s = max|x| / 127, y = x * (127 / max|x|), hi and lo the first two int8 digits of y."""
    A = A.astype(np.float32)
    amax = np.abs(A).max(axis=1).astype(np.float32)
    assert (amax > 1e-30).all()
    q = (np.float32(127.0) / amax).astype(np.float32)
    y = (A * q[:, None]).astype(np.float32)
    hi, lo, _ = int8_digits(y)
    s = (amax / np.float32(127.0)).astype(np.float32)
    return hi.astype(np.int64), lo.astype(np.int64), s


def emulate(A, q8, scale, C0=None):
    hi, lo, s = split_rows(A)
    # Integer sums below 2^31 are exact in float64 whatever the summation order, so BLAS
    # gives the same integers as the tensor cores.
    W = q8.astype(np.float64)
    Hi, Lo = hi.astype(np.float64) @ W, lo.astype(np.float64) @ W
    assert np.abs(Hi).max() < 2**31 and np.abs(Lo).max() < 2**31
    Hi, Lo = Hi.astype(np.int64), Lo.astype(np.int64)
    # fmaf(float(Lo), 2^-8, float(Hi)): one rounding of the exact sum (exact in float64 here).
    t = (Hi.astype(np.float32).astype(np.float64) +
         Lo.astype(np.float32).astype(np.float64) / 256.0).astype(np.float32)
    rsc = (s[:, None] * scale[None, :].astype(np.float32)).astype(np.float32)
    out = (t * rsc).astype(np.float32)
    if C0 is not None:
        out = (C0.astype(np.float32) + out).astype(np.float32)
    return out


def run(A, q8, scale, C0=None, accumulate=False, rms=None, kernel="tiled"):
    m, k = A.shape
    n = q8.shape[1]
    assert L.plan(m, n, k, q8=True, kernel=kernel, math=L.MATH_TENSOR,
                  rms_addr=256 if rms is not None else 0)["path_name"] == "tcgen05_q8"
    dC = torch.from_numpy(C0.copy()).cuda() if C0 is not None else \
        torch.full((m, n), float("nan"), device="cuda")
    L.matmul(torch.from_numpy(A).cuda(), torch.from_numpy(q8).cuda(),
             scale=torch.from_numpy(scale).cuda(), C=dC, kernel=kernel, accumulate=accumulate,
             rms_weight=torch.from_numpy(rms).cuda() if rms is not None else None)
    torch.cuda.synchronize()
    return dC.cpu().numpy()


@pytest.fixture(scope="module", autouse=True, params=["single", "pairs"])
def _tensor_math(request):
    """Every test twice: single CTAs (default) and CTA pairs (LLME_B200_CTA_PAIRS=1)."""
    L.load()
    prev = L.set_math(L.MATH_TENSOR)
    old = os.environ.get("LLME_B200_CTA_PAIRS")
    os.environ["LLME_B200_CTA_PAIRS"] = "1" if request.param == "pairs" else "0"
    yield
    if old is None:
        del os.environ["LLME_B200_CTA_PAIRS"]
    else:
        os.environ["LLME_B200_CTA_PAIRS"] = old
    L.set_math(prev)
    L.device_status()


# (m, k, n): tile edges, ragged m, k not a multiple of 16 or 128, n a multiple of 16 but not
# of 128, both column tiles (128 and 256 wide), and the 7B prefill shapes
# (m = 512 through the 4096 x 4096, 4096 x 11008 and 11008 x 4096 weights).
SHAPES = [(128, 128, 256), (128, 32, 128), (256, 512, 512), (130, 72, 1040), (300, 1000, 272),
          (129, 4100, 48), (512, 4096, 4096), (512, 4096, 11008), (512, 11008, 4096),
          (513, 100, 11008), (1024, 256, 8192)]


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_q8_gemm_matches_oracle_and_emulation(m, k, n):
    rng = np.random.default_rng(m + 3 * k + 7 * n)
    A = uni(rng, m, k)
    q, s = weights(rng, k, n)
    got = run(A, q, s)
    want = oracle.matmul_naive_q8(A, q, s)
    err = row_rel_err(got, want)
    print(f"q8 tcgen05 m={m} k={k} n={n}: row-rel {err:.2e}")
    assert err <= 5e-3
    assert err <= 1e-4
    np.testing.assert_array_equal(got, emulate(A, q, s))


def test_q8_gemm_accumulate_bit_exact():
    rng = np.random.default_rng(11)
    m, k, n = 200, 640, 528
    A, C0 = uni(rng, m, k), uni(rng, m, n)
    q, s = weights(rng, k, n)
    got = run(A, q, s, C0=C0, accumulate=True)
    np.testing.assert_array_equal(got, emulate(A, q, s, C0=C0))
    assert row_rel_err(got, C0 + oracle.matmul_naive_q8(A, q, s)) <= 1e-4


def test_q8_gemm_rmsnorm_fusion():
    # MatmulFusion{accumulate, rms_weight} (tests/test_cuda.cpp:190-212 with int8 weights).
    rng = np.random.default_rng(12)
    m, k, n = 260, 1024, 768
    A, C0, w = uni(rng, m, k), uni(rng, m, n), uni(rng, k)
    q, s = weights(rng, k, n)
    got = run(A, q, s, C0=C0, accumulate=True, rms=w)
    want = C0 + oracle.matmul_naive_q8(oracle.rmsnorm(A, w), q, s)
    assert row_rel_err(got, want) <= 1e-4


def test_q8_gemm_rows_of_zeros_and_scaled_rows():
    # A zero row (row scale 0), a row of tiny values and one of huge values: the split is
    # relative to each row's own largest magnitude.
    rng = np.random.default_rng(13)
    m, k, n = 128, 256, 256
    A = uni(rng, m, k)
    A[3] = 0.0
    A[5] *= 1e-20
    A[7] *= 1e20
    q, s = weights(rng, k, n)
    got = run(A, q, s)
    want = oracle.matmul_naive_q8(A.astype(np.float64).astype(np.float32), q, s)
    assert (got[3] == 0).all()
    for r in (5, 7, 9):
        rel = np.abs(got[r] - want[r]).max() / np.linalg.norm(want[r])
        assert rel <= 1e-4, (r, rel)


def test_q8_gemm_automatic_kernel_and_repeat():
    rng = np.random.default_rng(14)
    A = uni(rng, 384, 2048)
    q, s = weights(rng, 2048, 1536)
    a = run(A, q, s, kernel="automatic")
    b = run(A, q, s, kernel="automatic")
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(a, emulate(A, q, s))
