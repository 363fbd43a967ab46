"""Decode-shaped int8 products on the tensor cores (LLME_PATH_TCGEN05_SKINNY): activation rows
split into three int8 terms, kind::i8 MMAs, the k slices of a tile one thread-block cluster
adding exact int64 sums through distributed shared memory.

Held to the decode path's accuracy bound: max over rows of
||C - C_ref||_inf / ||C_ref row||_2 <= 1e-5 against the oracle (matmul_naive on the dequantised
weights, tests/test_quant.cpp:57-79); bit for bit against a numpy restatement of the kernel's
own arithmetic for rows without RMSNorm, at every cluster size from 1 to 8 that the shapes
below reach (integer sums: the same bits whatever the slice count); repeats bit-identical; and
the decode sweep's int8 shapes (m = 16, 64 x 4096^2) at full size.
"""
from __future__ import annotations

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


def split3(A):
    """The split pass with three terms, as the kernel computes it in fp32."""
    A = A.astype(np.float32)
    amax = np.abs(A).max(axis=1).astype(np.float32)
    q = (np.float32(127.0) / amax).astype(np.float32)
    y = (A * q[:, None]).astype(np.float32)
    t0, t1, t2 = int8_digits(y)
    s = (amax / np.float32(127.0)).astype(np.float32)
    return t0, t1, t2, s


def emulate(A, q8, scale, C0=None):
    t0, t1, t2, s = split3(A)
    W = q8.astype(np.float64)  # integer sums below 2^31 are exact in float64
    S = ((t0.astype(np.float64) @ W).astype(np.int64) * 65536 +
         (t1.astype(np.float64) @ W).astype(np.int64) * 256 +
         (t2.astype(np.float64) @ W).astype(np.int64))
    t = (S.astype(np.float32) * np.float32(1.0 / 65536)).astype(np.float32)
    out = (t * (s[:, None] * scale[None, :].astype(np.float32)).astype(np.float32)).astype(np.float32)
    if C0 is not None:
        out = (C0 + out).astype(np.float32)
    return out


def run(A, q8, scale, C0=None, accumulate=False, rms=None, kernel="automatic"):
    m, k = A.shape
    n = q8.shape[1]
    assert L.plan(m, n, k, q8=True, kernel=kernel, math=L.MATH_TENSOR,
                  rms_addr=256 if rms is not None else 0)["path_name"] == "tcgen05_skinny"
    dC = torch.from_numpy(C0.copy()).cuda() if C0 is not None else \
        torch.full((m, n), float("nan"), device="cuda")
    L.matmul(torch.from_numpy(A).cuda(), torch.from_numpy(q8).cuda(),
             scale=torch.from_numpy(scale).cuda(), C=dC, kernel=kernel, accumulate=accumulate,
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


# (m, k, n): every row tile (16 / 32 / 64, two 64-row tiles), ragged m, k not a multiple of 16
# or 128, n a multiple of 16 but not of 128, one k slice and many.
SHAPES = [(9, 4096, 4096), (16, 4096, 4096), (17, 1000, 272), (32, 512, 1040), (33, 4100, 48),
          (64, 4096, 4096), (65, 300, 4096), (100, 11008, 4096), (127, 72, 256), (12, 11008, 11008)]


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_skinny_matches_oracle_and_emulation(m, k, n):
    rng = np.random.default_rng(m * 7 + k + 3 * n)
    A = uni(rng, m, k)
    q, s = weights(rng, k, n)
    got = run(A, q, s)
    err = row_rel_err(got, oracle.matmul_naive_q8(A, q, s))
    print(f"skinny m={m} k={k} n={n}: row-rel {err:.2e}")
    assert err <= 1e-5
    np.testing.assert_array_equal(got, emulate(A, q, s))


@pytest.mark.parametrize("outlier", [100.0, 1000.0])
def test_skinny_outlier_activations(outlier):
    # A few activation channels far above the rest, as in real models. The split scales each
    # row by its maximum, so the ordinary values keep fewer of their bits; three terms still
    # hold the decode bound (a float64 emulation of the split gives about 1e-7 here, where two
    # terms give 2.5e-5), and the result is the kernel's arithmetic bit for bit.
    rng = np.random.default_rng(int(outlier))
    m, k, n = 16, 4096, 4096
    A = uni(rng, m, k)
    A[:, rng.integers(0, k, 8)] *= np.float32(outlier)
    q, s = weights(rng, k, n)
    got = run(A, q, s)
    assert row_rel_err(got, oracle.matmul_naive_q8(A, q, s)) <= 1e-5
    np.testing.assert_array_equal(got, emulate(A, q, s))


def test_skinny_half_way_digits():
    # Rows whose scale is exactly 1 (max |x| = 127) and whose other values lie half way between
    # integers: the first digit rounds to even, the remainder is exactly 1/2, and the second
    # digit is carried (+128 -> first digit + 1, second digit -128). The three digits then
    # hold every value exactly, so the result is the oracle's within fp32 rounding.
    rng = np.random.default_rng(77)
    m, k, n = 12, 4096, 2048
    A = (rng.integers(-126, 126, (m, k)) + 0.5).astype(np.float32)
    A[:, 0] = 127.0
    q, s = weights(rng, k, n)
    got = run(A, q, s)
    np.testing.assert_array_equal(got, emulate(A, q, s))
    assert row_rel_err(got, oracle.matmul_naive_q8(A, q, s)) <= 1e-6


@pytest.mark.parametrize("m", [2, 4, 8])
def test_skinny_small_m_through_tiled_split(m):
    rng = np.random.default_rng(40 + m)
    A = uni(rng, m, 2048)
    q, s = weights(rng, 2048, 1024)
    got = run(A, q, s, kernel="tiled_split")
    assert row_rel_err(got, oracle.matmul_naive_q8(A, q, s)) <= 1e-5
    np.testing.assert_array_equal(got, emulate(A, q, s))


def test_skinny_fusion():
    # MatmulFusion{accumulate, rms_weight} (tests/test_cuda.cpp:190-212, int8 weights).
    rng = np.random.default_rng(8)
    m, k, n = 24, 3000, 1536
    A, C0, w = uni(rng, m, k), uni(rng, m, n), uni(rng, k)
    q, s = weights(rng, k, n)
    got = run(A, q, s, C0=C0, accumulate=True)
    np.testing.assert_array_equal(got, emulate(A, q, s, C0=C0))
    got = run(A, q, s, C0=C0, accumulate=True, rms=w)
    want = C0 + oracle.matmul_naive_q8(oracle.rmsnorm(A, w), q, s)
    assert row_rel_err(got, want) <= 1e-5


def test_skinny_repeats_bit_identical_and_scratch_settles():
    rng = np.random.default_rng(9)
    A = uni(rng, 48, 4096)
    q, s = weights(rng, 4096, 4096)
    first = run(A, q, s)
    gen = L.scratch_generation()
    for _ in range(5):
        np.testing.assert_array_equal(run(A, q, s), first)
    assert L.scratch_generation() == gen


def test_config1_int8_decode_sweep_full_size():
    # The decode sweep, int8 half: m in {16, 64} (the rows this path takes), 4096 x 4096.
    rng = np.random.default_rng(1)
    q, s = weights(rng, 4096, 4096)
    for m in (16, 64):
        A = uni(rng, m, 4096)
        assert row_rel_err(run(A, q, s), oracle.matmul_naive_q8(A, q, s)) <= 1e-5
