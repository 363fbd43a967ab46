"""The CPU oracle, pinned against the reference (no GPU).

Two anchors: the known answers and invariants the reference's own tests hold
(tests/test_matmul.cpp, tests/test_quant.cpp), and bit-exact agreement with golden vectors
the reference's own sources produced (tests/golden/make_golden.py).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import close_to


def bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype == np.float32 else np.uint8)


def test_known_values():
    # tests/test_matmul.cpp:40-52
    A = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    B = np.array([[7, 8], [9, 10], [11, 12]], np.float32)
    C = oracle.matmul_naive(A, B)
    assert C.tolist() == [[58.0, 64.0], [139.0, 154.0]]
    assert oracle.matmul_parallel(A, B, threads=2).tolist() == [[58.0, 64.0], [139.0, 154.0]]


def test_known_values_golden(golden):
    np.testing.assert_array_equal(oracle.matmul_naive(golden["known_A"], golden["known_B"]),
                                  golden["known_C"])


@pytest.mark.parametrize("i", range(3))
def test_quantize_matches_reference_bits(golden, i):
    q, s = oracle.quantize_q8(golden[f"quant{i}_B"])
    np.testing.assert_array_equal(q, golden[f"quant{i}_q"])
    np.testing.assert_array_equal(bits(s), bits(golden[f"quant{i}_scale"]))
    np.testing.assert_array_equal(bits(oracle.dequantize(q, s)), bits(golden[f"quant{i}_deq"]))


def test_quantize_invariants():
    # tests/test_quant.cpp:33-51: half a step of error, max -> +-127, zero column -> scale 0.
    rng = np.random.default_rng(3)
    B = rng.uniform(-2, 2, (37, 21)).astype(np.float32)
    B[5, :] *= np.arange(1, 22, dtype=np.float32)
    B[:, 4] = 0
    q, s = oracle.quantize_q8(B)
    d = oracle.dequantize(q, s)
    assert s[4] == 0.0
    for c in range(B.shape[1]):
        assert np.all(np.abs(d[:, c] - B[:, c]) <= s[c] * 0.5 * (1 + 1e-5))
        assert np.abs(q[:, c].astype(int)).max() == (0 if c == 4 else 127)


def test_quantize_rounds_half_away_from_zero():
    # std::lround: ties away from zero, then the +-127 clamp.
    B = np.array([[127.0], [0.5], [-0.5], [1.5], [-1.5], [2.5]], np.float32)
    q, s = oracle.quantize_q8(B)
    assert s[0] == np.float32(1.0)
    assert q[:, 0].tolist() == [127, 1, -1, 2, -2, 3]


@pytest.mark.parametrize("i", range(15))
def test_matmul_naive_matches_reference_bits(golden, i):
    C = oracle.matmul_naive(golden[f"mm{i}_A"], golden[f"mm{i}_B"])
    np.testing.assert_array_equal(bits(C), bits(golden[f"mm{i}_C"]))


@pytest.mark.parametrize("i", range(7))
def test_q8_paths_match_reference_bits(golden, i):
    A, q, s = golden[f"q8_{i}_A"], golden[f"q8_{i}_q"], golden[f"q8_{i}_scale"]
    np.testing.assert_array_equal(bits(oracle.matmul_naive_q8(A, q, s)), bits(golden[f"q8_{i}_naive"]))
    # The CPU-baseline port splits work as matmul_parallel does, so it matches bit for bit too.
    for t in (1, 3):
        got = oracle.matmul_parallel(A, q=q, scale=s, threads=t)
        np.testing.assert_array_equal(bits(got), bits(golden[f"q8_{i}_par{t}"]))


@pytest.mark.parametrize("i", range(3))
def test_rmsnorm_matches_reference_bits(golden, i):
    y = oracle.rmsnorm(golden[f"rms{i}_x"], golden[f"rms{i}_w"])
    np.testing.assert_array_equal(bits(y), bits(golden[f"rms{i}_y"]))


@pytest.mark.parametrize("m,k,n", [(301, 129, 47), (1, 1029, 1000), (4, 300, 77), (70, 33, 900)])
def test_parallel_thread_counts(m, k, n):
    # tests/test_matmul.cpp:117-132
    rng = np.random.default_rng(7)
    A = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    B = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    want = oracle.matmul_naive(A, B)
    for t in (1, 2, 3, 5, 64, 0):
        assert close_to(oracle.matmul_parallel(A, B, threads=t), want, k)


def test_checker_catches_a_planted_error(golden):
    # A mistake planted in the oracle's output must fail the comparison the GPU tests use.
    C = oracle.matmul_naive(golden["mm5_A"], golden["mm5_B"]).copy()
    k = golden["mm5_A"].shape[1]
    assert close_to(C, golden["mm5_C"], k)
    C[3, 7] += 1e-5 * k * 1.5
    assert not close_to(C, golden["mm5_C"], k)


@pytest.mark.skipif(not oracle.Reference.available(), reason="oracle/_ref not built")
def test_restatement_matches_reference_on_fresh_inputs():
    ref = oracle.Reference()
    rng = np.random.default_rng(123)
    for m, k, n in [(1, 4096, 256), (4, 513, 129), (9, 64, 33), (2, 0, 5)]:
        A = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        W = (rng.standard_normal((k, n)) * 0.02).astype(np.float32)
        q, s = oracle.quantize_q8(W)
        rq, rs = ref.quantize_q8(W)
        np.testing.assert_array_equal(q, rq)
        np.testing.assert_array_equal(bits(s), bits(rs))
        np.testing.assert_array_equal(bits(oracle.matmul_naive(A, W)), bits(ref.matmul_naive(A, W)))
        h = ref.qtensor(q, s)
        np.testing.assert_array_equal(bits(oracle.matmul_parallel(A, q=q, scale=s, threads=2)),
                                      bits(ref.matmul_parallel_q8(A, h, threads=2)))


@pytest.mark.skipif(not oracle.Reference.available(), reason="oracle/_ref not built")
def test_reference_shape_error_names_both_shapes():
    # tests/test_matmul.cpp:56-66: the message carries "2x3" and "4x2".
    ref = oracle.Reference()
    with pytest.raises(ValueError) as e:
        ref.matmul_naive(np.zeros((2, 3), np.float32), np.zeros((4, 2), np.float32))
    assert "2x3" in str(e.value) and "4x2" in str(e.value)
