"""The C restatement (oracle/oracle.c) against the reference's own CPU code compiled from its
sources (oracle/_ref/libllme_ref.so, contraction off) over random shapes and value families,
bit for bit: quantize_q8 / dequantize (src/quant.cpp:6-36), matmul_naive (src/matmul.cpp:
205-217), the int8 naive product the reference's tests use (tests/test_quant.cpp:57-79),
rmsnorm (src/ops.cpp:13-26) and the thread-pooled matmul_parallel (src/matmul.cpp:240-318)
for fp32 and int8 weights at several thread counts. No GPU."""
from __future__ import annotations

import numpy as np
import pytest
from hypothesis import given, settings, strategies as st

import oracle

pytestmark = pytest.mark.skipif(not oracle.Reference.available(), reason="oracle/_ref not built")


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype == np.float32 else np.uint8)


def values(rng, shape, family):
    if family == "uniform":
        return rng.uniform(-1, 1, shape).astype(np.float32)
    if family == "weights":
        return (rng.standard_normal(shape) * 0.02).astype(np.float32)
    if family == "halves":  # products of the scale land exactly on .5: the rounding ties
        return (rng.integers(-254, 255, shape) / 2.0).astype(np.float32)
    if family == "wide":    # magnitudes from 1e-30 to 1e30, signs mixed
        return (rng.choice([-1, 1], shape) * 10.0 ** rng.uniform(-30, 30, shape)).astype(np.float32)
    x = rng.uniform(-1, 1, shape).astype(np.float32)  # "zero columns"
    if x.ndim == 2 and x.shape[1]:
        x[:, rng.integers(0, x.shape[1], max(1, x.shape[1] // 4))] = 0.0
    return x


FAMILIES = ["uniform", "weights", "halves", "wide", "zero columns"]


@settings(max_examples=400, deadline=None)
@given(m=st.integers(0, 12), k=st.integers(0, 300), n=st.integers(0, 140),
       wf=st.sampled_from(FAMILIES), af=st.sampled_from(["uniform", "halves", "zero columns"]),
       seed=st.integers(0, 2**31 - 1))
def test_restatement_matches_the_reference_bit_for_bit(m, k, n, wf, af, seed):
    ref = oracle.Reference()
    rng = np.random.default_rng(seed)
    W = values(rng, (k, n), wf)
    A = values(rng, (m, k), af)
    q, s = oracle.quantize_q8(W)
    rq, rs = ref.quantize_q8(W)
    np.testing.assert_array_equal(q, rq)
    np.testing.assert_array_equal(bits(s), bits(rs))
    np.testing.assert_array_equal(bits(oracle.dequantize(q, s)), bits(ref.dequantize(q, s)))
    np.testing.assert_array_equal(bits(oracle.matmul_naive(A, W)), bits(ref.matmul_naive(A, W)))
    np.testing.assert_array_equal(bits(oracle.matmul_naive_q8(A, q, s)),
                                  bits(ref.matmul_naive(A, ref.dequantize(q, s))))
    if k:
        w = values(rng, (k,), "uniform")
        np.testing.assert_array_equal(bits(oracle.rmsnorm(A, w)), bits(ref.rmsnorm(A, w)))


@settings(max_examples=150, deadline=None)
@given(m=st.integers(1, 20), k=st.integers(1, 400), n=st.integers(1, 200),
       threads=st.sampled_from([1, 2, 3, 5]), seed=st.integers(0, 2**31 - 1))
def test_parallel_port_matches_the_reference_bit_for_bit(m, k, n, threads, seed):
    ref = oracle.Reference()
    rng = np.random.default_rng(seed)
    A = values(rng, (m, k), "uniform")
    W = values(rng, (k, n), "weights")
    q, s = ref.quantize_q8(W)
    h = ref.qtensor(q, s)
    np.testing.assert_array_equal(bits(oracle.matmul_parallel(A, q=q, scale=s, threads=threads)),
                                  bits(ref.matmul_parallel_q8(A, h, threads=threads)))
    np.testing.assert_array_equal(bits(oracle.matmul_parallel(A, W, threads=threads)),
                                  bits(ref.matmul_parallel(A, W, threads=threads)))
