"""The GPU quantiser (llme_quantize_q8) against the reference's quantize_q8 (src/quant.cpp:6-28),
bit for bit: the oracle's restatement, itself pinned bit for bit to the reference's compiled
code (tests/test_oracle.py), on the same fp32 weights. Shapes: the benchmark's weights
(N(0, 0.02^2)), ragged column counts, a single row, columns of zeros, exact halfway products
(round half away from zero) and values that hit the +-127 clamp."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import llme_b200 as L

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def gpu_quantize(W):
    q, s = L.quantize_q8(torch.from_numpy(np.ascontiguousarray(W)).cuda())
    torch.cuda.synchronize()
    return q.cpu().numpy(), s.cpu().numpy()


@pytest.mark.parametrize("k,n", [(4096, 4096), (4096, 11008), (11008, 4096), (1, 1), (1, 37),
                                 (300, 129), (7, 4100), (2049, 3)])
def test_quantize_matches_reference(k, n):
    rng = np.random.default_rng(k * 31 + n)
    W = (rng.standard_normal((k, n)) * 0.02).astype(np.float32)
    q, s = gpu_quantize(W)
    qr, sr = oracle.quantize_q8(W)
    np.testing.assert_array_equal(s, sr)
    np.testing.assert_array_equal(q, qr)


def test_quantize_edge_values():
    rng = np.random.default_rng(5)
    W = rng.uniform(-3, 3, (64, 96)).astype(np.float32)
    W[:, 0] = 0.0                      # a column of zeros: scale 0, q 0
    W[:, 1] = -0.0
    # column 2: max 127, so inv = 1 and x * inv = x: exact halves round away from zero
    W[:, 2] = np.linspace(-126.5, 126.5, 64).astype(np.float32)
    W[0, 2] = 127.0
    W[:, 3] = 1e-30                    # tiny column: scale 7.9e-33, inv 1.3e32 (finite)
    W[5, 4] = 1e30                     # one huge value dominates its column
    q, s = gpu_quantize(W)
    qr, sr = oracle.quantize_q8(W)
    np.testing.assert_array_equal(s, sr)
    np.testing.assert_array_equal(q, qr)
    assert (q[:, 0] == 0).all() and s[0] == 0


def test_quantize_feeds_the_gemv_exactly():
    # A weight quantised on the GPU, multiplied on the GPU, equals the oracle's product of the
    # oracle's quantisation of the same weight.
    rng = np.random.default_rng(6)
    W = (rng.standard_normal((1024, 2048)) * 0.02).astype(np.float32)
    A = rng.uniform(-1, 1, (1, 1024)).astype(np.float32)
    dW = torch.from_numpy(W).cuda()
    q, s = L.quantize_q8(dW)
    C = L.matmul(torch.from_numpy(A).cuda(), q, scale=s)
    torch.cuda.synchronize()
    qr, sr = oracle.quantize_q8(W)
    want = oracle.matmul_naive_q8(A, qr, sr)
    assert np.abs(C.cpu().numpy() - want).max() <= 1e-5 * 1024


def test_quantize_rejects_and_empty():
    d = torch.zeros(4, device="cuda")
    L.quantize_q8_cuda(0, 5, d.data_ptr(), d.data_ptr(), d.data_ptr())  # no-op
    with pytest.raises(L.InvalidArgument):
        L.quantize_q8_cuda(4, 4, 0, d.data_ptr(), d.data_ptr())
    with pytest.raises(L.InvalidArgument):
        L.quantize_q8_cuda(1 << 16, 1 << 15, d.data_ptr(), d.data_ptr(), d.data_ptr())
