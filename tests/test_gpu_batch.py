"""Grouped products (llme_batch_q8_create / llme_batch_run): independent int8 products of
the same m in one persistent launch, against the oracle on identical inputs (the reference's
1e-5 * k bound, 2e-5 * k with the residual add, for the m <= 8 GEMV batches), bit-identical on
repeat and with programmatic dependent launch, and the argument checks. Batches with m >= 128
run on the tensor cores and must equal the single-call results bit for bit (and the oracle
within 1e-4 of each row's L2 norm)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import llme_b200 as L
from conftest import close_to, row_rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

# The chain's three weight shapes, its 4096 x 32000 classifier, and ragged ones.
SHAPES = [(4096, 4096), (4096, 11008), (11008, 4096), (4096, 32000), (64, 288), (1000, 4096),
          (4100, 32)]


def make(rng, m, shapes):
    prods, keep, wants = [], [], []
    for idx, (k, n) in enumerate(shapes):
        A = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        q, s = oracle.quantize_q8((rng.standard_normal((k, n)) * 0.02).astype(np.float32))
        acc = idx % 2 == 1
        C0 = rng.uniform(-1, 1, (m, n)).astype(np.float32)
        dA, dq, ds = (torch.from_numpy(x).cuda() for x in (A, q, s))
        dC = torch.from_numpy(C0.copy()).cuda()
        keep += [dA, dq, ds, dC]
        prods.append((n, k, dA.data_ptr(), dq.data_ptr(), ds.data_ptr(), dC.data_ptr(), int(acc)))
        want = oracle.matmul_naive_q8(A, q, s)
        wants.append((C0 + want if acc else want, k, acc, dC, C0))
    return prods, keep, wants


@pytest.mark.parametrize("m", [1, 2, 4, 8])
def test_batch_matches_oracle(m):
    rng = np.random.default_rng(100 + m)
    prods, keep, wants = make(rng, m, SHAPES)
    batch = L.Batch(m, prods)
    try:
        batch.run(stream=L.torch_stream_handle())
        torch.cuda.synchronize()
        first = []
        for want, k, acc, dC, C0 in wants:
            got = dC.cpu().numpy()
            assert close_to(got, want, k, 2.0 if acc else 1.0), (m, k, np.abs(got - want).max())
            first.append(got)
            dC.copy_(torch.from_numpy(C0))
        # Again, with programmatic dependent launch: the same bits.
        batch.run(flags=L.FLAG_WEIGHTS_STATIC, stream=L.torch_stream_handle())
        torch.cuda.synchronize()
        for (want, k, acc, dC, C0), prev in zip(wants, first):
            np.testing.assert_array_equal(dC.cpu().numpy(), prev)
        L.device_status()
    finally:
        batch.destroy()


def test_batch_rejects_ragged_rows():
    d = torch.zeros(8, device="cuda")
    with pytest.raises(L.InvalidArgument):
        L.Batch(1, [(100, 64, d.data_ptr(), d.data_ptr(), d.data_ptr(), d.data_ptr(), 0)])
    with pytest.raises(L.InvalidArgument):
        L.Batch(9, [(128, 64, d.data_ptr(), d.data_ptr(), d.data_ptr(), d.data_ptr(), 0)])


# ---- m >= 128: grouped tcgen05 products ------------------------------------------------------

TC_SHAPES = [(512, 512), (1000, 272), (2048, 1040), (4100, 48), (300, 4096), (4096, 4096)]


@pytest.mark.parametrize("pairs", ["0", "1"])
@pytest.mark.parametrize("m", [128, 200, 512])
def test_tc_batch_matches_single_calls_bit_for_bit(m, pairs, monkeypatch):
    # pairs = "1": the batch and the single calls run on CTA pairs (cta_group::2).
    monkeypatch.setenv("LLME_B200_CTA_PAIRS", pairs)
    rng = np.random.default_rng(200 + m)
    prev = L.set_math(L.MATH_TENSOR)
    try:
        prods, keep, wants = make(rng, m, TC_SHAPES)
        # The same products one call at a time, into separate outputs.
        singles = []
        for (n, k, a, b, s, c, acc), (want, _, _, dC, C0) in zip(prods, wants):
            out = torch.from_numpy(C0.copy()).cuda()
            L.matmul_cuda_q8(m, n, k, a, b, s, out.data_ptr(), "automatic", bool(acc), 0, 0,
                             L.torch_stream_handle())
            keep.append(out)
            singles.append(out)
        batch = L.Batch(m, prods)
        try:
            batch.run(stream=L.torch_stream_handle())
            torch.cuda.synchronize()
            for (want, k, acc, dC, C0), single in zip(wants, singles):
                got = dC.cpu().numpy()
                np.testing.assert_array_equal(got, single.cpu().numpy())
                assert row_rel_err(got, want) <= 1e-4, (m, k)
            L.device_status()
        finally:
            batch.destroy()
    finally:
        L.set_math(prev)


def test_tc_batch_repeats_and_rejects():
    rng = np.random.default_rng(300)
    prev = L.set_math(L.MATH_TENSOR)
    try:
        prods, keep, wants = make(rng, 256, [(1024, 1024), (2048, 512)])
        prods = [(n, k, a, b, s, c, 0) for (n, k, a, b, s, c, _) in prods]
        batch = L.Batch(256, prods)
        try:
            batch.run(stream=L.torch_stream_handle())
            torch.cuda.synchronize()
            first = [w[3].cpu().numpy() for w in wants]
            batch.run(stream=L.torch_stream_handle())
            torch.cuda.synchronize()
            for w, f in zip(wants, first):
                np.testing.assert_array_equal(w[3].cpu().numpy(), f)
        finally:
            batch.destroy()
        d = torch.zeros(8, device="cuda")
        with pytest.raises(L.InvalidArgument):   # m between the two regimes
            L.Batch(100, [(128, 64, d.data_ptr(), d.data_ptr(), d.data_ptr(), d.data_ptr(), 0)])
        with pytest.raises(L.InvalidArgument):   # n % 16
            L.Batch(128, [(100, 64, d.data_ptr(), d.data_ptr(), d.data_ptr(), d.data_ptr(), 0)])
        L.set_math(L.MATH_FP32)
        with pytest.raises(L.CudaError):          # LLME_E_UNSUPPORTED outside tensor math
            L.Batch(128, [(128, 64, d.data_ptr(), d.data_ptr(), d.data_ptr(), d.data_ptr(), 0)])
    finally:
        L.set_math(prev)
