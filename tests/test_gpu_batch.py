"""Grouped products (llme_batch_q8_create / llme_batch_run): independent int8 products of
the same m in one persistent launch, against the oracle on identical inputs (the reference's
1e-5 * k bound, 2e-5 * k with the residual add), bit-identical on repeat and with
programmatic dependent launch, and the argument checks."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import llme_b200 as L
from conftest import close_to

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SHAPES = [(4096, 4096), (4096, 11008), (11008, 4096), (64, 288), (1000, 4096), (4100, 32)]


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
