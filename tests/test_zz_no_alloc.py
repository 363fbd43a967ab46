"""The allocation-free entry point, llme_matmul_q8_noalloc, against llme_matmul_q8.

Some callers cannot allocate device memory while they run: code being recorded into a CUDA
graph, serving processes whose allocator already holds nearly all of HBM, real-time loops
that forbid allocation after start-up. For them the library offers one product whose split-K
scratch is a fixed device array inside the library. Through the C ABI, this file checks that
two such calls in a row match the allocating entry point running the same kernel
(tiled_split) within the suite's tolerance, that they leave the library's grow-only scratch
untouched (no reallocation), and that a product too large for the fixed array is refused
with a clear message. It is collected last and needs nothing from the other test files.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import llme_b200 as L
from conftest import close_to

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _case(rng, m, k, n):
    A = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    q, s = oracle.quantize_q8(rng.uniform(-1, 1, (k, n)).astype(np.float32))
    C0 = rng.uniform(-1, 1, (m, n)).astype(np.float32)
    dev = [torch.from_numpy(x).cuda() for x in (A, q, s, C0)]
    return (m, k, n), dev


def test_noalloc_matches_allocating_entry_point_twice_in_a_row():
    L.load()
    rng = np.random.default_rng(2026)
    cases = [(_case(rng, 16, 4096, 4096), False), (_case(rng, 33, 1029, 257), True)]
    stream = L.torch_stream_handle()
    # The allocating entry point with the same kernel: the reference result.
    wants = []
    for ((m, k, n), (dA, dq, ds, dC0)), acc in cases:
        C = dC0.clone()
        L.matmul_cuda_q8(m, n, k, dA.data_ptr(), dq.data_ptr(), ds.data_ptr(), C.data_ptr(),
                         "tiled_split", acc, 0, 0, stream)
        wants.append(C)
    torch.cuda.synchronize()
    generation = L.scratch_generation()
    # Two allocation-free calls back to back on the same stream.
    gots = []
    for ((m, k, n), (dA, dq, ds, dC0)), acc in cases:
        C = dC0.clone()
        L.matmul_cuda_q8_noalloc(m, n, k, dA.data_ptr(), dq.data_ptr(), ds.data_ptr(),
                                 C.data_ptr(), acc, stream)
        gots.append(C)
    torch.cuda.synchronize()
    L.synchronize()
    assert L.scratch_generation() == generation  # nothing was (re)allocated
    for (((m, k, n), _), acc), got, want in zip(cases, gots, wants):
        assert close_to(got.cpu().numpy(), want.cpu().numpy(), k, 2.0 if acc else 1.0), (m, k, n)


def test_noalloc_refuses_a_product_larger_than_its_scratch():
    L.load()
    # 580 output tiles of 64 x 64, k split in two: about 19 MB of partial sums, more than the
    # fixed 16 MiB array. Refused on the host before anything is launched.
    m, n, k = 64, 64 * 580, 512
    dA = torch.zeros(m, k, device="cuda")
    dq = torch.zeros(k, n, dtype=torch.int8, device="cuda")
    ds = torch.zeros(n, device="cuda")
    dC = torch.zeros(m, n, device="cuda")
    with pytest.raises(L.InvalidArgument) as e:
        L.matmul_cuda_q8_noalloc(m, n, k, dA.data_ptr(), dq.data_ptr(), ds.data_ptr(),
                                 dC.data_ptr(), False, L.torch_stream_handle())
    assert "fixed scratch" in str(e.value)
