"""The allocation-free entry point, llme_matmul_q8_noalloc, against llme_matmul_q8.

Some callers of this library cannot allocate device memory once they are running: a serving
process whose memory pool reserved nearly all of the GPU's HBM at start-up (a cudaMalloc from
inside the library would fail, or carve up what the pool meant to own), a latency-bound loop
that may not take cudaMalloc's device-wide synchronisation after start-up, and a plug-in
inside a host runtime that owns all device memory. For them the library offers one product
whose split-K scratch is a fixed device array inside the library itself.

Through the C ABI this file checks that two such calls in a row give, bit for bit, what the
allocating entry point gives when it runs the same kernel (the SIMT split-K tiles, selected
with LLME_MATH_FP32 and tiled_split), that both sit within the reference's 1e-5 * k of the
oracle, that the calls leave the library's grow-only scratch untouched (no reallocation), that
calls captured in a CUDA graph replay correctly with new inputs, and that a product too large
for the fixed array is refused with a clear message. It is collected last and needs nothing
from the other test files.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import llme_b200 as L
from conftest import close_to

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _case(rng, m, k, n, accumulate):
    A = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    q, s = oracle.quantize_q8((rng.standard_normal((k, n)) * 0.02).astype(np.float32))
    C0 = rng.uniform(-1, 1, (m, n)).astype(np.float32)
    want = oracle.matmul_naive_q8(A, q, s)
    if accumulate:
        want = C0 + want
    dev = [torch.from_numpy(x).cuda() for x in (A, q, s, C0)]
    return (m, k, n, accumulate), dev, want


def test_noalloc_matches_allocating_entry_point_twice_in_a_row():
    L.load()
    rng = np.random.default_rng(2026)
    cases = [_case(rng, 16, 4096, 4096, False), _case(rng, 33, 1029, 257, True)]
    stream = L.torch_stream_handle()
    # The allocating entry point on the kernel the allocation-free one runs: the SIMT tiles
    # with k split across CTAs (tiled_split in fp32 arithmetic).
    prev = L.set_math(L.MATH_FP32)
    try:
        wants = []
        for (m, k, n, acc), (dA, dq, ds, dC0), _ in cases:
            assert L.plan(m, n, k, q8=True, kernel="tiled_split", a_addr=dA.data_ptr(),
                          b_addr=dq.data_ptr(), math=L.MATH_FP32)["path_name"] == "tiled_simt"
            C = dC0.clone()
            L.matmul_cuda_q8(m, n, k, dA.data_ptr(), dq.data_ptr(), ds.data_ptr(), C.data_ptr(),
                             "tiled_split", acc, 0, 0, stream)
            wants.append(C)
        torch.cuda.synchronize()
    finally:
        L.set_math(prev)
    generation = L.scratch_generation()
    # Two allocation-free calls back to back on the same stream; the second reuses the
    # tickets the first left behind.
    gots = []
    for (m, k, n, acc), (dA, dq, ds, dC0), _ in cases:
        C = dC0.clone()
        L.matmul_cuda_q8_noalloc(m, n, k, dA.data_ptr(), dq.data_ptr(), ds.data_ptr(),
                                 C.data_ptr(), acc, stream)
        gots.append(C)
    torch.cuda.synchronize()
    L.synchronize()
    assert L.scratch_generation() == generation  # nothing was (re)allocated
    for ((m, k, n, acc), _, oracle_want), got, want in zip(cases, gots, wants):
        g = got.cpu().numpy()
        np.testing.assert_array_equal(g, want.cpu().numpy())
        assert close_to(g, oracle_want, k, 2.0 if acc else 1.0), (m, k, n)


def test_noalloc_calls_replay_from_a_cuda_graph():
    # The callers this entry point is for record graphs: two calls captured once (the second
    # accumulating, so it starts from tickets the first left at zero) are replayed with new
    # inputs copied into the captured buffers; every replay matches the oracle and nothing is
    # allocated.
    L.load()
    rng = np.random.default_rng(77)
    m, k, n = 16, 2048, 1024
    q, s = oracle.quantize_q8((rng.standard_normal((k, n)) * 0.02).astype(np.float32))
    dA = torch.zeros(m, k, device="cuda")
    dq, ds = torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()
    dC1 = torch.zeros(m, n, device="cuda")
    dC2 = torch.zeros(m, n, device="cuda")
    args = (m, n, k, dA.data_ptr(), dq.data_ptr(), ds.data_ptr())
    L.matmul_cuda_q8_noalloc(*args, dC1.data_ptr(), False, L.torch_stream_handle())  # set-up
    torch.cuda.synchronize()
    generation = L.scratch_generation()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        st = L.torch_stream_handle()
        L.matmul_cuda_q8_noalloc(*args, dC1.data_ptr(), False, st)
        L.matmul_cuda_q8_noalloc(*args, dC2.data_ptr(), True, st)
    for _ in range(3):
        A = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        C0 = rng.uniform(-1, 1, (m, n)).astype(np.float32)
        dA.copy_(torch.from_numpy(A))
        dC2.copy_(torch.from_numpy(C0))
        graph.replay()
        torch.cuda.synchronize()
        want = oracle.matmul_naive_q8(A, q, s)
        assert close_to(dC1.cpu().numpy(), want, k)
        assert close_to(dC2.cpu().numpy(), C0 + want, k, 2.0)
    del graph
    L.synchronize()
    assert L.scratch_generation() == generation


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
