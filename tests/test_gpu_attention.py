"""Causal decode attention (llme_attention, the interface of the reference's
src/cuda_attention.h) against a float64 restatement of its definition, the way the reference's
tests/test_cuda_attention.cpp checks its own kernels: the same shapes (multi-head,
grouped-query with every heads-per-block case, multi-query, tiny heads), positions on and
around chunk boundaries, 1 / 3 / 8 / 12 rows, every kernel, tolerance 5e-5 absolute, and a
second identical call giving the same bits; a context past single_block's shared-memory cap."""
from __future__ import annotations

import numpy as np
import pytest

import llme_b200 as L

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 5e-5


def reference(shape, rows, pos, q, kc, vc):
    hs, group = shape.head_size, shape.n_heads // shape.n_kv_heads
    out = np.zeros((rows, shape.out_stride))
    for i in range(rows):
        n_ctx = pos + i + 1
        for h in range(shape.n_heads):
            off = (h // group) * hs
            qv = q[i, h * hs:(h + 1) * hs].astype(np.float64)
            sc = kc[:n_ctx, off:off + hs].astype(np.float64) @ qv / np.sqrt(hs)
            p = np.exp(sc - sc.max())
            out[i, h * hs:(h + 1) * hs] = p @ vc[:n_ctx, off:off + hs].astype(np.float64) / p.sum()
    return out


def run_case(heads, kv_heads, hs, seq_len, kernel, positions, rows, rng):
    kv = kv_heads * hs
    dim = heads * hs
    shape = L.AttentionShape(heads, kv_heads, hs, seq_len, dim + 2 * kv, kv, dim)
    L.attention_check(shape, kernel)
    q = rng.uniform(-1, 1, (rows, shape.q_stride)).astype(np.float32)
    kc = rng.uniform(-1, 1, (seq_len, kv)).astype(np.float32)
    vc = rng.uniform(-1, 1, (seq_len, kv)).astype(np.float32)
    dq, dk, dv = (torch.from_numpy(x).cuda() for x in (q, kc, vc))
    out = torch.zeros(rows, dim, device="cuda")
    n_scr = L.attention_scratch_floats(shape, rows, kernel)
    scratch = torch.zeros(max(1, n_scr), device="cuda")
    pos_dev = torch.zeros(1, dtype=torch.int32, device="cuda")
    worst = 0.0
    for pos in positions:
        if pos + rows > seq_len:
            continue
        pos_dev.fill_(pos)
        L.attention(shape, rows, pos_dev.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                    out.data_ptr(), scratch.data_ptr(), kernel, L.torch_stream_handle())
        got = out.cpu().numpy().copy()
        L.attention(shape, rows, pos_dev.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                    out.data_ptr(), scratch.data_ptr(), kernel, L.torch_stream_handle())
        again = out.cpu().numpy()
        want = reference(shape, rows, pos, q, kc, vc)
        diff = np.abs(got - want).max()
        worst = max(worst, diff)
        assert diff <= TOL, (kernel, heads, kv_heads, hs, seq_len, pos, rows, diff)
        np.testing.assert_array_equal(got, again)
    return worst


@pytest.fixture(scope="module", autouse=True)
def _dev():
    L.load()
    yield
    L.device_status()


# tests/test_cuda_attention.cpp:140-146: heads, kv heads, head size, seq_len
CASES = [(6, 6, 48, 256), (8, 2, 64, 1000), (8, 1, 32, 600), (4, 2, 16, 300), (6, 2, 32, 300)]


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("kernel", ["single_block", "split", "automatic"])
def test_attention_matches_float64(case, kernel):
    rng = np.random.default_rng(hash((case, kernel)) % 2**32)
    heads, kv_heads, hs, seq_len = case
    for rows in (1, 3, 8, 12):
        worst = run_case(heads, kv_heads, hs, seq_len, kernel,
                         [0, 31, 32, 33, 200, seq_len - rows], rows, rng)
    print(f"{kernel} {case}: max |diff| {worst:.1e}")


def test_attention_long_context():
    # Past single_block's shared-memory cap (tests/test_cuda_attention.cpp:157-172).
    rng = np.random.default_rng(11)
    shape = L.AttentionShape(4, 1, 128, 20000, 4 * 128 + 2 * 128, 128, 4 * 128)
    with pytest.raises(L.InvalidArgument):
        L.attention_check(shape, "single_block")
    run_case(4, 1, 128, 20000, "split", [0, 5000, 19999], 1, rng)
    run_case(4, 1, 128, 20000, "automatic", [12345, 19990], 10, rng)


@pytest.mark.parametrize("case", [(4, 4, 256, 900), (2, 1, 320, 700), (16, 4, 128, 1100)])
def test_attention_wide_heads_and_long_chunks(case):
    # The widest head TMA boxes take (256), a head past them (320: per-position bulk copies),
    # and a grouped case with chunks of many boxes; rows 1 and 5.
    rng = np.random.default_rng(sum(case))
    heads, kv_heads, hs, seq_len = case
    for rows in (1, 5):
        run_case(heads, kv_heads, hs, seq_len, "split", [0, 17, 16 * 37, seq_len - rows], rows, rng)


def test_attention_scratch_reused_across_row_counts():
    # One scratch, zero-filled once, sized for the most rows; calls of 3, 1, 8, 1 and 5 rows in
    # turn on a context long enough to split into chunks (tickets in use), as a model's prefill
    # and decode share it: each call must leave the scratch ready for the next whatever its
    # row count (tests/test_cuda_attention.cpp's contract).
    rng = np.random.default_rng(21)
    heads, kv_heads, hs, seq_len = 8, 2, 64, 1200
    kv, dim = kv_heads * hs, heads * hs
    shape = L.AttentionShape(heads, kv_heads, hs, seq_len, dim + 2 * kv, kv, dim)
    kc = rng.uniform(-1, 1, (seq_len, kv)).astype(np.float32)
    vc = rng.uniform(-1, 1, (seq_len, kv)).astype(np.float32)
    dk, dv = torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()
    scratch = torch.zeros(max(1, L.attention_scratch_floats(shape, 8, "split")), device="cuda")
    pos_dev = torch.zeros(1, dtype=torch.int32, device="cuda")
    pos = 700
    for rows in (3, 1, 8, 1, 5):
        q = rng.uniform(-1, 1, (rows, shape.q_stride)).astype(np.float32)
        out = torch.zeros(rows, dim, device="cuda")
        pos_dev.fill_(pos)
        L.attention(shape, rows, pos_dev.data_ptr(), torch.from_numpy(q).cuda().data_ptr(),
                    dk.data_ptr(), dv.data_ptr(), out.data_ptr(), scratch.data_ptr(), "split",
                    L.torch_stream_handle())
        diff = np.abs(out.cpu().numpy() - reference(shape, rows, pos, q, kc, vc)).max()
        assert diff <= TOL, (rows, pos, diff)
        pos += rows
