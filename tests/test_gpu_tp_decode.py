"""The tensor-parallel transformer (llm-engine_b200/tp_decode.py) against the reference's own CPU
Transformer (src/model.cpp, built into oracle/_ref) on the same llama2.c checkpoint and token
stream: token-by-token decoding, then a prefill continuing the cache, fp32 and int8 weights.

* one rank: every step's logits within the reference model test's tolerance
  (tests/test_cuda_model.cpp:30, 1e-4, here relative to the largest logit);
* 2 and 4 ranks emulated in one process on one GPU: each rank holds only its heads, hidden
  slice and vocabulary slice; the test sums the yielded buffers over ranks in rank order, as
  the all-reduce does -- the decomposition must reproduce the unsharded model;
* 2 GPUs (skipped with fewer): one process per GPU, the library's communicator with its
  NVLink peer all-reduce fused into the residual add; both ranks must end with the same
  logits. Child processes keep NVLS off (NCCL_NVLS_ENABLE=0).
"""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import oracle
import llme_b200 as L
from checkpoint import load_checkpoint
from model_fixture import make_model, write_checkpoint
from tp_decode import TPTransformer

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not oracle.RefModel.available(), reason="reference model not built")]

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENV = dict(os.environ, NCCL_NVLS_ENABLE="0")
# token-by-token over the first positions, then a prefill of the next three, then one more
STREAM = [([5], 0), ([17], 1), ([2], 2), ([44], 3), ([9], 4), ([31, 0, 12], 5), ([7], 8)]
MODELS = {"gqa": dict(dim=64, hidden=96, layers=2, heads=8, kv_heads=4, vocab=50, seq_len=16),
          "mha": dict(dim=64, hidden=80, layers=2, heads=4, kv_heads=4, vocab=53, seq_len=16)}


def close(got, want):
    return float(np.abs(got - want).max()) <= 1e-4 * max(1.0, float(np.abs(want).max()))


@pytest.fixture(scope="module", autouse=True)
def _lib():
    L.load()
    yield
    L.device_status()


def checkpoint(tmp_path, name, seed=7):
    p = str(tmp_path / f"{name}.bin")
    write_checkpoint(make_model(seed=seed, **MODELS[name]), p)
    return p


def emulated_run(shards, tokens, pos):
    """One pass over shards that stand for the ranks of one model: at every reduction point
    the yielded buffers are summed in rank order and the sum written back to each."""
    gens = [s.steps(tokens, pos) for s in shards]
    while True:
        bufs = [next(g, None) for g in gens]
        if all(b is None for b in bufs):
            break
        assert all(b is not None for b in bufs), "ranks disagree on the reduction points"
        total = bufs[0].clone()
        for b in bufs[1:]:
            total += b
        for b in bufs:
            b.copy_(total)
    return shards[0].logits.cpu().numpy()


@pytest.mark.parametrize("q8", [False, True])
@pytest.mark.parametrize("name", ["gqa", "mha"])
def test_one_rank_matches_the_reference_model(tmp_path, name, q8):
    p = checkpoint(tmp_path, name)
    ref = oracle.RefModel(p, q8)
    tp = TPTransformer(load_checkpoint(p), q8=q8)
    for tokens, pos in STREAM:
        got, want = tp.run(tokens, pos), ref.run(tokens, pos)
        assert close(got, want), (tokens, pos, float(np.abs(got - want).max()))


@pytest.mark.parametrize("q8", [False, True])
@pytest.mark.parametrize("world", [2, 4])
def test_emulated_ranks_match_the_reference_model(tmp_path, world, q8):
    p = checkpoint(tmp_path, "gqa", seed=8)
    ref = oracle.RefModel(p, q8)
    ck = load_checkpoint(p)
    shards = [TPTransformer(ck, world=world, rank=r, q8=q8) for r in range(world)]
    assert sum(s.nq for s in shards) == ck.config.n_heads
    assert all(s.hc < ck.config.hidden_dim for s in shards)
    for tokens, pos in STREAM:
        got, want = emulated_run(shards, tokens, pos), ref.run(tokens, pos)
        assert close(got, want), (world, tokens, pos, float(np.abs(got - want).max()))


@pytest.mark.parametrize("q8", [False, True])
def test_graph_decode_matches_the_reference_model(tmp_path, q8):
    # The one-token step captured once (after an eager step) and replayed at later positions,
    # including a rewind that overwrites a cached position, as the reference's graph serves
    # every position (src/cuda_model.cu:190-220).
    p = checkpoint(tmp_path, "gqa", seed=10)
    ref = oracle.RefModel(p, q8)
    tp = TPTransformer(load_checkpoint(p), q8=q8)
    assert close(tp.run([3], 0), ref.run([3], 0))
    tp.capture_decode()
    for token, pos in [(8, 1), (21, 2), (4, 3), (40, 2), (6, 3), (11, 4)]:
        got, want = tp.forward(token, pos), ref.run([token], pos)
        assert close(got, want), (token, pos, float(np.abs(got - want).max()))


@pytest.mark.parametrize("q8", [False, True])
def test_graph_recaptured_after_a_longer_prefill(tmp_path, q8):
    # A prefill longer than any run before replaces the activation buffers the graph points
    # at; the next decode() sees the generation move and captures again, as the reference's
    # CudaTransformer does (src/cuda_model.cu:175-177, 196-227).
    p = checkpoint(tmp_path, "mha", seed=12)
    ref = oracle.RefModel(p, q8)
    tp = TPTransformer(load_checkpoint(p), q8=q8)
    assert close(tp.run([3], 0), ref.run([3], 0))
    tp.capture_decode()
    captured = tp.graph_generation
    assert close(tp.forward(8, 1), ref.run([8], 1))
    assert tp.graph_generation == captured
    assert close(tp.prefill([4, 9, 1, 30], 2), ref.run([4, 9, 1, 30], 2))
    assert tp.buffers_generation() != captured
    for token, pos in [(5, 6), (12, 7), (2, 8)]:
        got, want = tp.forward(token, pos), ref.run([token], pos)
        assert close(got, want), (token, pos, float(np.abs(got - want).max()))
    assert tp.graph_generation == tp.buffers_generation() != captured


def test_positions_are_checked(tmp_path):
    tp = TPTransformer(load_checkpoint(checkpoint(tmp_path, "gqa")))
    with pytest.raises(IndexError):
        tp.run([1], 3)          # skips cached positions
    with pytest.raises(IndexError):
        tp.run([50], 0)         # outside the vocabulary
    tp.run([1], 0)
    with pytest.raises(IndexError):
        tp.run([1] * 16, 1)     # past seq_len


WORKER = r"""
import os, sys, datetime
import numpy as np
sys.path.insert(0, "llm-engine_b200"); sys.path.insert(0, "tests")
import torch, torch.distributed as dist
import llme_b200 as L
from checkpoint import load_checkpoint
from tp_decode import TPTransformer
rank, world, port, ckpt, q8, out = (int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]),
                                    sys.argv[4], sys.argv[5] == "1", sys.argv[6])
torch.cuda.set_device(rank)
dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                        world_size=world, timeout=datetime.timedelta(seconds=60))
uid = [L.Comm.unique_id() if rank == 0 else None]
dist.broadcast_object_list(uid, src=0)
comm = L.Comm(world, rank, uid[0], timeout_s=60.0)
comm.enable_peer(1 << 16)
tp = TPTransformer(load_checkpoint(ckpt), world=world, rank=rank, q8=q8, comm=comm)
stream = eval(sys.argv[7])
for i, (tokens, pos) in enumerate(stream):
    np.save(f"{out}/logits_{i}_{rank}.npy", tp.run(tokens, pos))
torch.cuda.synchronize()
L.Comm.status()
comm.destroy()
dist.destroy_process_group()
print("OK", rank)
"""


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("q8", [False, True])
def test_two_gpus_match_the_reference_model(tmp_path, q8):
    world = 2
    p = checkpoint(tmp_path, "gqa", seed=9)
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    procs = [subprocess.Popen([sys.executable, "-c", WORKER, str(r), str(world), str(port), p,
                               "1" if q8 else "0", str(tmp_path), repr(STREAM)], cwd=REPO,
                              env=ENV, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
             for r in range(world)]
    outs = [pr.communicate(timeout=300)[0] for pr in procs]
    for pr, o in zip(procs, outs):
        assert pr.returncode == 0 and "OK" in o, o[-3000:]
    ref = oracle.RefModel(p, q8)
    for i, (tokens, pos) in enumerate(STREAM):
        want = ref.run(tokens, pos)
        got = [np.load(tmp_path / f"logits_{i}_{r}.npy") for r in range(world)]
        np.testing.assert_array_equal(got[0], got[1])
        assert close(got[0], want), (tokens, pos, float(np.abs(got[0] - want).max()))
