"""The transformer engine (the library's C++ llme_model_*, llm-engine_b200/csrc/model.cu) against
the reference's own CPU Transformer (src/model.cpp, built into oracle/_ref) on the same llama2.c
checkpoint and token stream: token-by-token decoding, prefills continuing the cache (three
tokens: the fused GEMV epilogues; nine tokens: the separate RoPE and SwiGLU kernels), fp32 and
int8 weights.

* one rank: every step's logits within the reference model test's tolerance
  (tests/test_cuda_model.cpp:30, 1e-4, here relative to the largest logit);
* 2 and 4 ranks emulated in one process on one GPU (llme_model_group_forward): each rank holds
  only its heads, hidden slice and vocabulary slice, and the partials are summed in rank order
  at every reduction point, as the all-reduce does -- the decomposition must reproduce the
  unsharded model;
* the one-token step captured as a CUDA graph and replayed at later and rewound positions,
  and captured again after a longer prefill reallocated its buffers;
* 2 GPUs (skipped with fewer): one process per GPU, the library's communicator with its
  NVLink peer all-reduce; both ranks must end with the same logits. Child processes keep NVLS
  off (NCCL_NVLS_ENABLE=0).
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
from model_fixture import make_model, write_checkpoint

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not oracle.RefModel.available(), reason="reference model not built")]

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENV = dict(os.environ, NCCL_NVLS_ENABLE="0")
# token-by-token over the first positions, a prefill of the next three, one more token, then a
# nine-token prefill that rewinds to position 4
STREAM = [([5], 0), ([17], 1), ([2], 2), ([44], 3), ([9], 4), ([31, 0, 12], 5), ([7], 8),
          ([3, 1, 4, 1, 5, 9, 2, 6, 5], 4)]
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


@pytest.mark.parametrize("q8", [False, True])
@pytest.mark.parametrize("name", ["gqa", "mha"])
def test_one_rank_matches_the_reference_model(tmp_path, name, q8):
    p = checkpoint(tmp_path, name)
    ref = oracle.RefModel(p, q8)
    model = L.Model.load(p, q8=q8)
    for tokens, pos in STREAM:
        got, want = model.forward(tokens, pos), ref.run(tokens, pos)
        assert close(got, want), (tokens, pos, float(np.abs(got - want).max()))


@pytest.mark.parametrize("q8", [False, True])
@pytest.mark.parametrize("world", [2, 4])
def test_emulated_ranks_match_the_reference_model(tmp_path, world, q8):
    p = checkpoint(tmp_path, "gqa", seed=8)
    ref = oracle.RefModel(p, q8)
    ranks = [L.Model.load(p, q8=q8, world=world, rank=r) for r in range(world)]
    cfg = ranks[0].config
    assert sum(r.local["q_heads"] for r in ranks) == cfg["n_heads"]
    assert sum(r.local["hidden"] for r in ranks) == cfg["hidden_dim"]
    assert sum(r.local["vocab"] for r in ranks) == cfg["vocab_size"]
    for tokens, pos in STREAM:
        got, want = L.Model.group_forward(ranks, tokens, pos), ref.run(tokens, pos)
        assert close(got, want), (world, tokens, pos, float(np.abs(got - want).max()))
    with pytest.raises(L.InvalidArgument):
        ranks[1].forward([1], 0)  # a rank without a communicator runs only in its group


@pytest.mark.parametrize("q8", [False, True])
def test_graph_decode_matches_the_reference_model(tmp_path, q8):
    # The one-token step runs eagerly once and is captured, then replayed at later positions,
    # including a rewind that overwrites a cached position, as the reference's graph serves
    # every position (src/cuda_model.cu:190-220).
    p = checkpoint(tmp_path, "gqa", seed=10)
    ref = oracle.RefModel(p, q8)
    model = L.Model.load(p, q8=q8)
    assert model.captures == 0
    for token, pos in [(3, 0), (8, 1), (21, 2), (4, 3), (40, 2), (6, 3), (11, 4)]:
        got, want = model.decode(token, pos), ref.run([token], pos)
        assert close(got, want), (token, pos, float(np.abs(got - want).max()))
        assert model.captures == 1
    model.replay(3)  # more replays of the last step on the current stream
    torch.cuda.synchronize()
    L.device_status()


@pytest.mark.parametrize("q8", [False, True])
def test_graph_recaptured_after_a_longer_prefill(tmp_path, q8):
    # A prefill longer than any step before replaces the activation buffers the graph points
    # at; the next decode sees the buffers' generation move and captures again, as the
    # reference's CudaTransformer does (src/cuda_model.cu:175-177, 196-227).
    p = checkpoint(tmp_path, "mha", seed=12)
    ref = oracle.RefModel(p, q8)
    model = L.Model.load(p, q8=q8)
    assert close(model.decode(3, 0), ref.run([3], 0))
    assert close(model.decode(8, 1), ref.run([8], 1))
    assert model.captures == 1
    assert close(model.forward([4, 9, 1, 30], 2), ref.run([4, 9, 1, 30], 2))
    for token, pos in [(5, 6), (12, 7), (2, 8)]:
        got, want = model.decode(token, pos), ref.run([token], pos)
        assert close(got, want), (token, pos, float(np.abs(got - want).max()))
    assert model.captures == 2


def test_positions_are_checked(tmp_path):
    model = L.Model.load(checkpoint(tmp_path, "gqa"))
    with pytest.raises(IndexError):
        model.forward([1], 3)          # skips cached positions
    with pytest.raises(IndexError):
        model.forward([50], 0)         # outside the vocabulary
    with pytest.raises(IndexError):
        model.decode(-1, 0)
    model.forward([1], 0)
    with pytest.raises(IndexError):
        model.forward([1] * 16, 1)     # past seq_len
    with pytest.raises(L.InvalidArgument):
        model.forward([], 0)


def test_synthetic_model_runs_and_repeats():
    # The benchmark's model: weights drawn on the device, a cache history filled, one token
    # decoded twice at the same position gives the same logits bit for bit (eager, then the
    # captured graph).
    cfg = dict(dim=256, hidden_dim=512, n_layers=2, n_heads=4, n_kv_heads=2, vocab_size=1000,
               seq_len=64)
    model = L.Model.synthetic(cfg, q8=True, seed=3)
    model.fill_history(40, seed=1)
    a = model.decode(7, 40)
    b = model.decode(7, 40)
    assert np.isfinite(a).all() and np.abs(a).max() > 0
    np.testing.assert_array_equal(a, b)
    w, kv = model.stream_bytes()
    assert w > 2 * 256 * 256 and kv == 2 * 2 * 2 * 64 * 4


WORKER = r"""
import os, sys, datetime
import numpy as np
sys.path.insert(0, "llm-engine_b200"); sys.path.insert(0, "tests")
import torch, torch.distributed as dist
import llme_b200 as L
rank, world, port, ckpt, q8, out = (int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]),
                                    sys.argv[4], sys.argv[5] == "1", sys.argv[6])
torch.cuda.set_device(rank)
dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                        world_size=world, timeout=datetime.timedelta(seconds=60))
uid = [L.Comm.unique_id() if rank == 0 else None]
dist.broadcast_object_list(uid, src=0)
comm = L.Comm(world, rank, uid[0], timeout_s=60.0)
comm.enable_peer(1 << 16)
model = L.Model.load(ckpt, q8=q8, world=world, rank=rank, comm=comm)
stream = eval(sys.argv[7])
for i, (tokens, pos) in enumerate(stream):
    np.save(f"{out}/logits_{i}_{rank}.npy", model.forward(tokens, pos))
np.save(f"{out}/decode_{rank}.npy", np.stack([model.decode(t, p) for t, p in [(4, 13), (9, 14)]]))
torch.cuda.synchronize()
L.Comm.status()
model.destroy()
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
    dec = [np.load(tmp_path / f"decode_{r}.npy") for r in range(world)]
    np.testing.assert_array_equal(dec[0], dec[1])
    for j, (t, p_) in enumerate([(4, 13), (9, 14)]):
        assert close(dec[0][j], ref.run([t], p_))
