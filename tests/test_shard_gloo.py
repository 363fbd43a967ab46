"""Tensor-parallel sharding logic on CPU ranks (gloo, world_size 2), no GPU.

Each rank computes its shard of the product with the oracle and the ranks exchange results
the way the GPU path does: column-parallel outputs are disjoint column blocks, row-parallel
partial outputs are summed by an all-reduce with only rank 0 adding the residual. The
gathered / reduced result must equal the unsharded product within the reference's tolerance.
A second test makes one rank fail before the exchange and checks that the other learns of it
through the process group's timeout instead of hanging.
"""
from __future__ import annotations

import datetime
import os
import socket
import sys

import numpy as np
import pytest

import oracle
import shard

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("total,world", [(4096, 8), (11008, 8), (32000, 8), (10, 3), (7, 4), (3, 4)])
def test_shard_range_covers_everything_once(total, world):
    seen = []
    for r in range(world):
        s, c = shard.shard_range(total, world, r)
        seen.extend(range(s, s + c))
    assert seen == list(range(total))
    counts = [shard.shard_range(total, world, r)[1] for r in range(world)]
    assert max(counts) - min(counts) <= 1


def test_only_wo_and_w2_are_row_parallel():
    assert [k for k, v in shard.PARALLELISM.items() if v == "row"] == ["wo", "w2"]


def _tp_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    import torch
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    sys.path.insert(0, os.path.join(REPO, "llm-engine_b200"))
    import oracle as orc
    import shard as sh
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    rng = np.random.default_rng(7)  # same inputs on every rank
    m, k, n = 3, 96, 40
    A = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    q, s = orc.quantize_q8((rng.standard_normal((k, n)) * 0.02).astype(np.float32))
    C0 = rng.uniform(-1, 1, (m, n)).astype(np.float32)
    # Column-parallel: this rank's columns, gathered.
    qc, sc = sh.column_shard(q, s, world, rank)
    part = torch.from_numpy(orc.matmul_naive_q8(A, qc, sc))
    gathered = [torch.empty(m, sh.shard_range(n, world, r)[1]) for r in range(world)]
    dist.all_gather(gathered, part)
    col = torch.cat(gathered, dim=1).numpy()
    # Row-parallel with a residual add: partial sums, rank 0 adds C0, then one all-reduce.
    Ar = sh.activation_columns(A, world, rank)
    qr = sh.row_shard(q, world, rank)
    partial = orc.matmul_naive_q8(Ar, qr, s)
    if sh.accumulate_on_this_rank(True, rank):
        partial = partial + C0
    t = torch.from_numpy(partial)
    dist.all_reduce(t)
    np.save(os.path.join(out_dir, f"col{rank}.npy"), col)
    np.save(os.path.join(out_dir, f"row{rank}.npy"), t.numpy())
    dist.destroy_process_group()


def test_tensor_parallel_products_on_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    world, port = 2, _free_port()
    mp.start_processes(_tp_worker, args=(world, port, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    rng = np.random.default_rng(7)
    m, k, n = 3, 96, 40
    A = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    q, s = oracle.quantize_q8((rng.standard_normal((k, n)) * 0.02).astype(np.float32))
    C0 = rng.uniform(-1, 1, (m, n)).astype(np.float32)
    full = oracle.matmul_naive_q8(A, q, s)
    for r in range(world):
        col = np.load(tmp_path / f"col{r}.npy")
        row = np.load(tmp_path / f"row{r}.npy")
        np.testing.assert_array_equal(col, full)  # same products, only split by column
        assert np.abs(row - (C0 + full)).max() <= 2e-5 * k


def _failing_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        # This rank fails between steps: it leaves without joining the exchange.
        os._exit(0)
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        outcome = "completed"
    except Exception as e:  # the survivor learns of it through the timeout
        outcome = "error: " + type(e).__name__
    with open(os.path.join(out_dir, "outcome.txt"), "w") as f:
        f.write(outcome)
    os._exit(0)


def test_a_rank_that_leaves_is_detected_by_timeout(tmp_path):
    import torch.multiprocessing as mp
    world, port = 2, _free_port()
    ctx = mp.start_processes(_failing_worker, args=(world, port, str(tmp_path)), nprocs=world,
                             join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=60)
        assert not p.is_alive()
    outcome = (tmp_path / "outcome.txt").read_text()
    assert outcome.startswith("error"), outcome
