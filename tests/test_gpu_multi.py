"""Tensor-parallel products through the library's NCCL communicator.

* A communicator whose second rank never joins must end in LLME_E_TIMEOUT within its
  deadline, not hang (host-side failure: nothing runs on the GPU; one GPU is enough).
* On two GPUs (skipped with fewer): the library's NVLink peer all-reduce, six calls back to
  back with exactly known sums; column-parallel products on n-shards and row-parallel products
  on k-shards (llme_matmul_q8_rowpar, all-reduce inside, residual added once), through the C
  ABI, against the oracle on the unsharded weights; with equal shards (LLME_FLAG_SAME_SHARDS)
  the rank sum taken inside the GEMV, bit for bit the separate all-reduce's result on every
  rank, over repeated back-to-back calls; and a grouped row-parallel batch with the rank sum
  inside its launch (llme_batch_run_rowpar), against the plain batch + all-reduce and the
  oracle.
Child processes keep NVLS off (NCCL_NVLS_ENABLE=0), as failure tests on this pool require.
"""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import oracle
from conftest import close_to

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENV = dict(os.environ, NCCL_NVLS_ENABLE="0")

NEVER_JOINS = r"""
import sys, time
sys.path.insert(0, "llm-engine_b200")
import llme_b200 as L
uid = L.Comm.unique_id()
t0 = time.time()
try:
    L.Comm(2, 0, uid, timeout_s=3.0)
    print("JOINED")
except L.DeviceTimeout as e:
    print("TIMEOUT", round(time.time() - t0, 1), e)
"""


def test_comm_init_times_out_when_a_rank_never_joins():
    r = subprocess.run([sys.executable, "-c", NEVER_JOINS], cwd=REPO, env=ENV, timeout=120,
                       stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    assert r.returncode == 0, r.stdout[-2000:]
    assert "TIMEOUT" in r.stdout, r.stdout[-2000:]


TP_WORKER = r"""
import os, sys, datetime
import numpy as np
sys.path.insert(0, "llm-engine_b200"); sys.path.insert(0, "oracle")
import torch, torch.distributed as dist
import llme_b200 as L, shard, oracle
rank, world, port, out = int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]), sys.argv[4]
SAME_SHARDS = eval(sys.argv[5])
BATCH = eval(sys.argv[6])
torch.cuda.set_device(rank)
dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                        world_size=world, timeout=datetime.timedelta(seconds=60))
uid = [L.Comm.unique_id() if rank == 0 else None]
dist.broadcast_object_list(uid, src=0)
comm = L.Comm(world, rank, uid[0], timeout_s=60.0)
comm.enable_peer(1 << 20)   # the library's NVLink peer all-reduce for up to 1 Mi floats
# Back-to-back peer all-reduces with no host sync in between (both slots reused several times):
# rank r contributes (r + 1) * (i + 1) + j, so every sum is known exactly.
bufs = []
for i in range(6):
    x = (torch.arange(300003, dtype=torch.float32, device="cuda") % 7) + (rank + 1) * (i + 1)
    comm.allreduce_sum_f32(x.data_ptr(), x.numel(), stream=L.torch_stream_handle())
    bufs.append(x)
torch.cuda.synchronize()
L.Comm.status()
for i, x in enumerate(bufs):
    want = world * (torch.arange(300003, dtype=torch.float32, device="cuda") % 7) + \
        sum((r + 1) * (i + 1) for r in range(world))
    assert torch.equal(x, want), ("peer all-reduce", i)
rng = np.random.default_rng(31)
for (m, k, n) in [(1, 4096, 4096), (4, 11008, 4096), (8, 1024, 2048), (130, 512, 1024)]:
    A = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    q, s = oracle.quantize_q8((rng.standard_normal((k, n)) * 0.02).astype(np.float32))
    C0 = rng.uniform(-1, 1, (m, n)).astype(np.float32)
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()
    # column-parallel: this rank's columns
    qc, sc = shard.column_shard(q, s, world, rank)
    Cc = torch.empty(m, qc.shape[1], device="cuda")
    L.matmul(dev(A), dev(qc), scale=dev(sc), C=Cc)
    # row-parallel with the residual add
    Ar, qr = shard.activation_columns(A, world, rank), shard.row_shard(q, world, rank)
    Cr = dev(C0)
    dAr, dqr, ds = dev(Ar), dev(qr), dev(s)  # kept alive until the async product has run
    comm.matmul_q8_rowpar(m, n, Ar.shape[1], dAr.data_ptr(), dqr.data_ptr(), ds.data_ptr(),
                          Cr.data_ptr(), accumulate=True, stream=L.torch_stream_handle())
    torch.cuda.synchronize()
    np.save(f"{out}/col_{m}_{rank}.npy", Cc.cpu().numpy())
    np.save(f"{out}/row_{m}_{rank}.npy", Cr.cpu().numpy())
# Row-parallel products with every rank's shard the same size (FLAG_SAME_SHARDS): the sum over
# the ranks runs inside the GEMV. Several calls back to back with no host sync (both slots of
# every CTA reused), each against the separate-all-reduce path on the same inputs.
fused = {}
for it in range(3):
    for (m, k, n) in SAME_SHARDS:
        A = rng.uniform(-1, 1, (m, k)).astype(np.float32) + it
        q, s = oracle.quantize_q8((rng.standard_normal((k, n)) * 0.02).astype(np.float32))
        C0 = rng.uniform(-1, 1, (m, n)).astype(np.float32)
        Ar, qr = shard.activation_columns(A, world, rank), shard.row_shard(q, world, rank)
        dAr, dqr, ds = dev(Ar), dev(qr), dev(s)
        Cf, Cs = dev(C0), dev(C0)
        for C, fl in ((Cf, L.FLAG_SAME_SHARDS | L.FLAG_WEIGHTS_STATIC), (Cs, L.FLAG_WEIGHTS_STATIC)):
            comm.matmul_q8_rowpar(m, n, Ar.shape[1], dAr.data_ptr(), dqr.data_ptr(), ds.data_ptr(),
                                  C.data_ptr(), accumulate=True, flags=fl,
                                  stream=L.torch_stream_handle())
        fused[(it, m, k, n)] = (Cf, Cs, dAr, dqr, ds)
torch.cuda.synchronize()
L.Comm.status()
for (it, m, k, n), (Cf, Cs, *_) in fused.items():
    np.save(f"{out}/fused_{it}_{m}_{k}_{rank}.npy", Cf.cpu().numpy())
    np.save(f"{out}/sep_{it}_{m}_{k}_{rank}.npy", Cs.cpu().numpy())
# A row-parallel batch (equal shards) with the sum over the ranks inside the launch, against
# the same batch run plainly and summed by the peer all-reduce; rank 0 adds C0 (accumulate).
prods = []
for (k, n) in BATCH:
    A = rng.uniform(-1, 1, (1, k)).astype(np.float32)
    q, s = oracle.quantize_q8((rng.standard_normal((k, n)) * 0.02).astype(np.float32))
    prods.append((dev(shard.activation_columns(A, world, rank)), dev(shard.row_shard(q, world, rank)),
                  dev(s), k // world, n))
C0 = [rng.uniform(-1, 1, (1, n)).astype(np.float32) for (_, n) in BATCH]
offs = np.cumsum([0] + [(n + 3) // 4 * 4 for (_, n) in BATCH])
Cf = torch.zeros(int(offs[-1]), device="cuda")
Cs = torch.zeros(int(offs[-1]), device="cuda")
acc = 1 if rank == 0 else 0
def batch(C):
    return L.Batch(1, [(n, kl, a.data_ptr(), b.data_ptr(), sc.data_ptr(), C.data_ptr() + 4 * int(o), acc)
                       for (a, b, sc, kl, n), o in zip(prods, offs[:-1])])
bf, bs = batch(Cf), batch(Cs)
h = L.torch_stream_handle()
runs = []
for it in range(3):
    for C in (Cf, Cs):
        for (kk, n), o, c0 in zip(BATCH, offs[:-1], C0):
            C[int(o):int(o) + n].copy_(torch.from_numpy(c0[0]))
    bf.run_rowpar(comm, L.FLAG_WEIGHTS_STATIC, h)
    bs.run(L.FLAG_WEIGHTS_STATIC, h)
    comm.allreduce_sum_f32(Cs.data_ptr(), Cs.numel(), stream=h)
    runs.append((Cf.clone(), Cs.clone()))
torch.cuda.synchronize()
L.Comm.status()
for it, (f, sp) in enumerate(runs):
    np.save(f"{out}/batchf_{it}_{rank}.npy", f.cpu().numpy())
    np.save(f"{out}/batchs_{it}_{rank}.npy", sp.cpu().numpy())
bf.destroy(); bs.destroy()
L.synchronize()
L.Comm.status()
comm.destroy()
dist.destroy_process_group()
print("OK", rank)
"""


# (m, k, n) of the row-parallel products with equal shards (k splits evenly over 2 ranks): the
# 7B decode's wo and w2, several rows, one k slice per strip (a 2 x 128-row k shard).
SAME_SHARDS = [(1, 4096, 4096), (1, 11008, 4096), (4, 4096, 4096), (8, 11008, 4096),
               (2, 256, 8192), (3, 2048, 1040)]
# (k, n) of a grouped row-parallel step: the decode's wo / w2 shapes and enough small products
# that CTAs run several units each.
BATCH = [(4096, 4096), (11008, 4096), (2048, 1040)] + [(256, 2048)] * 24


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tensor_parallel_products_on_two_gpus(tmp_path):
    world = 2
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    procs = [subprocess.Popen([sys.executable, "-c", TP_WORKER, str(r), str(world), str(port),
                               str(tmp_path), repr(SAME_SHARDS), repr(BATCH)], cwd=REPO, env=ENV,
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
             for r in range(world)]
    outs = [p.communicate(timeout=300)[0] for p in procs]
    for p, o in zip(procs, outs):
        assert p.returncode == 0 and "OK" in o, o[-3000:]
    import shard
    rng = np.random.default_rng(31)
    for (m, k, n) in [(1, 4096, 4096), (4, 11008, 4096), (8, 1024, 2048), (130, 512, 1024)]:
        A = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        q, s = oracle.quantize_q8((rng.standard_normal((k, n)) * 0.02).astype(np.float32))
        C0 = rng.uniform(-1, 1, (m, n)).astype(np.float32)
        full = oracle.matmul_naive_q8(A, q, s)
        cols = np.concatenate([np.load(tmp_path / f"col_{m}_{r}.npy") for r in range(world)], axis=1)
        assert close_to(cols, full, k), m
        for r in range(world):
            assert close_to(np.load(tmp_path / f"row_{m}_{r}.npy"), C0 + full, k, 2.0), (m, r)
    # The in-kernel rank sum adds the same values in the same order as the separate all-reduce,
    # so both give the same bits, on every rank, and match the oracle.
    report = []
    for it in range(3):
        for (m, k, n) in SAME_SHARDS:
            A = rng.uniform(-1, 1, (m, k)).astype(np.float32) + it
            q, s = oracle.quantize_q8((rng.standard_normal((k, n)) * 0.02).astype(np.float32))
            C0 = rng.uniform(-1, 1, (m, n)).astype(np.float32)
            want = C0 + oracle.matmul_naive_q8(A, q, s)
            got = [np.load(tmp_path / f"fused_{it}_{m}_{k}_{r}.npy") for r in range(world)]
            sep = [np.load(tmp_path / f"sep_{it}_{m}_{k}_{r}.npy") for r in range(world)]
            bad = []
            for r in range(world):
                if not np.array_equal(got[r], sep[0], equal_nan=True):
                    diff = np.argwhere(~((got[r] == sep[0]) | (np.isnan(got[r]) & np.isnan(sep[0]))))
                    bad.append(f"rank {r}: {len(diff)} differ from the separate sum, first at "
                               f"{diff[0].tolist()}")
                for name, x in (("fused", got[r]), ("separate", sep[r])):
                    if not close_to(x, want, k, 2.0):
                        bad.append(f"{name} rank {r}: {int(np.isnan(x).sum())} NaN, "
                                   f"{int((np.abs(x - want) > 2e-5 * k).sum())} off the oracle")
            if bad:
                report.append(f"it {it} (m, k, n) = {(m, k, n)}: " + "; ".join(bad))
    # The grouped row-parallel step: the in-launch sum equals the plain batch + all-reduce bit
    # for bit on both ranks, and the oracle on the unsharded products (C0 added once).
    want = []
    for (k, n) in BATCH:
        A = rng.uniform(-1, 1, (1, k)).astype(np.float32)
        q, s = oracle.quantize_q8((rng.standard_normal((k, n)) * 0.02).astype(np.float32))
        want.append(oracle.matmul_naive_q8(A, q, s))
    C0 = [rng.uniform(-1, 1, (1, n)).astype(np.float32) for (_, n) in BATCH]
    offs = np.cumsum([0] + [(n + 3) // 4 * 4 for (_, n) in BATCH])
    for it in range(3):
        f = [np.load(tmp_path / f"batchf_{it}_{r}.npy") for r in range(world)]
        sp = np.load(tmp_path / f"batchs_{it}_0.npy")
        for r in range(world):
            if not np.array_equal(f[r], sp):
                report.append(f"batch it {it} rank {r}: {int((f[r] != sp).sum())} differ from the "
                              "plain batch + all-reduce")
        for (k, n), o, w, c0 in zip(BATCH, offs[:-1], want, C0):
            got = f[0][int(o):int(o) + n][None, :]
            if not close_to(got, c0 + w, k, 2.0):
                report.append(f"batch it {it} (k, n) = {(k, n)}: off the oracle")
    assert not report, "\n".join(report)
