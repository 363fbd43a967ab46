"""Benchmark: the 7B-shaped int8 decode matmul chain (default) and the other workloads.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one pass of the chain: 32 layers x {wq, wk, wv, wo: 4096x4096; w1, w3:
4096->11008; w2: 11008->4096} + the 4096->32000 classifier = 225 int8 weight x fp32
activation products at m = 1, each on a fresh U(-1, 1) activation vector. Weights are
N(0, 0.02^2), quantised per column as the reference's quant.cpp does. On N GPUs the
column-parallel weights (wq, wk, wv, w1, w3, classifier) are split along n and the
row-parallel ones (wo, w2) along k, followed by a sum all-reduce of the partial outputs.

`value` is whole-job algorithmic bytes (int8 weights + scales + fp32 activations and
outputs) per second with everything resident in HBM, timed with CUDA events around K graph
replays, max over ranks. `e2e` is the same metric through the C ABI with the activations
copied in from pinned host memory and every output copied back inside the timed region.
The weights (6.6 GB / N per GPU) are far larger than L2, so no L2 flush is needed.
`--impl reference` times the reference's own CPU matmul_parallel (compiled from its sources
into oracle/_ref) on a bounded sample of the chain, on the host cores; with
`--workload attention` or `--workload sweep` it times the reference's own GPU code for that
path (src/cuda_attention.cu, src/cuda_matmul.cu built for sm_100a) on the same B200 and
inputs as this library's arm.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "llm-engine_b200"))

DIM, HIDDEN, VOCAB, LAYERS = 4096, 11008, 32000, 32
METRIC = "int8 decode-GEMV HBM GB/s (7B-shaped chain, m=1)"
WORKLOAD_CONFIG = {
    "chain": {"workload": "7B-shaped int8 decode matmul chain, m=1 (BASELINE configs[3])",
              "dim": DIM, "hidden": HIDDEN, "vocab": VOCAB,
              "l2": "no flush: 6.6 GB of weights per step (>> 126 MB L2)"},
    "gemv": {"workload": "decode GEMV m=1, 4096x4096 int8 (BASELINE configs[0]), 16 weight "
                         "copies per step",
             "l2": "no flush: 16 distinct 16.8 MB weights per step (268 MB > 2 x L2)"},
}
UNIT = "GB/s"


def chain_shapes(layers=LAYERS):
    """(name, k, n, row_parallel) for every product of one step, in order."""
    out = []
    for layer in range(layers):
        for name in ("wq", "wk", "wv"):
            out.append((f"{name}{layer}", DIM, DIM, False))
        out.append((f"wo{layer}", DIM, DIM, True))
        out.append((f"w1{layer}", DIM, HIDDEN, False))
        out.append((f"w3{layer}", DIM, HIDDEN, False))
        out.append((f"w2{layer}", HIDDEN, DIM, True))
    out.append(("cls", DIM, VOCAB, False))
    return out


def algorithmic_bytes(k, n, m=1):
    # int8 weights + fp32 column scales + fp32 activations + fp32 outputs
    return k * n + 4 * n + 4 * m * k + 4 * m * n


def _oracle():
    """The checker (oracle/): used after the timed regions to compare sampled outputs with the
    reference's arithmetic, and by the CPU-baseline legs; never inside a timed region."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    return oracle


def _row_rel_err(got, want):
    """max over rows of ||C - C_ref||_inf / ||C_ref row||_2 (the path's error metric)."""
    g, w = np.atleast_2d(got).astype(np.float64), np.atleast_2d(want).astype(np.float64)
    den = np.linalg.norm(w, axis=1)
    den = np.where(den == 0, 1.0, den)
    return float((np.abs(g - w).max(axis=1) / den).max()) if g.size else 0.0


# ---- clocks during the timed region (NVML, read-only) -------------------------------------

class ClockSampler:
    def __init__(self, device_index: int):
        self.samples, self.reasons = [], set()
        self.raw = 0  # union of the raw NVML clocks-event-reason bits seen
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        nv = self.nv
        names = {
            "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
            "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
            "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
        }
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.raw |= r
                for k, bit in names.items():
                    if r & bit and k != "gpu_idle":
                        self.reasons.add(k)
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self.nv:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread:
            self._stop.set()
            self._thread.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "samples": len(self.samples),
                "reasons": sorted(self.reasons), "reason_bits": hex(self.raw & ~0x1)}


# ---- distributed plumbing -----------------------------------------------------------------

def dist_setup(n_gpus: int):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---- the chain on the GPU -----------------------------------------------------------------

def quantize_on_device(W):
    """Synthetic-weight preparation (not timed): the library's GPU quantiser, bit for bit the
    reference's quantize_q8 (quant.cpp:6-28)."""
    import llme_b200 as L
    return L.quantize_q8(W.contiguous())


def gemv_shapes(copies=16):
    """Config 0: m = 1, 4096 x 4096 int8, over `copies` distinct weight matrices per step
    (16 x 16.8 MB = 268 MB > 2 x L2, so every product streams from HBM)."""
    return [(f"gemv{i}", DIM, DIM, False) for i in range(copies)]


class Chain:
    def __init__(self, world, rank, shapes, seed=3):
        import torch
        self.world, self.rank = world, rank
        self.shapes = shapes
        g = torch.Generator(device="cuda")
        self.mats = []  # (q, scale, k_loc, n_loc, row_parallel)
        for idx, (name, k, n, rowp) in enumerate(self.shapes):
            g.manual_seed(seed * 100003 + idx)
            W = torch.randn(k, n, generator=g, device="cuda") * 0.02
            q, s = quantize_on_device(W)
            del W
            if world > 1:
                import shard
                if rowp:
                    q = shard.row_shard(q, world, rank).contiguous()
                    kl, nl = q.shape[0], n
                else:
                    q, s = shard.column_shard(q, s, world, rank)
                    s = s.contiguous()
                    kl, nl = k, q.shape[1]
            else:
                kl, nl = k, n
            self.mats.append((q, s, kl, nl, rowp))
        torch.cuda.synchronize()
        # Activations: a fresh U(-1, 1) row per product, the same on every rank (a row shard
        # takes its slice of it). Outputs: one slot each, the row-parallel ones contiguous at
        # the end so one all-reduce covers them all.
        import shard
        self.a_off, self.c_off = [None] * len(self.mats), [None] * len(self.mats)
        a_tot = c_tot = 0
        for i, (_, _, kl, nl, _) in enumerate(self.mats):
            self.a_off[i] = a_tot
            a_tot += (kl + 3) // 4 * 4   # keep every vector 16-byte aligned
        for rowp_pass in (False, True):
            if rowp_pass:
                self.rp_off = c_tot
            for i, (_, _, kl, nl, rowp) in enumerate(self.mats):
                if rowp == rowp_pass:
                    self.c_off[i] = c_tot
                    c_tot += (nl + 3) // 4 * 4
        self.rp_count = c_tot - self.rp_off
        ga = torch.Generator(device="cpu")
        ga.manual_seed(seed * 7)
        a_host = torch.empty(a_tot)
        for i, (_, k, n, rowp) in enumerate(self.shapes):
            full = torch.rand(k, generator=ga) * 2 - 1
            kl = self.mats[i][2]
            s0 = shard.shard_range(k, world, rank)[0] if (rowp and world > 1) else 0
            a_host[self.a_off[i]:self.a_off[i] + kl] = full[s0:s0 + kl]
        self.a_host = a_host.pin_memory()
        self.c_host = torch.empty(c_tot, dtype=torch.float32).pin_memory()
        self.a_dev = self.a_host.cuda()
        self.c_dev = torch.empty(c_tot, dtype=torch.float32, device="cuda")
        self.bytes_per_step = sum(algorithmic_bytes(kl, nl) for (_, _, kl, nl, _) in self.mats) \
            * 1  # this rank's share
        self.total_bytes = sum(algorithmic_bytes(k, n) for (_, k, n, _) in self.shapes)

    def io(self):
        """The current activation / output buffers (and their batches)."""
        return (self.a_host, self.c_host, self.a_dev, self.c_dev, getattr(self, "batches", None))

    def use_io(self, io):
        self.a_host, self.c_host, self.a_dev, self.c_dev, b = io
        if b is not None:
            self.batches = b

    def add_io_set(self):
        """Switches to a second set of activation / output buffers (same inputs, same weights;
        batches rebuilt for them), so consecutive steps can overlap their copies."""
        import torch
        self.a_host = self.a_host.clone().pin_memory()
        self.c_host = torch.empty_like(self.c_host).pin_memory()
        self.a_dev = torch.empty_like(self.a_dev)
        self.c_dev = torch.empty_like(self.c_dev)
        if getattr(self, "batches", None) is not None:
            self.make_batch()
        return self.io()

    def make_batch(self):
        """The step's products as grouped launches (they are independent): one batch on one
        GPU; on several, the row-parallel products first (their partial outputs are summed
        while the column-parallel batch runs) and the column-parallel ones second."""
        import llme_b200 as L
        prods = {False: [], True: []}
        for i, (q, s, kl, nl, rowp) in enumerate(self.mats):
            prods[rowp and self.world > 1].append(
                (nl, kl, self.a_dev.data_ptr() + 4 * self.a_off[i], q.data_ptr(), s.data_ptr(),
                 self.c_dev.data_ptr() + 4 * self.c_off[i], 0))
        self.batches = [L.Batch(1, prods[True])] if prods[True] else []
        self.batches.append(L.Batch(1, prods[False]))
        self.all_batches = getattr(self, "all_batches", []) + self.batches

    def launch_grouped(self, stream_handle, tp=None, comm_stream=None, fused=False):
        import torch
        import llme_b200 as L
        if tp is None or len(self.batches) == 1:
            for b in self.batches:
                b.run(L.FLAG_WEIGHTS_STATIC, stream_handle)
            return
        row, col = self.batches
        if fused:
            # The rank sum of the row-parallel products inside their grouped launch.
            row.run_rowpar(tp, L.FLAG_WEIGHTS_STATIC, stream_handle)
            col.run(L.FLAG_WEIGHTS_STATIC, stream_handle)
            return
        row.run(L.FLAG_WEIGHTS_STATIC, stream_handle)
        comm_stream.wait_stream(torch.cuda.current_stream())
        tp.allreduce_sum_f32(self.c_dev.data_ptr() + 4 * self.rp_off, self.rp_count,
                             comm_stream.cuda_stream)
        col.run(L.FLAG_WEIGHTS_STATIC, stream_handle)
        torch.cuda.current_stream().wait_stream(comm_stream)

    def destroy_batches(self):
        for b in getattr(self, "all_batches", []):
            b.destroy()

    def launch_all(self, stream_handle, comm=None, join=None):
        import llme_b200 as L
        for i, (q, s, kl, nl, rowp) in enumerate(self.mats):
            a = self.a_dev.data_ptr() + 4 * self.a_off[i]
            c = self.c_dev.data_ptr() + 4 * self.c_off[i]
            L.matmul_cuda_q8(1, nl, kl, a, q.data_ptr(), s.data_ptr(), c, "automatic", False, 0,
                             L.FLAG_WEIGHTS_STATIC, stream_handle)
            if rowp and comm is not None:
                comm(c, nl)
        if join is not None:
            join()

    def n_launches(self):
        return len(self.mats)


def capture(fn, stream):
    import torch
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        fn()  # warm (lazy module loading, tensor-map cache, scratch growth)
    torch.cuda.synchronize()
    with torch.cuda.graph(g, stream=stream):
        fn()
    torch.cuda.synchronize()
    return g


def time_graph(graph, steps, warmup, stream, world, sampler=None):
    import torch
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx = sampler if sampler is not None else _Null()
    # LLME_PROFILE_REGION=1 brackets the timed replays with cudaProfilerStart/Stop, so
    # `ncu --profile-from-start off` sees exactly the timed launches.
    profile = os.environ.get("LLME_PROFILE_REGION") == "1"
    with ctx:
        if profile:
            torch.cuda.cudart().cudaProfilerStart()
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(steps):
                graph.replay()
            end.record(stream)
        torch.cuda.synchronize()
        if profile:
            torch.cuda.cudart().cudaProfilerStop()
    barrier(world)
    torch.cuda.synchronize()
    return start.elapsed_time(end) / 1e3


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def gemv_4096_probe(steps=200):
    """Config 0 in isolation: m = 1, 4096 x 4096 int8, back to back over 16 weight copies
    (268 MB > 2 x L2), with and without programmatic dependent launch; and, where it is built,
    the reference's own GPU matmul on the same weights and activation (reference_gpu)."""
    import torch
    import llme_b200 as L
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    copies = 16
    qs, ss = [], []
    for i in range(copies):
        W = torch.randn(DIM, DIM, generator=g, device="cuda") * 0.02
        q, s = quantize_on_device(W)
        qs.append(q)
        ss.append(s)
    A = torch.rand(DIM, generator=g, device="cuda") * 2 - 1
    C = torch.empty(copies, DIM, device="cuda")
    stream = torch.cuda.Stream()
    h = stream.cuda_stream
    nbytes = algorithmic_bytes(DIM, DIM)
    res = {}
    for label, flags in (("pdl", L.FLAG_WEIGHTS_STATIC), ("serial", 0)):
        def fn():
            for i in range(copies):
                L.matmul_cuda_q8(1, DIM, DIM, A.data_ptr(), qs[i].data_ptr(), ss[i].data_ptr(),
                                 C[i].data_ptr(), "automatic", False, 0, flags, h)
        graph = capture(fn, stream)
        secs = time_graph(graph, steps, 5, stream, 1)
        us = secs / (steps * copies) * 1e6
        res[label] = {"us_per_gemv": round(us, 3), "GB_s": round(nbytes / (us * 1e-6) / 1e9, 1)}
        del graph
    ref = ref_matmul_gpu()
    if ref is not None:
        C_ref = torch.empty(copies, DIM, device="cuda")

        def calls(ok):
            for i in range(copies):
                ok(ref.ref_gpu_matmul_q8(1, DIM, DIM, A.data_ptr(), qs[i].data_ptr(),
                                         ss[i].data_ptr(), C_ref[i].data_ptr(), 0, 0, None))
        secs = time_ref_matmul_gpu(ref, calls, steps, 5)
        us = secs / (steps * copies) * 1e6
        torch.cuda.synchronize()
        diff = float((C - C_ref).abs().max())
        res["reference_gpu"] = {
            "us_per_gemv": round(us, 3), "GB_s": round(nbytes / (us * 1e-6) / 1e9, 1),
            "impl": "the reference's matmul_cuda (src/cuda_matmul.cu built for sm_100a), "
                    "GpuKernel::automatic, 16 calls captured on its per-thread stream",
            "max_abs_diff_vs_ours": float(f"{diff:.3e}"), "tolerance": 2e-5 * DIM}
    return res


def chain_per_call_beside_reference(chain, steps=50, warmup=5):
    """Layer 0's seven products and the classifier, one call each (the reference's
    CudaTransformer call pattern), on the chain's own weights and activations: this library's
    llme_matmul_q8 against the reference's own matmul_cuda built for sm_100a, each captured
    as one CUDA graph. None where the reference's GPU library is not built."""
    import torch
    import llme_b200 as L
    ref = ref_matmul_gpu()
    if ref is None:
        return None
    idx = list(range(7)) + [len(chain.mats) - 1]
    outs = {"ours": torch.empty_like(chain.c_dev), "reference": torch.empty_like(chain.c_dev)}
    nbytes = sum(algorithmic_bytes(chain.mats[i][2], chain.mats[i][3]) for i in idx)
    stream = torch.cuda.Stream()
    h = stream.cuda_stream

    def ours():
        for i in idx:
            q, s, kl, nl, _ = chain.mats[i]
            L.matmul_cuda_q8(1, nl, kl, chain.a_dev.data_ptr() + 4 * chain.a_off[i], q.data_ptr(),
                             s.data_ptr(), outs["ours"].data_ptr() + 4 * chain.c_off[i],
                             "automatic", False, 0, L.FLAG_WEIGHTS_STATIC, h)

    def theirs(ok):
        for i in idx:
            q, s, kl, nl, _ = chain.mats[i]
            ok(ref.ref_gpu_matmul_q8(1, nl, kl, chain.a_dev.data_ptr() + 4 * chain.a_off[i],
                                     q.data_ptr(), s.data_ptr(),
                                     outs["reference"].data_ptr() + 4 * chain.c_off[i], 0, 0,
                                     None))
    graph = capture(ours, stream)
    secs_ours = time_graph(graph, steps, warmup, stream, 1)
    del graph
    secs_ref = time_ref_matmul_gpu(ref, theirs, steps, warmup)
    torch.cuda.synchronize()
    diff = max(float((outs["ours"][chain.c_off[i]:chain.c_off[i] + chain.mats[i][3]] -
                      outs["reference"][chain.c_off[i]:chain.c_off[i] + chain.mats[i][3]])
                     .abs().max()) for i in idx)
    us_o, us_r = secs_ours / steps * 1e6, secs_ref / steps * 1e6
    return {"products": "layer 0 (wq, wk, wv, wo, w1, w3, w2) + classifier, m=1, one call each",
            "ours": {"us_per_step": round(us_o, 2), "GB_s": round(nbytes / us_o / 1e3, 1)},
            "reference_gpu": {"us_per_step": round(us_r, 2), "GB_s": round(nbytes / us_r / 1e3, 1)},
            "speedup": round(us_r / us_o, 2),
            "max_abs_diff": float(f"{diff:.3e}"),
            "impl": "the reference's matmul_cuda (src/cuda_matmul.cu built for sm_100a), "
                    "GpuKernel::automatic, captured on its per-thread stream"}


def chain_parity(chain, world):
    """After the timed regions: the outputs of one grouped step (run again on the first buffer
    set) for layer 0's seven products, the last layer's w2 and the classifier, against the
    oracle's matmul_naive_q8 on the same int8 weights and activations, within the reference's
    own test bound of 1e-5 * k. On several GPUs only the column-parallel products (complete
    local slices) are compared."""
    oracle = _oracle()
    n = len(chain.mats)
    pick = sorted(set([i for i in range(min(7, n))] + [max(0, n - 2), n - 1]))
    a = chain.a_dev.cpu().numpy()
    c = chain.c_dev.cpu().numpy()
    worst_ratio, worst_rel, checked = 0.0, 0.0, []
    for i in pick:
        q, s, kl, nl, rowp = chain.mats[i]
        if rowp and world > 1:
            continue
        A = a[chain.a_off[i]:chain.a_off[i] + kl][None]
        got = c[chain.c_off[i]:chain.c_off[i] + nl][None]
        want = oracle.matmul_naive_q8(A, q.cpu().numpy(), s.cpu().numpy())
        worst_ratio = max(worst_ratio, float(np.abs(got.astype(np.float64) - want).max())
                          / (1e-5 * kl))
        worst_rel = max(worst_rel, _row_rel_err(got, want))
        checked.append(chain.shapes[i][0])
    return {"ok": bool(worst_ratio <= 1.0), "max_err_over_tolerance": float(f"{worst_ratio:.3e}"),
            "row_rel_err": float(f"{worst_rel:.3e}"),
            "tolerance": "1e-5 * k per element (the reference's tests/test_cuda.cpp bound)",
            "products_checked": checked,
            "against": "oracle matmul_naive_q8 on the same int8 weights and activations"}


def sgemm_line(n, steps, warmup, world, local, check_rows=0):
    """The square SGEMM: C = A x B, fp32 N x N, A and B ~ U(-1, 1) (seed 2), through the
    C ABI on the tcgen05 TF32 path (B read as stored, MN-major). Inputs 768 MB > L2. With
    check_rows > 0, that many rows of C are compared with the oracle after the timed region."""
    import torch
    import llme_b200 as L
    g = torch.Generator(device="cuda")
    g.manual_seed(2)
    A = torch.rand(n, n, generator=g, device="cuda") * 2 - 1
    B = torch.rand(n, n, generator=g, device="cuda") * 2 - 1
    C = torch.empty(n, n, device="cuda")
    plan = L.plan(n, n, n, q8=False, a_addr=A.data_ptr(), b_addr=B.data_ptr())
    stream = torch.cuda.Stream()
    h = stream.cuda_stream
    graph = capture(lambda: L.matmul_cuda_f32(n, n, n, A.data_ptr(), B.data_ptr(), C.data_ptr(),
                                              "automatic", False, 0, L.FLAG_WEIGHTS_STATIC, h),
                    stream)
    sampler = ClockSampler(local)
    secs = max_over_ranks(time_graph(graph, steps, warmup, stream, world, sampler), world)
    del graph
    flops = 2.0 * n ** 3
    tflops = flops * steps * world / secs / 1e12
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            bf16 = float(json.load(f)["bf16_tflops"])
        peak, kind = bf16 / 2, "half of measured bf16 burst (TF32 runs at half the bf16 rate)"
    except Exception:
        peak, kind = 1590.0 / 2, "half of fallback bf16"
    line = {"metric": f"TF32 GEMM TFLOP/s ({n}^3, fp32 in/out)", "value": round(tflops, 1),
            "unit": "TFLOP/s", "n_gpus": world, "steps": steps, "warmup": warmup,
            "ms_per_step": round(secs / steps * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "tf32",
            "data": "synthetic U(-1,1)",
            "config": {"workload": "square fp32 SGEMM on the TF32 tcgen05 path (BASELINE configs[2])",
                       "N": n, "path": plan["path_name"],
                       "l2": "no flush: 768 MB of operands (> 126 MB L2)"},
            "roofline": {"bound": "tensor", "achieved": round(tflops / world, 1), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(tflops / world / peak, 4),
                         "peak_kind": kind, "kernel": "gemm_tf32_kernel",
                         "traffic": None},
            "gpu_launches": steps, "clocks": sampler.summary()}
    if check_rows:
        # The checker (oracle/) after the timed region: sampled rows of C against
        # matmul_naive of those rows of A, at the TF32 path's 5e-3 row bound.
        oracle = _oracle()
        rng = np.random.default_rng(2)
        rows = np.unique(np.concatenate([[0, n - 1], rng.choice(n, check_rows - 2, replace=False)]))
        got = C[torch.from_numpy(rows).cuda()].cpu().numpy()
        want = oracle.matmul_naive(A[torch.from_numpy(rows).cuda()].cpu().numpy(), B.cpu().numpy())
        err = _row_rel_err(got, want)
        line["parity"] = {"ok": bool(err <= 5e-3), "row_rel_err": float(f"{err:.3e}"),
                          "bound": 5e-3, "rows_checked": int(rows.size),
                          "against": "oracle matmul_naive on the sampled rows"}
    del A, B, C
    return line


def run_sgemm(args, world, rank, local):
    line = sgemm_line(args.size, args.steps, args.warmup, world, local,
                      check_rows=0 if args.no_extras else 16)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if "parity" in line and not line["parity"]["ok"]:
        raise SystemExit(3)


# ---- the decode-shaped sweep ------------------------------------------------------------

SWEEP_ROWS = (1, 4, 16, 64)
SWEEP_COPIES = 12  # distinct 4096 x 4096 weights per case (201 MB int8 / 805 MB fp32 > L2)
SWEEP_METRIC = "decode sweep GB/s (m in {1,4,16,64} x 4096^2, fp32 and int8 W, per call)"


def ref_matmul_gpu():
    """The reference's own GPU matmul (src/cuda_matmul.cu for sm_100a, built into
    oracle/_ref/libref_matmul_gpu.so by `make -C oracle refmatmul`), or None: timed only by
    the reference arm (`--impl reference --workload sweep`)."""
    import ctypes
    path = os.path.join(REPO, "oracle", "_ref", "libref_matmul_gpu.so")
    if not os.path.exists(path):
        return None
    lib = ctypes.CDLL(path)
    sz, vp, ci = ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int
    lib.ref_gpu_matmul_f32.argtypes = [sz, sz, sz, vp, vp, vp, ci, ci, vp]
    lib.ref_gpu_matmul_q8.argtypes = [sz, sz, sz, vp, vp, vp, vp, ci, ci, vp]
    lib.ref_gpu_error.restype = ctypes.c_char_p
    lib.ref_gpu_capture_end.argtypes = [ctypes.POINTER(vp)]
    lib.ref_gpu_time_graph.argtypes = [vp, ci, ci, ctypes.POINTER(ctypes.c_float)]
    lib.ref_gpu_graph_destroy.argtypes = [vp]
    return lib


def time_ref_matmul_gpu(ref, calls, steps, warmup):
    """Seconds for `steps` replays of the reference's calls captured as one CUDA graph on the
    stream they launch on (its per-thread default stream), after one eager pass that grows its
    scratch -- the way its CudaTransformer captures its decode step."""
    import ctypes
    import torch

    def ok(rc):
        if rc:
            raise RuntimeError("reference GPU matmul: " + ref.ref_gpu_error().decode())
    torch.cuda.synchronize()  # inputs written on torch's streams are in place
    calls(ok)
    ok(ref.ref_gpu_synchronize())
    ok(ref.ref_gpu_capture_begin())
    calls(ok)
    graph = ctypes.c_void_p()
    ok(ref.ref_gpu_capture_end(ctypes.byref(graph)))
    ms = ctypes.c_float()
    try:
        ok(ref.ref_gpu_time_graph(graph, steps, warmup, ctypes.byref(ms)))
    finally:
        ref.ref_gpu_graph_destroy(graph)
    return ms.value / 1e3


def run_sweep(args, world, rank, local):
    """m in {1, 4, 16, 64} x 4096 x 4096, fp32 and int8 weights (N(0, 0.02^2), seed 1, the
    int8 ones quantised as quant.cpp does), U(-1, 1) activations: one C-ABI call per product,
    12 distinct weights per case captured in one CUDA graph. `value` is the sweep's total
    algorithmic bytes over its total time; every case is reported in `cases`."""
    import torch
    import llme_b200 as L
    g = torch.Generator(device="cuda")
    g.manual_seed(1)
    stream = torch.cuda.Stream()
    h = stream.cuda_stream
    sampler = ClockSampler(local)
    cases, tot_bytes, tot_s, launches = [], 0, 0.0, 0
    for q8 in (False, True):
        Ws = [torch.randn(DIM, DIM, generator=g, device="cuda") * 0.02 for _ in range(SWEEP_COPIES)]
        if q8:
            Ws = [quantize_on_device(w) for w in Ws]
        for m in SWEEP_ROWS:
            A = torch.rand(m, DIM, generator=g, device="cuda") * 2 - 1
            C = torch.empty(m, DIM, device="cuda")

            def fn():
                for i in range(SWEEP_COPIES):
                    if q8:
                        q, sc = Ws[i]
                        L.matmul_cuda_q8(m, DIM, DIM, A.data_ptr(), q.data_ptr(), sc.data_ptr(),
                                         C.data_ptr(), "automatic", False, 0,
                                         L.FLAG_WEIGHTS_STATIC, h)
                    else:
                        L.matmul_cuda_f32(m, DIM, DIM, A.data_ptr(), Ws[i].data_ptr(),
                                          C.data_ptr(), "automatic", False, 0,
                                          L.FLAG_WEIGHTS_STATIC, h)
            graph = capture(fn, stream)
            secs = max_over_ranks(time_graph(graph, args.steps, args.warmup, stream, world,
                                             sampler if q8 and m == 64 else None), world)
            del graph
            nbytes = (algorithmic_bytes(DIM, DIM, m) if q8 else
                      4 * DIM * DIM + 4 * m * DIM + 4 * m * DIM)
            us = secs / (args.steps * SWEEP_COPIES) * 1e6
            path = L.plan(m, DIM, DIM, q8=q8)["path_name"]
            # launches per call: the split pass before the three-term int8 kernel, else one
            per_call = 2 if path == "tcgen05_skinny" else 1
            launches += per_call * SWEEP_COPIES * args.steps
            cases.append({"w": "int8" if q8 else "fp32", "m": m, "us": round(us, 2),
                          "GB_s": round(nbytes / us / 1e3, 1), "path": path,
                          "launches_per_call": per_call})
            tot_bytes += nbytes * args.steps * SWEEP_COPIES
            tot_s += secs
    hbm, hbm_kind = peaks()
    value = tot_bytes / tot_s / 1e9
    cpu = cpu_sweep_sample() if rank == 0 and world == 1 and not args.no_extras else None
    line = {"metric": SWEEP_METRIC,
            "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(tot_s / args.steps * 1e3, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: N(0,0.02^2) weights (seed 1), U(-1,1) activations",
            "config": {"workload": "decode-shaped sweep (BASELINE configs[1]), one C-ABI call "
                                   "per product, 12 distinct weights per case in a CUDA graph",
                       "l2": "no flush: 12 distinct weights per case (201 MB int8, 805 MB fp32)"},
            "cases": cases,
            "roofline": {"bound": "hbm", "achieved": round(value, 1), "peak": hbm,
                         "unit": "GB/s", "frac": round(value / hbm, 4), "peak_kind": hbm_kind,
                         "kernel": "per case (see cases[].path)", "traffic": None},
            "gpu_launches": launches, "clocks": sampler.summary()}
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if rank == 0:
        print(json.dumps(line), flush=True)


def cpu_sweep_sample(budget_s=2.0):
    """The reference's matmul_parallel on each sweep case (one 4096 x 4096 weight, fp32 and
    int8), on all host cores: the same total-bytes / total-time figure as the GPU line."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle  # the CPU baseline leg only
    rng = np.random.default_rng(1)
    W = (rng.standard_normal((DIM, DIM), dtype=np.float32) * 0.02).astype(np.float32)
    kind = "reference" if oracle.Reference.available(fast=True) else "port"
    ref = oracle.Reference(fast=True) if kind == "reference" else None
    q, sc = ref.quantize_q8(W) if ref else oracle.quantize_q8(W)
    qh = ref.qtensor(q, sc) if ref else None
    wh = ref.tensor(W) if ref else None  # weights held on the reference side, not copied per call
    cases, tb, ts = [], 0, 0.0
    for q8 in (False, True):
        for m in SWEEP_ROWS:
            A = rng.uniform(-1, 1, (m, DIM)).astype(np.float32)
            if ref:
                one = (lambda: ref.matmul_parallel_q8(A, qh)) if q8 else \
                    (lambda: ref.matmul_parallel_h(A, wh))
            else:
                one = (lambda: oracle.matmul_parallel(A, q=q, scale=sc)) if q8 else \
                    (lambda: oracle.matmul_parallel(A, W))
            one()
            times, t_end = [], time.perf_counter() + budget_s
            while time.perf_counter() < t_end or len(times) < 3:
                t0 = time.perf_counter()
                one()
                times.append(time.perf_counter() - t0)
            med = statistics.median(times)
            nbytes = algorithmic_bytes(DIM, DIM, m) if q8 else 4 * DIM * DIM + 8 * m * DIM
            cases.append({"w": "int8" if q8 else "fp32", "m": m, "us": round(med * 1e6, 1)})
            tb += nbytes
            ts += med
    return {"value": round(tb / ts / 1e9, 2), "unit": "GB/s",
            "cores": ref.threads() if ref else oracle.default_threads(), "kind": kind,
            "sample": "each sweep case once (median of repeated calls, about 2 s per case)",
            "cases": cases}


# ---- decode attention over a KV cache (the path after wqkv) ----------------------------------

ATTN_CASES = [  # (name, heads, kv heads, head size, cached positions)
    ("7B MHA", 32, 32, 128, 4096),
    ("7B GQA 32/8", 32, 8, 128, 4096),
    ("MQA long context", 4, 1, 128, 20000),
]
ATTN_LAYERS = 8  # distinct caches per step, so the keys and values come from HBM
ATTN_METRIC = "decode attention GB/s (KV-cache bytes, 1 row)"


def run_tp_decode(args, world, rank, local):
    """Decode tokens/s of a 7B-shaped int8 transformer (32 layers, dim 4096, 32 heads, hidden
    11008, vocab 32000; the reference's CudaTransformer architecture, src/cuda_model.cu) run by
    the library's C++ engine (llme_model_*), split over N GPUs: heads by kv head,
    column-parallel wqkv / w13 / classifier, row-parallel wo / w2 with the NVLink peer
    all-reduce carrying the residual add. One step = one token at context length --context (a
    synthetic history in the caches), the engine's captured CUDA graph of the step replayed.
    Synthetic weights drawn on the device."""
    import time
    import torch
    import llme_b200 as L
    ctx = args.context
    cfg = dict(dim=DIM, hidden_dim=HIDDEN, n_layers=args.layers, n_heads=32, n_kv_heads=32,
               vocab_size=VOCAB, seq_len=ctx + 16)
    comm = None
    if world > 1:
        import torch.distributed as dist
        uid = [L.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = L.Comm(world, rank, uid[0], timeout_s=60.0)
        comm.enable_peer(VOCAB)  # the largest all-reduce of a decode step: the logits
    model = L.Model.synthetic(cfg, q8=True, world=world, rank=rank, comm=comm, seed=5)
    model.fill_history(ctx, seed=11)  # the keys and values of ctx earlier positions
    model.decode(1, ctx)  # eager step (grows every buffer), then the step is captured
    model.decode(1, ctx)  # one replay through the captured graph
    stream = torch.cuda.Stream()
    h = stream.cuda_stream
    for _ in range(args.warmup):
        model.replay(1, h)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with sampler:
        e0.record(stream)
        model.replay(args.steps, h)
        e1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    secs = max_over_ranks(e0.elapsed_time(e1) / 1e3, world)
    tokens_s = args.steps / secs
    # Kernels of one token: embed; per layer wqkv (+ RoPE + cache write in its epilogue),
    # attention, wo, w13 (+ SwiGLU in its epilogue), w2; the classifier (+ its all-reduce at
    # N > 1). At N > 1 the sums after wo and w2 run inside those GEMVs when every rank's shard
    # has the same size (hidden % N == 0), else as two more all-reduce launches per layer.
    separate_sums = world > 1 and cfg["hidden_dim"] % world != 0
    # the attention: its split kernel, and the merge launch when the context spans chunks (the
    # engine's per-rank shape: this rank's heads over the qkv row it writes)
    part = L.model_partition(cfg, world, rank)
    hs = cfg["dim"] // cfg["n_heads"]
    attn_launches = L.attention_launches(L.AttentionShape(
        part["nq"], part["nkv"], hs, cfg["seq_len"], (part["nq"] + 2 * part["nkv"]) * hs,
        part["nkv"] * hs, part["nq"] * hs), 1)
    launches_per_token = (1 + cfg["n_layers"] * (4 + attn_launches + (2 if separate_sums else 0))
                          + 1 + (1 if world > 1 else 0))
    w_bytes, kv_per_pos = model.stream_bytes()
    per_gpu = w_bytes + kv_per_pos * (ctx + 1)
    hbm, hbm_kind = peaks()
    achieved = per_gpu / (secs / args.steps) / 1e9

    # e2e: llme_model_decode per token -- the token and position copied in, the logits copied
    # out and the host waiting for them, as a caller sampling tokens does.
    for _ in range(3):
        model.decode(1, ctx)
    barrier(world)
    t0 = time.perf_counter()
    e2e_steps = min(args.steps, 100)
    for _ in range(e2e_steps):
        model.decode(1, ctx)
    e2e_secs = max_over_ranks(time.perf_counter() - t0, world)
    line = {"metric": f"decode tokens/s (7B-shaped int8 transformer, tensor-parallel over N GPUs, "
                      f"context {ctx})",
            "value": round(tokens_s, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(secs / args.steps * 1e3, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8 W, f32",
            "data": "synthetic: N(0,0.02^2) weights drawn on the device, quantised per column; "
                    "U(-1,1) embedding and KV history",
            "config": {"workload": "tensor-parallel transformer decode, one token per step",
                       "layers": cfg["n_layers"], "dim": DIM, "hidden": HIDDEN, "heads": 32,
                       "vocab": VOCAB, "context": ctx, "parallelism": f"tp{world}",
                       "engine": "the library's C++ transformer engine (llme_model_*)",
                       "launch": "one CUDA graph per token: embed, per layer rmsnorm+wqkv with "
                                 "RoPE and the cache write in the GEMV epilogue, attention, "
                                 "wo with the residual, rmsnorm+w13 with SwiGLU in the GEMV "
                                 "epilogue, w2 with the residual; classifier. At N > 1 the rank "
                                 "sums of wo and w2 run inside their GEMVs (each CTA exchanges "
                                 "its columns with the same CTA of every rank over NVLink); "
                                 "the classifier's logits are summed by the peer all-reduce",
                       "l2": f"no flush: {per_gpu / 1e9:.2f} GB per token per GPU (> L2)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm,
                         "unit": "GB/s", "frac": round(achieved / hbm, 4), "peak_kind": hbm_kind,
                         "kernel": "whole decode step (per GPU)",
                         "bytes_per_token_per_gpu": per_gpu, "traffic": None},
            "e2e": {"value": round(e2e_steps / e2e_secs, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4 * VOCAB},
            "gpu_launches": launches_per_token * args.steps, "cpu_baseline": None,
            "cpu_baseline_note": "the reference's CPU Transformer needs a 27 GB fp32 checkpoint at "
                                 "this size; its parity is tested on small checkpoints",
            "clocks": sampler.summary()}
    model.destroy()
    torch.cuda.synchronize()
    if comm is not None:
        comm.destroy()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def attention_case_inputs(torch, g, heads, kvh, hs, T):
    """One attention case's inputs drawn from `g` in a fixed order, so both arms of the
    attention benchmark see the same bytes: the query row, ATTN_LAYERS key and value caches of
    T positions, and the position (the last cached one) in device memory."""
    kv, dim = kvh * hs, heads * hs
    q = torch.rand(1, dim + 2 * kv, generator=g, device="cuda") * 2 - 1
    ks = [torch.rand(T, kv, generator=g, device="cuda") * 2 - 1 for _ in range(ATTN_LAYERS)]
    vs = [torch.rand(T, kv, generator=g, device="cuda") * 2 - 1 for _ in range(ATTN_LAYERS)]
    pos = torch.full((1,), T - 1, dtype=torch.int32, device="cuda")
    return q, ks, vs, pos


def attention_case_bytes(heads, kvh, hs, T):
    """Algorithmic bytes of one call: the context's keys and values, the query and output rows."""
    return 2 * T * kvh * hs * 4 + heads * hs * 4 * 2


def run_attention(args, world, rank, local):
    """One decode row (position = the last cached one) through each case, per layer cache,
    one call each, in a CUDA graph through this library's llme_attention (split kernel).
    `--impl reference --workload attention` times the reference's own GPU kernel on the same
    inputs. Bytes per call: the keys and values of the context + the query row + the output
    row."""
    import torch
    import llme_b200 as L
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    stream = torch.cuda.Stream()
    h = stream.cuda_stream
    sampler = ClockSampler(local)
    cases = []
    tot_bytes = tot_s = 0.0
    for name, heads, kvh, hs, T in ATTN_CASES:
        kv, dim = kvh * hs, heads * hs
        shape = L.AttentionShape(heads, kvh, hs, T, dim + 2 * kv, kv, dim)
        q, ks, vs, pos = attention_case_inputs(torch, g, heads, kvh, hs, T)
        nbytes = attention_case_bytes(heads, kvh, hs, T)
        out = torch.zeros(ATTN_LAYERS, dim, device="cuda")
        scratch = torch.zeros(max(1, L.attention_scratch_floats(shape, 1, "automatic")),
                              device="cuda")

        def fn():
            for l in range(ATTN_LAYERS):
                L.attention(shape, 1, pos.data_ptr(), q.data_ptr(), ks[l].data_ptr(),
                            vs[l].data_ptr(), out[l].data_ptr(), scratch.data_ptr(),
                            "automatic", h)
        graph = capture(fn, stream)
        secs = max_over_ranks(time_graph(graph, args.steps, args.warmup, stream, world,
                                         sampler if name == "7B MHA" else None), world)
        del graph
        us = secs / (args.steps * ATTN_LAYERS) * 1e6
        cases.append({"case": name, "heads": heads, "kv_heads": kvh, "head_size": hs,
                      "positions": T, "ours": {"us": round(us, 2),
                                               "GB_s": round(nbytes / us / 1e3, 1)}})
        tot_bytes += nbytes * args.steps * ATTN_LAYERS
        tot_s += secs
    hbm, hbm_kind = peaks()
    value = tot_bytes / tot_s / 1e9
    line = {"metric": ATTN_METRIC,
            "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(tot_s / args.steps * 1e3, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic U(-1,1) queries and caches",
            "config": {"workload": "decode attention over KV caches (the path after wqkv, "
                                   "reference cuda_attention.cu), 8 layer caches per case",
                       "l2": "no flush: 8 distinct caches per case"},
            "cases": cases,
            "roofline": {"bound": "hbm", "achieved": round(value, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(value / hbm, 4), "peak_kind": hbm_kind,
                         "kernel": "attn_split_kernel", "traffic": None},
            "gpu_launches": sum(L.attention_launches(L.AttentionShape(
                h, kvh, hs, T, h * hs + 2 * kvh * hs, kvh * hs, h * hs), 1)
                for _, h, kvh, hs, T in ATTN_CASES) * ATTN_LAYERS * args.steps,
            "clocks": sampler.summary()}
    if rank == 0:
        print(json.dumps(line), flush=True)


# ---- the 7B-shaped prefill (m = 512) ---------------------------------------------------

PREFILL_ROWS = 512
PREFILL_METRIC = "prefill GEMM TFLOP/s (7B-shaped int8 weights, m=512)"


class Prefill:
    """Every product of the 7B-shaped layer stack at m = 512 rows (the classifier on the last
    row only), int8 weights drawn N(0, 0.02^2) with seed 4 and quantised per column, a fresh
    U(-1, 1) activation matrix per product. On N GPUs: column-parallel weights split along n,
    row-parallel (wo, w2) along k with a sum all-reduce of the m x 4096 partial outputs."""

    def __init__(self, world, rank, seed=4, layers=LAYERS):
        import torch
        import shard
        self.world, self.rank = world, rank
        self.shapes = chain_shapes(layers)
        g = torch.Generator(device="cuda")
        ga = torch.Generator(device="cuda")
        ga.manual_seed(seed * 7)
        self.items = []  # (q, s, m, k_loc, n_loc, rowp, A_dev, C_dev)
        for idx, (name, k, n, rowp) in enumerate(self.shapes):
            g.manual_seed(seed * 100003 + idx)
            W = torch.randn(k, n, generator=g, device="cuda") * 0.02
            q, s = quantize_on_device(W)
            del W
            m = 1 if name == "cls" else PREFILL_ROWS
            A = torch.rand(m, k, generator=ga, device="cuda") * 2 - 1  # same on every rank
            if world > 1:
                if rowp:
                    q = shard.row_shard(q, world, rank).contiguous()
                    s0, kl = shard.shard_range(k, world, rank)
                    A = A[:, s0:s0 + kl].contiguous()
                else:
                    q, s = shard.column_shard(q, s, world, rank)
                    q, s = q.contiguous(), s.contiguous()
            kl, nl = q.shape
            C = torch.empty(m, nl, device="cuda")
            self.items.append((q, s, m, kl, nl, rowp, A, C))
        torch.cuda.synchronize()
        self.flops_total = sum(2.0 * (1 if nm == "cls" else PREFILL_ROWS) * k * n
                               for (nm, k, n, _) in self.shapes)
        self.flops_rank = sum(2.0 * m * kl * nl for (_, _, m, kl, nl, _, _, _) in self.items)
        # This rank's algorithmic bytes: the GEMMs read W, the hi/lo rows and write C; the
        # split reads A and writes hi/lo (the classifier GEMV's bytes are in the GEMM share).
        self.gemm_bytes = sum(kl * nl + 4 * nl + 2 * m * kl + 4 * m * nl
                              for (_, _, m, kl, nl, _, _, _) in self.items)
        self.split_bytes = sum(6 * m * kl for (_, _, m, kl, nl, _, _, _) in self.items if m > 1)
        self.a_host = [it[6].cpu().pin_memory() for it in self.items]
        self.c_host = [torch.empty(it[7].shape).pin_memory() for it in self.items]

    def launch_all(self, stream_handle, comm=None, join=None):
        import llme_b200 as L
        for (q, s, m, kl, nl, rowp, A, C) in self.items:
            L.matmul_cuda_q8(m, nl, kl, A.data_ptr(), q.data_ptr(), s.data_ptr(), C.data_ptr(),
                             "automatic", False, 0, L.FLAG_WEIGHTS_STATIC, stream_handle)
            if rowp and comm is not None:
                comm(C.data_ptr(), m * nl)
        if join is not None:
            join()

    def make_batch(self):
        """The m = 512 products as grouped launches (they are independent): one batch on one
        GPU; on several, the row-parallel products first (their partial outputs are summed
        while the column-parallel batch runs) and the column-parallel ones second. The
        classifier (last row only, m = 1) stays a single GEMV call."""
        import llme_b200 as L
        prods = {False: [], True: []}
        for (q, s, m, kl, nl, rowp, A, C) in self.items:
            if m == PREFILL_ROWS:
                prods[rowp and self.world > 1].append(
                    (nl, kl, A.data_ptr(), q.data_ptr(), s.data_ptr(), C.data_ptr(), 0))
        self.batches = [L.Batch(PREFILL_ROWS, prods[True])] if prods[True] else []
        self.batches.append(L.Batch(PREFILL_ROWS, prods[False]))
        self.all_batches = self.batches

    def launch_grouped(self, stream_handle, comm=None, join=None):
        import llme_b200 as L
        for b in self.batches:
            b.run(0, stream_handle)
            if comm is not None and b is self.batches[0] and len(self.batches) > 1:
                for (q, s, m, kl, nl, rowp, A, C) in self.items:
                    if rowp:
                        comm(C.data_ptr(), m * nl)
        for (q, s, m, kl, nl, rowp, A, C) in self.items:
            if m != PREFILL_ROWS:
                L.matmul_cuda_q8(m, nl, kl, A.data_ptr(), q.data_ptr(), s.data_ptr(),
                                 C.data_ptr(), "automatic", False, 0, L.FLAG_WEIGHTS_STATIC,
                                 stream_handle)
        if join is not None:
            join()

    def destroy_batches(self):
        for b in getattr(self, "all_batches", []):
            b.destroy()

    def launches(self):
        import llme_b200 as L
        n = 0
        for (q, s, m, kl, nl, rowp, A, C) in self.items:
            p = L.plan(m, nl, kl, q8=True, a_addr=A.data_ptr(), b_addr=q.data_ptr())
            n += 2 if p["path_name"] == "tcgen05_q8" else 1
        return n

    def h2d(self):
        for it, h in zip(self.items, self.a_host):
            it[6].copy_(h, non_blocking=True)

    def d2h(self):
        for it, h in zip(self.items, self.c_host):
            h.copy_(it[7], non_blocking=True)


def cpu_prefill_sample(pf, budget_s=10.0):
    """The reference's matmul_parallel (its packed GEMM for m > 4, matmul.cpp:240-306) on
    layer 0's wq product at m = 512 (the same int8 weights), on all host cores."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle  # the CPU baseline leg only
    kind = "reference" if oracle.Reference.available(fast=True) else "port"
    q, s, m, kl, nl = (pf.items[0][0].cpu().numpy(), pf.items[0][1].cpu().numpy(),
                       pf.items[0][2], pf.items[0][3], pf.items[0][4])
    A = pf.items[0][6].cpu().numpy()
    flops = 2.0 * m * kl * nl
    if kind == "reference":
        ref = oracle.Reference(fast=True)
        hq = ref.qtensor(q, s)
        cores = ref.threads()
        one = lambda: ref.matmul_parallel_q8(A, hq)  # noqa: E731
    else:
        cores = oracle.default_threads()
        one = lambda: oracle.matmul_parallel(A, q=q, scale=s)  # noqa: E731
    one()
    times, t_end = [], time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": round(flops / med / 1e12, 4), "unit": "TFLOP/s", "cores": cores,
            "kind": kind, "sample": f"layer 0 wq ({m} x {kl} x {nl}, int8 weights), median of "
                                    f"{len(times)} calls"}


def prefill_parity(pf, world):
    """After the timed region: one grouped step again, then rows 0, 255 and 511 of layer 0's
    wq, wo, w1 and w2 and the last layer's w3 (and the classifier's row) against the oracle's
    matmul_naive_q8 on the same bytes, at the tensor-core path's 5e-3 row bound. On several
    GPUs only the column-parallel products, whose local slices are complete, are checked."""
    oracle = _oracle()
    want_idx = [0, 3, 4, 6, len(pf.items) - 3, len(pf.items) - 1]
    worst, checked = 0.0, []
    for i in want_idx:
        q, s, m, kl, nl, rowp, A, C = pf.items[i]
        if rowp and world > 1:
            continue
        rows = [0] if m == 1 else [0, 255, m - 1]
        A_h = A[rows].cpu().numpy()
        got = C[rows].cpu().numpy()
        want = oracle.matmul_naive_q8(A_h, q.cpu().numpy(), s.cpu().numpy())
        worst = max(worst, _row_rel_err(got, want))
        checked.append(pf.shapes[i][0])
    return {"ok": bool(worst <= 5e-3), "row_rel_err": float(f"{worst:.3e}"), "bound": 5e-3,
            "products_checked": checked, "rows": "0, 255, 511 (the classifier's one row)",
            "against": "oracle matmul_naive_q8 on the same int8 weights and activations"}


def prefill_line(world, rank, local, steps, warmup, layers, grouped=True, per_call=True,
                 e2e=True, cpu=True, check=True):
    import torch
    import llme_b200 as L
    prev_math = L.set_math(L.MATH_TENSOR)
    pf = Prefill(world, rank, layers=layers)
    stream = torch.cuda.Stream()
    h = stream.cuda_stream
    tp = comm = join = None
    if world > 1:
        import torch.distributed as dist
        uid = [L.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        # NCCL for the m x 4096 partials: bandwidth-bound sums, where the library's peer
        # all-reduce (one tagged 64-bit word a value, made for small latency-bound sums)
        # measured 11.3 against 6.0 ms a step at N = 2
        tp = L.Comm(world, rank, uid[0], timeout_s=60.0)
        comm_stream = torch.cuda.Stream()

        def comm(c_ptr, n):
            comm_stream.wait_stream(torch.cuda.current_stream())
            tp.allreduce_sum_f32(c_ptr, n, comm_stream.cuda_stream)

        def join():
            torch.cuda.current_stream().wait_stream(comm_stream)
    if grouped:
        pf.make_batch()
        step_fn = lambda: pf.launch_grouped(h, comm, join)  # noqa: E731
    else:
        step_fn = lambda: pf.launch_all(h, comm, join)  # noqa: E731
    graph = capture(step_fn, stream)
    sampler = ClockSampler(local)
    secs = max_over_ranks(time_graph(graph, steps, warmup, stream, world, sampler), world)
    tflops = pf.flops_total * steps / secs / 1e12
    pc = None
    if grouped and per_call:
        pc_graph = capture(lambda: pf.launch_all(h, comm, join), stream)
        pc_secs = max_over_ranks(time_graph(pc_graph, steps, warmup, stream, world), world)
        pc = {"value": round(pf.flops_total * steps / pc_secs / 1e12, 1),
              "unit": "TFLOP/s", "ms_per_step": round(pc_secs / steps * 1e3, 4),
              "launches_per_step": pf.launches()}
        del pc_graph
    e2e_d = None
    if e2e:
        def e2e_fn():
            pf.h2d()
            step_fn()
            pf.d2h()
        e2e_graph = capture(e2e_fn, stream)
        e2e_secs = max_over_ranks(time_graph(e2e_graph, steps, warmup, stream, world), world)
        e2e_d = {"value": round(pf.flops_total * steps / e2e_secs / 1e12, 1), "unit": "TFLOP/s",
                 "h2d_bytes_per_step": int(sum(t.numel() * 4 for t in pf.a_host)),
                 "d2h_bytes_per_step": int(sum(t.numel() * 4 for t in pf.c_host)),
                 "ms_per_step": round(e2e_secs / steps * 1e3, 4)}
        del e2e_graph
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops_sustained"])
        peak_kind = "measured bf16 sustained"
    except Exception:
        peak, peak_kind = 1400.0, "fallback bf16 sustained"
    achieved = pf.flops_rank * steps / secs / 1e12
    launches = 2 * len(pf.batches) + 1 if grouped else pf.launches()
    n_rowpar = sum(1 for it in pf.items if it[5]) if world > 1 else 0
    line = {
        "metric": PREFILL_METRIC, "value": round(tflops, 1), "unit": "TFLOP/s", "n_gpus": world,
        "steps": steps, "warmup": warmup,
        "ms_per_step": round(secs / steps * 1e3, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8 x (int8 hi + int8 lo) -> s32",
        "data": "synthetic: N(0,0.02^2) weights (seed 4) quantised per column to int8, "
                "U(-1,1) activations",
        "config": {"workload": "7B-shaped batched prefill, m=512, int8 weights (BASELINE "
                               "configs[4]); classifier on the last row",
                   "layers": layers, "rows": PREFILL_ROWS, "products_per_step": len(pf.items),
                   "launches_per_step": launches, "flops_per_step": pf.flops_total,
                   "parallelism": f"tp{world}" if world > 1 else "single",
                   "launch": ("grouped: one split launch + one persistent tcgen05 launch over "
                              "every m=512 product (llme_batch_run; the products are "
                              "independent) + the classifier GEMV, one CUDA graph per step")
                             if grouped else
                             "one C-ABI call per product (split pass + tcgen05 GEMM), one CUDA "
                             "graph per step",
                   "l2": "no flush: 6.6 GB of weights and 2.3 GB of activations per step"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                     "peak_kind": peak_kind + " (each product is two int8 MMAs, together the "
                                              "bf16 rate)",
                     "kernel": "gemm_q8_tc_kernel (+ split_rows_kernel)",
                     # DRAM read+write bytes of the step's launches: the full ncu capture of the
                     # same kernels on the 2-layer case measured 1.02 x the GEMM's algorithmic
                     # bytes (weights read once) and the split's reads exactly; scaled here to
                     # the step: GEMM (W + hi/lo + C) x 1.02 + split (4mk + 2mk).
                     "traffic": int(1.02 * pf.gemm_bytes + pf.split_bytes),
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the "
                                       "2-layer case: 1.02 x the GEMM's algorithmic bytes, "
                                       "scaled to the step",
                     "bytes_per_step": int(pf.gemm_bytes + pf.split_bytes)},
        "gpu_launches": launches * steps, "clocks": sampler.summary(),
    }
    if world > 1:
        line["exchange"] = (f"the {n_rowpar} wo/w2 partial outputs ({PREFILL_ROWS} x {DIM} floats "
                            "each) summed over the ranks on a side stream by NCCL (library "
                            "communicator)")
    if e2e_d is not None:
        line["e2e"] = e2e_d
    if pc is not None:
        line["per_call"] = pc
    if check:
        with torch.cuda.stream(stream):
            step_fn()
        torch.cuda.synchronize()
        line["parity"] = prefill_parity(pf, world)
    if cpu and rank == 0 and world == 1:
        line["cpu_baseline"] = cpu_prefill_sample(pf)
    del graph
    torch.cuda.synchronize()
    if grouped:
        pf.destroy_batches()
    if tp is not None:
        tp.destroy()
    del pf
    torch.cuda.synchronize()
    L.set_math(prev_math)
    return line


def run_prefill(args, world, rank, local):
    line = prefill_line(world, rank, local, args.steps, args.warmup, args.layers,
                        grouped=args.launch == "grouped", cpu=not args.no_extras,
                        check=not args.no_extras)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if "parity" in line and not line["parity"]["ok"]:
        raise SystemExit(3)


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def cpu_baseline_sample(chain, budget_s=8.0):
    """The reference's matmul_parallel on layer 0's seven products + the classifier (the same
    int8 bytes the GPU uses), on all host cores; GB/s of algorithmic bytes."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle  # the CPU baseline leg only
    kind = "reference" if oracle.Reference.available(fast=True) else "port"
    idx = list(range(7)) + [len(chain.mats) - 1]
    mats = [(chain.mats[i][0].cpu().numpy(), chain.mats[i][1].cpu().numpy()) for i in idx]
    rng = np.random.default_rng(1)
    acts = [rng.uniform(-1, 1, (1, q.shape[0])).astype(np.float32) for q, _ in mats]
    nbytes = sum(algorithmic_bytes(q.shape[0], q.shape[1]) for q, _ in mats)
    if kind == "reference":
        ref = oracle.Reference(fast=True)
        hs = [ref.qtensor(q, s) for q, s in mats]
        cores = ref.threads()

        def one():
            for a, h in zip(acts, hs):
                ref.matmul_parallel_q8(a, h)
    else:
        cores = oracle.default_threads()

        def one():
            for a, (q, s) in zip(acts, mats):
                oracle.matmul_parallel(a, q=q, scale=s)
    one()
    times, t_end = [], time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": round(nbytes / med / 1e9, 2), "unit": UNIT, "cores": cores, "kind": kind,
            "sample": f"layer 0 (7 products) + classifier, m=1, {nbytes / 1e6:.0f} MB of "
                      f"algorithmic bytes per pass, median of {len(times)} passes"}


def run_ours(args):
    import torch
    import llme_b200 as L
    if not torch.cuda.is_available():
        raise SystemExit("this benchmark needs an sm_100 (B200) GPU; none is visible")
    world, rank, local = dist_setup(args.gpus)
    L.load()
    if not L.device_supported():
        raise SystemExit("this benchmark needs an sm_100 (B200) GPU")
    if args.workload == "sgemm":
        return run_sgemm(args, world, rank, local)
    if args.workload == "prefill":
        return run_prefill(args, world, rank, local)
    if args.workload == "sweep":
        return run_sweep(args, world, rank, local)
    if args.workload == "attention":
        return run_attention(args, world, rank, local)
    if args.workload == "tp_decode":
        return run_tp_decode(args, world, rank, local)
    if args.workload == "chain":
        chain = Chain(world, rank, chain_shapes(args.layers), seed=3)
    else:
        chain = Chain(world, rank, gemv_shapes(), seed=0)
    comm = tp = None
    stream = torch.cuda.Stream()
    h = stream.cuda_stream
    if world > 1:
        # The library's own NCCL communicator; each row-parallel all-reduce runs on a side
        # stream so it overlaps the products that follow, and the step joins it at the end.
        import torch.distributed as dist
        uid = [L.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        tp = L.Comm(world, rank, uid[0], timeout_s=60.0)
        if args.allreduce in ("peer", "fused"):
            tp.enable_peer(chain.rp_count)  # NVLink peer receive areas
        comm_stream = torch.cuda.Stream()

        def comm(c_ptr, n):  # noqa: F811
            comm_stream.wait_stream(torch.cuda.current_stream())
            tp.allreduce_sum_f32(c_ptr, n, comm_stream.cuda_stream)
    join = (lambda: torch.cuda.current_stream().wait_stream(comm_stream)) if world > 1 else None
    grouped = args.launch == "grouped"
    if grouped:
        chain.make_batch()
        step_fn = lambda: chain.launch_grouped(h, tp, comm_stream if world > 1 else None,  # noqa: E731
                                               fused=args.allreduce == "fused")
    else:
        step_fn = lambda: chain.launch_all(h, comm, join)  # noqa: E731
    graph = capture(step_fn, stream)
    sampler = ClockSampler(local)
    secs = time_graph(graph, args.steps, args.warmup, stream, world, sampler)
    secs = max_over_ranks(secs, world)
    value = chain.total_bytes * args.steps / secs / 1e9
    ms_per_step = secs / args.steps * 1e3
    # The same step as one C-ABI call per product (the reference's call pattern), for comparison.
    per_call = None
    if grouped:
        pc_graph = capture(lambda: chain.launch_all(h, comm, join), stream)
        pc_secs = max_over_ranks(time_graph(pc_graph, args.steps, args.warmup, stream, world), world)
        per_call = {"value": round(chain.total_bytes * args.steps / pc_secs / 1e9, 1),
                    "unit": UNIT, "ms_per_step": round(pc_secs / args.steps * 1e3, 4),
                    "launches_per_step": chain.n_launches()}
        del pc_graph

    # e2e: every step copies its inputs in from pinned host memory and its outputs back out
    # inside the timed region, software-pipelined over two buffer sets: step i + 1's inputs go
    # up and step i - 1's outputs come down while step i computes (three streams ordered by
    # events: a set is reloaded only after the step that read it, and its outputs are copied
    # out before the next step on that set overwrites them).
    ios = [chain.io(), chain.add_io_set()]
    e2e_graphs = []
    for io in ios:
        chain.use_io(io)
        e2e_graphs.append(capture(step_fn, stream))
    chain.use_io(ios[0])
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    ev_up = [torch.cuda.Event() for _ in ios]
    ev_comp = [torch.cuda.Event() for _ in ios]
    ev_down = [torch.cuda.Event() for _ in ios]
    for e in ev_up + ev_comp + ev_down:
        e.record(stream)

    def e2e_step(i):
        j = i % 2
        a_host, c_host, a_dev, c_dev, _ = ios[j]
        up.wait_event(ev_comp[j])
        with torch.cuda.stream(up):
            a_dev.copy_(a_host, non_blocking=True)
            ev_up[j].record(up)
        stream.wait_event(ev_up[j])
        stream.wait_event(ev_down[j])
        with torch.cuda.stream(stream):
            e2e_graphs[j].replay()
            ev_comp[j].record(stream)
        down.wait_event(ev_comp[j])
        with torch.cuda.stream(down):
            c_host.copy_(c_dev, non_blocking=True)
            ev_down[j].record(down)

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_start.record(up)
    for i in range(args.steps):
        e2e_step(i)
    t_end.record(down)
    torch.cuda.synchronize()
    e2e_secs = max_over_ranks(t_start.elapsed_time(t_end) / 1e3, world)
    barrier(world)
    e2e = {"value": round(chain.total_bytes * args.steps / e2e_secs / 1e9, 1), "unit": UNIT,
           "h2d_bytes_per_step": int(chain.a_host.numel() * 4),
           "d2h_bytes_per_step": int(chain.c_host.numel() * 4),
           "ms_per_step": round(e2e_secs / args.steps * 1e3, 4),
           "pipelined": "two buffer sets: the next step's inputs copied in and the previous "
                        "step's outputs copied out while a step computes"}

    peak, peak_kind = peaks()
    launches = len(chain.batches) if grouped else chain.n_launches()
    if world > 1 and not (grouped and args.allreduce == "fused"):
        launches += 1 if grouped else sum(1 for m in chain.mats if m[4])  # the all-reduces
    per_launch_bytes = chain.bytes_per_step / launches
    per_launch_s = (secs / args.steps) / launches
    achieved = per_launch_bytes / per_launch_s / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                "kernel": "gemv_batch_kernel<1> (int8)" if grouped else "gemv_tma_kernel<1,int8>",
                "bytes_per_launch": int(per_launch_bytes),
                # DRAM read+write bytes per launch: ncu on the same grouped launch of the
                # 8-layer chain measured 1.0014 x its algorithmic bytes, and on one per-call
                # GEMV 1.0002 x (traffic grows with the weights streamed); scaled here.
                "traffic": int((1.0014 if grouped else 1.0002) * per_launch_bytes),
                "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                                   + ("grouped launch of the 8-layer chain: 1.0014"
                                      if grouped else "per-call 4096^2 GEMV: 1.0002")
                                   + " x the algorithmic bytes, scaled to this launch")}
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: N(0,0.02^2) weights quantised per column to int8, U(-1,1) activations",
        "exchange": (None if world == 1 else
                     "the wo/w2 partial outputs summed over the ranks inside their grouped launch "
                     "(each CTA sends its strips to the same CTA of every rank over NVLink peer "
                     "stores and writes the rank-ordered sums; llme_batch_run_rowpar)"
                     if grouped and args.allreduce == "fused" else
                     (("one-shot all-reduce over NVLink peer memory (library kernel)"
                       if args.allreduce in ("peer", "fused") else
                       "NCCL all-reduce (library communicator)")
                      + " of the wo/w2 partial outputs, on a side stream overlapping the "
                        "column-parallel products")),
        "config": WORKLOAD_CONFIG[args.workload] | {
                   "layers": args.layers if args.workload == "chain" else None,
                   "products_per_step": chain.n_launches(), "launches_per_step": launches,
                   "algorithmic_bytes_per_step": int(chain.total_bytes),
                   "parallelism": f"tp{world}" if world > 1 else "single",
                   "launch": ("one grouped launch of all products per step (llme_batch_run; the "
                              "products are independent), in a CUDA graph with PDL") if grouped
                             else "one C-ABI call per product, one CUDA graph per step, PDL"},
        "roofline": roofline, "e2e": e2e, "gpu_launches": launches * args.steps,
        "per_call": per_call,
        "clocks": sampler.summary(),
    }
    # The checker after every timed region: one grouped step again, sampled outputs against
    # the oracle (every rank takes the same collective steps).
    if not args.no_extras:
        chain.use_io(ios[0])
        with torch.cuda.stream(stream):
            step_fn()
        torch.cuda.synchronize()
        line["parity"] = chain_parity(chain, world)
    if rank == 0 and world == 1 and not args.no_extras and args.workload == "chain":
        line["gemv_4096x4096"] = gemv_4096_probe()
        for v in line["gemv_4096x4096"].values():
            v["frac"] = round(v["GB_s"] / peak, 4)
        beside = chain_per_call_beside_reference(chain)
        if beside is not None:
            line["reference_gpu"] = beside
        line["cpu_baseline"] = cpu_baseline_sample(chain)
        # The other two north-star targets, each its own short timed region.
        keep = ("metric", "value", "unit", "ms_per_step", "steps", "warmup", "roofline",
                "clocks", "parity", "gpu_launches")
        sg = sgemm_line(8192, 20, 5, 1, local, check_rows=16)
        line["sgemm_8192"] = {k: sg[k] for k in keep if k in sg} | {
            "workload": "configs[2]: square fp32 SGEMM, N=8192, TF32 tcgen05"}
        pre = prefill_line(1, 0, local, 20, 5, LAYERS, per_call=False, e2e=False, cpu=False,
                           check=True)
        line["prefill"] = {k: pre[k] for k in keep if k in pre} | {
            "workload": "configs[4]: 7B-shaped int8 prefill, m=512, one grouped step"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    failed = [k for k in ("parity",) if k in line and not line[k]["ok"]] + \
        [k for k in ("sgemm_8192", "prefill") if k in line and not line[k]["parity"]["ok"]]
    # Graphs holding NCCL calls go first, then the communicator, then the process group.
    del graph, e2e_graphs
    torch.cuda.synchronize()
    if grouped:
        chain.destroy_batches()
    if tp is not None:
        tp.destroy()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if failed:
        raise SystemExit(f"parity failed after the timed regions: {failed}")


def ref_gpu_attention(args, path):
    """The reference's own GPU attention (src/cuda_attention.cu for sm_100a) on the attention
    workload's cases and inputs, called through its attention_cuda() on its per-thread default
    stream, not captured, timed with events around synchronised batches of calls."""
    import ctypes
    import torch
    ref = ctypes.CDLL(path)
    sz, vp, ci = ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int
    ref.ref_attention_scratch_floats.argtypes = [ci, ci, ci, ci, sz, sz, sz, sz, ci]
    ref.ref_attention_scratch_floats.restype = sz
    ref.ref_attention.argtypes = [ci, ci, ci, ci, sz, sz, sz, sz, vp, vp, vp, vp, vp, vp, ci]
    g = torch.Generator(device="cuda")
    g.manual_seed(5)  # the same draws, in the same order, as run_attention
    cases, tot_bytes, tot_s = [], 0.0, 0.0
    for name, heads, kvh, hs, T in ATTN_CASES:
        kv, dim = kvh * hs, heads * hs
        q, ks, vs, pos = attention_case_inputs(torch, g, heads, kvh, hs, T)
        nbytes = attention_case_bytes(heads, kvh, hs, T)
        out = torch.zeros(ATTN_LAYERS, dim, device="cuda")
        n = ref.ref_attention_scratch_floats(heads, kvh, hs, T, dim + 2 * kv, kv, dim, 1, 0)
        scratch = torch.zeros(max(1, n), device="cuda")

        def fn():
            for l in range(ATTN_LAYERS):
                if ref.ref_attention(heads, kvh, hs, T, dim + 2 * kv, kv, dim, 1, pos.data_ptr(),
                                     q.data_ptr(), ks[l].data_ptr(), vs[l].data_ptr(),
                                     out[l].data_ptr(), scratch.data_ptr(), 0):
                    raise RuntimeError("reference attention failed")
        torch.cuda.synchronize()
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(torch.cuda.default_stream())  # the legacy stream orders the per-thread one
        for _ in range(args.steps):
            fn()
        torch.cuda.synchronize()
        e1.record(torch.cuda.default_stream())
        torch.cuda.synchronize()
        secs = e0.elapsed_time(e1) / 1e3
        us = secs / (args.steps * ATTN_LAYERS) * 1e6
        cases.append({"case": name, "heads": heads, "kv_heads": kvh, "head_size": hs,
                      "positions": T, "reference_gpu": {"us": round(us, 2),
                                                        "GB_s": round(nbytes / us / 1e3, 1)}})
        tot_bytes += nbytes * args.steps * ATTN_LAYERS
        tot_s += secs
    value = tot_bytes / tot_s / 1e9
    return {"metric": ATTN_METRIC, "value": round(value, 1), "unit": "GB/s",
            "ms_per_step": round(tot_s / args.steps * 1e3, 4),
            "data": "synthetic U(-1,1) queries and caches, the same bytes as this library's arm",
            "config": {"workload": "decode attention over KV caches, 8 layer caches per case",
                       "reference": "src/cuda_attention.cu built for sm_100a, attention_cuda() "
                                    "uncaptured on its per-thread default stream"},
            "cases": cases}


def ref_gpu_sweep(args):
    """The reference's own GPU matmul (src/cuda_matmul.cu for sm_100a) on the sweep's cases
    and inputs, automatic kernel choice, each case's 12 calls captured as one CUDA graph on its
    per-thread default stream (as its CudaTransformer captures), timed with events there."""
    import torch
    ref = ref_matmul_gpu()
    g = torch.Generator(device="cuda")
    g.manual_seed(1)  # the same draws, in the same order, as run_sweep
    cases, tot_bytes, tot_s = [], 0, 0.0
    for q8 in (False, True):
        Ws = [torch.randn(DIM, DIM, generator=g, device="cuda") * 0.02 for _ in range(SWEEP_COPIES)]
        if q8:
            Ws = [quantize_on_device(w) for w in Ws]  # bit-identical to its quantize_q8
        for m in SWEEP_ROWS:
            A = torch.rand(m, DIM, generator=g, device="cuda") * 2 - 1
            C = torch.empty(m, DIM, device="cuda")

            def calls(ok):
                for i in range(SWEEP_COPIES):
                    if q8:
                        q, sc = Ws[i]
                        ok(ref.ref_gpu_matmul_q8(m, DIM, DIM, A.data_ptr(), q.data_ptr(),
                                                 sc.data_ptr(), C.data_ptr(), 0, 0, None))
                    else:
                        ok(ref.ref_gpu_matmul_f32(m, DIM, DIM, A.data_ptr(), Ws[i].data_ptr(),
                                                  C.data_ptr(), 0, 0, None))
            secs = time_ref_matmul_gpu(ref, calls, args.steps, args.warmup)
            nbytes = (algorithmic_bytes(DIM, DIM, m) if q8 else
                      4 * DIM * DIM + 4 * m * DIM + 4 * m * DIM)
            us = secs / (args.steps * SWEEP_COPIES) * 1e6
            cases.append({"w": "int8" if q8 else "fp32", "m": m, "us": round(us, 2),
                          "GB_s": round(nbytes / us / 1e3, 1)})
            tot_bytes += nbytes * args.steps * SWEEP_COPIES
            tot_s += secs
    value = tot_bytes / tot_s / 1e9
    return {"metric": SWEEP_METRIC, "value": round(value, 1), "unit": "GB/s",
            "ms_per_step": round(tot_s / args.steps * 1e3, 4),
            "data": "synthetic: N(0,0.02^2) weights (seed 1), U(-1,1) activations, the same "
                    "bytes as this library's arm",
            "config": {"workload": "decode-shaped sweep, one call per product, 12 distinct "
                                   "weights per case in a CUDA graph",
                       "reference": "src/cuda_matmul.cu built for sm_100a, matmul_cuda() with "
                                    "GpuKernel::automatic, captured on its per-thread default "
                                    "stream"},
            "cases": cases}


def run_reference_gpu(args):
    """`--impl reference` for the attention and sweep workloads: the reference's own GPU code
    for the path (built from its sources for sm_100a into oracle/_ref by `make -C oracle
    refgpu` / `make -C oracle refmatmul`), on the same B200 and the same inputs as this
    library's arm, through its public API."""
    import torch
    lib, target = (("libref_attention.so", "refgpu") if args.workload == "attention"
                   else ("libref_matmul_gpu.so", "refmatmul"))
    path = os.path.join(REPO, "oracle", "_ref", lib)
    if not torch.cuda.is_available() or not os.path.exists(path):
        why = (f"the reference's GPU code for --workload {args.workload} needs a CUDA device"
               if not torch.cuda.is_available() else
               f"oracle/_ref/{lib} is not built (make -C oracle {target})")
        print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
        return
    sampler = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")))
    with sampler:
        body = ref_gpu_attention(args, path) if args.workload == "attention" else ref_gpu_sweep(args)
    line = {"impl": "reference", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            **body,
            "e2e": {"value": body["value"], "unit": body["unit"], "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "clocks": sampler.summary()}
    print(json.dumps(line), flush=True)


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.workload in ("attention", "sweep"):
        return run_reference_gpu(args)
    if args.workload not in ("chain", "gemv"):
        # The other workloads time the reference's CPU code inside their own line
        # (cpu_baseline) on a bounded sample; tp_decode's reference model would need a 27 GB
        # fp32 checkpoint at 7B size.
        why = ("the reference's CPU Transformer at 7B size needs a 27 GB fp32 checkpoint; its "
               "parity is tested on small checkpoints" if args.workload == "tp_decode" else
               f"the reference arm times the decode chain; --workload {args.workload} reports "
               f"the reference's CPU code in its own line (cpu_baseline)")
        print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
        return
    oracle = _oracle()  # the reference arm: the reference's own CPU code (oracle/_ref)
    kind = "reference" if oracle.Reference.available(fast=True) else "port"
    shapes = chain_shapes(args.layers) if args.workload == "chain" else gemv_shapes()
    seed = 3 if args.workload == "chain" else 0
    t_setup = time.perf_counter()
    ref = oracle.Reference(fast=True) if kind == "reference" else None
    handles, acts, source = reference_chain_inputs(shapes, seed, ref, oracle)
    setup_s = time.perf_counter() - t_setup
    nbytes = sum(algorithmic_bytes(k, n) for (_, k, n, _) in shapes)
    outs = [np.empty((1, n), np.float32) for (_, k, n, _) in shapes]
    if ref is not None:
        cores = ref.threads()

        def step():
            for a, hq, o in zip(acts, handles, outs):
                ref.matmul_parallel_q8(a, hq, out=o)
    else:
        cores = oracle.default_threads()

        def step():
            for a, (q, s), o in zip(acts, handles, outs):
                o[...] = oracle.matmul_parallel(a, q=q, scale=s)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    secs = time.perf_counter() - t0
    value = nbytes * args.steps / secs / 1e9
    sample_desc = (f"the whole step: all {len(shapes)} products, m=1, "
                   f"{nbytes / 1e9:.3f} GB of algorithmic bytes per step; {source}")
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(secs / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: N(0,0.02^2) weights quantised per column to int8, U(-1,1) "
                    "activations (the same bytes as this library's arm)",
            "config": WORKLOAD_CONFIG[args.workload] | {
                "layers": args.layers if args.workload == "chain" else None,
                "products_per_step": len(shapes), "algorithmic_bytes_per_step": int(nbytes),
                "parallelism": "host threads (the reference's thread pool)",
                "isa": ref.isa() if ref is not None else "the C port, -O2"},
            "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": cores,
                             "kind": kind, "sample": sample_desc},
            "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "setup_s": round(setup_s, 1)}
    print(json.dumps(line), flush=True)


def reference_chain_inputs(shapes, seed, ref, oracle):
    """The chain's int8 weights and activations as the same bytes this library's arm uses:
    each weight drawn by torch with the same generator and seed as Chain (on the GPU where one
    is visible, as Chain draws it), copied to the host and quantised there by the reference's
    own quantize_q8 (quant.cpp:6-28; the port where the reference is not built), on a few host
    threads; activations drawn as Chain draws them. Returns (weights as reference-side
    QTensors or (q, scale) pairs, activation rows, a note on where the weights came from)."""
    import concurrent.futures as cf
    import torch
    cuda = torch.cuda.is_available()
    dev = "cuda" if cuda else "cpu"
    g = torch.Generator(device=dev)
    quant = ref.quantize_q8 if ref is not None else oracle.quantize_q8
    workers = max(1, min(8, os.cpu_count() or 1))

    def one(W):
        q, s = quant(W)
        return ref.qtensor(q, s) if ref is not None else (q, s)
    handles, futs = [None] * len(shapes), {}
    with cf.ThreadPoolExecutor(workers) as pool:
        for idx, (_, k, n, _) in enumerate(shapes):
            g.manual_seed(seed * 100003 + idx)
            W = (torch.randn(k, n, generator=g, device=dev) * 0.02).cpu().numpy()
            futs[pool.submit(one, W)] = idx
            if len(futs) >= 2 * workers:  # bound the fp32 copies held at once
                done, _ = cf.wait(futs, return_when=cf.FIRST_COMPLETED)
                for f in done:
                    handles[futs.pop(f)] = f.result()
        for f in cf.as_completed(list(futs)):
            handles[futs.pop(f)] = f.result()
    ga = torch.Generator(device="cpu")
    ga.manual_seed(seed * 7)
    acts = [(torch.rand(k, generator=ga) * 2 - 1).numpy().reshape(1, k) for (_, k, n, _) in shapes]
    source = ("weights drawn by torch on the GPU exactly as the library's arm draws them, "
              "quantised by the reference's quantize_q8" if cuda else
              "weights drawn by torch on the host (no GPU visible: other values, the same "
              "distribution), quantised by the reference's quantize_q8")
    if ref is None:
        source = source.replace("the reference's quantize_q8", "the C port of quantize_q8")
    return handles, acts, source


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["chain", "gemv", "sgemm", "prefill", "sweep",
                                           "attention", "tp_decode"],
                    default="chain",
                    help="chain: m = 1 through the 32 layers of 7B-shaped int8 weights (default); "
                         "gemv: one int8 4096 x 4096 weight at m = 1; sgemm: square TF32 "
                         "GEMM (--size); prefill: m = 512 through the 7B-shaped int8 weights; "
                         "sweep: m in {1,4,16,64} x 4096^2, fp32 and int8 W, per call; attention: "
                         "decode attention over KV caches; tp_decode: tokens/s of the "
                         "7B-shaped int8 transformer, tensor-parallel over --gpus")
    ap.add_argument("--size", type=int, default=8192, help="N for --workload sgemm")
    ap.add_argument("--context", type=int, default=1024,
                    help="cached positions before the decoded token (--workload tp_decode)")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="layers of the chain / prefill (32 = a 7B model; fewer only "
                         "for small profiling cases)")
    ap.add_argument("--allreduce", choices=["peer", "fused", "nccl"], default="peer",
                    help="N>1: the library's NVLink peer all-reduce on a side stream, hidden "
                         "under the column-parallel launch (default); the rank sum inside the "
                         "row-parallel grouped launch (fused: 0.520 against 0.490 ms per step "
                         "at N = 2, its wait is not hidden); or NCCL")
    ap.add_argument("--launch", choices=["grouped", "per_call"], default="grouped",
                    help="grouped: one llme_batch_run per step (default); per_call: one "
                         "llme_matmul_q8 per product (also reported as per_call)")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the isolated 4096^2 GEMV probe and the CPU baseline")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
