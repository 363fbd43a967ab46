"""Tensor-parallel decoding of the reference's Llama-architecture transformer.

The reference runs the whole model on one GPU (CudaTransformer, src/cuda_model.cu:232-270);
here each of `world` GPUs (one process per GPU) holds a slice of every layer and the ranks
exchange one all-reduce after each row-parallel projection:

* attention heads are split by kv head: rank r holds kv heads [r * nkv, (r + 1) * nkv) and the
  query heads that read them, so attention, RoPE and the KV cache are rank-local;
* wqkv (column-parallel): this rank's q, k and v columns; wo (row-parallel): the rows that
  multiply this rank's heads' outputs; w13 (column-parallel): this rank's slice of the gate
  and the matching slice of the up projection, so SwiGLU is local; w2 (row-parallel): the
  rows of that hidden slice; the classifier (column-parallel): a slice of the vocabulary;
* the residual stream x is replicated; each row-parallel product is the library's fused
  `matmul_*_rowpar`: rank 0 adds x to its partial, the others write their partial, and one
  all-reduce leaves x + sum of partials on every rank (the residual add fused into the
  collective); the classifier's slices are joined the same way (zeros elsewhere, summed).

int8 weights are quantised as the reference quantises them -- per column over all rows of the
full matrix (quant.cpp:6-28) -- so the row-parallel shards keep the full scale vector, and a
rank's int8 values are exactly the reference's for its slice.

Per layer and token: rmsnorm + wqkv (fused), RoPE + cache write, attention over the local
heads, wo + all-reduce (+ residual), rmsnorm + w13, SwiGLU, w2 + all-reduce (+ residual); then
rmsnorm + classifier + one all-reduce of the logits. Everything runs on the current torch
stream through the library's C ABI (matmul, attention, the decode-step helpers).
"""
from __future__ import annotations

import numpy as np

import llme_b200 as L
from checkpoint import Checkpoint
from shard import shard_range


def head_partition(n_heads: int, n_kv_heads: int, world: int, rank: int):
    """(first query head, query heads, first kv head, kv heads) of `rank`."""
    if n_kv_heads % world != 0:
        raise L.InvalidArgument(f"tensor parallel: {n_kv_heads} kv heads do not split over "
                                f"{world} ranks")
    nkv = n_kv_heads // world
    group = n_heads // n_kv_heads
    return rank * nkv * group, nkv * group, rank * nkv, nkv


def shard_layer(lw, cfg, world: int, rank: int) -> dict:
    """This rank's slices of one layer's weights (numpy, fp32)."""
    hs, D, KV, H = cfg.head_size, cfg.dim, cfg.kv_dim, cfg.hidden_dim
    q0, nq, kv0, nkv = head_partition(cfg.n_heads, cfg.n_kv_heads, world, rank)
    cols = np.concatenate([np.arange(q0 * hs, (q0 + nq) * hs),
                           D + np.arange(kv0 * hs, (kv0 + nkv) * hs),
                           D + KV + np.arange(kv0 * hs, (kv0 + nkv) * hs)])
    h0, hc = shard_range(H, world, rank)
    return {
        "wqkv": np.ascontiguousarray(lw.wqkv[:, cols]),
        "wo_rows": (q0 * hs, nq * hs),
        "w13": np.ascontiguousarray(np.concatenate([lw.w13[:, h0:h0 + hc],
                                                    lw.w13[:, H + h0:H + h0 + hc]], axis=1)),
        "w2_rows": (h0, hc),
    }


class TPTransformer:
    """One rank of a tensor-parallel transformer over a loaded Checkpoint.

    comm: the library's communicator (llme_b200.Comm) when world > 1 and the ranks run as
    processes; None with world > 1 hands every reduction to the caller through steps() (a
    single process emulating the ranks). run(tokens, pos) has the reference's position rules
    (check_feed, src/model.cpp:162-169) and returns the last row's logits (numpy)."""

    def __init__(self, ckpt: Checkpoint, world: int = 1, rank: int = 0, q8: bool = False,
                 comm=None):
        self._setup(ckpt.config, world, rank, q8, comm)
        torch, dev, cfg = self.torch, self.dev, self.cfg

        def dev_f32(a):
            return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)

        def proj(full, cols=None, rows=None):
            """A projection shard: fp32, or int8 + scales quantised over the full matrix."""
            if not q8:
                w = full if cols is None else full[:, cols[0]:cols[0] + cols[1]]
                w = w if rows is None else w[rows[0]:rows[0] + rows[1]]
                return (dev_f32(w), None)
            if rows is not None:  # row-parallel: scales over all rows, then the row slice
                q, s = L.quantize_q8(dev_f32(full))
                return (q[rows[0]:rows[0] + rows[1]].contiguous(), s)
            w = full if cols is None else full[:, cols[0]:cols[0] + cols[1]]
            return L.quantize_q8(dev_f32(w))

        self.emb = dev_f32(ckpt.token_embedding)
        self.rms_final = dev_f32(ckpt.rms_final)
        self.wcls = proj(ckpt.wcls, cols=(self.v0, self.vc))
        for lw in ckpt.layers:
            sh = shard_layer(lw, cfg, world, rank)
            self._add_layer(dev_f32(lw.rms_att), dev_f32(lw.rms_ffn), proj(sh["wqkv"]),
                            proj(lw.wo, rows=sh["wo_rows"]), proj(sh["w13"]),
                            proj(lw.w2, rows=sh["w2_rows"]))
        self._finish()

    @classmethod
    def synthetic(cls, cfg, world: int = 1, rank: int = 0, q8: bool = True, comm=None,
                  seed: int = 0):
        """A model of cfg's shape with random weights drawn on the device (projections
        N(0, 0.02^2), embedding U(-1, 1), unit RMSNorm weights), each rank drawing only its
        own shards -- for benchmarks at full size, where a host checkpoint would not fit."""
        self = cls.__new__(cls)
        self._setup(cfg, world, rank, q8, comm)
        torch, dev = self.torch, self.dev
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 1009 + rank)

        def proj(rows, cols):
            w = torch.randn(rows, cols, generator=g, device=dev) * 0.02
            return L.quantize_q8(w) if q8 else (w, None)

        D, hs = cfg.dim, cfg.head_size
        self.emb = torch.rand(cfg.vocab_size, D, generator=g, device=dev) * 2 - 1
        self.rms_final = torch.ones(D, device=dev)
        self.wcls = proj(D, self.vc)
        for _ in range(cfg.n_layers):
            self._add_layer(torch.ones(D, device=dev), torch.ones(D, device=dev),
                            proj(D, self.qkv_cols), proj(self.nq * hs, D),
                            proj(D, 2 * self.hc), proj(self.hc, D))
        self._finish()
        return self

    def _setup(self, cfg, world, rank, q8, comm):
        import torch
        self.torch = torch
        self.cfg = cfg
        self.world, self.rank, self.q8, self.comm = world, rank, q8, comm
        self.dev = torch.device("cuda", torch.cuda.current_device())
        hs = cfg.head_size
        self.q0, self.nq, self.kv0, self.nkv = head_partition(cfg.n_heads, cfg.n_kv_heads,
                                                              world, rank)
        self.h0, self.hc = shard_range(cfg.hidden_dim, world, rank)
        self.v0, self.vc = shard_range(cfg.vocab_size, world, rank)
        self.qkv_cols = (self.nq + 2 * self.nkv) * hs
        self.shape = L.AttentionShape(self.nq, self.nkv, hs, cfg.seq_len, self.qkv_cols,
                                      self.nkv * hs, self.nq * hs)
        L.attention_check(self.shape)
        self.layers = []
        self.graph = None
        # Reallocations of this model's activation buffers; with the library's scratch
        # generation it tells whether a captured graph still points at live buffers.
        self.own_generation = 0
        self.graph_generation = -1

    def _add_layer(self, rms_att, rms_ffn, wqkv, wo, w13, w2):
        t, cfg = self.torch, self.cfg
        kv = self.nkv * cfg.head_size
        self.layers.append({"rms_att": rms_att, "rms_ffn": rms_ffn, "wqkv": wqkv, "wo": wo,
                            "w13": w13, "w2": w2,
                            "kc": t.zeros(cfg.seq_len, kv, device=self.dev),
                            "vc": t.zeros(cfg.seq_len, kv, device=self.dev)})

    def _finish(self):
        t, cfg = self.torch, self.cfg
        cos, sin = L.rope_tables(cfg.seq_len, cfg.head_size)
        self.cos, self.sin = t.from_numpy(cos).to(self.dev), t.from_numpy(sin).to(self.dev)
        self.feed_host = t.zeros(cfg.seq_len + 1, dtype=t.int32).pin_memory()
        self.feed = t.zeros(cfg.seq_len + 1, dtype=t.int32, device=self.dev)
        self.logits = t.zeros(cfg.vocab_size, device=self.dev)
        self.rows = 0
        self.filled = 0
        self._reserve(1)

    def _reserve(self, n: int) -> None:
        if n <= self.rows:
            return
        t, cfg, dev = self.torch, self.cfg, self.dev
        self.x = t.zeros(n, cfg.dim, device=dev)
        self.qkv = t.zeros(n, self.qkv_cols, device=dev)
        self.att = t.zeros(n, self.nq * cfg.head_size, device=dev)
        self.gu = t.zeros(n, 2 * self.hc, device=dev)
        self.hb = t.zeros(n, self.hc, device=dev)
        self.scratch = t.zeros(max(1, L.attention_scratch_floats(self.shape, n)), device=dev)
        self.rows = n
        self.own_generation += 1

    def buffers_generation(self) -> int:
        """Changes whenever a buffer a captured step points at is replaced: this model's
        activation rows or the library's scratch (src/cuda_model.cu:175-177)."""
        return self.own_generation + L.scratch_generation()

    # ---- the products --------------------------------------------------------------------
    def _matmul(self, m, n, k, A, w, C, accumulate=False, rms=0):
        B, scale = w
        h = L.torch_stream_handle()
        if scale is None:
            L.matmul_cuda_f32(m, n, k, A, B.data_ptr(), C, "automatic", accumulate, rms,
                              L.FLAG_WEIGHTS_STATIC, h)
        else:
            L.matmul_cuda_q8(m, n, k, A, B.data_ptr(), scale.data_ptr(), C, "automatic",
                             accumulate, rms, L.FLAG_WEIGHTS_STATIC, h)

    def _rowpar(self, m, n, k_local, A, w, C):
        """C (the x tensor) <- x + sum over ranks of A_r W_r; yields C for an external
        reduction when the ranks are emulated in one process."""
        B, scale = w
        acc = self.rank == 0
        if self.comm is not None:
            h = L.torch_stream_handle()
            if scale is None:
                self.comm.matmul_f32_rowpar(m, n, k_local, A, B.data_ptr(), C.data_ptr(),
                                            "automatic", acc, L.FLAG_WEIGHTS_STATIC, h)
            else:
                self.comm.matmul_q8_rowpar(m, n, k_local, A, B.data_ptr(), scale.data_ptr(),
                                           C.data_ptr(), "automatic", acc, L.FLAG_WEIGHTS_STATIC,
                                           h)
            return
        self._matmul(m, n, k_local, A, w, C.data_ptr(), accumulate=acc)
        if self.world > 1:
            yield C

    def steps(self, tokens, pos: int):
        """Queues one pass over tokens at positions [pos, pos + n) on the current stream.
        A generator: with world > 1 and no communicator it yields each buffer that must be
        summed over the ranks (x after wo and w2, then the logits) and continues once the
        caller has written the sum into every rank's buffer (the yielded torch tensor)."""
        cfg = self.cfg
        n = len(tokens)
        if n == 0:
            raise L.InvalidArgument("prefill: no tokens")
        for t in tokens:
            if not 0 <= int(t) < cfg.vocab_size:
                raise IndexError(f"forward: token {int(t)} outside vocab")
        if pos + n > cfg.seq_len or pos > self.filled:
            raise IndexError(f"forward: positions {pos}..{pos + n - 1} with {self.filled} cached "
                             f"of {cfg.seq_len}")
        self._reserve(n)
        D, hs = cfg.dim, cfg.head_size
        h = L.torch_stream_handle()
        self.feed_host[0] = pos
        self.feed_host[1:n + 1] = self.torch.tensor([int(t) for t in tokens], dtype=self.torch.int32)
        self.feed[:n + 1].copy_(self.feed_host[:n + 1], non_blocking=True)
        fp, x = self.feed.data_ptr(), self.x.data_ptr()
        L.embed_rows(n, D, fp, self.emb.data_ptr(), x, h)
        for lw in self.layers:
            self._matmul(n, self.qkv_cols, D, x, lw["wqkv"], self.qkv.data_ptr(),
                         rms=lw["rms_att"].data_ptr())
            L.rope_cache(n, self.nq, self.nkv, hs, fp, self.cos.data_ptr(), self.sin.data_ptr(),
                         self.qkv.data_ptr(), lw["kc"].data_ptr(), lw["vc"].data_ptr(), h)
            L.attention(self.shape, n, fp, self.qkv.data_ptr(), lw["kc"].data_ptr(),
                        lw["vc"].data_ptr(), self.att.data_ptr(), self.scratch.data_ptr(),
                        stream=h)
            yield from self._rowpar(n, D, self.nq * hs, self.att.data_ptr(), lw["wo"], self.x)
            self._matmul(n, 2 * self.hc, D, x, lw["w13"], self.gu.data_ptr(),
                         rms=lw["rms_ffn"].data_ptr())
            L.swiglu(n, self.hc, self.gu.data_ptr(), self.hb.data_ptr(), h)
            yield from self._rowpar(n, D, self.hc, self.hb.data_ptr(), lw["w2"], self.x)
        # The last row's logits: this rank's vocabulary slice, zeros elsewhere, then summed.
        self.logits.zero_()
        last = x + (n - 1) * D * 4
        self._matmul(1, self.vc, D, last, self.wcls, self.logits.data_ptr() + self.v0 * 4,
                     rms=self.rms_final.data_ptr())
        if self.world > 1:
            if self.comm is not None:
                self.comm.allreduce_sum_f32(self.logits.data_ptr(), cfg.vocab_size, h)
            else:
                yield self.logits
        self.filled = pos + n

    def run(self, tokens, pos: int) -> np.ndarray:
        """Feeds tokens at [pos, pos + n) and returns the last row's logits."""
        if self.world > 1 and self.comm is None:
            raise L.InvalidArgument("tensor parallel: run() needs a communicator; drive steps() "
                                    "to reduce across emulated ranks")
        for _ in self.steps(tokens, pos):
            raise L.InvalidArgument("tensor parallel: unexpected reduction point")
        return self.logits.cpu().numpy()

    def forward(self, token: int, pos: int) -> np.ndarray:
        if self.graph is not None:
            return self.decode(token, pos).cpu().numpy()
        return self.run([token], pos)

    def capture_decode(self):
        """Captures the one-token step as a CUDA graph, as the reference's CudaTransformer
        does (src/cuda_model.cu:190-220): token and position are read from device memory, so
        one graph serves every position. Call after an eager one-token run(), which has grown
        every buffer the step uses, so capturing allocates nothing; nothing runs while
        capturing. Returns the graph; decode() replays it."""
        t = self.torch
        if self.filled == 0:
            raise L.InvalidArgument("capture_decode: run one token eagerly first")
        saved = self.filled
        s = t.cuda.Stream()
        s.wait_stream(t.cuda.current_stream())
        g = t.cuda.CUDAGraph()
        with t.cuda.stream(s):
            with t.cuda.graph(g, stream=s):
                for _ in self.steps([0], saved - 1):
                    raise L.InvalidArgument("tensor parallel: graphs need a communicator")
        t.cuda.current_stream().wait_stream(s)
        self.filled = saved
        self.graph = g
        self.graph_generation = self.buffers_generation()
        return g

    def decode(self, token: int, pos: int):
        """One token through the captured graph on the current stream; returns the logits
        (device tensor, valid once the stream reaches this point)."""
        cfg = self.cfg
        if not 0 <= int(token) < cfg.vocab_size:
            raise IndexError(f"forward: token {int(token)} outside vocab")
        if pos + 1 > cfg.seq_len or pos > self.filled:
            raise IndexError(f"forward: positions {pos}..{pos} with {self.filled} cached of "
                             f"{cfg.seq_len}")
        self.torch.cuda.current_stream().synchronize()  # the previous replay read the feed
        if self.graph_generation != self.buffers_generation():
            # A longer prefill replaced the buffers the graph was captured on (the reference
            # re-captures in the same case, src/cuda_model.cu:196-227).
            self.capture_decode()
        self.feed_host[0] = pos
        self.feed_host[1] = int(token)
        self.graph.replay()
        self.filled = max(self.filled, pos + 1)
        return self.logits

    def prefill(self, tokens, pos: int) -> np.ndarray:
        return self.run(list(tokens), pos)
