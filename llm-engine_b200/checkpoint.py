"""llama2.c checkpoints (legacy version-0 format) for the transformer, as the reference loads
them (src/model.cpp:113-169, load_checkpoint): seven int32 header fields (dim, hidden_dim,
n_layers, n_heads, n_kv_heads, vocab_size -- negative when the classifier is stored apart from
the embedding -- and seq_len), then fp32 weights grouped by kind across all layers: embedding,
rms_att, wq, wk, wv, wo, rms_ffn, w1, w2, w3, rms_final, the legacy RoPE tables (skipped), and
the classifier when it is not shared.

Projections are returned (in x out), the transpose of the file's (out x in), and concatenated
as the reference's Transformer keeps them (src/model.h:24-37): wqkv = [wq | wk | wv] and
w13 = [w1 | w3] by columns. The same header checks and size check as the reference, with the
same error texts.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field

import numpy as np


@dataclass
class Config:
    dim: int
    hidden_dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    vocab_size: int
    seq_len: int

    @property
    def head_size(self) -> int:
        return self.dim // self.n_heads

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_size


@dataclass
class LayerWeights:
    rms_att: np.ndarray   # dim
    wqkv: np.ndarray      # dim x (dim + 2 kv_dim): q | k | v
    wo: np.ndarray        # dim x dim
    rms_ffn: np.ndarray   # dim
    w13: np.ndarray       # dim x 2 hidden_dim: gate (w1) | up (w3)
    w2: np.ndarray        # hidden_dim x dim


@dataclass
class Checkpoint:
    config: Config
    token_embedding: np.ndarray            # vocab x dim
    layers: list = field(default_factory=list)
    rms_final: np.ndarray | None = None    # dim
    wcls: np.ndarray | None = None         # dim x vocab


def _parse_header(h, path: str) -> tuple[Config, bool]:
    shared = int(h[5]) > 0
    for i in range(7):
        if h[i] == 0 or (i != 5 and h[i] < 0):
            raise RuntimeError(f"checkpoint {path}: bad header field {i} = {int(h[i])}")
    c = Config(*[abs(int(v)) for v in h])
    if c.dim % c.n_heads != 0 or c.head_size % 2 != 0 or c.n_heads % c.n_kv_heads != 0:
        raise RuntimeError(f"checkpoint {path}: dim must split into even-sized heads, and query "
                           "heads into whole groups per kv head")
    return c, shared


def expected_size(c: Config, shared: bool) -> int:
    """File size implied by the header, in bytes (src/model.cpp:79-87)."""
    D, H, KV, V = c.dim, c.hidden_dim, c.kv_dim, c.vocab_size
    per_layer = 2 * D + 2 * D * D + 2 * D * KV + 3 * D * H
    floats = V * D + c.n_layers * per_layer + D + c.seq_len * c.head_size
    if not shared:
        floats += V * D
    return 7 * 4 + floats * 4


def load_checkpoint(path: str) -> Checkpoint:
    if not os.path.exists(path):
        raise RuntimeError(f"cannot open checkpoint {path}")
    size = os.path.getsize(path)
    if size < 28:
        raise RuntimeError(f"checkpoint {path} ended early")
    header = np.fromfile(path, dtype="<i4", count=7)
    c, shared = _parse_header(header, path)
    want = expected_size(c, shared)
    if size != want:
        raise RuntimeError(f"checkpoint {path} is {size} bytes, header implies {want}")
    data = np.memmap(path, dtype="<f4", mode="r", offset=28)
    D, H, KV, V, NL = c.dim, c.hidden_dim, c.kv_dim, c.vocab_size, c.n_layers
    off = 0

    def take(count: int, shape=None) -> np.ndarray:
        nonlocal off
        a = np.array(data[off:off + count], dtype=np.float32)
        off += count
        return a if shape is None else a.reshape(shape)

    def per_layer(rows: int, cols: int) -> list:
        return [take(rows * cols, (rows, cols)) for _ in range(NL)]

    emb = take(V * D, (V, D))
    rms_att = per_layer(1, D)
    wq, wk, wv = per_layer(D, D), per_layer(KV, D), per_layer(KV, D)
    wo = per_layer(D, D)
    rms_ffn = per_layer(1, D)
    w1, w2, w3 = per_layer(H, D), per_layer(D, H), per_layer(H, D)
    rms_final = take(D)
    off += c.seq_len * c.head_size  # legacy RoPE tables: recomputed, as llama2.c does
    wcls = emb.T.copy() if shared else take(V * D, (V, D)).T.copy()

    ck = Checkpoint(c, emb, [], rms_final, np.ascontiguousarray(wcls))
    for l in range(NL):
        ck.layers.append(LayerWeights(
            rms_att=rms_att[l].reshape(D),
            wqkv=np.ascontiguousarray(np.concatenate([wq[l].T, wk[l].T, wv[l].T], axis=1)),
            wo=np.ascontiguousarray(wo[l].T),
            rms_ffn=rms_ffn[l].reshape(D),
            w13=np.ascontiguousarray(np.concatenate([w1[l].T, w3[l].T], axis=1)),
            w2=np.ascontiguousarray(w2[l].T)))
    return ck
