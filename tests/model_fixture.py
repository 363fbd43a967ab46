"""Small random llama2.c checkpoints for the transformer tests (legacy version-0 format, as
the reference's loader reads it, src/model.cpp:113-169): seven int32 header fields, then the
fp32 weights grouped by kind across layers, the legacy RoPE tables (filled with a constant the
loader must ignore) and the classifier when it is not shared with the embedding."""
from __future__ import annotations

import numpy as np


def make_model(dim=64, hidden=96, layers=2, heads=8, kv_heads=4, vocab=50, seq_len=16,
               shared=False, seed=0) -> dict:
    """Weights in the file's own (out x in) layout, drawn from a seeded generator."""
    rng = np.random.default_rng(seed)
    hs = dim // heads
    kv = kv_heads * hs

    def u(shape, scale):
        return rng.uniform(-scale, scale, shape).astype(np.float32)

    m = {"dim": dim, "hidden": hidden, "layers": layers, "heads": heads, "kv_heads": kv_heads,
         "vocab": vocab, "seq_len": seq_len, "shared": shared,
         "emb": u((vocab, dim), 1.0)}
    for name in ("rms_att", "wq", "wk", "wv", "wo", "rms_ffn", "w1", "w2", "w3"):
        m[name] = []
    for _ in range(layers):
        m["rms_att"].append(1.0 + u(dim, 0.2))
        m["rms_ffn"].append(1.0 + u(dim, 0.2))
        m["wq"].append(u((dim, dim), 0.4))
        m["wk"].append(u((kv, dim), 0.4))
        m["wv"].append(u((kv, dim), 0.4))
        m["wo"].append(u((dim, dim), 0.3))
        m["w1"].append(u((hidden, dim), 0.3))
        m["w2"].append(u((dim, hidden), 0.3))
        m["w3"].append(u((hidden, dim), 0.3))
    m["rms_final"] = 1.0 + u(dim, 0.2)
    m["wcls"] = None if shared else u((vocab, dim), 1.0)
    return m


def write_checkpoint(m: dict, path: str, drop_bytes: int = 0) -> None:
    header = np.array([m["dim"], m["hidden"], m["layers"], m["heads"], m["kv_heads"],
                       m["vocab"] if m["shared"] else -m["vocab"], m["seq_len"]], dtype="<i4")
    parts = [header.tobytes(), m["emb"].astype("<f4").tobytes()]
    for name in ("rms_att", "wq", "wk", "wv", "wo", "rms_ffn", "w1", "w2", "w3"):
        parts += [a.astype("<f4").tobytes() for a in m[name]]
    parts.append(m["rms_final"].astype("<f4").tobytes())
    hs = m["dim"] // m["heads"]
    parts.append(np.full(m["seq_len"] * hs, 123.0, dtype="<f4").tobytes())
    if not m["shared"]:
        parts.append(m["wcls"].astype("<f4").tobytes())
    data = b"".join(parts)
    with open(path, "wb") as f:
        f.write(data[:len(data) - drop_bytes] if drop_bytes else data)
