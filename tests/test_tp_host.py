"""Host side of the transformer engine (no GPU): the C++ checkpoint reader's header and size
rules (llme_checkpoint_config, the same checks llme_model_load makes) on files the reference
reads, the RoPE tables against the reference's own (rope_tables, model.cpp:171-184, compiled
into oracle/_ref), the tensor-parallel partition of heads, hidden units and vocabulary, the
reference CPU Transformer that the GPU tests use as their oracle, and the argument checks of
the decode-step kernels."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import llme_b200 as L
from model_fixture import make_model, write_checkpoint


def test_checkpoint_config_reads_the_header(tmp_path):
    m = make_model(dim=32, hidden=48, layers=2, heads=4, kv_heads=2, vocab=20, seq_len=8, seed=3)
    p = str(tmp_path / "m.bin")
    write_checkpoint(m, p)
    assert L.checkpoint_config(p) == dict(dim=32, hidden_dim=48, n_layers=2, n_heads=4,
                                          n_kv_heads=2, vocab_size=20, seq_len=8)
    ms = make_model(dim=32, hidden=48, layers=1, heads=4, kv_heads=4, vocab=20, seq_len=8,
                    shared=True, seed=4)
    write_checkpoint(ms, p)  # classifier shared with the embedding: vocab stored positive
    assert L.checkpoint_config(p)["vocab_size"] == 20


def test_checkpoint_reader_rejects_what_the_reference_rejects(tmp_path):
    m = make_model(dim=32, hidden=48, layers=1, heads=4, kv_heads=2, vocab=20, seq_len=8)
    p = str(tmp_path / "m.bin")
    write_checkpoint(m, p, drop_bytes=4)
    with pytest.raises(L.InvalidArgument, match="header implies"):
        L.checkpoint_config(p)
    bad = dict(m, heads=3)  # 32 does not split into 3 heads
    write_checkpoint(bad, p)
    with pytest.raises(L.InvalidArgument, match="even-sized heads"):
        L.checkpoint_config(p)
    with pytest.raises(L.InvalidArgument, match="cannot open"):
        L.checkpoint_config(str(tmp_path / "missing.bin"))


@pytest.mark.skipif(not oracle.RefModel.available(), reason="reference model not built here")
@pytest.mark.parametrize("seq_len,dim,heads", [(16, 64, 8), (256, 4096, 32), (64, 96, 2)])
def test_rope_tables_match_the_reference_bit_for_bit(seq_len, dim, heads):
    cos, sin = L.rope_tables(seq_len, dim // heads)
    rc, rs = oracle.ref_rope_tables(seq_len, dim, heads)
    np.testing.assert_array_equal(cos, rc)
    np.testing.assert_array_equal(sin, rs)


@pytest.mark.parametrize("cfg", [
    dict(dim=64, hidden_dim=96, n_layers=1, n_heads=8, n_kv_heads=4, vocab_size=50, seq_len=8),
    dict(dim=4096, hidden_dim=11008, n_layers=32, n_heads=32, n_kv_heads=32, vocab_size=32000,
         seq_len=2048),
    dict(dim=4096, hidden_dim=14336, n_layers=32, n_heads=32, n_kv_heads=8, vocab_size=128256,
         seq_len=8192)])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_partition_covers_every_head_unit_and_token_once(cfg, world):
    if cfg["n_kv_heads"] % world:
        with pytest.raises(L.InvalidArgument, match="do not split"):
            L.model_partition(cfg, world, 0)
        return
    group = cfg["n_heads"] // cfg["n_kv_heads"]
    q, kv, hid, voc = [], [], [], []
    for r in range(world):
        s = L.model_partition(cfg, world, r)
        assert s["nq"] == s["nkv"] * group and s["q0"] == s["kv0"] * group
        q += list(range(s["q0"], s["q0"] + s["nq"]))
        kv += list(range(s["kv0"], s["kv0"] + s["nkv"]))
        hid += list(range(s["h0"], s["h0"] + s["hc"]))
        voc.append((s["v0"], s["vc"]))
        # contiguous blocks, sizes differing by at most one
        assert abs(s["hc"] - cfg["hidden_dim"] / world) < 1
        assert abs(s["vc"] - cfg["vocab_size"] / world) < 1
    assert q == list(range(cfg["n_heads"])) and kv == list(range(cfg["n_kv_heads"]))
    assert hid == list(range(cfg["hidden_dim"]))
    assert [v0 for v0, _ in voc] == list(np.cumsum([0] + [vc for _, vc in voc[:-1]]))
    assert sum(vc for _, vc in voc) == cfg["vocab_size"]


def test_partition_rejects_bad_configurations():
    good = dict(dim=64, hidden_dim=96, n_layers=1, n_heads=8, n_kv_heads=4, vocab_size=50,
                seq_len=8)
    for bad in (dict(good, n_heads=6), dict(good, n_kv_heads=3), dict(good, dim=0)):
        with pytest.raises(L.InvalidArgument):
            L.model_partition(bad, 1, 0)
    with pytest.raises(L.InvalidArgument):
        L.model_partition(good, 2, 2)


@pytest.mark.skipif(not oracle.RefModel.available(), reason="reference model not built here")
@pytest.mark.parametrize("q8", [False, True])
def test_reference_model_oracle(q8, tmp_path):
    # The oracle harness itself: the reference's prefill equals its token-by-token forward
    # (its own contract, model.h:91-99), and a call past the cache is refused.
    m = make_model(dim=32, hidden=48, layers=2, heads=4, kv_heads=2, vocab=20, seq_len=8, seed=6)
    p = str(tmp_path / "m.bin")
    write_checkpoint(m, p)
    a, b = oracle.RefModel(p, q8), oracle.RefModel(p, q8)
    toks = [3, 7, 1, 19, 0]
    for i, t in enumerate(toks):
        last = a.run([t], i)
    pre = b.run(toks, 0)
    assert np.isfinite(pre).all()
    np.testing.assert_allclose(pre, last, rtol=1e-4, atol=1e-4)
    with pytest.raises(RuntimeError, match="positions"):
        a.run([1], 7 + 2)


def test_decode_step_arguments_are_checked_before_any_launch():
    # Every refusal here happens on the host; nothing is launched and the fake addresses are
    # never read. Empty work is a no-op that touches no GPU either.
    P = 256
    L.embed_rows(0, 64, P, P, P)
    L.rope_cache(0, 4, 2, 8, P, P, P, P, P, P)
    L.swiglu(0, 96, P, P)
    bad = [lambda: L.embed_rows(1, 64, 0, P, P),
           lambda: L.embed_rows(65536, 64, P, P, P),
           lambda: L.embed_rows(1 << 15, 1 << 16, P, P, P),           # 2^31 elements
           lambda: L.rope_cache(1, 4, 2, 7, P, P, P, P, P, P),        # odd head_size
           lambda: L.rope_cache(1, 4, 0, 8, P, P, P, P, P, P),        # no kv heads
           lambda: L.rope_cache(65536, 4, 2, 8, P, P, P, P, P, P),
           lambda: L.rope_cache(1, 4, 2, 8, P, P, P, 0, P, P),
           lambda: L.swiglu(1, 1 << 30, P, P),
           lambda: L.swiglu(1, 96, P, 0),
           lambda: L.rope_tables(4, 7)]
    for call in bad:
        with pytest.raises(L.InvalidArgument):
            call()
