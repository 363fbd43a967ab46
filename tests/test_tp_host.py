"""Host side of the tensor-parallel transformer (no GPU): the checkpoint loader against the
llama2.c layout the reference reads (src/model.cpp:113-169), the RoPE tables against the
reference's own (rope_tables, model.cpp:171-184, compiled into oracle/_ref), the head / hidden
partition, and the reference CPU Transformer that the GPU tests use as their oracle."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import llme_b200 as L
from checkpoint import load_checkpoint
from model_fixture import make_model, write_checkpoint
from tp_decode import head_partition, shard_layer


def test_loader_concatenates_and_transposes_like_the_reference(tmp_path):
    m = make_model(dim=32, hidden=48, layers=2, heads=4, kv_heads=2, vocab=20, seq_len=8, seed=3)
    p = str(tmp_path / "m.bin")
    write_checkpoint(m, p)
    ck = load_checkpoint(p)
    c = ck.config
    assert (c.dim, c.hidden_dim, c.n_layers, c.n_heads, c.n_kv_heads, c.vocab_size, c.seq_len) == \
        (32, 48, 2, 4, 2, 20, 8)
    assert c.head_size == 8 and c.kv_dim == 16
    for l, lw in enumerate(ck.layers):
        np.testing.assert_array_equal(lw.wqkv, np.concatenate([m["wq"][l].T, m["wk"][l].T,
                                                               m["wv"][l].T], axis=1))
        np.testing.assert_array_equal(lw.w13, np.concatenate([m["w1"][l].T, m["w3"][l].T], axis=1))
        np.testing.assert_array_equal(lw.wo, m["wo"][l].T)
        np.testing.assert_array_equal(lw.w2, m["w2"][l].T)
        np.testing.assert_array_equal(lw.rms_att, m["rms_att"][l])
    np.testing.assert_array_equal(ck.wcls, m["wcls"].T)
    np.testing.assert_array_equal(ck.token_embedding, m["emb"])
    ms = make_model(dim=32, hidden=48, layers=1, heads=4, kv_heads=4, vocab=20, seq_len=8,
                    shared=True, seed=4)
    write_checkpoint(ms, p)
    np.testing.assert_array_equal(load_checkpoint(p).wcls, ms["emb"].T)


def test_loader_rejects_what_the_reference_rejects(tmp_path):
    m = make_model(dim=32, hidden=48, layers=1, heads=4, kv_heads=2, vocab=20, seq_len=8)
    p = str(tmp_path / "m.bin")
    write_checkpoint(m, p, drop_bytes=4)
    with pytest.raises(RuntimeError, match="header implies"):
        load_checkpoint(p)
    bad = dict(m, heads=3)  # 32 does not split into 3 heads
    write_checkpoint(bad, p)
    with pytest.raises(RuntimeError, match="even-sized heads"):
        load_checkpoint(p)
    with pytest.raises(RuntimeError, match="cannot open"):
        load_checkpoint(str(tmp_path / "missing.bin"))


@pytest.mark.skipif(not oracle.RefModel.available(), reason="reference model not built here")
@pytest.mark.parametrize("seq_len,dim,heads", [(16, 64, 8), (256, 4096, 32), (64, 96, 2)])
def test_rope_tables_match_the_reference_bit_for_bit(seq_len, dim, heads):
    cos, sin = L.rope_tables(seq_len, dim // heads)
    rc, rs = oracle.ref_rope_tables(seq_len, dim, heads)
    np.testing.assert_array_equal(cos, rc)
    np.testing.assert_array_equal(sin, rs)


@pytest.mark.parametrize("world", [1, 2, 4])
def test_shards_reassemble_the_layer(world, tmp_path):
    # Column shards cover every q / k / v / gate / up column once; row-parallel partial
    # products sum to the unsharded product (numpy, float64).
    m = make_model(dim=64, hidden=96, layers=1, heads=8, kv_heads=4, vocab=50, seq_len=8, seed=5)
    p = str(tmp_path / "m.bin")
    write_checkpoint(m, p)
    ck = load_checkpoint(p)
    cfg, lw = ck.config, ck.layers[0]
    rng = np.random.default_rng(1)
    x = rng.uniform(-1, 1, (3, cfg.dim))
    qkv_full = x @ lw.wqkv.astype(np.float64)
    att = rng.uniform(-1, 1, (3, cfg.dim))
    hb = rng.uniform(-1, 1, (3, cfg.hidden_dim))
    hs, D, KV, H = cfg.head_size, cfg.dim, cfg.kv_dim, cfg.hidden_dim
    wo_sum = np.zeros((3, D))
    w2_sum = np.zeros((3, D))
    seen_q, seen_kv, seen_h = [], [], []
    for r in range(world):
        q0, nq, kv0, nkv = head_partition(cfg.n_heads, cfg.n_kv_heads, world, r)
        assert nq == nkv * (cfg.n_heads // cfg.n_kv_heads)
        sh = shard_layer(lw, cfg, world, r)
        local = x @ sh["wqkv"].astype(np.float64)
        np.testing.assert_allclose(local[:, :nq * hs], qkv_full[:, q0 * hs:(q0 + nq) * hs])
        np.testing.assert_allclose(local[:, nq * hs:(nq + nkv) * hs],
                                   qkv_full[:, D + kv0 * hs:D + (kv0 + nkv) * hs])
        np.testing.assert_allclose(local[:, (nq + nkv) * hs:],
                                   qkv_full[:, D + KV + kv0 * hs:D + KV + (kv0 + nkv) * hs])
        r0, rc = sh["wo_rows"]
        wo_sum += att[:, r0:r0 + rc] @ lw.wo[r0:r0 + rc].astype(np.float64)
        h0, hc = sh["w2_rows"]
        assert sh["w13"].shape == (D, 2 * hc)
        np.testing.assert_array_equal(sh["w13"][:, :hc], lw.w13[:, h0:h0 + hc])
        np.testing.assert_array_equal(sh["w13"][:, hc:], lw.w13[:, H + h0:H + h0 + hc])
        w2_sum += hb[:, h0:h0 + hc] @ lw.w2[h0:h0 + hc].astype(np.float64)
        seen_q += list(range(q0, q0 + nq))
        seen_kv += list(range(kv0, kv0 + nkv))
        seen_h += list(range(h0, h0 + hc))
    assert seen_q == list(range(cfg.n_heads)) and seen_kv == list(range(cfg.n_kv_heads))
    assert seen_h == list(range(H))
    np.testing.assert_allclose(wo_sum, att @ lw.wo.astype(np.float64), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(w2_sum, hb @ lw.w2.astype(np.float64), rtol=1e-12, atol=1e-12)


def test_kv_heads_must_split_evenly():
    with pytest.raises(L.InvalidArgument):
        head_partition(8, 2, 4, 0)


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
