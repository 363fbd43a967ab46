"""The transformer engine's C++ checkpoint reader (llme_checkpoint_config: the header and size
checks llme_model_load makes, llm-engine_b200/csrc/model.cu) against the reference's own
load_checkpoint (src/model.cpp:113-163, compiled into oracle/_ref/libref_model.so) on corrupted
llama2.c files: header fields set to zero, negative or inconsistent values, truncated or
over-long files, a missing file. Both readers must accept the same files and reject the others
with the same message. No GPU."""
from __future__ import annotations

import os

import numpy as np
import pytest
from hypothesis import given, settings, strategies as st

import oracle
import llme_b200 as L
from model_fixture import make_model, write_checkpoint

pytestmark = pytest.mark.skipif(not oracle.RefModel.available(), reason="reference model not built")


def outcome_ours(path):
    try:
        L.checkpoint_config(path)
        return "ok"
    except L.InvalidArgument as e:
        return str(e)


def outcome_reference(path):
    try:
        oracle.RefModel(path, False).close()
        return "ok"
    except RuntimeError as e:
        return str(e)


@settings(max_examples=120, deadline=None)
@given(field=st.integers(0, 6), value=st.sampled_from([0, -1, -7, 1, 3, 5, 6, 64, 1 << 20]),
       tail=st.sampled_from([0, -4, -1, 4, 1]), shared=st.booleans())
def test_corrupted_headers_and_sizes(tmp_path_factory, field, value, tail, shared):
    path = str(tmp_path_factory.mktemp("ck") / "m.bin")
    m = make_model(dim=32, hidden=48, layers=1, heads=4, kv_heads=2, vocab=20, seq_len=8,
                   shared=shared, seed=1)
    write_checkpoint(m, path)
    raw = bytearray(open(path, "rb").read())
    header = np.frombuffer(bytes(raw[:28]), dtype="<i4").copy()
    header[field] = value
    raw[:28] = header.tobytes()
    if tail < 0:
        raw = raw[:tail]
    elif tail > 0:
        raw += b"\0" * tail
    with open(path, "wb") as f:
        f.write(bytes(raw))
    assert outcome_ours(path) == outcome_reference(path)


def test_missing_and_short_files(tmp_path):
    missing = str(tmp_path / "missing.bin")
    assert outcome_ours(missing) == outcome_reference(missing) != "ok"
    for size in (0, 5, 27):
        p = str(tmp_path / f"short{size}.bin")
        with open(p, "wb") as f:
            f.write(b"\1" * size)
        assert outcome_ours(p) == outcome_reference(p) != "ok", size
