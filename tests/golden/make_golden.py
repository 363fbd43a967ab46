"""Generates the golden vectors in tests/golden/ from the reference engine's own code.

    make -C oracle ref && python tests/golden/make_golden.py

The reference's matmul.cpp / quant.cpp / ops.cpp are compiled from its sources by
oracle/Makefile into oracle/_ref/libllme_ref.so (with -ffp-contract=off, so a product and
the add after it round separately); this script feeds them seeded numpy inputs and stores
inputs and outputs as .npz. The reference ships no golden data of its own (its tests draw
from std::mt19937 at run time), so these files pin the oracle restatement to the
reference's actual outputs. Shapes follow the reference's own test lists
(tests/test_matmul.cpp:89-100, tests/test_quant.cpp:33-79), with wide dimensions trimmed
to keep the file small; every block edge of the CPU kernels is still crossed.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import oracle  # noqa: E402  (test infrastructure)

# tests/test_matmul.cpp:89-100 (every block edge of the CPU kernels) and decode shapes.
MATMUL_SHAPES = [(1, 1, 1), (1, 17, 1), (3, 5, 7), (4, 256, 16), (5, 257, 17), (63, 300, 65),
                 (64, 255, 40), (1, 300, 130), (2, 64, 41), (3, 1000, 17), (4, 4097, 9),
                 (5, 200, 30), (8, 513, 49), (1, 0, 5), (6, 0, 3)]
# tests/test_quant.cpp:57-79
Q8_SHAPES = [(1, 1, 1), (1, 300, 130), (3, 1000, 17), (4, 4097, 9), (5, 257, 17),
             (64, 255, 40), (2, 0, 5)]


def main() -> None:
    ref = oracle.Reference(fast=False)
    rng = np.random.default_rng(20261201)
    out = {}

    # Known answer, tests/test_matmul.cpp:40-52.
    A = np.arange(1, 7, dtype=np.float32).reshape(2, 3)
    B = np.arange(7, 13, dtype=np.float32).reshape(3, 2)
    out["known_A"], out["known_B"], out["known_C"] = A, B, ref.matmul_naive(A, B)

    # Quantiser: tests/test_quant.cpp:33-51 (spread scales, an all-zero column), BASELINE's
    # N(0, 0.02^2) weights, and values landing exactly on rounding ties.
    B0 = rng.uniform(-2, 2, (37, 21)).astype(np.float32)
    B0[5, :] *= np.arange(1, 22, dtype=np.float32)
    B0[:, 4] = 0.0
    B1 = (rng.standard_normal((96, 80)) * 0.02).astype(np.float32)
    B2 = np.array([[127.0, -127.0, 2.5, 0.0], [0.5, -0.5, -2.5, 0.0], [1.5, 63.5, 127.0, 0.0],
                   [-1.5, -63.5, 0.25, 0.0]], dtype=np.float32)
    for i, Bq in enumerate((B0, B1, B2)):
        q, s = ref.quantize_q8(Bq)
        out[f"quant{i}_B"], out[f"quant{i}_q"], out[f"quant{i}_scale"] = Bq, q, s
        out[f"quant{i}_deq"] = ref.dequantize(q, s)

    # matmul_naive on fp32.
    for i, (m, k, n) in enumerate(MATMUL_SHAPES):
        A = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        B = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        out[f"mm{i}_A"], out[f"mm{i}_B"], out[f"mm{i}_C"] = A, B, ref.matmul_naive(A, B)

    # int8: naive on the dequantised weights, and the thread-pool path (1 and 3 threads).
    for i, (m, k, n) in enumerate(Q8_SHAPES):
        A = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        q, s = ref.quantize_q8(rng.uniform(-0.5, 0.5, (k, n)).astype(np.float32))
        out[f"q8_{i}_A"], out[f"q8_{i}_q"], out[f"q8_{i}_scale"] = A, q, s
        out[f"q8_{i}_naive"] = ref.matmul_naive(A, ref.dequantize(q, s))
        h = ref.qtensor(q, s)
        out[f"q8_{i}_par1"] = ref.matmul_parallel_q8(A, h, threads=1)
        out[f"q8_{i}_par3"] = ref.matmul_parallel_q8(A, h, threads=3)

    # RMSNorm (ops.cpp:8-26), used by MatmulFusion's oracle.
    for i, (r, c) in enumerate([(1, 288), (3, 100), (8, 1024)]):
        x = rng.uniform(-1, 1, (r, c)).astype(np.float32)
        w = rng.uniform(-1, 1, c).astype(np.float32)
        out[f"rms{i}_x"], out[f"rms{i}_w"], out[f"rms{i}_y"] = x, w, ref.rmsnorm(x, w)

    path = os.path.join(HERE, "reference_vectors.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
