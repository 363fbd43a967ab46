"""Tensor-parallel sharding of the matmul path (host side).

The reference runs on one GPU (one CudaTransformer, src/cuda_model.h); this module
splits the 7B-shaped chain across the GPUs of one box:

* column-parallel weights (wq, wk, wv, w1, w3, classifier): B (k x n) is split along n;
  each rank holds the contiguous k x n_r block and the matching slice of the column scales,
  multiplies the full activation row and owns those output columns -- no exchange;
* row-parallel weights (wo, w2): B is split along k; each rank holds rows [k0, k0 + k_r), the
  matching columns of A and the *whole* scale vector (the column scale multiplies each
  partial sum, which is linear), and the partial m x n products are summed by one all-reduce
  (llme_allreduce_sum_f32 / llme_matmul_*_rowpar). With MatmulFusion::accumulate only rank 0
  adds the existing C, so the sum counts it once.

Works on numpy arrays and torch tensors alike (only slicing is used).
"""
from __future__ import annotations

PARALLELISM = {"wq": "column", "wk": "column", "wv": "column", "wo": "row",
               "w1": "column", "w3": "column", "w2": "row", "cls": "column"}


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, start + count) of `total` for `rank`; the first total % world ranks
    take one extra element, so shards differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def column_shard(B, scale, world: int, rank: int):
    """This rank's k x n_r block of B (made contiguous) and its slice of the scales."""
    s, c = shard_range(B.shape[1], world, rank)
    blk = B[:, s:s + c]
    blk = blk.contiguous() if hasattr(blk, "contiguous") else blk.copy()
    return blk, (None if scale is None else scale[s:s + c])


def row_shard(B, world: int, rank: int):
    """This rank's k_r x n block of B (rows are contiguous already)."""
    s, c = shard_range(B.shape[0], world, rank)
    return B[s:s + c]


def activation_columns(A, world: int, rank: int):
    """The columns of A (m x k) that multiply this rank's row shard."""
    s, c = shard_range(A.shape[1], world, rank)
    blk = A[:, s:s + c]
    return blk.contiguous() if hasattr(blk, "contiguous") else blk.copy()


def accumulate_on_this_rank(accumulate: bool, rank: int) -> bool:
    """Row-parallel residual add: only rank 0 adds C before the sum."""
    return bool(accumulate) and rank == 0
