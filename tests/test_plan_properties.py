"""Properties of the dispatch plan (llme_plan, host only) over random shapes, kernels, weight
types, arithmetic modes, SM counts and pointer alignments: every plan either refuses the call
with LLME_E_INVALID or describes launches that cover C and k exactly once within the
hardware's grid and cluster limits, and a path that reads an operand by TMA or computes on the
tensor cores is only chosen when its alignment and arithmetic-mode preconditions hold. The
argument checks follow the reference's matmul_impl (src/cuda_matmul.cu:399-422)."""
from __future__ import annotations

from hypothesis import given, settings, strategies as st

import llme_b200 as L

KERNELS = ["automatic", "naive", "tiled", "tiled_split", "skinny"]
TENSOR_PATHS = {"tcgen05", "tcgen05_q8", "tcgen05_skinny", "tcgen05_f32_skinny"}
TMA_PATHS = {"gemv_tma"} | TENSOR_PATHS
LIMIT = 1 << 31
NAMES = {v: name for name, v in L.KERNELS.items()}


def dims():
    # Mostly small and ragged, sometimes exactly on or next to a tile edge, sometimes large.
    edges = st.sampled_from([1, 4, 8, 9, 16, 31, 32, 33, 64, 127, 128, 129, 255, 256, 1000,
                             4096, 4100, 6144, 11008])
    return st.one_of(st.integers(0, 300), edges, st.integers(0, 70000))


@settings(max_examples=3000, deadline=None)
@given(m=dims(), n=dims(), k=dims(), q8=st.booleans(), kernel=st.sampled_from(KERNELS),
       accumulate=st.booleans(), math=st.sampled_from([L.MATH_TENSOR, L.MATH_FP32]),
       sms=st.sampled_from([148, 132, 20, 1]),
       a_off=st.sampled_from([0, 4, 8, 12]), b_off=st.sampled_from([0, 1, 4, 8]),
       rms=st.sampled_from([0, 256, 260]))
def test_every_plan_covers_c_and_k_within_limits(m, n, k, q8, kernel, accumulate, math, sms,
                                                 a_off, b_off, rms):
    a_addr, b_addr = 256 + a_off, 256 + (b_off if q8 else b_off // 4 * 4)
    try:
        p = L.plan(m, n, k, q8=q8, kernel=kernel, accumulate=accumulate, a_addr=a_addr,
                   b_addr=b_addr, rms_addr=rms, sm_count=sms, math=math)
    except L.InvalidArgument as e:
        msg = str(e)
        too_big = m * k >= LIMIT or k * n >= LIMIT or m * n >= LIMIT
        assert (kernel == "skinny" and m > 8) or too_big or "exceed the grid's 65535" in msg, msg
        return
    assert not (kernel == "skinny" and m > 8)
    assert max(m * k, k * n, m * n) < LIMIT
    path = p["path_name"]
    assert kernel == "automatic" or NAMES[p["kernel"]] == kernel
    if kernel == "automatic":
        assert NAMES[p["kernel"]] == ("skinny" if m <= 8 else "tiled_split" if m < 128 else "tiled")
    kernel = NAMES[p["kernel"]]  # the kernel after resolving automatic
    if m == 0 or n == 0:
        assert path == "none"
        return
    if k == 0:
        assert path == ("none" if accumulate else "zero")
        return
    assert p["grid_x"] >= 1 and 1 <= p["grid_y"] <= 65535
    assert p["grid_x"] <= LIMIT - 1
    s, span = p["slices"], p["span"]
    assert s >= 1 and span >= 1 and (s - 1) * span < k <= s * span, p
    assert 1 <= p["cluster"] <= 8 or p["cluster"] == 0

    # arithmetic mode and operand preconditions of the path
    if path in TENSOR_PATHS:
        assert math == L.MATH_TENSOR
    if path in TMA_PATHS:
        assert b_addr % 16 == 0
    if path == "gemv_ldg":
        assert m <= 8 and kernel == "skinny"
    if path == "gemv_tma":
        # m <= 8 through skinny; fp32 B with 9..16 rows through tiled_split (automatic) or
        # tiled, in fp32 arithmetic.
        assert (m <= 8 and kernel == "skinny") or (not q8 and 9 <= m <= 16 and math == L.MATH_FP32
                                                   and kernel in ("tiled", "tiled_split"))
    if path == "gemv_tma":
        assert a_addr % 16 == 0 and k % 4 == 0 and (n * (1 if q8 else 4)) % 16 == 0
        assert rms == 0 or rms % 16 == 0
        assert span % 128 == 0 and s <= 8 and p["cluster"] == s
        # RMSNorm inside the kernel up to 8 rows; the 16-row fp32 form takes the row pass
        assert p["split_bytes"] == 0 and p["rms_prepass"] == (1 if rms and m > 8 else 0)
    if path == "naive":
        assert kernel == "naive" and s == 1
    if path == "tcgen05":
        assert not q8 and m >= 128 and k % 4 == 0 and n % 4 == 0 and kernel == "tiled"
        assert rms or a_addr % 16 == 0
        assert p["operand_bytes"] == (4 * k * n if m >= 6144 else 0)
    if path == "tcgen05_q8":
        assert q8 and m >= 128 and n % 16 == 0 and kernel == "tiled"
        assert p["grid_x"] <= sms and p["operand_bytes"] > 0
    if path == "tcgen05_skinny":
        assert q8 and n % 16 == 0 and kernel in ("tiled", "tiled_split")
        assert span % 128 == 0 and p["operand_bytes"] > 0
        assert s <= 8 and p["cluster"] == s and p["split_bytes"] == 0
    if path == "tcgen05_f32_skinny":
        assert not q8 and n % 4 == 0 and k % 4 == 0 and kernel in ("tiled", "tiled_split")
        assert rms or a_addr % 16 == 0
        assert s <= 8 and p["cluster"] == s and span % 32 == 0
    if path == "tiled_simt":
        assert span % 16 == 0

    # C is covered: columns by grid x (or the persistent GEMM's tile loop), rows by grid y
    if path in ("tcgen05", "tcgen05_q8"):
        assert p["grid_y"] == 1 and s == 1
    else:
        assert p["grid_x"] * p["tile_n"] >= n
        if path in ("gemv_tma", "gemv_ldg"):
            # every row in one CTA (16 for fp32 B past 8 rows); grid y holds the k slices
            assert p["tile_m"] == (m if m <= 8 else 16)
        else:
            assert p["grid_y"] * p["tile_m"] >= m
    # scratch is asked for only when the path uses it, and the normalised copy of A only
    # when RMSNorm runs as a separate pass
    if p["rms_prepass"]:
        assert rms and p["norm_bytes"] == 4 * m * k
    else:
        assert p["norm_bytes"] == 0


@settings(max_examples=1500, deadline=None)
@given(n=dims(), k=dims(), q8=st.booleans(), m=st.integers(1, 8),
       sms=st.sampled_from([148, 132, 20]),
       shrink=st.lists(st.floats(0.3, 1.0), min_size=8, max_size=8))
def test_gemv_clusters_fit_the_device_capacity(n, k, q8, m, sms, shrink):
    # For any device capacity table (clusters of c CTAs it holds at once, at most the model's
    # 2 x SMs / c and not growing with c), the GEMV's k slices leave every cluster resident
    # at once and still cover k exactly once; the device never takes more slices than the
    # model would.
    model = [2 * sms // c for c in range(1, 9)]
    table, prev = [], None
    for c in range(8):
        v = max(1, int(model[c] * shrink[c]))
        v = min(v, prev) if prev is not None else v
        table.append(v)
        prev = v
    kw = dict(q8=q8, kernel="skinny", sm_count=sms)
    try:
        base = L.plan(m, n, k, **kw)
    except L.InvalidArgument:
        return
    if base["path_name"] != "gemv_tma":
        return
    p = L.plan(m, n, k, gemv_clusters=table, **kw)
    s, span = p["slices"], p["span"]
    assert p["path_name"] == "gemv_tma" and p["grid_x"] == base["grid_x"]
    assert s == 1 or p["grid_x"] <= table[s - 1], (table, p)
    assert (s - 1) * span < k <= s * span and span % 128 == 0
    assert p["cluster"] == s and s <= base["slices"]
