"""The device side of the dispatch plan: the weight-streaming GEMV's thread-block cluster capacity
as the driver reports it (llme_gemv_cluster_capacity), the plan a call then takes
(llme_plan_clusters with that table), and that call's product against the oracle
(matmul_naive_q8, the reference's src/matmul.cpp restated and pinned)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import llme_b200 as L
from conftest import close_to

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_gemv_cluster_capacity_is_a_packing_of_the_sms():
    L.load()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    cap = L.gemv_cluster_capacity()
    print("GEMV cluster capacity, sizes 1..8:", cap)
    assert sms <= cap[0] <= 2 * sms                 # clusters of one: up to two CTAs per SM
    for c in range(2, 9):
        assert 0 < cap[c - 1] <= 2 * sms // c       # never more CTAs than the SMs hold
        assert cap[c - 1] <= cap[c - 2]


def test_decode_product_on_the_device_plan_matches_the_oracle():
    # The 7B wqkv shape (96 column strips): its slices are chosen so every cluster is resident
    # at once on this device; the product is the oracle's within the reference's tolerance.
    L.load()
    cap = L.gemv_cluster_capacity()
    m, n, k = 1, 12288, 4096
    p = L.plan(m, n, k, q8=True, gemv_clusters=cap)
    assert p["path_name"] == "gemv_tma" and p["grid_x"] <= cap[p["grid_y"] - 1]
    rng = np.random.default_rng(31)
    A = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    q, s = oracle.quantize_q8((rng.standard_normal((k, n)) * 0.02).astype(np.float32))
    got = L.matmul(torch.from_numpy(A).cuda(), torch.from_numpy(q).cuda(),
                   scale=torch.from_numpy(s).cuda()).cpu().numpy()
    assert close_to(got, oracle.matmul_naive_q8(A, q, s), k)
