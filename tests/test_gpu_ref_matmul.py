"""The reference's own GPU matmul (src/cuda_matmul.cu built for sm_100a into
oracle/_ref/libref_matmul_gpu.so by `make -C oracle refmatmul`) as a second oracle on the
B200: on the shapes of the reference's tests/test_cuda.cpp:66-72 and every kernel choice, its
output must sit within the reference's own tolerance of matmul_naive (1e-5 * k), and this
library's output within twice that of it (the TF32 GEMM within its 5e-3 row bound). Skipped
where that library is not built."""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest

import oracle
import llme_b200 as L
from conftest import close_to, row_rel_err

torch = pytest.importorskip("torch")

REF = os.path.join(os.path.dirname(oracle.HERE), "oracle", "_ref", "libref_matmul_gpu.so")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.exists(REF), reason="oracle/_ref/libref_matmul_gpu.so not built")]

KERNELS = ["automatic", "naive", "tiled", "tiled_split", "skinny"]  # GpuKernel order
SHAPES = [(1, 1, 1), (3, 5, 7), (8, 8, 128), (9, 9, 129), (127, 300, 129), (128, 256, 128),
          (130, 70, 1030), (1, 4096, 288), (4, 4097, 33), (16, 4096, 300), (64, 2000, 4096)]


@pytest.fixture(scope="module")
def ref():
    lib = ctypes.CDLL(REF)
    sz, vp, ci = ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int
    lib.ref_gpu_matmul_f32.argtypes = [sz, sz, sz, vp, vp, vp, ci, ci, vp]
    lib.ref_gpu_matmul_q8.argtypes = [sz, sz, sz, vp, vp, vp, vp, ci, ci, vp]
    lib.ref_gpu_error.restype = ctypes.c_char_p
    L.load()
    yield lib
    L.device_status()


def run_ref(ref, A, B=None, q=None, s=None, kernel=0):
    m, k = A.shape
    n = (q if q is not None else B).shape[1]
    dA = torch.from_numpy(A).cuda()
    dC = torch.full((m, n), float("nan"), device="cuda")
    if q is not None:
        dq, ds = torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()
        torch.cuda.synchronize()
        rc = ref.ref_gpu_matmul_q8(m, n, k, dA.data_ptr(), dq.data_ptr(), ds.data_ptr(),
                                   dC.data_ptr(), kernel, 0, None)
    else:
        dB = torch.from_numpy(B).cuda()
        torch.cuda.synchronize()
        rc = ref.ref_gpu_matmul_f32(m, n, k, dA.data_ptr(), dB.data_ptr(), dC.data_ptr(),
                                    kernel, 0, None)
    assert rc == 0, ref.ref_gpu_error().decode()
    assert ref.ref_gpu_synchronize() == 0, ref.ref_gpu_error().decode()
    return dC.cpu().numpy()


def run_ours(A, B=None, q=None, s=None, kernel="automatic"):
    dA = torch.from_numpy(A).cuda()
    if q is not None:
        C = L.matmul(dA, torch.from_numpy(q).cuda(), scale=torch.from_numpy(s).cuda(), kernel=kernel)
    else:
        C = L.matmul(dA, torch.from_numpy(B).cuda(), kernel=kernel)
    torch.cuda.synchronize()
    return C.cpu().numpy()


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_reference_gpu_matmul_is_an_oracle_and_ours_agrees(ref, m, k, n):
    rng = np.random.default_rng(7 + m + 3 * k + 5 * n)
    A = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    B = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    q, s = oracle.quantize_q8(rng.uniform(-1, 1, (k, n)).astype(np.float32))
    want_f, want_q = oracle.matmul_naive(A, B), oracle.matmul_naive_q8(A, q, s)
    for kid, name in enumerate(KERNELS):
        if name == "skinny" and m > 8:
            continue
        rf, rq = run_ref(ref, A, B=B, kernel=kid), run_ref(ref, A, q=q, s=s, kernel=kid)
        assert close_to(rf, want_f, k), (name, "fp32", float(np.abs(rf - want_f).max()))
        assert close_to(rq, want_q, k), (name, "int8", float(np.abs(rq - want_q).max()))
        of, oq = run_ours(A, B=B, kernel=name), run_ours(A, q=q, s=s, kernel=name)
        if L.plan(m, n, k, q8=False, kernel=name, math=L.get_math())["path_name"] == "tcgen05":
            assert row_rel_err(of, rf) <= 5e-3, (name, "fp32 TF32", row_rel_err(of, rf))
        else:
            assert close_to(of, rf, k, 2.0), (name, "fp32", float(np.abs(of - rf).max()))
        assert close_to(oq, rq, k, 2.0), (name, "int8", float(np.abs(oq - rq).max()))
