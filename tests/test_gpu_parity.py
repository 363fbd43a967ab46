"""GPU parity: every kernel through the C ABI against the CPU oracle.

Mirrors the reference's tests/test_cuda.cpp: the shape list on and around tile edges
(:66-72) for every GpuKernel, output reuse (:93-105), every MatmulFusion case (:126-165),
int8 weights plain and fused (:170-213), back-to-back split-K launches that must repeat
bit for bit (:221-275) and the argument errors (:277-287). Tolerance as the reference:
|got - want| <= 1e-5 * k (2e-5 * k fused) against matmul_naive on identical inputs (the
dequantised weights for int8). The benchmark's decode shapes run at full size against the
decode path's accuracy bound, max over rows of ||C - C_ref||_inf / ||C_ref row||_2 <= 1e-5.
"""
from __future__ import annotations

import os
import subprocess

import numpy as np
import pytest

import oracle
import llme_b200 as L
from conftest import close_to, row_rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

KERNELS = [("naive", None), ("tiled", None), ("tiled_split", None), ("skinny", 8),
           ("automatic", None)]
# tests/test_cuda.cpp:66-72 (m, k, n)
SHAPES = [(1, 1, 1), (1, 17, 1), (3, 5, 7), (8, 8, 128), (9, 9, 129), (127, 300, 129),
          (128, 256, 128), (200, 513, 33), (130, 70, 1030), (1, 4096, 288), (1, 288, 4096),
          (2, 1000, 70), (4, 4097, 33), (7, 64, 4111), (8, 513, 2049), (16, 4096, 300),
          (33, 1029, 257), (64, 2000, 4096), (1, 0, 5), (12, 0, 3)]
Q8_EXTRA = [(3, 100, 1028), (8, 1000, 4100), (6, 20, 36), (1, 4096, 4)]


def uni(rng, *shape, scale=1.0):
    return rng.uniform(-scale, scale, shape).astype(np.float32)


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def path_of(m, n, k, q8, kernel, accumulate=False, rms=False):
    return L.plan(m, n, k, q8=q8, kernel=kernel, accumulate=accumulate,
                  rms_addr=256 if rms else 0, math=L.get_math())["path_name"]


def check(got, want, k, factor, path):
    """The reference's absolute 1e-5 * k bound for fp32-product paths; the tensor-core
    bound (5e-3 of the row's L2 norm) for the tensor-core paths."""
    if path in ("tcgen05", "tcgen05_q8"):
        return row_rel_err(got, want) <= 5e-3
    return close_to(got, want, k, factor)


def gpu_matmul(A, B=None, q=None, scale=None, kernel="automatic", C0=None, accumulate=False,
               rms=None, weights_static=False):
    m, k = A.shape
    n = (q if q is not None else B).shape[1]
    dA = dev(A)
    dC = dev(C0) if C0 is not None else torch.full((m, n), float("nan"), device="cuda")
    dW = dev(rms) if rms is not None else None
    if q is not None:
        L.matmul(dA, dev(q), scale=dev(scale), C=dC, kernel=kernel, accumulate=accumulate,
                 rms_weight=dW, weights_static=weights_static)
    else:
        L.matmul(dA, dev(B), C=dC, kernel=kernel, accumulate=accumulate, rms_weight=dW,
                 weights_static=weights_static)
    torch.cuda.synchronize()
    return dC.cpu().numpy()


@pytest.fixture(scope="module", autouse=True)
def _device():
    L.load()
    assert L.available() and L.device_supported(), "needs an sm_100 GPU"
    yield
    L.device_status()  # no bounded device wait gave up during the module


def test_native_library_is_loaded():
    L.load()
    maps = open("/proc/self/maps").read()
    assert L.library_path() in maps


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_fp32_every_kernel(m, k, n):
    rng = np.random.default_rng(42 + m * 7 + k * 3 + n)
    A, B = uni(rng, m, k), uni(rng, k, n)
    want = oracle.matmul_naive(A, B)
    for name, max_m in KERNELS:
        if max_m is not None and m > max_m:
            continue
        got = gpu_matmul(A, B=B, kernel=name)
        assert check(got, want, k, 1.0, path_of(m, n, k, False, name)), \
            (name, m, k, n, np.abs(got - want).max())


@pytest.mark.parametrize("m,k,n", SHAPES + Q8_EXTRA)
def test_q8_every_kernel(m, k, n):
    rng = np.random.default_rng(11 + m * 5 + k + n)
    A = uni(rng, m, k)
    q, s = oracle.quantize_q8(uni(rng, k, n))
    want = oracle.matmul_naive_q8(A, q, s)
    for name, max_m in KERNELS:
        if max_m is not None and m > max_m:
            continue
        got = gpu_matmul(A, q=q, scale=s, kernel=name)
        assert close_to(got, want, k), (name, m, k, n, np.abs(got - want).max())


@pytest.mark.parametrize("m,k,n", [(1, 288, 300), (3, 100, 70), (8, 513, 129), (9, 64, 33),
                                   (70, 40, 130)])
def test_fusion_every_kernel(m, k, n):
    # tests/test_cuda.cpp:126-165
    rng = np.random.default_rng(9 + m)
    A, B, C0, w = uni(rng, m, k), uni(rng, k, n), uni(rng, m, n), uni(rng, k)
    plain = oracle.matmul_naive(A, B)
    normed = oracle.matmul_naive(oracle.rmsnorm(A, w), B)
    cases = [("accumulate", True, None, C0 + plain), ("rms", False, w, normed),
             ("rms + accumulate", True, w, C0 + normed)]
    for name, max_m in KERNELS:
        if max_m is not None and m > max_m:
            continue
        for case, acc, rms, want in cases:
            got = gpu_matmul(A, B=B, kernel=name, C0=C0, accumulate=acc, rms=rms)
            path = path_of(m, n, k, False, name, acc, rms is not None)
            assert check(got, want, k, 2.0, path), (name, case, m, k, n)


@pytest.mark.parametrize("m,k,n", [(1, 288, 300), (5, 768, 288), (2, 20, 64), (3, 288, 30),
                                   (70, 40, 130)])
def test_q8_fused_every_kernel(m, k, n):
    # tests/test_cuda.cpp:190-212
    rng = np.random.default_rng(19 + m)
    A = uni(rng, m, k)
    q, s = oracle.quantize_q8(uni(rng, k, n))
    C0, w = uni(rng, m, n), uni(rng, k)
    want = C0 + oracle.matmul_naive_q8(oracle.rmsnorm(A, w), q, s)
    for name, max_m in KERNELS:
        if max_m is not None and m > max_m:
            continue
        got = gpu_matmul(A, q=q, scale=s, kernel=name, C0=C0, accumulate=True, rms=w)
        assert close_to(got, want, k, 2.0), (name, m, k, n)


def test_reuse_across_shapes():
    # tests/test_cuda.cpp:93-105: the split scratch is shared by calls of different shapes.
    rng = np.random.default_rng(5)
    for m, k, n in [(1, 2000, 300), (4, 100, 5000), (64, 3000, 64), (200, 64, 64)]:
        A, B = uni(rng, m, k), uni(rng, k, n)
        assert check(gpu_matmul(A, B=B), oracle.matmul_naive(A, B), k, 1.0,
                     path_of(m, n, k, False, "automatic"))


def test_split_k_queue_is_deterministic():
    # tests/test_cuda.cpp:221-275: back-to-back launches, no host sync in between; each
    # result matches the oracle and repeats give the same bits.
    rng = np.random.default_rng(13)
    cases = [((1, 4096, 4096), False, False), ((8, 4096, 4100), True, True),
             ((1, 288, 32000), True, False), ((3, 768, 288), False, True),
             ((1, 288, 864), True, True), ((5, 1000, 70), True, False),
             ((1, 11008, 4096), True, True), ((4, 4096, 11008), True, False)]
    repeats = 3
    for _ in range(2):
        outs, wants, keep = [], [], []
        for (m, k, n), q8, acc in cases:
            A, B, C0 = uni(rng, m, k), uni(rng, k, n), uni(rng, m, n)
            q, s = oracle.quantize_q8(B)
            prod = oracle.matmul_naive_q8(A, q, s) if q8 else oracle.matmul_naive(A, B)
            dA, dB, dq, ds = dev(A), dev(B), dev(q), dev(s)
            keep += [dA, dB, dq, ds]
            for _r in range(repeats):
                dC = dev(C0)
                if q8:
                    L.matmul(dA, dq, scale=ds, C=dC, kernel="skinny", accumulate=acc)
                else:
                    L.matmul(dA, dB, C=dC, kernel="skinny", accumulate=acc)
                outs.append(dC)
                wants.append((C0 + prod if acc else prod, k))
        torch.cuda.synchronize()
        for i, dC in enumerate(outs):
            got = dC.cpu().numpy()
            want, k = wants[i]
            assert close_to(got, want, k, 2.0), i
            if i % repeats:
                np.testing.assert_array_equal(got, outs[i - 1].cpu().numpy())


def test_scratch_settles_after_one_pass():
    # cuda_scratch_generation() contract (cuda_matmul.h:109-112): once a fixed sequence of
    # calls has run, repeating it allocates nothing, so it can be captured in a CUDA graph.
    rng = np.random.default_rng(17)
    shapes = [(1, 4096, 4096), (1, 4096, 11008), (1, 11008, 4096), (1, 4096, 32000),
              (16, 4096, 300), (3, 288, 4100)]
    ops = []
    for m, k, n in shapes:
        q, s = oracle.quantize_q8(uni(rng, k, n))
        ops.append((dev(uni(rng, m, k)), dev(q), dev(s), torch.empty(m, n, device="cuda")))

    def one_pass():
        for dA, dq, ds, dC in ops:
            L.matmul(dA, dq, scale=ds, C=dC, weights_static=True)
    one_pass()
    torch.cuda.synchronize()
    gen = L.scratch_generation()
    one_pass()
    one_pass()
    torch.cuda.synchronize()
    assert L.scratch_generation() == gen


@pytest.mark.parametrize("m,k", [(8, 5504), (6, 5504), (5, 5504), (8, 2816), (7, 11008)])
def test_cluster_reduction_with_a_short_last_slice(m, k):
    # k slices of a column strip reduced across their cluster while the last, one-box slice
    # finishes long before the others: every CTA's sums must be complete before it sends
    # them (a missing barrier there once let a few owners read half-written values). Repeated
    # calls, since the failure depended on timing.
    rng = np.random.default_rng(70 + m + k)
    n = 4096
    q, s = oracle.quantize_q8((rng.standard_normal((k, n)) * 0.02).astype(np.float32))
    dq, ds = dev(q), dev(s)
    assert L.plan(m, n, k, q8=True)["slices"] > 1
    runs = []
    for _ in range(8):
        A = uni(rng, m, k)
        C = torch.full((m, n), float("nan"), device="cuda")
        L.matmul(dev(A), dq, scale=ds, C=C, weights_static=True)
        runs.append((A, C))
    torch.cuda.synchronize()
    for A, C in runs:
        got, want = C.cpu().numpy(), oracle.matmul_naive_q8(A, q, s)
        assert close_to(got, want, k), (m, k, int((np.abs(got - want) > 1e-5 * k).sum()))


def test_programmatic_launch_gives_identical_bits():
    rng = np.random.default_rng(21)
    A = uni(rng, 2, 4096)
    q, s = oracle.quantize_q8(uni(rng, 4096, 11008, scale=0.05))
    a = gpu_matmul(A, q=q, scale=s, kernel="skinny")
    b = gpu_matmul(A, q=q, scale=s, kernel="skinny", weights_static=True)
    np.testing.assert_array_equal(a, b)


def test_unaligned_weights_take_the_plain_load_path():
    rng = np.random.default_rng(23)
    m, k, n = 3, 1000, 4096
    A = uni(rng, m, k)
    q, s = oracle.quantize_q8(uni(rng, k, n))
    buf = torch.empty(k * n + 16, dtype=torch.int8, device="cuda")
    dq = buf[1:1 + k * n].view(k, n)
    dq.copy_(dev(q))
    assert L.plan(m, n, k, q8=True, b_addr=dq.data_ptr())["path_name"] == "gemv_ldg"
    dC = torch.empty(m, n, device="cuda")
    L.matmul(dev(A), dq, scale=dev(s), C=dC)
    torch.cuda.synchronize()
    assert close_to(dC.cpu().numpy(), oracle.matmul_naive_q8(A, q, s), k)


def test_bad_shapes_raise_invalid_argument():
    dA = torch.zeros(9, 2, device="cuda")
    dB = torch.zeros(2, 2, device="cuda")
    with pytest.raises(L.InvalidArgument) as e:
        L.matmul(dA, dB, kernel="skinny")
    assert "9x2" in str(e.value)
    with pytest.raises(L.InvalidArgument) as e:
        L.matmul(torch.zeros(2, 3, device="cuda"), torch.zeros(4, 2, device="cuda"))
    assert "2x3" in str(e.value) and "4x2" in str(e.value)


# ---- the benchmark's decode shapes at full size -----------------------------------------

def baseline_weights(seed, k, n):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((k, n)) * 0.02).astype(np.float32)
    return rng, W


def test_config0_decode_gemv_int8():
    rng, W = baseline_weights(0, 4096, 4096)
    q, s = oracle.quantize_q8(W)
    A = uni(rng, 1, 4096)
    want = oracle.matmul_naive_q8(A, q, s)
    got = gpu_matmul(A, q=q, scale=s)
    assert row_rel_err(got, want) <= 1e-5


@pytest.mark.parametrize("m", [1, 4, 16, 64])
def test_config1_decode_sweep(m):
    rng, W = baseline_weights(1, 4096, 4096)
    q, s = oracle.quantize_q8(W)
    A = uni(rng, m, 4096)
    assert row_rel_err(gpu_matmul(A, B=W), oracle.matmul_naive(A, W)) <= 1e-5
    assert row_rel_err(gpu_matmul(A, q=q, scale=s), oracle.matmul_naive_q8(A, q, s)) <= 1e-5


@pytest.mark.parametrize("k,n", [(4096, 11008), (11008, 4096), (4096, 32000)])
def test_config3_chain_shapes(k, n):
    rng, W = baseline_weights(3, k, n)
    q, s = oracle.quantize_q8(W)
    A = uni(rng, 1, k)
    want = oracle.matmul_naive_q8(A, q, s)
    got = gpu_matmul(A, q=q, scale=s, weights_static=True)
    assert row_rel_err(got, want) <= 1e-5


def test_linearity_at_full_size():
    # A size-independent property: C(A1 + A2) = C(A1) + C(A2) within rounding.
    rng, W = baseline_weights(4, 4096, 11008)
    q, s = oracle.quantize_q8(W)
    A1, A2 = uni(rng, 4, 4096), uni(rng, 4, 4096)
    dq, ds = dev(q), dev(s)
    c = [L.matmul(dev(a), dq, scale=ds) for a in (A1, A2, A1 + A2)]
    torch.cuda.synchronize()
    lhs = c[2].cpu().numpy().astype(np.float64)
    rhs = c[0].cpu().numpy().astype(np.float64) + c[1].cpu().numpy()
    assert row_rel_err(lhs, rhs) <= 2e-5


# ---- the reference's own GPU test, compiled against this library ------------------------

DROPIN = os.path.join(os.path.dirname(oracle.HERE), "oracle", "_ref", "test_cuda_dropin")


@pytest.mark.skipif(not os.path.exists(DROPIN), reason="oracle/_ref/test_cuda_dropin not built")
def test_reference_test_cuda_passes_unmodified():
    env = dict(os.environ, LLME_B200_MATH="fp32")
    r = subprocess.run([DROPIN], env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-4000:]
    assert "all tests passed" in r.stdout


MODEL_DROPIN = os.path.join(os.path.dirname(oracle.HERE), "oracle", "_ref",
                            "test_cuda_model_dropin")


@pytest.mark.skipif(not os.path.exists(MODEL_DROPIN),
                    reason="oracle/_ref/test_cuda_model_dropin not built")
@pytest.mark.parametrize("math", ["tensor", "fp32"])
def test_reference_cuda_model_runs_on_the_library(math):
    """The real caller: the reference's CudaTransformer (src/cuda_model.cu, built from its
    sources) with every projection and the classifier going through this library's
    matmul_cuda, checked by the reference's own tests/test_cuda_model.cpp against its CPU
    Transformer (decode, chunked prefill, rewinds, bad inputs; tolerance 1e-4), f32 and int8
    weights, in both arithmetic modes."""
    env = dict(os.environ, LLME_B200_MATH=math)
    r = subprocess.run([MODEL_DROPIN], env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-4000:]
    assert "all tests passed" in r.stdout


ATTN_DROPIN = os.path.join(os.path.dirname(oracle.HERE), "oracle", "_ref",
                           "test_cuda_attention_dropin")


@pytest.mark.skipif(not os.path.exists(ATTN_DROPIN),
                    reason="oracle/_ref/test_cuda_attention_dropin not built")
def test_reference_cuda_attention_test_passes_on_the_library():
    """The reference's tests/test_cuda_attention.cpp, unmodified, against this library's
    attention (include/cuda_attention.h): every kernel and shape case against its float64
    reference (5e-5), repeat bits, the long context and the rejections."""
    r = subprocess.run([ATTN_DROPIN], stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stdout[-4000:]
    assert "all tests passed" in r.stdout
