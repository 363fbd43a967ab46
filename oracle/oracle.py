"""TEST INFRASTRUCTURE ONLY: numpy bindings of the CPU oracle.

Two libraries, both built by oracle/Makefile:
  * liboracle.so      -- the plain-C restatement of the reference's CPU matmul path
                         (oracle.c; each function cites the reference file:line it follows);
  * _ref/libllme_ref*.so -- the reference's own matmul.cpp / quant.cpp / ops.cpp /
                         thread_pool.cpp compiled from its sources (present only where the
                         reference tree was available at build time).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import this module,
and only as the checker or the timed CPU baseline; the product never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libllme_ref.so")
REF_FAST_V3_SO = os.path.join(HERE, "_ref", "libllme_ref_fast.so")
REF_FAST_V4_SO = os.path.join(HERE, "_ref", "libllme_ref_fast_v4.so")
# The reference checkout (read-only): LLME_REFERENCE_SRC, else the directory beside this repo.
REF_SRC = os.environ.get("LLME_REFERENCE_SRC") or os.path.join(
    os.path.dirname(os.path.dirname(HERE)), "reference")


def _host_has_avx512() -> bool:
    """The x86-64-v4 level: AVX-512 F, BW, CD, DQ and VL, as the kernel reports them."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    flags = set(line.split(":", 1)[1].split())
                    return {"avx512f", "avx512bw", "avx512cd", "avx512dq", "avx512vl"} <= flags
    except OSError:
        pass
    return False


def _fast_so() -> str:
    """The timed CPU baseline: the reference's sources at -O3 for the widest vector ISA this
    host runs (its own build uses -march=native, CMakeLists.txt:20)."""
    if os.path.exists(REF_FAST_V4_SO) and _host_has_avx512():
        return REF_FAST_V4_SO
    return REF_FAST_V3_SO


REF_FAST_SO = _fast_so()

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(dtype=np.int8, flags="C_CONTIGUOUS")
_sz = ctypes.c_size_t


def build() -> None:
    """Builds liboracle.so (and oracle/_ref when the reference sources are present)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if os.path.isdir(os.path.join(REF_SRC, "src")):
        subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)


_oracle = None


def oracle_lib() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_SO):
            build()
        lib = ctypes.CDLL(ORACLE_SO)
        lib.orc_quantize_q8.argtypes = [_sz, _sz, _f32p, _i8p, _f32p]
        lib.orc_dequantize.argtypes = [_sz, _sz, _i8p, _f32p, _f32p]
        lib.orc_matmul_naive.argtypes = [_sz, _sz, _sz, _f32p, _f32p, _f32p]
        lib.orc_matmul_naive_q8.argtypes = [_sz, _sz, _sz, _f32p, _i8p, _f32p, _f32p]
        lib.orc_rmsnorm.argtypes = [_sz, _sz, _f32p, _f32p, ctypes.c_float, _f32p]
        vp = ctypes.c_void_p
        lib.orc_matmul_parallel.argtypes = [_sz, _sz, _sz, vp, vp, vp, vp, vp, ctypes.c_uint]
        lib.orc_default_threads.restype = ctypes.c_uint
        _oracle = lib
    return _oracle


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def quantize_q8(B: np.ndarray):
    """quant.cpp:6-28 -> (q int8 [rows, cols], scale fp32 [cols])."""
    B = _c(B, np.float32)
    rows, cols = B.shape
    q = np.empty((rows, cols), np.int8)
    s = np.empty(cols, np.float32)
    oracle_lib().orc_quantize_q8(rows, cols, B, q, s)
    return q, s


def dequantize(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    q = _c(q, np.int8)
    rows, cols = q.shape
    out = np.empty((rows, cols), np.float32)
    oracle_lib().orc_dequantize(rows, cols, q, _c(scale, np.float32), out)
    return out


def matmul_naive(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """matmul.cpp:205-217 (fp32, i-k-j order)."""
    A, B = _c(A, np.float32), _c(B, np.float32)
    m, k = A.shape
    n = B.shape[1]
    C = np.empty((m, n), np.float32)
    oracle_lib().orc_matmul_naive(m, n, k, A, B, C)
    return C


def matmul_naive_q8(A: np.ndarray, q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """matmul_naive(A, dequantize(q)) without materialising the fp32 weights."""
    A, q = _c(A, np.float32), _c(q, np.int8)
    m, k = A.shape
    n = q.shape[1]
    C = np.empty((m, n), np.float32)
    oracle_lib().orc_matmul_naive_q8(m, n, k, A, q, _c(scale, np.float32), C)
    return C


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """ops.cpp:8-26 (double accumulation)."""
    x = _c(x, np.float32)
    rows, cols = x.shape
    y = np.empty_like(x)
    oracle_lib().orc_rmsnorm(rows, cols, x, _c(w, np.float32), eps, y)
    return y


def matmul_parallel(A: np.ndarray, B=None, q=None, scale=None, threads: int = 0) -> np.ndarray:
    """The CPU-baseline port of matmul.cpp:240-306 (pthreads)."""
    A = _c(A, np.float32)
    m, k = A.shape
    if q is not None:
        q, scale = _c(q, np.int8), _c(scale, np.float32)
        n = q.shape[1]
        args = (None, q.ctypes.data, scale.ctypes.data)
    else:
        B = _c(B, np.float32)
        n = B.shape[1]
        args = (B.ctypes.data, None, None)
    C = np.empty((m, n), np.float32)
    oracle_lib().orc_matmul_parallel(m, n, k, A.ctypes.data, *args, C.ctypes.data, threads)
    return C


def default_threads() -> int:
    return int(oracle_lib().orc_default_threads())


# ---- the reference's own code (oracle/_ref) --------------------------------------------------

class Reference:
    """The reference engine's CPU matmul / quant / rmsnorm, compiled from its sources."""

    def __init__(self, fast: bool = False):
        path = REF_FAST_SO if fast else REF_SO
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.path = path
        lib = ctypes.CDLL(path)
        lib.ref_last_error.restype = ctypes.c_char_p
        lib.ref_pool_threads.restype = ctypes.c_uint
        lib.ref_matmul_naive.argtypes = [_sz, _sz, _sz, _sz, _f32p, _f32p, _f32p]
        lib.ref_matmul_parallel_f32.argtypes = [_sz, _sz, _sz, _f32p, _f32p, _f32p, ctypes.c_uint]
        lib.ref_quantize_q8.argtypes = [_sz, _sz, _f32p, _i8p, _f32p]
        lib.ref_dequantize.argtypes = [_sz, _sz, _i8p, _f32p, _f32p]
        lib.ref_rmsnorm.argtypes = [_sz, _sz, _f32p, _f32p, _f32p]
        lib.ref_qtensor_new.argtypes = [_sz, _sz, _i8p, _f32p]
        lib.ref_qtensor_new.restype = ctypes.c_void_p
        lib.ref_qtensor_free.argtypes = [ctypes.c_void_p]
        lib.ref_matmul_parallel_q8.argtypes = [ctypes.c_void_p, _sz, _sz, _f32p, _f32p,
                                               ctypes.c_uint]
        lib.ref_tensor_new.argtypes = [_sz, _sz, _f32p]
        lib.ref_tensor_new.restype = ctypes.c_void_p
        lib.ref_tensor_free.argtypes = [ctypes.c_void_p]
        lib.ref_matmul_parallel_f32_h.argtypes = [ctypes.c_void_p, _sz, _sz, _f32p, _f32p,
                                                  ctypes.c_uint]
        self.lib = lib

    @staticmethod
    def available(fast: bool = False) -> bool:
        return os.path.exists(REF_FAST_SO if fast else REF_SO)

    def _check(self, st: int) -> None:
        if st == 1:
            raise ValueError(self.lib.ref_last_error().decode())
        if st:
            raise RuntimeError(self.lib.ref_last_error().decode())

    def threads(self) -> int:
        return int(self.lib.ref_pool_threads())

    def isa(self) -> str:
        """The vector ISA the loaded library was built for."""
        return "x86-64-v4 (AVX-512)" if self.path == REF_FAST_V4_SO else (
            "x86-64-v3 (AVX2+FMA)" if self.path == REF_FAST_V3_SO else "-O2, contraction off")

    def matmul_naive(self, A, B, b_rows=None):
        A, B = _c(A, np.float32), _c(B, np.float32)
        m, k = A.shape
        n = B.shape[1]
        C = np.empty((m, n), np.float32)
        self._check(self.lib.ref_matmul_naive(m, n, k, B.shape[0] if b_rows is None else b_rows,
                                              A, B, C))
        return C

    def matmul_parallel(self, A, B, threads: int = 0):
        A, B = _c(A, np.float32), _c(B, np.float32)
        m, k = A.shape
        n = B.shape[1]
        C = np.empty((m, n), np.float32)
        self._check(self.lib.ref_matmul_parallel_f32(m, n, k, A, B, C, threads))
        return C

    def quantize_q8(self, B):
        B = _c(B, np.float32)
        rows, cols = B.shape
        q = np.empty((rows, cols), np.int8)
        s = np.empty(cols, np.float32)
        self._check(self.lib.ref_quantize_q8(rows, cols, B, q, s))
        return q, s

    def dequantize(self, q, scale):
        q = _c(q, np.int8)
        out = np.empty(q.shape, np.float32)
        self._check(self.lib.ref_dequantize(q.shape[0], q.shape[1], q, _c(scale, np.float32), out))
        return out

    def rmsnorm(self, x, w):
        x = _c(x, np.float32)
        y = np.empty_like(x)
        self._check(self.lib.ref_rmsnorm(x.shape[0], x.shape[1], x, _c(w, np.float32), y))
        return y

    def qtensor(self, q, scale):
        """A QTensor kept alive on the reference side; pass to matmul_parallel_q8."""
        q, scale = _c(q, np.int8), _c(scale, np.float32)
        h = self.lib.ref_qtensor_new(q.shape[0], q.shape[1], q, scale)
        return _QHandle(self, h, q.shape)

    def matmul_parallel_q8(self, A, qh: "_QHandle", threads: int = 0, out=None):
        A = _c(A, np.float32)
        m, k = A.shape
        C = out if out is not None else np.empty((m, qh.shape[1]), np.float32)
        self._check(self.lib.ref_matmul_parallel_q8(qh.handle, m, k, A, C, threads))
        return C


    def tensor(self, B):
        """An fp32 Tensor kept alive on the reference side; pass to matmul_parallel_h."""
        B = _c(B, np.float32)
        return _QHandle(self, self.lib.ref_tensor_new(B.shape[0], B.shape[1], B), B.shape,
                        self.lib.ref_tensor_free)

    def matmul_parallel_h(self, A, th: "_QHandle", threads: int = 0, out=None):
        """matmul_parallel(A, B) with B from tensor(): the weight is not copied per call."""
        A = _c(A, np.float32)
        m, k = A.shape
        C = out if out is not None else np.empty((m, th.shape[1]), np.float32)
        self._check(self.lib.ref_matmul_parallel_f32_h(th.handle, m, k, A, C, threads))
        return C


class _QHandle:
    def __init__(self, ref: Reference, handle, shape, free=None):
        self.ref, self.handle, self.shape = ref, handle, shape
        self.free = free if free is not None else ref.lib.ref_qtensor_free

    def __del__(self):
        try:
            self.free(self.handle)
        except Exception:
            pass


# ---- the reference's CPU Transformer (oracle/_ref/libref_model.so) ---------------------------

REF_MODEL_SO = os.path.join(HERE, "_ref", "libref_model.so")
_ref_model_lib = None


def _model_lib() -> ctypes.CDLL:
    global _ref_model_lib
    if _ref_model_lib is None:
        if not os.path.exists(REF_MODEL_SO):
            raise FileNotFoundError(REF_MODEL_SO)
        lib = ctypes.CDLL(REF_MODEL_SO)
        vp = ctypes.c_void_p
        lib.ref_model_error.restype = ctypes.c_char_p
        lib.ref_model_load.argtypes = [ctypes.c_char_p, ctypes.c_int]
        lib.ref_model_load.restype = vp
        lib.ref_model_free.argtypes = [vp]
        lib.ref_model_vocab.argtypes = [vp]
        lib.ref_model_vocab.restype = _sz
        lib.ref_model_run.argtypes = [vp, np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS"),
                                      _sz, _sz, _f32p]
        lib.ref_rope_tables.argtypes = [_sz, _sz, _sz, _f32p, _f32p]
        _ref_model_lib = lib
    return _ref_model_lib


class RefModel:
    """The reference's CPU Transformer (model.cpp) over a llama2.c checkpoint file: the oracle
    of the tensor-parallel transformer. run(tokens, pos) feeds tokens at [pos, pos + n) and
    returns the last row's logits."""

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_MODEL_SO)

    def __init__(self, path: str, q8: bool):
        lib = _model_lib()
        self.handle = lib.ref_model_load(path.encode(), int(q8))
        if not self.handle:
            raise RuntimeError(lib.ref_model_error().decode())
        self.vocab = int(lib.ref_model_vocab(self.handle))

    def run(self, tokens, pos: int) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros(self.vocab, np.float32)
        if _model_lib().ref_model_run(self.handle, t, t.size, pos, out):
            raise RuntimeError(_model_lib().ref_model_error().decode())
        return out

    def close(self) -> None:
        if self.handle:
            _model_lib().ref_model_free(self.handle)
            self.handle = None

    def __del__(self):
        self.close()


def ref_rope_tables(seq_len: int, dim: int, n_heads: int):
    """The reference's rope_tables (model.cpp:171-184) for head_size = dim / n_heads."""
    half = dim // n_heads // 2
    cos = np.zeros(seq_len * half, np.float32)
    sin = np.zeros(seq_len * half, np.float32)
    _model_lib().ref_rope_tables(seq_len, dim, n_heads, cos, sin)
    return cos.reshape(seq_len, half), sin.reshape(seq_len, half)
