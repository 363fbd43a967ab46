"""Python binding of the B200 matmul library's C ABI (include/llme_b200.h).

A thin ctypes layer with the reference's operator interface for this path
(src/cuda_matmul.h:94-107): matmul_cuda on raw device pointers for fp32 or int8
weights, with the MatmulFusion fields (accumulate, rms_weight), the GpuKernel
names, cuda_scratch_generation, cuda_synchronize and cuda_available. Errors
follow the reference's exception split: InvalidArgument (a ValueError, for the
reference's std::invalid_argument) and CudaError (a RuntimeError, for its
std::runtime_error "cuda: ..." messages).

PyTorch is used only to hand over device memory and streams (the `matmul`
helper); the arithmetic is entirely in libllme_b200.so. There is no fallback:
if the library is missing, loading raises.
"""
from __future__ import annotations

import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "lib", "libllme_b200.so")

KERNELS = {"automatic": 0, "naive": 1, "tiled": 2, "tiled_split": 3, "skinny": 4}
PATHS = {0: "none", 1: "zero", 2: "naive", 3: "gemv_tma", 4: "gemv_ldg", 5: "tiled_simt",
         6: "tcgen05", 7: "tcgen05_q8", 8: "tcgen05_skinny",
         9: "tcgen05_f32_skinny"}
MATH_TENSOR, MATH_FP32 = 0, 1
FLAG_WEIGHTS_STATIC = 1
FLAG_SAME_SHARDS = 2

OK, E_INVALID, E_CUDA, E_TIMEOUT, E_UNSUPPORTED, E_NCCL, E_HOST, E_RANGE = range(8)

# cudaStreamLegacy: torch's default stream has handle 0, which the C ABI would read as
# "per-thread default stream"; pass the legacy handle instead so both sides agree.
_STREAM_LEGACY = 1


class InvalidArgument(ValueError):
    """std::invalid_argument in the reference (shape mismatch, skinny with m > 8, 2^31)."""


class CudaError(RuntimeError):
    """std::runtime_error("cuda: <what>: <message>") in the reference."""


class DeviceTimeout(RuntimeError):
    """A bounded device-side wait gave up (LLME_E_TIMEOUT)."""


class Plan(ctypes.Structure):
    _fields_ = [
        ("path", ctypes.c_int), ("kernel", ctypes.c_int), ("rms_prepass", ctypes.c_int),
        ("grid_x", ctypes.c_int), ("grid_y", ctypes.c_int), ("slices", ctypes.c_int),
        ("cluster", ctypes.c_int),
        ("span", ctypes.c_int), ("tile_m", ctypes.c_int), ("tile_n", ctypes.c_int),
        ("split_bytes", ctypes.c_size_t), ("counter_slots", ctypes.c_size_t),
        ("norm_bytes", ctypes.c_size_t), ("operand_bytes", ctypes.c_size_t),
    ]

    def as_dict(self) -> dict:
        d = {name: getattr(self, name) for name, _ in self._fields_}
        d["path_name"] = PATHS.get(self.path, "?")
        return d


class Q8Product(ctypes.Structure):
    """llme_q8_product: one product of a grouped launch (device pointers)."""
    _fields_ = [("n", ctypes.c_size_t), ("k", ctypes.c_size_t), ("A", ctypes.c_void_p),
                ("B", ctypes.c_void_p), ("scale", ctypes.c_void_p), ("C", ctypes.c_void_p),
                ("accumulate", ctypes.c_int)]


class ModelConfig(ctypes.Structure):
    """llme_model_config: the llama2.c header fields."""
    _fields_ = [(f, ctypes.c_int) for f in ("dim", "hidden_dim", "n_layers", "n_heads",
                                            "n_kv_heads", "vocab_size", "seq_len")]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


class ModelSlice(ctypes.Structure):
    """llme_model_slice: one rank's heads, hidden units and vocabulary."""
    _fields_ = [("q0", ctypes.c_int), ("nq", ctypes.c_int), ("kv0", ctypes.c_int),
                ("nkv", ctypes.c_int), ("h0", ctypes.c_size_t), ("hc", ctypes.c_size_t),
                ("v0", ctypes.c_size_t), ("vc", ctypes.c_size_t)]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


_lib = None


def library_path() -> str:
    return LIB_PATH


def load() -> ctypes.CDLL:
    """Loads libllme_b200.so (built by llm-engine_b200/build.py); raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python llm-engine_b200/build.py` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    sz, vp, i, u = ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int, ctypes.c_uint
    lib.llme_matmul_f32.argtypes = [sz, sz, sz, vp, vp, vp, i, i, vp, u, vp]
    lib.llme_matmul_q8.argtypes = [sz, sz, sz, vp, vp, vp, vp, i, i, vp, u, vp]
    lib.llme_matmul_f32.restype = lib.llme_matmul_q8.restype = i
    lib.llme_matmul_q8_noalloc.argtypes = [sz, sz, sz, vp, vp, vp, vp, i, vp]
    lib.llme_matmul_q8_noalloc.restype = i
    lib.llme_quantize_q8.argtypes = [sz, sz, vp, vp, vp, vp]
    lib.llme_attention_check.argtypes = [ctypes.POINTER(AttentionShape), i]
    lib.llme_attention_scratch_floats.argtypes = [ctypes.POINTER(AttentionShape), sz, i]
    lib.llme_attention_scratch_floats.restype = sz
    lib.llme_attention_launches.argtypes = [ctypes.POINTER(AttentionShape), sz, i]
    lib.llme_attention_launches.restype = sz
    lib.llme_attention.argtypes = [ctypes.POINTER(AttentionShape), sz, vp, vp, vp, vp, vp, vp, i,
                                   vp]
    lib.llme_embed_rows.argtypes = [sz, sz, vp, vp, vp, vp]
    lib.llme_rope_cache.argtypes = [sz, i, i, i, vp, vp, vp, vp, vp, vp, vp]
    lib.llme_swiglu.argtypes = [sz, sz, vp, vp, vp]
    lib.llme_rope_tables.argtypes = [sz, sz, vp, vp]
    mp, ip = ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)
    cfgp = ctypes.POINTER(ModelConfig)
    lib.llme_model_load.argtypes = [ctypes.c_char_p, i, i, i, vp, ctypes.POINTER(vp)]
    lib.llme_model_synthetic.argtypes = [cfgp, i, i, i, vp, ctypes.c_ulonglong, ctypes.POINTER(vp)]
    lib.llme_checkpoint_config.argtypes = [ctypes.c_char_p, cfgp]
    lib.llme_model_partition.argtypes = [cfgp, i, i, ctypes.POINTER(ModelSlice)]
    lib.llme_model_get_config.argtypes = [mp, cfgp]
    lib.llme_model_local.argtypes = [mp, ip, ip, ip, ip]
    lib.llme_model_stream_bytes.argtypes = [mp, ctypes.POINTER(sz), ctypes.POINTER(sz)]
    lib.llme_model_forward.argtypes = [mp, vp, sz, sz, vp]
    lib.llme_model_decode.argtypes = [mp, i, sz, vp]
    lib.llme_model_captures.argtypes = [mp]
    lib.llme_model_captures.restype = sz
    lib.llme_model_fill_history.argtypes = [mp, sz, ctypes.c_ulonglong]
    lib.llme_model_replay.argtypes = [mp, sz, vp]
    lib.llme_model_group_forward.argtypes = [ctypes.POINTER(vp), i, vp, sz, sz, vp]
    lib.llme_model_destroy.argtypes = [mp]
    for f in ("llme_model_load", "llme_model_synthetic", "llme_checkpoint_config",
              "llme_model_partition", "llme_model_get_config", "llme_model_local",
              "llme_model_stream_bytes", "llme_model_forward", "llme_model_decode",
              "llme_model_fill_history", "llme_model_replay", "llme_model_group_forward",
              "llme_model_destroy"):
        getattr(lib, f).restype = i
    for f in ("llme_embed_rows", "llme_rope_cache", "llme_swiglu", "llme_rope_tables"):
        getattr(lib, f).restype = i
    lib.llme_batch_q8_create.argtypes = [ctypes.POINTER(vp), sz, sz, ctypes.POINTER(Q8Product)]
    lib.llme_batch_run.argtypes = [vp, u, vp]
    lib.llme_batch_destroy.argtypes = [vp]
    lib.llme_batch_run_rowpar.argtypes = [vp, vp, u, vp]
    for f in ("llme_batch_q8_create", "llme_batch_run", "llme_batch_destroy", "llme_batch_run_rowpar"):
        getattr(lib, f).restype = i
    lib.llme_comm_unique_id.argtypes = [ctypes.c_char_p]
    lib.llme_comm_init.argtypes = [ctypes.POINTER(vp), i, i, ctypes.c_char_p, ctypes.c_double]
    lib.llme_comm_destroy.argtypes = lib.llme_comm_abort.argtypes = [vp]
    lib.llme_comm_size.argtypes = lib.llme_comm_rank.argtypes = [vp]
    lib.llme_allreduce_sum_f32.argtypes = [vp, sz, vp, vp]
    lib.llme_matmul_q8_rowpar.argtypes = [sz, sz, sz, vp, vp, vp, vp, i, i, u, vp, vp]
    lib.llme_matmul_f32_rowpar.argtypes = [sz, sz, sz, vp, vp, vp, i, i, u, vp, vp]
    lib.llme_comm_enable_peer.argtypes = [vp, sz]
    lib.llme_comm_status.argtypes = []
    for f in ("llme_comm_enable_peer", "llme_comm_status",
              "llme_comm_unique_id", "llme_comm_init", "llme_comm_destroy", "llme_comm_abort",
              "llme_comm_size", "llme_comm_rank", "llme_allreduce_sum_f32",
              "llme_matmul_q8_rowpar", "llme_matmul_f32_rowpar"):
        getattr(lib, f).restype = i
    lib.llme_last_error.restype = ctypes.c_char_p
    lib.llme_scratch_generation.restype = sz
    for f in ("llme_synchronize", "llme_device_available", "llme_device_supported",
              "llme_device_status", "llme_get_math"):
        getattr(lib, f).restype = i
        getattr(lib, f).argtypes = []
    lib.llme_set_math.argtypes = [i]
    lib.llme_set_math.restype = i
    lib.llme_plan.argtypes = [sz, sz, sz, i, i, i, ctypes.c_size_t, ctypes.c_size_t,
                              ctypes.c_size_t, i, i, ctypes.POINTER(Plan)]
    lib.llme_plan.restype = i
    lib.llme_plan_clusters.argtypes = [sz, sz, sz, i, i, i, ctypes.c_size_t, ctypes.c_size_t,
                                       ctypes.c_size_t, i, i, ctypes.POINTER(ctypes.c_int),
                                       ctypes.POINTER(Plan)]
    lib.llme_plan_clusters.restype = i
    lib.llme_gemv_cluster_capacity.argtypes = [ctypes.POINTER(ctypes.c_int)]
    lib.llme_gemv_cluster_capacity.restype = i
    lib.llme_alloc.argtypes = [ctypes.POINTER(vp), sz]
    lib.llme_free.argtypes = [vp]
    lib.llme_copy_to_device.argtypes = [vp, vp, sz]
    lib.llme_copy_to_host.argtypes = [vp, vp, sz]
    for f in ("llme_alloc", "llme_free", "llme_copy_to_device", "llme_copy_to_host"):
        getattr(lib, f).restype = i
    _lib = lib
    return lib


def last_error() -> str:
    return load().llme_last_error().decode()


def _check(status: int) -> None:
    if status == OK:
        return
    msg = last_error()
    if status == E_INVALID:
        raise InvalidArgument(msg)
    if status == E_TIMEOUT:
        raise DeviceTimeout(msg)
    if status == E_HOST:
        raise MemoryError(msg) if "out of memory" in msg else RuntimeError(msg)
    if status == E_RANGE:
        raise IndexError(msg)
    raise CudaError(msg or f"cuda: error {status}")


def _kernel_id(kernel) -> int:
    if isinstance(kernel, int):
        return kernel
    return KERNELS[kernel]


def matmul_cuda_f32(m: int, n: int, k: int, A: int, B: int, C: int, kernel="automatic",
                    accumulate: bool = False, rms_weight: int = 0, flags: int = 0,
                    stream: int | None = None) -> None:
    """C (+)= [rmsnorm(A)] x B on device pointers (cuda_matmul.h:97-99)."""
    _check(load().llme_matmul_f32(m, n, k, A, B, C, _kernel_id(kernel), int(bool(accumulate)),
                                  rms_weight or None, flags, stream or None))


def matmul_cuda_q8(m: int, n: int, k: int, A: int, B: int, scale: int, C: int,
                   kernel="automatic", accumulate: bool = False, rms_weight: int = 0,
                   flags: int = 0, stream: int | None = None) -> None:
    """C (+)= [rmsnorm(A)] x (B * scale) with int8 B on device pointers (cuda_matmul.h:105-107)."""
    _check(load().llme_matmul_q8(m, n, k, A, B, scale, C, _kernel_id(kernel),
                                 int(bool(accumulate)), rms_weight or None, flags, stream or None))


class AttentionShape(ctypes.Structure):
    """llme_attention_shape (the reference's AttentionShape, src/cuda_attention.h:8-14)."""
    _fields_ = [("n_heads", ctypes.c_int), ("n_kv_heads", ctypes.c_int),
                ("head_size", ctypes.c_int), ("seq_len", ctypes.c_int),
                ("q_stride", ctypes.c_size_t), ("kv_stride", ctypes.c_size_t),
                ("out_stride", ctypes.c_size_t)]


ATTN_KERNELS = {"automatic": 0, "single_block": 1, "split": 2}


def attention_check(shape: AttentionShape, kernel="automatic") -> None:
    _check(load().llme_attention_check(ctypes.byref(shape), ATTN_KERNELS[kernel]))


def attention_scratch_floats(shape: AttentionShape, rows: int, kernel="automatic") -> int:
    return load().llme_attention_scratch_floats(ctypes.byref(shape), rows, ATTN_KERNELS[kernel])


def attention_launches(shape: AttentionShape, rows: int, kernel="automatic") -> int:
    """Kernels one attention call enqueues (1, or 2 with the split path's merge); 0: invalid."""
    return load().llme_attention_launches(ctypes.byref(shape), rows, ATTN_KERNELS[kernel])


def attention(shape: AttentionShape, rows: int, pos_dev: int, q: int, k_cache: int, v_cache: int,
              out: int, scratch: int, kernel="automatic", stream: int | None = None) -> None:
    """Causal attention over a KV cache on device pointers (cuda_attention.h:38-45)."""
    _check(load().llme_attention(ctypes.byref(shape), rows, pos_dev, q, k_cache, v_cache, out,
                                 scratch or None, ATTN_KERNELS[kernel], stream or None))


def embed_rows(n: int, dim: int, feed: int, table: int, x: int, stream: int | None = None) -> None:
    """x[i] = table[feed[1 + i]] on device pointers (the reference's embed, cuda_model.cu:27-31)."""
    _check(load().llme_embed_rows(n, dim, feed, table, x, stream or None))


def rope_cache(n: int, nq: int, nkv: int, head_size: int, feed: int, cos: int, sin: int, qkv: int,
               key_cache: int, value_cache: int, stream: int | None = None) -> None:
    """RoPE on a rank's q / k heads at positions feed[0] + i and the KV-cache write
    (the reference's rope_and_cache, cuda_model.cu:33-66), on device pointers."""
    _check(load().llme_rope_cache(n, nq, nkv, head_size, feed, cos, sin, qkv, key_cache,
                                  value_cache, stream or None))


def swiglu(n: int, hidden: int, gu: int, hb: int, stream: int | None = None) -> None:
    """hb = silu(gate) * up for n rows of [gate | up] (cuda_model.cu:68-75), device pointers."""
    _check(load().llme_swiglu(n, hidden, gu, hb, stream or None))


def rope_tables(seq_len: int, head_size: int):
    """The RoPE cos / sin tables (seq_len x head_size / 2, numpy float32), computed by the
    library's host code with the reference's float expressions (model.cpp:171-184)."""
    import numpy as np
    half = head_size // 2
    cos = np.zeros((seq_len, half), np.float32)
    sin = np.zeros((seq_len, half), np.float32)
    _check(load().llme_rope_tables(seq_len, head_size, cos.ctypes.data, sin.ctypes.data))
    return cos, sin


def quantize_q8_cuda(k: int, n: int, W: int, q: int, scale: int, stream: int | None = None) -> None:
    """The reference's quantize_q8 (quant.cpp:6-28) on device pointers: W (k x n fp32) ->
    q (k x n int8) and scale (n fp32), bit for bit."""
    _check(load().llme_quantize_q8(k, n, W, q, scale, stream or None))


def quantize_q8(W):
    """quantize_q8 over a torch CUDA tensor W (k x n fp32): returns (q int8, scale fp32)."""
    import torch
    if W.dtype != torch.float32 or W.dim() != 2 or not W.is_contiguous():
        raise InvalidArgument("quantize_q8: W must be a contiguous 2-D float32 tensor")
    if W.device.type != "cuda":
        raise InvalidArgument(f"quantize_q8: W is on {W.device}; it must be in CUDA device memory")
    k, n = W.shape
    q = torch.empty((k, n), dtype=torch.int8, device=W.device)
    scale = torch.empty(n, dtype=torch.float32, device=W.device)
    quantize_q8_cuda(k, n, W.data_ptr(), q.data_ptr(), scale.data_ptr(), torch_stream_handle())
    return q, scale


def matmul_cuda_q8_noalloc(m: int, n: int, k: int, A: int, B: int, scale: int, C: int,
                           accumulate: bool = False, stream: int | None = None) -> None:
    """The allocation-free split-K product (llme_matmul_q8_noalloc): its scratch is a fixed
    device array inside the library, so the call never allocates device memory."""
    _check(load().llme_matmul_q8_noalloc(m, n, k, A, B, scale, C, int(bool(accumulate)),
                                         stream or None))


class Batch:
    """Independent int8 products of the same m run in one persistent launch
    (llme_batch_q8_create / llme_batch_run). products: (n, k, A, B, scale, C, accumulate)
    tuples of device pointers that stay valid for the batch's lifetime."""

    def __init__(self, m: int, products):
        arr = (Q8Product * len(products))(*[Q8Product(*p) for p in products])
        h = ctypes.c_void_p()
        _check(load().llme_batch_q8_create(ctypes.byref(h), m, len(products), arr))
        self.handle = h.value

    def run(self, flags: int = 0, stream: int | None = None) -> None:
        _check(load().llme_batch_run(self.handle, flags, stream or None))

    def run_rowpar(self, comm, flags: int = 0, stream: int | None = None) -> None:
        """The batch with the sum over the ranks taken inside the launch (row-parallel products,
        every rank running a batch of the same shapes)."""
        _check(load().llme_batch_run_rowpar(self.handle, comm.handle, flags, stream or None))

    def destroy(self) -> None:
        if self.handle:
            h, self.handle = self.handle, None
            _check(load().llme_batch_destroy(h))


COMM_ID_BYTES = 128


class Comm:
    """An NCCL communicator owned by the library (one per GPU, one process per GPU)."""

    def __init__(self, nranks: int, rank: int, unique_id: bytes, timeout_s: float = 60.0):
        if len(unique_id) != COMM_ID_BYTES:
            raise InvalidArgument("communicator id must be 128 bytes")
        h = ctypes.c_void_p()
        _check(load().llme_comm_init(ctypes.byref(h), nranks, rank, unique_id, timeout_s))
        self.handle = h.value
        self.nranks, self.rank = nranks, rank

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(COMM_ID_BYTES)
        _check(load().llme_comm_unique_id(buf))
        return buf.raw

    def enable_peer(self, max_floats: int) -> None:
        """Use the library's NVLink peer all-reduce for up to max_floats values (collective)."""
        _check(load().llme_comm_enable_peer(self.handle, max_floats))

    @staticmethod
    def status() -> None:
        _check(load().llme_comm_status())

    def allreduce_sum_f32(self, ptr: int, count: int, stream: int | None = None) -> None:
        _check(load().llme_allreduce_sum_f32(ptr, count, self.handle, stream or None))

    def matmul_q8_rowpar(self, m, n, k_local, A, B, scale, C, kernel="automatic",
                         accumulate=False, flags=0, stream=None) -> None:
        _check(load().llme_matmul_q8_rowpar(m, n, k_local, A, B, scale, C, _kernel_id(kernel),
                                            int(bool(accumulate)), flags, self.handle,
                                            stream or None))

    def matmul_f32_rowpar(self, m, n, k_local, A, B, C, kernel="automatic", accumulate=False,
                          flags=0, stream=None) -> None:
        _check(load().llme_matmul_f32_rowpar(m, n, k_local, A, B, C, _kernel_id(kernel),
                                             int(bool(accumulate)), flags, self.handle,
                                             stream or None))

    def destroy(self) -> None:
        if self.handle:
            h, self.handle = self.handle, None
            _check(load().llme_comm_destroy(h))

    def abort(self) -> None:
        if self.handle:
            h, self.handle = self.handle, None
            _check(load().llme_comm_abort(h))


def plan(m: int, n: int, k: int, q8: bool, kernel="automatic", accumulate: bool = False,
         a_addr: int = 256, b_addr: int = 256, rms_addr: int = 0, sm_count: int = 148,
         math: int = MATH_TENSOR, gemv_clusters=None) -> dict:
    """The dispatch decision for a call, computed on the host only (no GPU needed).
    gemv_clusters: a device's GEMV cluster capacity (8 counts, gemv_cluster_capacity());
    None models it as 2 x sm_count / cluster size."""
    p = Plan()
    args = (m, n, k, int(bool(q8)), _kernel_id(kernel), int(bool(accumulate)), a_addr, b_addr,
            rms_addr, sm_count, math)
    if gemv_clusters is None:
        _check(load().llme_plan(*args, ctypes.byref(p)))
    else:
        table = (ctypes.c_int * 8)(*gemv_clusters)
        _check(load().llme_plan_clusters(*args, table, ctypes.byref(p)))
    return p.as_dict()


def gemv_cluster_capacity() -> list:
    """The current device's capacity for GEMV clusters of 1..8 CTAs (needs a GPU)."""
    out = (ctypes.c_int * 8)()
    _check(load().llme_gemv_cluster_capacity(out))
    return list(out)


def scratch_generation() -> int:
    return load().llme_scratch_generation()


def synchronize() -> None:
    _check(load().llme_synchronize())


def device_status() -> None:
    _check(load().llme_device_status())


def available() -> bool:
    return bool(load().llme_device_available())


def device_supported() -> bool:
    return bool(load().llme_device_supported())


def set_math(mode: int) -> int:
    prev = load().llme_set_math(mode)
    if prev < 0:
        _check(E_INVALID)
    return prev


def get_math() -> int:
    return load().llme_get_math()


def torch_stream_handle(stream=None) -> int:
    """The cudaStream_t of a torch stream (default: current), mapped for the C ABI."""
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    h = s.cuda_stream
    return h if h else _STREAM_LEGACY


def matmul(A, B, scale=None, C=None, kernel="automatic", accumulate: bool = False,
           rms_weight=None, weights_static: bool = False, stream=None):
    """Convenience over torch CUDA tensors: A (m x k fp32), B (k x n fp32 or int8), scale
    (n fp32, int8 only), C (m x n fp32, allocated if None). Returns C. Runs on the current
    torch stream unless `stream` is given."""
    import torch
    if A.dim() != 2 or B.dim() != 2:
        raise InvalidArgument("matmul: A and B must be matrices")
    m, k = A.shape
    kb, n = B.shape
    if kb != k:
        raise InvalidArgument(f"matmul_cuda: inner dimensions differ (A is {m}x{k}, B is {kb}x{n})")
    # Everything the kernels will read or write, checked before any pointer leaves Python: a
    # host tensor's address or a short C would otherwise reach the GPU as a bad address.
    f32 = (torch.float32,)
    expect = [("A", A, f32, (m, k)), ("B", B, (torch.float32, torch.int8), (k, n)),
              ("C", C, f32, (m, n)), ("scale", scale, f32, (n,)),
              ("rms_weight", rms_weight, f32, (k,))]
    for name, t, dtypes, shape in expect:
        if t is None:
            continue
        if t.dtype not in dtypes:
            raise InvalidArgument(f"matmul: {name} is {t.dtype}, expected "
                                  + " or ".join(str(d) for d in dtypes))
        if tuple(t.shape) != shape:
            raise InvalidArgument(f"matmul: {name} has shape {tuple(t.shape)}, expected {shape}")
        if not t.is_contiguous():
            raise InvalidArgument("matmul: tensors must be contiguous row-major")
    for name, t, _, _ in expect:
        if t is not None and (t.device.type != "cuda" or t.device != A.device):
            raise InvalidArgument(f"matmul: {name} is on {t.device}; every tensor must be in the "
                                  "memory of one CUDA device")
    if C is None:
        C = torch.empty((m, n), dtype=torch.float32, device=A.device)
    flags = FLAG_WEIGHTS_STATIC if weights_static else 0
    h = torch_stream_handle(stream)
    rms = rms_weight.data_ptr() if rms_weight is not None else 0
    if B.dtype == torch.int8:
        if scale is None:
            raise InvalidArgument("matmul: int8 B needs a scale vector")
        matmul_cuda_q8(m, n, k, A.data_ptr(), B.data_ptr(), scale.data_ptr(), C.data_ptr(),
                       kernel, accumulate, rms, flags, h)
    else:
        matmul_cuda_f32(m, n, k, A.data_ptr(), B.data_ptr(), C.data_ptr(), kernel, accumulate,
                        rms, flags, h)
    return C


# ---- the transformer engine (C++, model.cu) ----------------------------------------------------

def _config(cfg) -> "ModelConfig":
    if isinstance(cfg, ModelConfig):
        return cfg
    if isinstance(cfg, dict):
        return ModelConfig(**cfg)
    return ModelConfig(*cfg)


def checkpoint_config(path: str) -> dict:
    """The header and size checks of llme_model_load on the host (no GPU); the configuration."""
    c = ModelConfig()
    _check(load().llme_checkpoint_config(path.encode(), ctypes.byref(c)))
    return c.as_dict()


def model_partition(cfg, world: int, rank: int) -> dict:
    """Rank `rank`'s query heads, kv heads, hidden units and vocabulary (host only)."""
    out = ModelSlice()
    _check(load().llme_model_partition(ctypes.byref(_config(cfg)), world, rank, ctypes.byref(out)))
    return out.as_dict()


class Model:
    """One rank (or the whole) of the reference's transformer on the current GPU, run by the
    library's C++ engine (llme_model_*). forward()/decode() return the last row's logits as a
    numpy array (the whole vocabulary on every rank)."""

    def __init__(self, handle: int):
        self.handle = handle
        c = ModelConfig()
        _check(load().llme_model_get_config(handle, ctypes.byref(c)))
        self.config = c.as_dict()
        nq, nkv, hc, vc = (ctypes.c_int() for _ in range(4))
        _check(load().llme_model_local(handle, ctypes.byref(nq), ctypes.byref(nkv),
                                       ctypes.byref(hc), ctypes.byref(vc)))
        self.local = {"q_heads": nq.value, "kv_heads": nkv.value, "hidden": hc.value,
                      "vocab": vc.value}

    @classmethod
    def load(cls, path: str, q8: bool = False, world: int = 1, rank: int = 0, comm=None):
        h = ctypes.c_void_p()
        _check(load().llme_model_load(path.encode(), int(bool(q8)), world, rank,
                                      comm.handle if comm is not None else None, ctypes.byref(h)))
        return cls(h.value)

    @classmethod
    def synthetic(cls, cfg, q8: bool = True, world: int = 1, rank: int = 0, comm=None,
                  seed: int = 0):
        h = ctypes.c_void_p()
        _check(load().llme_model_synthetic(ctypes.byref(_config(cfg)), int(bool(q8)), world, rank,
                                           comm.handle if comm is not None else None, seed,
                                           ctypes.byref(h)))
        return cls(h.value)

    def _logits(self):
        import numpy as np
        return np.zeros(self.config["vocab_size"], np.float32)

    def forward(self, tokens, pos: int):
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        out = self._logits()
        _check(load().llme_model_forward(self.handle, t.ctypes.data, t.size, pos,
                                          out.ctypes.data))
        return out

    def decode(self, token: int, pos: int):
        out = self._logits()
        _check(load().llme_model_decode(self.handle, int(token), pos, out.ctypes.data))
        return out

    @property
    def captures(self) -> int:
        return int(load().llme_model_captures(self.handle))

    def stream_bytes(self) -> tuple[int, int]:
        w, kv = ctypes.c_size_t(), ctypes.c_size_t()
        _check(load().llme_model_stream_bytes(self.handle, ctypes.byref(w), ctypes.byref(kv)))
        return w.value, kv.value

    def fill_history(self, positions: int, seed: int = 0) -> None:
        _check(load().llme_model_fill_history(self.handle, positions, seed))

    def replay(self, times: int, stream: int | None = None) -> None:
        _check(load().llme_model_replay(self.handle, times, stream or None))

    @staticmethod
    def group_forward(models, tokens, pos: int):
        """One forward over emulated ranks (Models built with world > 1 and no communicator,
        ranks 0..world-1); their partials summed in rank order. Rank 0's logits."""
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        arr = (ctypes.c_void_p * len(models))(*[m.handle for m in models])
        out = models[0]._logits()
        _check(load().llme_model_group_forward(arr, len(models), t.ctypes.data, t.size, pos,
                                                out.ctypes.data))
        return out

    def destroy(self) -> None:
        if self.handle:
            _check(load().llme_model_destroy(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass
