"""The C ABI boundary and the host-side dispatch logic (no GPU).

Checks that libllme_b200.so loads and exports every entry point include/llme_b200.h
declares, that libllme_b200_cxx.so exports the reference's C++ API (cuda_matmul.h), and
the plan the dispatcher makes: kernel choice (cuda_matmul.cu:406-410), the argument
errors and their messages (:411-417, test_cuda.cpp:277-287), empty and k == 0 handling
(:418-422), the TMA / plain-load choice and the split-K sizing.
"""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

import llme_b200 as L

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "llme_b200.h")
CXX_LIB = os.path.join(REPO, "llm-engine_b200", "lib", "libllme_b200_cxx.so")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(llme_\w+)\s*\(", text)))


def exported(path: str, demangle: bool = False) -> str:
    args = ["nm", "-D", "--defined-only"] + (["-C"] if demangle else []) + [path]
    return subprocess.run(args, check=True, stdout=subprocess.PIPE, text=True).stdout


def test_library_loads_and_exports_every_declared_symbol():
    L.load()
    names = declared_functions()
    assert "llme_matmul_q8" in names and "llme_matmul_f32" in names
    syms = exported(L.library_path())
    for name in names:
        assert re.search(rf"\bT {name}$", syms, re.M), name
        assert hasattr(L.load(), name)


def test_cxx_shim_exports_reference_api():
    syms = exported(CXX_LIB, demangle=True)
    for sig in ["matmul_cuda(DeviceTensor const&, DeviceTensor const&, DeviceTensor&, GpuKernel)",
                "matmul_cuda(unsigned long, unsigned long, unsigned long, float const*, float const*, float*, GpuKernel, MatmulFusion const&)",
                "matmul_cuda(unsigned long, unsigned long, unsigned long, float const*, signed char const*, float const*, float*, GpuKernel, MatmulFusion const&)",
                "matmul_cuda(Tensor const&, Tensor const&, GpuKernel)",
                "matmul_cuda(Tensor const&, QTensor const&, GpuKernel)",
                "cuda_scratch_generation()", "cuda_synchronize()", "cuda_available()",
                "DeviceTensor::upload(Tensor const&)", "DeviceTensor::download() const",
                "DeviceQTensor::DeviceQTensor(QTensor const&)"]:
        assert sig in syms, sig


C_CLIENT = r"""
#include <stdio.h>
#include <string.h>
#include "llme_b200.h"

int main(void) {
    llme_plan_t p;
    if (llme_plan(1, 4096, 4096, 1, LLME_KERNEL_AUTOMATIC, 0, 256, 256, 0, 148, LLME_MATH_TENSOR,
                  &p) != LLME_OK || p.path != LLME_PATH_GEMV_TMA)
        return 1;
    if (llme_plan(9, 2, 2, 0, LLME_KERNEL_SKINNY, 0, 256, 256, 0, 148, LLME_MATH_TENSOR, &p) !=
            LLME_E_INVALID || strstr(llme_last_error(), "at most 8 rows") == NULL)
        return 2;
    printf("%d %d %d\n", p.path, LLME_PATH_TCGEN05_F32_SKINNY, (int)sizeof(llme_plan_t));
    return 0;
}
"""


@pytest.mark.skipif(subprocess.run(["which", "gcc"], stdout=subprocess.DEVNULL).returncode != 0,
                    reason="no C compiler")
def test_header_is_plain_c_and_links_from_c(tmp_path):
    # The boundary a cgo / FFI binding sees: strict C99, no C++ or CUDA types, and a program
    # linked to the library plans a call and reads an error message without touching a GPU.
    src, exe = tmp_path / "client.c", tmp_path / "client"
    src.write_text(C_CLIENT)
    libdir = os.path.dirname(L.library_path())
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror",
                    "-I", os.path.join(REPO, "include"), str(src), "-o", str(exe), "-L", libdir,
                    "-lllme_b200", f"-Wl,-rpath,{libdir}"], check=True)
    out = subprocess.run([str(exe)], stdout=subprocess.PIPE, text=True)
    assert out.returncode == 0, out.returncode
    assert int(out.stdout.split()[2]) == ctypes.sizeof(L.Plan)


def test_cxx_headers_compile_against_the_bundled_tensor_layout():
    src = '#include "llme_b200.h"\n#include "cuda_matmul.h"\n#include "cuda_attention.h"\n'
    inc = os.path.join(REPO, "include")
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", inc,
                    "-I", os.path.join(inc, "tensor"), "-x", "c++", "-fsyntax-only", "-"],
                   input=src, text=True, check=True)


@pytest.mark.parametrize("m,kernel", [(1, "skinny"), (8, "skinny"), (9, "tiled_split"),
                                      (64, "tiled_split"), (127, "tiled_split"), (128, "tiled"),
                                      (512, "tiled")])
def test_automatic_kernel_choice(m, kernel):
    p = L.plan(m, 4096, 4096, q8=True)
    assert p["kernel"] == L.KERNELS[kernel]


def test_skinny_rejects_more_than_8_rows():
    with pytest.raises(L.InvalidArgument) as e:
        L.plan(9, 2, 2, q8=False, kernel="skinny")
    assert "at most 8 rows" in str(e.value)
    assert "9x2" in str(e.value)


def test_rejects_2_pow_31_elements():
    with pytest.raises(L.InvalidArgument) as e:
        L.plan(1, 1 << 16, 1 << 15, q8=True)
    assert "2^31" in str(e.value)
    L.plan(1, (1 << 16) - 1, 1 << 15, q8=True)  # just below the limit


def test_unknown_kernel_is_invalid():
    with pytest.raises(L.InvalidArgument):
        L.plan(1, 4, 4, q8=False, kernel=7)


@pytest.mark.parametrize("m,n,k,acc,path", [(0, 5, 5, False, "none"), (3, 0, 5, False, "none"),
                                            (1, 5, 0, False, "zero"), (12, 3, 0, True, "none"),
                                            (12, 3, 0, False, "zero")])
def test_empty_and_zero_k(m, n, k, acc, path):
    assert L.plan(m, n, k, q8=False, accumulate=acc)["path_name"] == path


def test_tma_path_needs_aligned_rows_and_pointers():
    assert L.plan(1, 4096, 4096, q8=True)["path_name"] == "gemv_tma"
    assert L.plan(1, 4100, 4096, q8=True)["path_name"] == "gemv_ldg"      # 4100 B rows
    assert L.plan(1, 4112, 4096, q8=True)["path_name"] == "gemv_tma"
    assert L.plan(1, 1028, 96, q8=False)["path_name"] == "gemv_tma"       # 4112 B rows
    assert L.plan(1, 1027, 96, q8=False)["path_name"] == "gemv_ldg"
    assert L.plan(1, 4096, 4096, q8=True, b_addr=257)["path_name"] == "gemv_ldg"
    assert L.plan(1, 4096, 4097, q8=True)["path_name"] == "gemv_ldg"      # k % 4 (A rows)
    assert L.plan(1, 4096, 4096, q8=True, rms_addr=260)["path_name"] == "gemv_ldg"
    assert L.plan(1, 4096, 4096, q8=True, rms_addr=272)["path_name"] == "gemv_tma"


@pytest.mark.parametrize("n,k", [(4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096),
                                 (288, 4096), (4, 4096), (4100, 1000), (1, 17)])
@pytest.mark.parametrize("q8", [True, False])
@pytest.mark.parametrize("sms", [148, 132, 20])
def test_split_k_plan_covers_k_exactly_once(n, k, q8, sms):
    p = L.plan(1, n, k, q8=q8, sm_count=sms)
    s, span = p["slices"], p["span"]
    assert s >= 1 and span >= 1
    assert (s - 1) * span < k <= s * span           # every row in exactly one slice
    assert p["grid_y"] == s
    assert p["grid_x"] * p["tile_n"] >= n
    if p["path_name"] == "gemv_tma":
        assert span % 128 == 0                      # boxes never straddle two slices
        assert s <= 8 and p["cluster"] == s         # the slices of a strip are one cluster
        assert p["grid_x"] * p["grid_y"] <= max(2 * sms, p["grid_x"])
        assert p["split_bytes"] == 0                # reduced through DSMEM, no scratch
    elif s > 1:
        assert p["split_bytes"] > 0 and p["counter_slots"] == p["grid_x"]
    else:
        assert p["split_bytes"] == 0


def test_decode_shapes_fill_the_gpu():
    # The 7B decode shapes launch close to two CTAs per SM on 148 SMs (host-only plans: the
    # model of the cluster capacity, 2 x SMs / cluster size).
    for n, k in [(4096, 4096), (11008, 4096), (4096, 11008), (12288, 4096)]:
        p = L.plan(1, n, k, q8=True)
        assert 0.8 * 296 <= p["grid_x"] * p["grid_y"] <= 296, (n, k, p)


def test_gemv_slices_fit_the_device_cluster_capacity():
    # The k slices of a strip form one cluster, and every cluster must be resident at once.
    # B200's measured capacity (clusters of 1..8 CTAs at two CTAs per SM) is below 296 / c.
    b200 = [296, 148, 93, 71, 56, 45, 37, 33]
    # the 7B wqkv: 96 strips; the model would take 3 slices, the device holds 93 clusters of 3
    assert L.plan(1, 12288, 4096, q8=True)["grid_y"] == 3
    p = L.plan(1, 12288, 4096, q8=True, gemv_clusters=b200)
    assert p["grid_y"] == 2 and p["cluster"] == 2 and p["span"] == 2048
    # the 86-strip w1 fits at 3; 32 strips fit at 8 (33 clusters)
    assert L.plan(1, 11008, 4096, q8=True, gemv_clusters=b200)["grid_y"] == 3
    assert L.plan(1, 4096, 4096, q8=True, gemv_clusters=b200)["grid_y"] == 8
    # one fewer cluster of 8 than strips: 7 slices, k still covered exactly once
    p = L.plan(1, 4096, 4096, q8=True, gemv_clusters=b200[:7] + [31])
    assert p["grid_y"] == 7 and (p["slices"] - 1) * p["span"] < 4096 <= p["slices"] * p["span"]
    # a table with no answer for a size falls back to the model
    assert L.plan(1, 12288, 4096, q8=True, gemv_clusters=[0] * 8)["grid_y"] == 3


def test_tcgen05_path_choice():
    # TF32 tensor cores for m >= 128 with TMA-addressable fp32 operands, in tensor math only.
    assert L.plan(128, 4096, 4096, q8=False)["path_name"] == "tcgen05"
    assert L.plan(8192, 8192, 8192, q8=False)["grid_x"] == 64 * 32
    # B read as stored (MN-major operand) below 6144 rows; a B^T pass from there on.
    assert L.plan(6143, 4096, 1024, q8=False)["operand_bytes"] == 0
    assert L.plan(6144, 4096, 1024, q8=False)["operand_bytes"] == 4096 * 1024 * 4
    assert L.plan(127, 4096, 4096, q8=False)["path_name"] == "tcgen05_f32_skinny"
    assert L.plan(127, 4096, 4096, q8=False, math=L.MATH_FP32)["path_name"] == "tiled_simt"
    assert L.plan(128, 4096, 4096, q8=False, math=L.MATH_FP32)["path_name"] == "tiled_simt"
    assert L.plan(128, 1030, 4096, q8=False)["path_name"] == "tiled_simt"   # n % 4
    assert L.plan(128, 1028, 513, q8=False)["path_name"] == "tiled_simt"    # k % 4
    assert L.plan(128, 1028, 512, q8=False, a_addr=260)["path_name"] == "tiled_simt"
    assert L.plan(128, 1028, 512, q8=False, a_addr=260, rms_addr=256)["path_name"] == "tcgen05"


def test_tcgen05_q8_path_choice():
    # int8 weights, m >= 128, tensor math: kind::i8 tensor cores on the split activations.
    p = L.plan(512, 4096, 4096, q8=True)
    assert p["path_name"] == "tcgen05_q8" and p["kernel"] == 2      # automatic -> tiled
    assert p["tile_m"] == 128 and p["tile_n"] == 128 and p["cluster"] == 1
    assert p["grid_x"] == 128


def test_tcgen05_skinny_plan():
    # Decode-shaped int8 (9..127 rows, or tiled_split / tiled below 128) in tensor math.
    p = L.plan(16, 4096, 4096, q8=True)
    assert p["path_name"] == "tcgen05_skinny" and p["kernel"] == 3       # -> tiled_split
    assert (p["tile_m"], p["tile_n"], p["grid_x"], p["grid_y"]) == (16, 128, 32, 1)
    assert p["slices"] == 8 and p["span"] == 512                          # 256 CTAs
    assert p["cluster"] == 8                    # the k slices of a tile are one cluster
    assert p["counter_slots"] == 0 and p["split_bytes"] == 0              # no scratch
    assert p["operand_bytes"] == 3 * 16 * 4096 + 16 * 4
    p = L.plan(64, 4096, 4096, q8=True)
    assert p["tile_m"] == 64 and p["slices"] == 4 and p["grid_x"] * p["slices"] <= 148
    p = L.plan(100, 11008, 4096, q8=True)
    assert (p["tile_m"], p["grid_y"], p["slices"]) == (64, 2, 1) and p["split_bytes"] == 0
    for m, k in [(9, 4096), (33, 11008), (127, 100)]:
        p = L.plan(m, 4096, k, q8=True)
        assert (p["slices"] - 1) * p["span"] < k <= p["slices"] * p["span"]
    assert L.plan(4, 4096, 4096, q8=True)["path_name"] == "gemv_tma"
    assert L.plan(4, 4096, 4096, q8=True, kernel="tiled_split")["path_name"] == "tcgen05_skinny"
    assert L.plan(16, 4096, 4096, q8=True, math=L.MATH_FP32)["path_name"] == "tiled_simt"
    assert L.plan(16, 4104, 4096, q8=True)["path_name"] == "tiled_simt"     # n % 16
    assert L.plan(16, 4096, 4096, q8=False)["path_name"] == "tcgen05_f32_skinny"  # fp32 W


def test_tcgen05_f32_skinny_plan():
    # Decode-shaped fp32 weights (tiled_split, or tiled below 128 rows) in tensor math: three
    # TF32 terms, k slices as one thread-block cluster of at most 8.
    p = L.plan(16, 4096, 4096, q8=False)
    assert p["path_name"] == "tcgen05_f32_skinny" and p["kernel"] == 3
    assert (p["tile_m"], p["tile_n"], p["grid_x"], p["grid_y"]) == (16, 128, 32, 1)
    assert p["slices"] == 4 and p["cluster"] == 4 and p["span"] == 1024  # 128 CTAs, 1 per SM
    assert p["split_bytes"] == 0 and p["counter_slots"] == 0 and p["operand_bytes"] == 0
    p = L.plan(64, 4096, 4096, q8=False)
    assert (p["tile_m"], p["slices"], p["span"]) == (64, 4, 1024)        # 128 CTAs, 1 per SM
    p = L.plan(100, 11008, 4096, q8=False)
    assert (p["tile_m"], p["grid_x"], p["grid_y"], p["slices"]) == (64, 86, 2, 1)
    for m, k in [(9, 4096), (33, 11008), (127, 100), (20, 4)]:
        p = L.plan(m, 4096, k, q8=False)
        assert p["slices"] <= 8 and p["span"] % 32 == 0
        assert (p["slices"] - 1) * p["span"] < k <= p["slices"] * p["span"]
    assert L.plan(4, 4096, 4096, q8=False, kernel="tiled_split")["path_name"] == \
        "tcgen05_f32_skinny"
    assert L.plan(4, 4096, 4096, q8=False)["path_name"] == "gemv_tma"
    p = L.plan(24, 1028, 512, q8=False, a_addr=260, rms_addr=256)
    assert p["path_name"] == "tcgen05_f32_skinny" and p["rms_prepass"] == 1
    assert L.plan(24, 1028, 512, q8=False, a_addr=260)["path_name"] == "tiled_simt"


def test_fp32_gemv_up_to_16_rows_plan():
    # fp32 weights with 9..16 rows (automatic -> tiled_split, or tiled) in fp32 arithmetic: the
    # TMA GEMV at 16 rows instead of the SIMT tiles. Tensor math keeps the TF32 kernel.
    F = L.MATH_FP32
    for m in (9, 12, 16):
        p = L.plan(m, 4096, 4096, q8=False, math=F)
        assert p["path_name"] == "gemv_tma" and p["kernel"] == 3
        assert (p["tile_m"], p["tile_n"], p["grid_x"]) == (16, 32, 128)
        assert p["slices"] == 2 and p["cluster"] == 2 and p["span"] == 2048   # 256 CTAs
        assert p["split_bytes"] == 0 and p["norm_bytes"] == 0 and p["rms_prepass"] == 0
        assert L.plan(m, 4096, 4096, q8=False)["path_name"] == "tcgen05_f32_skinny"
    assert L.plan(12, 4096, 4096, q8=False, kernel="tiled", math=F)["path_name"] == "gemv_tma"
    p = L.plan(12, 4096, 4096, q8=False, rms_addr=256, math=F)   # RMSNorm by the row pass
    assert p["path_name"] == "gemv_tma" and p["rms_prepass"] == 1
    assert p["norm_bytes"] == 12 * 4096 * 4
    assert L.plan(17, 4096, 4096, q8=False, math=F)["path_name"] == "tiled_simt"
    assert L.plan(16, 4096, 4096, q8=True, math=F)["path_name"] == "tiled_simt"   # int8 W
    # Operands the TMA cannot stream: the SIMT tiles, as before.
    assert L.plan(12, 4096, 4096, q8=False, a_addr=260, math=F)["path_name"] == "tiled_simt"
    assert L.plan(12, 4096, 4098, q8=False, math=F)["path_name"] == "tiled_simt"  # k % 4
    assert L.plan(24, 1030, 512, q8=False)["path_name"] == "tiled_simt"   # n % 4
    assert L.plan(24, 1028, 514, q8=False)["path_name"] == "tiled_simt"   # k % 4
    assert L.plan(24, 1028, 512, q8=False, b_addr=8)["path_name"] == "tiled_simt"


def test_tcgen05_q8_cta_pairs_plan(monkeypatch):
    # LLME_B200_CTA_PAIRS=1: cta_group::2, 128 x 256 tiles, 4 x 16 of them on 64 pairs.
    monkeypatch.setenv("LLME_B200_CTA_PAIRS", "1")
    p = L.plan(512, 4096, 4096, q8=True)
    assert p["tile_n"] == 256 and p["cluster"] == 2 and p["grid_x"] == 128
    assert L.plan(2048, 8192, 4096, q8=True)["grid_x"] == 148
    # an odd SM count keeps single CTAs with 128 x 128 tiles
    p1 = L.plan(512, 4096, 4096, q8=True, sm_count=147)
    assert p1["tile_n"] == 128 and p1["cluster"] == 1 and p1["grid_x"] == 128
    kp = 4096
    assert p["operand_bytes"] == 2 * ((512 * kp + 255) // 256 * 256) + 512 * 4
    p = L.plan(130, 1040, 72, q8=True, rms_addr=256)
    assert p["path_name"] == "tcgen05_q8" and p["rms_prepass"] == 0 and p["norm_bytes"] == 0
    assert p["operand_bytes"] == 2 * ((130 * 80 + 255) // 256 * 256) + 130 * 4   # pitch 80
    assert L.plan(2048, 8192, 4096, q8=True, sm_count=148)["grid_x"] == 148   # persistent
    assert L.plan(512, 4096, 4096, q8=True, math=L.MATH_FP32)["path_name"] == "tiled_simt"
    assert L.plan(127, 4096, 4096, q8=True)["path_name"] == "tcgen05_skinny"
    assert L.plan(512, 4104, 4096, q8=True)["path_name"] == "tiled_simt"     # n % 16
    assert L.plan(512, 4096, 4096, q8=True, b_addr=8)["path_name"] == "tiled_simt"
    assert L.plan(512, 4096, 131072, q8=True)["path_name"] == "tcgen05_q8"
    assert L.plan(512, 4096, 131073, q8=True)["path_name"] == "tiled_simt"   # s32 sums exact
    assert L.plan(512, 4096, 4096, q8=True, kernel="tiled_split")["path_name"] == "tcgen05_skinny"


def test_rms_prepass_only_outside_the_gemv():
    assert L.plan(4, 300, 288, q8=False, rms_addr=256)["rms_prepass"] == 0
    p = L.plan(70, 130, 40, q8=False, rms_addr=256)
    assert p["rms_prepass"] == 1 and p["norm_bytes"] == 70 * 40 * 4


def test_tiled_split_sizes():
    p = L.plan(16, 4096, 4096, q8=True, kernel="tiled_split", math=L.MATH_FP32)
    assert p["path_name"] == "tiled_simt" and p["slices"] > 1
    assert (p["slices"] - 1) * p["span"] < 4096 <= p["slices"] * p["span"]
    p = L.plan(200, 33, 513, q8=False, kernel="tiled")
    assert p["slices"] == 1


def test_math_mode_roundtrip():
    prev = L.get_math()
    assert L.set_math(L.MATH_FP32) == prev
    assert L.get_math() == L.MATH_FP32
    L.set_math(prev)
    with pytest.raises(L.InvalidArgument):
        L.set_math(5)


def test_attention_launch_counts():
    # Kernels one call enqueues (host only): the split kernel, plus the merge launch when the
    # context may span chunks; single_block is one launch; invalid arguments give 0.
    S = L.AttentionShape
    mha = S(32, 32, 128, 4096, 3 * 4096, 4096, 4096)
    assert L.attention_launches(mha, 1) == 2
    assert L.attention_launches(S(4, 1, 128, 20000, 768, 128, 512), 1) == 2
    assert L.attention_launches(S(4, 1, 128, 64, 768, 128, 512), 1) == 1     # one chunk
    assert L.attention_launches(S(32, 32, 128, 100, 3 * 4096, 4096, 4096), 20) == 1  # single
    assert L.attention_launches(S(32, 32, 128, 100, 3 * 4096, 4096, 4096), 20, "split") == 2
    assert L.attention_launches(mha, 0) == 0
    assert L.attention_launches(S(6, 4, 8, 64, 96, 32, 48), 1) == 0          # 6 heads / 4 kv


def test_attention_scratch_is_the_chunk_partials():
    # One block per row: every chunk's partial o (head_size floats) and its (m, l) pair, each
    # part a whole number of float4s -- nothing else (the merge is a second launch, so there
    # are no tickets or group partials).
    S = L.AttentionShape
    mha = S(32, 32, 128, 4096, 3 * 4096, 4096, 4096)      # 64 chunks of 64 positions
    chunks = 32 * 64
    assert L.attention_scratch_floats(mha, 1, "split") == chunks * 128 + 2 * chunks
    assert L.attention_scratch_floats(mha, 3, "split") == 3 * (chunks * 128 + 2 * chunks)


def test_attention_check_rules():
    # The reference's attention_check rules (src/cuda_attention.cu:306-325), host only.
    S = L.AttentionShape
    ok = S(8, 2, 64, 1000, 768, 128, 512)
    for k in ("automatic", "split", "single_block"):
        L.attention_check(ok, k)
    with pytest.raises(L.InvalidArgument):        # head_size % 4 for split
        L.attention_check(S(2, 2, 6, 64, 36, 12, 12), "split")
    L.attention_check(S(2, 2, 6, 64, 36, 12, 12), "single_block")
    with pytest.raises(L.InvalidArgument):        # 6 heads over 4 kv heads
        L.attention_check(S(6, 4, 8, 64, 96, 32, 48), "automatic")
    with pytest.raises(L.InvalidArgument):        # empty context
        L.attention_check(S(4, 4, 8, 0, 64, 32, 32), "automatic")
    long = S(4, 1, 128, 20000, 768, 128, 512)
    with pytest.raises(L.InvalidArgument):        # single_block's 48 KB of scores
        L.attention_check(long, "single_block")
    L.attention_check(long, "split")
    assert L.attention_scratch_floats(long, 1, "single_block") == 0
    assert L.attention_scratch_floats(long, 10, "automatic") >= 10 * 4 * 128
    # automatic splits at most 8 rows when single_block fits
    assert L.attention_scratch_floats(ok, 100, "automatic") == L.attention_scratch_floats(ok, 8, "split")
    # one block per row at a stride set by the shape alone (16-byte multiples): a call with
    # fewer rows uses a prefix of a larger call's blocks, tickets included
    for shape in (ok, long, S(32, 32, 128, 4112, 12288, 4096, 4096)):
        one = L.attention_scratch_floats(shape, 1, "split")
        assert one % 4 == 0
        for rows in (2, 3, 8, 13):
            assert L.attention_scratch_floats(shape, rows, "split") == rows * one


@pytest.mark.parametrize("q8,kernel,math,tile", [(False, "naive", L.MATH_TENSOR, 16),
                                                 (False, "tiled", L.MATH_FP32, 64),
                                                 (True, "tiled_split", L.MATH_TENSOR, 64),
                                                 (False, "tiled_split", L.MATH_TENSOR, 64)])
def test_row_tiles_beyond_the_grid_are_invalid(q8, kernel, math, tile):
    # Paths with row tiles on grid y take at most 65535 of them; the prefill GEMMs (all tiles
    # on x) take the same rows.
    rows = 65535 * tile
    assert L.plan(rows, 16, 16, q8=q8, kernel=kernel, math=math)["grid_y"] == 65535
    with pytest.raises(L.InvalidArgument) as e:
        L.plan(rows + 1, 16, 16, q8=q8, kernel=kernel, math=math)
    assert "exceed the grid's 65535" in str(e.value)
    big = L.plan(rows + 1, 16, 16, q8=q8, kernel="tiled", math=L.MATH_TENSOR)
    assert big["path_name"] in ("tcgen05", "tcgen05_q8") and big["grid_y"] == 1


def test_scratch_free_plans_are_the_ones_the_header_names():
    # Plans with split_bytes, norm_bytes and operand_bytes all zero touch no shared scratch.
    def scratch(p):
        return p["split_bytes"] + p["norm_bytes"] + p["operand_bytes"]
    for q8 in (False, True):
        for n, k in [(4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)]:
            for rms in (0, 256):
                p = L.plan(1, n, k, q8=q8, rms_addr=rms)
                assert p["path_name"] == "gemv_tma" and scratch(p) == 0
    p = L.plan(16, 4096, 4096, q8=False, math=L.MATH_TENSOR)
    assert p["path_name"] == "tcgen05_f32_skinny" and scratch(p) == 0
    p = L.plan(16, 4096, 4096, q8=False, rms_addr=256, math=L.MATH_TENSOR)
    assert p["path_name"] == "tcgen05_f32_skinny" and p["norm_bytes"] == 16 * 4096 * 4
    assert scratch(L.plan(16, 4096, 4096, q8=True, math=L.MATH_TENSOR)) > 0
    assert scratch(L.plan(512, 4096, 4096, q8=True, math=L.MATH_TENSOR)) > 0


def test_null_pointers_are_refused_before_any_device_work():
    # A pointer the call would read or write that is NULL is LLME_E_INVALID, decided on the host
    # before the device is queried; pointers a call never touches may be NULL.
    lib, P, INVALID = L.load(), 256, 1

    def refused(rc, text="null"):
        return rc == INVALID and text in L.last_error()

    assert refused(lib.llme_matmul_f32(2, 3, 4, None, P, P, 0, 0, None, 0, None))
    assert refused(lib.llme_matmul_f32(2, 3, 4, P, None, P, 0, 0, None, 0, None))
    assert refused(lib.llme_matmul_f32(2, 3, 4, P, P, None, 0, 0, None, 0, None))
    assert refused(lib.llme_matmul_q8(2, 3, 4, P, P, None, P, 0, 0, None, 0, None))
    assert refused(lib.llme_matmul_f32(2, 3, 0, None, None, None, 0, 0, None, 0, None))  # zeroes C
    assert refused(lib.llme_matmul_q8_noalloc(2, 3, 4, P, P, None, P, 0, None))
    # empty products and k == 0 with accumulate touch nothing: not refused (without a GPU they
    # go on to fail at the device query instead)
    assert lib.llme_matmul_f32(0, 3, 4, None, None, None, 0, 0, None, 0, None) != INVALID
    assert lib.llme_matmul_q8(2, 0, 4, None, None, None, None, 0, 0, None, 0, None) != INVALID
    assert lib.llme_matmul_f32(2, 3, 0, None, None, None, 0, 1, None, 0, None) != INVALID
    # plans, batches, communicators and attention
    assert refused(lib.llme_plan(1, 1, 1, 0, 0, 0, P, P, 0, 148, 0, None))
    assert refused(lib.llme_batch_q8_create(None, 1, 1, None))
    handle = ctypes.c_void_p()
    assert refused(lib.llme_batch_q8_create(ctypes.byref(handle), 1, 1, None))
    prods = (L.Q8Product * 2)(L.Q8Product(16, 16, P, P, P, P, 0), L.Q8Product(16, 16, P, P, None, P, 0))
    assert refused(lib.llme_batch_q8_create(ctypes.byref(handle), 1, 2, prods), "product 1")
    assert refused(lib.llme_batch_q8_create(ctypes.byref(handle), 128, 2, prods), "product 1")
    assert handle.value is None
    assert refused(lib.llme_comm_unique_id(None))
    assert refused(lib.llme_comm_init(None, 2, 0, b"x" * 128, 1.0))
    assert refused(lib.llme_comm_init(ctypes.byref(handle), 2, 0, None, 1.0))
    assert refused(lib.llme_allreduce_sum_f32(P, 4, None, None), "no communicator")
    shape = L.AttentionShape(8, 8, 64, 128, 512, 512, 512)
    assert refused(lib.llme_attention(ctypes.byref(shape), 1, None, P, P, P, P, P, 0, None))
    assert refused(lib.llme_attention(ctypes.byref(shape), 1, P, P, P, P, None, P, 0, None))
    assert lib.llme_attention(ctypes.byref(shape), 0, None, None, None, None, None, None, 0, None) == 0


def test_status_codes_match_the_header():
    text = open(HEADER).read()
    codes = dict((name, int(v)) for name, v in re.findall(r"\b(LLME_(?:OK|E_\w+))\s*=\s*(\d+)", text))
    assert codes == {"LLME_OK": L.OK, "LLME_E_INVALID": L.E_INVALID, "LLME_E_CUDA": L.E_CUDA,
                     "LLME_E_TIMEOUT": L.E_TIMEOUT, "LLME_E_UNSUPPORTED": L.E_UNSUPPORTED,
                     "LLME_E_NCCL": L.E_NCCL, "LLME_E_HOST": L.E_HOST, "LLME_E_RANGE": L.E_RANGE}


def test_no_exception_crosses_the_c_boundary():
    # Every status-returning entry point runs its body under a guard that turns a host-side
    # exception into LLME_E_HOST; the source holds one guard per such function.
    csrc = os.path.join(REPO, "llm-engine_b200", "csrc")
    unguarded = []
    for name in ("capi.cu", "comm.cu", "attention.cu", "model.cu"):
        src = open(os.path.join(csrc, name)).read()
        body = src[src.index('extern "C" {'):]
        for m in re.finditer(r"^int (llme_\w+)\([^{]*\) \{\n(.*?)^\}", body, re.S | re.M):
            fn, text = m.group(1), m.group(2)
            if "llme::guarded(" not in text and fn not in (
                    "llme_set_math", "llme_device_available", "llme_device_supported"):
                unguarded.append(fn)
    assert unguarded == []


def test_torch_wrapper_refuses_what_the_kernels_cannot_take():
    # Checked in Python before any pointer reaches the library: dtypes, shapes, contiguity,
    # and residency in one CUDA device's memory (a host tensor's address on the GPU faults).
    torch = pytest.importorskip("torch")
    A, B = torch.zeros(3, 5), torch.zeros(5, 7)
    q, s = torch.zeros(5, 7, dtype=torch.int8), torch.zeros(7)
    cases = [
        ((torch.zeros(3, 5, 2), B), {}, "matrices"),
        ((torch.zeros(2, 3), torch.zeros(4, 2)), {}, "2x3"),
        ((A.half(), B), {}, "A is torch.float16"),
        ((A, B.double()), {}, "B is torch.float64"),
        ((A, B), {"C": torch.zeros(3, 6)}, "C has shape (3, 6)"),
        ((A, q), {"scale": torch.zeros(6)}, "scale has shape (6,)"),
        ((A, B), {"rms_weight": torch.zeros(4)}, "rms_weight has shape (4,)"),
        ((A, B.t().contiguous().t()), {}, "contiguous"),
        ((A, B), {}, "CUDA device"),
        ((A, q), {"scale": s}, "CUDA device"),
    ]
    for args, kw, text in cases:
        with pytest.raises(L.InvalidArgument) as e:
            L.matmul(*args, **kw)
        assert text in str(e.value), (text, str(e.value))
    with pytest.raises(L.InvalidArgument, match="CUDA device memory"):
        L.quantize_q8(torch.zeros(4, 8))
    with pytest.raises(L.InvalidArgument, match="2-D float32"):
        L.quantize_q8(torch.zeros(4, 8, dtype=torch.float64))
