// TEST/BENCH INFRASTRUCTURE ONLY: a C entry point to the reference's own GPU attention
// (src/cuda_attention.cu, compiled from the reference's sources for sm_100a), so the
// benchmark can time it beside the library's kernels on the same inputs.
#include <cstddef>
#include <exception>

#include "cuda_attention.h"

extern "C" {

size_t ref_attention_scratch_floats(int n_heads, int n_kv_heads, int head_size, int seq_len,
                                    size_t q_stride, size_t kv_stride, size_t out_stride,
                                    size_t rows, int kernel) {
    const AttentionShape s{n_heads, n_kv_heads, head_size, seq_len, q_stride, kv_stride, out_stride};
    try {
        return attention_scratch_floats(s, rows, static_cast<AttentionKernel>(kernel));
    } catch (const std::exception&) {
        return 0;
    }
}

// 0 on success, 1 on a rejected shape or a CUDA error.
int ref_attention(int n_heads, int n_kv_heads, int head_size, int seq_len, size_t q_stride,
                  size_t kv_stride, size_t out_stride, size_t rows, const int* pos_dev,
                  const float* q, const float* k, const float* v, float* out, float* scratch,
                  int kernel) {
    const AttentionShape s{n_heads, n_kv_heads, head_size, seq_len, q_stride, kv_stride, out_stride};
    try {
        attention_cuda(s, rows, pos_dev, q, k, v, out, scratch, static_cast<AttentionKernel>(kernel));
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}

}  // extern "C"
