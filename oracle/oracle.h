/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the matmul path.
 *
 * A plain-C restatement of the reference engine's CPU matmul, int8 weight
 * format and RMSNorm. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs may load this library, and only as
 * the checker or the timed CPU baseline; the product (llm-engine_b200) never
 * links or calls it.
 *
 * Parity is pinned two ways (tests/test_oracle.py): against the known-answer
 * and invariant tests the reference's own tests hold (tests/test_matmul.cpp,
 * tests/test_quant.cpp), and bit for bit against golden vectors produced by
 * the reference's own sources compiled here (oracle/Makefile -> oracle/_ref,
 * fixtures in tests/golden/ made by tests/golden/make_golden.py).
 *
 * Layouts follow the reference: A is m x k fp32 row-major, B is k x n
 * (in x out) row-major, fp32 or int8 with one fp32 scale per column, C is
 * m x n fp32 row-major.
 */
#ifndef LLME_ORACLE_H
#define LLME_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* quant.cpp:6-28. scale[c] = max|B[:,c]| / 127; q = clamp(lround(B * (1/scale)), -127, 127);
 * an all-zero column gets scale 0 and q 0. */
void orc_quantize_q8(size_t rows, size_t cols, const float* B, int8_t* q, float* scale);

/* quant.cpp:30-36. out[r,c] = (float)q[r,c] * scale[c]. */
void orc_dequantize(size_t rows, size_t cols, const int8_t* q, const float* scale, float* out);

/* matmul.cpp:205-217. i-k-j loop, fp32, C zeroed first. */
void orc_matmul_naive(size_t m, size_t n, size_t k, const float* A, const float* B, float* C);

/* matmul_naive on the dequantized matrix, without materialising it:
 * C[i,j] += A[i,p] * (q[p,j] * scale[j]) in the same i-k-j order. */
void orc_matmul_naive_q8(size_t m, size_t n, size_t k, const float* A, const int8_t* q,
                         const float* scale, float* C);

/* ops.cpp:8-26. Row-wise y = x / sqrt(mean(x^2) + eps) * w, sum of squares in double. */
void orc_rmsnorm(size_t rows, size_t cols, const float* x, const float* w, float eps, float* y);

/* The CPU baseline port: matmul.cpp:240-306's work split on pthreads.
 * m <= 4: k split into contiguous spans (one per thread, at least 64 rows each), each span
 * summed raw into a private partial (gemm_stream, matmul.cpp:186-200), partials added in
 * span order, then the column scales applied once (matmul.cpp:273-281).
 * m > 4: columns split across threads, each thread running the i-k-j loop on its columns
 * with B dequantized as it is read (the packed path's arithmetic, matmul.cpp:84).
 * threads == 0 means one per online CPU. scale == NULL means fp32 B (Bf used). */
void orc_matmul_parallel(size_t m, size_t n, size_t k, const float* A, const float* Bf,
                         const int8_t* Bq, const float* scale, float* C, unsigned threads);

/* Number of threads orc_matmul_parallel uses for threads == 0. */
unsigned orc_default_threads(void);

#ifdef __cplusplus
}
#endif

#endif
