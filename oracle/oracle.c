/*
 * TEST INFRASTRUCTURE ONLY -- see oracle.h. CPU restatement of the reference
 * engine's matmul path; each function cites the reference file:line it follows
 * (paths inside the reference project).
 *
 * Built with -ffp-contract=off (oracle/Makefile) so a product a*b and the sum
 * that follows round separately, as the reference's own build in oracle/_ref
 * does; the golden vectors then match bit for bit.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* quant.cpp:6-28 */
void orc_quantize_q8(size_t rows, size_t cols, const float* B, int8_t* q, float* scale) {
    for (size_t c = 0; c < cols; ++c) scale[c] = 0.0f;
    /* max |B[:, c]|, with std::max's rule: keep the current value unless it is less. */
    for (size_t r = 0; r < rows; ++r)
        for (size_t c = 0; c < cols; ++c) {
            const float v = fabsf(B[r * cols + c]);
            if (scale[c] < v) scale[c] = v;
        }
    float* inv = (float*)malloc((cols ? cols : 1) * sizeof(float));
    for (size_t c = 0; c < cols; ++c) {
        scale[c] /= 127.0f;
        inv[c] = scale[c] > 0.0f ? 1.0f / scale[c] : 0.0f;
    }
    for (size_t r = 0; r < rows; ++r)
        for (size_t c = 0; c < cols; ++c) {
            /* round half away from zero, then clamp to the symmetric range */
            long v = lroundf(B[r * cols + c] * inv[c]);
            if (v < -127L) v = -127L;
            if (v > 127L) v = 127L;
            q[r * cols + c] = (int8_t)v;
        }
    free(inv);
}

/* quant.cpp:30-36 */
void orc_dequantize(size_t rows, size_t cols, const int8_t* q, const float* scale, float* out) {
    for (size_t r = 0; r < rows; ++r)
        for (size_t c = 0; c < cols; ++c) out[r * cols + c] = (float)q[r * cols + c] * scale[c];
}

/* matmul.cpp:205-217 */
void orc_matmul_naive(size_t m, size_t n, size_t k, const float* A, const float* B, float* C) {
    memset(C, 0, m * n * sizeof(float));
    for (size_t i = 0; i < m; ++i)
        for (size_t p = 0; p < k; ++p) {
            const float a = A[i * k + p];
            const float* b = B + p * n;
            float* c = C + i * n;
            for (size_t j = 0; j < n; ++j) c[j] += a * b[j];
        }
}

void orc_matmul_naive_q8(size_t m, size_t n, size_t k, const float* A, const int8_t* q,
                         const float* scale, float* C) {
    memset(C, 0, m * n * sizeof(float));
    for (size_t i = 0; i < m; ++i)
        for (size_t p = 0; p < k; ++p) {
            const float a = A[i * k + p];
            const int8_t* b = q + p * n;
            float* c = C + i * n;
            for (size_t j = 0; j < n; ++j) c[j] += a * ((float)b[j] * scale[j]);
        }
}

/* ops.cpp:8-26 */
void orc_rmsnorm(size_t rows, size_t cols, const float* x, const float* w, float eps, float* y) {
    if (cols == 0) return;
    for (size_t r = 0; r < rows; ++r) {
        const float* in = x + r * cols;
        float* out = y + r * cols;
        double ss = 0.0;
        for (size_t c = 0; c < cols; ++c) ss += (double)in[c] * in[c];
        const float s = (float)(1.0 / sqrt(ss / (double)cols + (double)eps));
        for (size_t c = 0; c < cols; ++c) out[c] = in[c] * s * w[c];
    }
}

/* ---- CPU baseline port: matmul.cpp:240-306 on pthreads ------------------------------- */

enum { kStreamMaxRows = 4, kStreamMinK = 64, kKC = 256 };

typedef struct {
    size_t m, n, k;
    const float* A;
    const float* Bf;
    const int8_t* Bq;
    const float* scale;
    float* out;   /* stream path: partial (m x n); packed path: C */
    size_t p0, p1; /* stream path: k range */
    size_t c0, c1; /* packed path: column range */
} Task;

/* gemm_stream, matmul.cpp:186-200: raw int8 (unscaled) or fp32 summed over [p0, p1). */
static void* stream_task(void* arg) {
    Task* t = (Task*)arg;
    memset(t->out, 0, t->m * t->n * sizeof(float));
    for (size_t p = t->p0; p < t->p1; ++p)
        for (size_t r = 0; r < t->m; ++r) {
            const float a = t->A[r * t->k + p];
            float* o = t->out + r * t->n;
            if (t->Bq) {
                const int8_t* b = t->Bq + p * t->n;
                for (size_t c = 0; c < t->n; ++c) o[c] += a * (float)b[c];
            } else {
                const float* b = t->Bf + p * t->n;
                for (size_t c = 0; c < t->n; ++c) o[c] += a * b[c];
            }
        }
    return NULL;
}

/* The packed path's per-element arithmetic (matmul.cpp:111-125, 131-163): for each KC-deep
 * block of k, a register sum over the block starting from zero, then C += that sum; int8 B
 * dequantized as it is packed (matmul.cpp:84). */
static void* packed_task(void* arg) {
    Task* t = (Task*)arg;
    const size_t w = t->c1 - t->c0;
    float* tmp = (float*)malloc((w ? w : 1) * sizeof(float));
    for (size_t i = 0; i < t->m; ++i) {
        float* crow = t->out + i * t->n;
        for (size_t pc = 0; pc < t->k; pc += kKC) {
            const size_t pe = pc + kKC < t->k ? pc + kKC : t->k;
            for (size_t j = 0; j < w; ++j) tmp[j] = 0.0f;
            for (size_t p = pc; p < pe; ++p) {
                const float a = t->A[i * t->k + p];
                for (size_t j = 0; j < w; ++j) {
                    const size_t c = t->c0 + j;
                    const float b = t->Bq ? (float)t->Bq[p * t->n + c] * t->scale[c]
                                          : t->Bf[p * t->n + c];
                    tmp[j] += a * b;
                }
            }
            for (size_t j = 0; j < w; ++j) crow[t->c0 + j] += tmp[j];
        }
    }
    free(tmp);
    return NULL;
}

unsigned orc_default_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (unsigned)n : 1u;
}

static void run_tasks(Task* tasks, size_t count, void* (*fn)(void*)) {
    if (count == 1) {
        fn(&tasks[0]);
        return;
    }
    pthread_t* th = (pthread_t*)malloc(count * sizeof(pthread_t));
    for (size_t i = 1; i < count; ++i) pthread_create(&th[i], NULL, fn, &tasks[i]);
    fn(&tasks[0]); /* the caller works too, as ThreadPool::run does */
    for (size_t i = 1; i < count; ++i) pthread_join(th[i], NULL);
    free(th);
}

void orc_matmul_parallel(size_t m, size_t n, size_t k, const float* A, const float* Bf,
                         const int8_t* Bq, const float* scale, float* C, unsigned threads) {
    memset(C, 0, m * n * sizeof(float));
    if (m == 0 || n == 0) return;
    const size_t workers = threads ? threads : orc_default_threads();
    if (m <= kStreamMaxRows) {
        /* matmul.cpp:255-282 */
        size_t tasks = (k + kStreamMinK - 1) / kStreamMinK;
        if (tasks > workers) tasks = workers;
        if (tasks < 1) tasks = 1;
        const size_t span = tasks ? (k + tasks - 1) / tasks : 0;
        float* partials = (float*)malloc(tasks * m * n * sizeof(float));
        Task* ts = (Task*)calloc(tasks, sizeof(Task));
        for (size_t t = 0; t < tasks; ++t) {
            size_t p0 = t * span;
            if (p0 > k) p0 = k;
            size_t p1 = p0 + span < k ? p0 + span : k;
            Task x = {m, n, k, A, Bf, Bq, scale, partials + t * m * n, p0, p1, 0, 0};
            ts[t] = x;
        }
        run_tasks(ts, tasks, stream_task);
        for (size_t t = 0; t < tasks; ++t) {
            const float* part = partials + t * m * n;
            for (size_t i = 0; i < m * n; ++i) C[i] += part[i];
        }
        if (Bq)
            for (size_t r = 0; r < m; ++r)
                for (size_t c = 0; c < n; ++c) C[r * n + c] *= scale[c];
        free(ts);
        free(partials);
        return;
    }
    /* Column slabs of at least 64 columns, one per worker. */
    size_t tasks = (n + 63) / 64;
    if (tasks > workers) tasks = workers;
    if (tasks < 1) tasks = 1;
    const size_t slab = (n + tasks - 1) / tasks;
    Task* ts = (Task*)calloc(tasks, sizeof(Task));
    size_t used = 0;
    for (size_t t = 0; t < tasks; ++t) {
        const size_t c0 = t * slab;
        if (c0 >= n) break;
        const size_t c1 = c0 + slab < n ? c0 + slab : n;
        Task x = {m, n, k, A, Bf, Bq, scale, C, 0, 0, c0, c1};
        ts[used++] = x;
    }
    run_tasks(ts, used, packed_task);
    free(ts);
}
