// TEST INFRASTRUCTURE ONLY. A C-callable wrapper around the reference engine's
// own CPU matmul API (matmul.h:9-22, quant.h:4-9, ops.h:11), compiled together
// with the reference's unmodified sources by oracle/Makefile into
// oracle/_ref/libllme_ref.so. Used to pin the oracle restatement (golden
// vectors) and, as "kind": "reference", as the timed CPU baseline. Nothing in
// the product links it.
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <exception>
#include <stdexcept>
#include <vector>
#include <string>

#include "matmul.h"
#include "ops.h"
#include "quant.h"
#include "tensor.h"
#include "thread_pool.h"

namespace {

thread_local std::string g_error;

Tensor make_tensor(std::size_t rows, std::size_t cols, const float* src) {
    Tensor t(rows, cols);
    if (rows * cols) std::memcpy(t.data.data(), src, rows * cols * sizeof(float));
    return t;
}

void copy_out(const Tensor& t, float* dst) {
    if (!t.data.empty()) std::memcpy(dst, t.data.data(), t.data.size() * sizeof(float));
}

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::invalid_argument& e) {
        g_error = e.what();
        return 1;
    } catch (const std::exception& e) {
        g_error = e.what();
        return 2;
    }
}

}  // namespace

extern "C" {

const char* ref_last_error() { return g_error.c_str(); }

unsigned ref_pool_threads() { return ThreadPool::global().size(); }

// matmul.cpp:205-217
int ref_matmul_naive(std::size_t m, std::size_t n, std::size_t k, std::size_t b_rows,
                     const float* A, const float* B, float* C) {
    return guarded([&] {
        copy_out(matmul_naive(make_tensor(m, k, A), make_tensor(b_rows, n, B)), C);
    });
}

// matmul.cpp:310-313
int ref_matmul_parallel_f32(std::size_t m, std::size_t n, std::size_t k, const float* A,
                            const float* B, float* C, unsigned threads) {
    return guarded([&] {
        copy_out(matmul_parallel(make_tensor(m, k, A), make_tensor(k, n, B), threads), C);
    });
}

// quant.cpp:6-28
int ref_quantize_q8(std::size_t rows, std::size_t cols, const float* B, std::int8_t* q,
                    float* scale) {
    return guarded([&] {
        const QTensor t = quantize_q8(make_tensor(rows, cols, B));
        if (!t.data.empty()) std::memcpy(q, t.data.data(), t.data.size());
        if (!t.scale.empty()) std::memcpy(scale, t.scale.data(), t.scale.size() * sizeof(float));
    });
}

// quant.cpp:30-36
int ref_dequantize(std::size_t rows, std::size_t cols, const std::int8_t* q, const float* scale,
                   float* out) {
    return guarded([&] {
        QTensor t;
        t.rows = rows;
        t.cols = cols;
        t.data.assign(q, q + rows * cols);
        t.scale.assign(scale, scale + cols);
        copy_out(dequantize(t), out);
    });
}

// ops.cpp:8-26
int ref_rmsnorm(std::size_t rows, std::size_t cols, const float* x, const float* w, float* y) {
    return guarded([&] {
        copy_out(rmsnorm(make_tensor(rows, cols, x), std::vector<float>(w, w + cols)), y);
    });
}

// A QTensor kept alive across calls, so timing matmul_parallel does not also
// time copying the weights into a std::vector.
void* ref_qtensor_new(std::size_t rows, std::size_t cols, const std::int8_t* q,
                      const float* scale) {
    auto* t = new QTensor;
    t->rows = rows;
    t->cols = cols;
    t->data.assign(q, q + rows * cols);
    t->scale.assign(scale, scale + cols);
    return t;
}

void ref_qtensor_free(void* h) { delete static_cast<QTensor*>(h); }

// The same for fp32 weights: a Tensor kept alive across calls of matmul_parallel.
void* ref_tensor_new(std::size_t rows, std::size_t cols, const float* B) {
    return new Tensor(make_tensor(rows, cols, B));
}

void ref_tensor_free(void* h) { delete static_cast<Tensor*>(h); }

// matmul.h:17-22 (fp32 weights, a handle from ref_tensor_new)
int ref_matmul_parallel_f32_h(void* h, std::size_t m, std::size_t k, const float* A, float* C,
                              unsigned threads) {
    return guarded([&] {
        const Tensor& B = *static_cast<const Tensor*>(h);
        copy_out(matmul_parallel(make_tensor(m, k, A), B, threads), C);
    });
}

// matmul.cpp:315-318, with B the QTensor made by ref_qtensor_new.
int ref_matmul_parallel_q8(void* h, std::size_t m, std::size_t k, const float* A, float* C,
                           unsigned threads) {
    return guarded([&] {
        const QTensor& B = *static_cast<const QTensor*>(h);
        copy_out(matmul_parallel(make_tensor(m, k, A), B, threads), C);
    });
}

}  // extern "C"
