#pragma once
// Drop-in replacement for the reference engine's src/cuda_matmul.h
// (cuda_matmul.h:1-122): the same classes, enum, struct and overloads, with
// the same meaning, so a caller rebuilt against this header and linked to
// libllme_b200_cxx.so + libllme_b200.so runs on the B200 kernels unchanged.
//
// Implemented in llm-engine_b200/csrc/cuda_matmul.cpp on top of the C ABI in
// llme_b200.h. Behaviour kept from the reference:
//  - every call is asynchronous on the calling thread's per-thread default
//    stream, except download() and the Tensor overloads of matmul_cuda(),
//    which wait; not safe from several host threads at once;
//  - std::invalid_argument for mismatched shapes (the message names both
//    shapes, "AxB"), for skinny with m > 8 and for matrices of 2^31 or more
//    elements; std::runtime_error("cuda: <what>: <message>") for CUDA errors;
//  - m == 0 or n == 0 does nothing, k == 0 zeroes C unless accumulating;
//  - results are bit-identical across repeats (no float atomics anywhere).
//
// Tensor and QTensor come from the reference's tensor.h; where that header is
// not on the include path, include/tensor/tensor.h provides the same layout.
#include <cstddef>
#include <cstdint>

#include "tensor.h"

// Row-major fp32 matrix in GPU memory. Move-only; frees its memory on
// destruction.
class DeviceTensor {
public:
    DeviceTensor() = default;
    DeviceTensor(std::size_t rows, std::size_t cols);  // contents undefined
    explicit DeviceTensor(const Tensor& t);            // copies t to the GPU
    ~DeviceTensor();

    DeviceTensor(DeviceTensor&& other) noexcept;
    DeviceTensor& operator=(DeviceTensor&& other) noexcept;
    DeviceTensor(const DeviceTensor&) = delete;
    DeviceTensor& operator=(const DeviceTensor&) = delete;

    // Copies t into this tensor, reallocating if the shape differs.
    void upload(const Tensor& t);
    Tensor download() const;

    std::size_t rows() const { return rows_; }
    std::size_t cols() const { return cols_; }
    float* data() { return data_; }
    const float* data() const { return data_; }

private:
    std::size_t rows_ = 0, cols_ = 0;
    float* data_ = nullptr;
};

// int8 matrix with one fp32 scale per column in GPU memory (QTensor's
// layout). Move-only; frees its memory on destruction.
class DeviceQTensor {
public:
    DeviceQTensor() = default;
    explicit DeviceQTensor(const QTensor& t);  // copies t to the GPU
    ~DeviceQTensor();

    DeviceQTensor(DeviceQTensor&& other) noexcept;
    DeviceQTensor& operator=(DeviceQTensor&& other) noexcept;
    DeviceQTensor(const DeviceQTensor&) = delete;
    DeviceQTensor& operator=(const DeviceQTensor&) = delete;

    std::size_t rows() const { return rows_; }
    std::size_t cols() const { return cols_; }
    const std::int8_t* data() const { return data_; }
    const float* scale() const { return scale_; }

private:
    std::size_t rows_ = 0, cols_ = 0;
    std::int8_t* data_ = nullptr;
    float* scale_ = nullptr;  // cols
};

// The kernel names of the reference. On the B200 build:
enum class GpuKernel {
    automatic,    // skinny for m <= 8, tiled_split up to m = 127, the tcgen05 GEMM beyond
    naive,        // one thread per element of C, the reference's summation order
    tiled,        // whole-k tiles; the tcgen05 GEMM where the shape allows it
    tiled_split,  // fp32 tiles with k split across CTAs, reduced in a fixed order
    skinny,       // m <= 8 only: the TMA-fed weight-streaming GEMV
};

// C = A x B; C is reallocated if it isn't m x n.
void matmul_cuda(const DeviceTensor& A, const DeviceTensor& B, DeviceTensor& C,
                 GpuKernel kernel = GpuKernel::automatic);

// Neighbouring ops folded into a product.
struct MatmulFusion {
    // C += A x B instead of C = A x B: a residual add.
    bool accumulate = false;
    // Multiply rmsnorm(A) instead of A: each row of A scaled by
    // 1 / sqrt(mean(row^2) + 1e-5) and by these k weights (device memory).
    const float* rms_weight = nullptr;
};

// Raw device pointers: A is m x k, B k x n, C m x n, dense and row-major.
void matmul_cuda(std::size_t m, std::size_t n, std::size_t k, const float* A, const float* B,
                 float* C, GpuKernel kernel = GpuKernel::automatic,
                 const MatmulFusion& fusion = {});

// int8 B: C = A x dequantize(B), B k x n int8 with n column scales.
void matmul_cuda(std::size_t m, std::size_t n, std::size_t k, const float* A,
                 const std::int8_t* B, const float* scale, float* C,
                 GpuKernel kernel = GpuKernel::automatic, const MatmulFusion& fusion = {});

// Bumped whenever matmul_cuda() reallocates internal scratch; a CUDA graph
// captured before the bump must be captured again.
std::size_t cuda_scratch_generation();

// Copy A and B to the GPU, multiply, copy C back (these wait).
Tensor matmul_cuda(const Tensor& A, const Tensor& B, GpuKernel kernel = GpuKernel::automatic);
Tensor matmul_cuda(const Tensor& A, const QTensor& B, GpuKernel kernel = GpuKernel::automatic);

// Waits for all queued GPU work; throws std::runtime_error if any failed.
void cuda_synchronize();

// False if there is no usable CUDA device.
bool cuda_available();
