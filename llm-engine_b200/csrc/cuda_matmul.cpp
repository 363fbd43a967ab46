// The drop-in C++ API (include/cuda_matmul.h) on top of the C ABI
// (include/llme_b200.h). Host code only: no CUDA headers, every device
// operation goes through an llme_* call, and a nonzero status becomes the
// exception the reference throws (src/cuda_matmul.cu:399-574):
// LLME_E_INVALID -> std::invalid_argument, anything else ->
// std::runtime_error with the library's "cuda: <what>: <message>" text.
#include "cuda_matmul.h"

#include <stdexcept>
#include <string>
#include <utility>

#include "llme_b200.h"

namespace {

void check(int status) {
    if (status == LLME_OK) return;
    const std::string msg = llme_last_error();
    if (status == LLME_E_INVALID) throw std::invalid_argument(msg);
    throw std::runtime_error(msg.empty() ? "cuda: error " + std::to_string(status) : msg);
}

std::string shape_str(std::size_t rows, std::size_t cols) {
    return std::to_string(rows) + "x" + std::to_string(cols);
}

int kernel_id(GpuKernel k) {
    switch (k) {
        case GpuKernel::automatic: return LLME_KERNEL_AUTOMATIC;
        case GpuKernel::naive: return LLME_KERNEL_NAIVE;
        case GpuKernel::tiled: return LLME_KERNEL_TILED;
        case GpuKernel::tiled_split: return LLME_KERNEL_TILED_SPLIT;
        case GpuKernel::skinny: return LLME_KERNEL_SKINNY;
    }
    return -1;
}

void inner_mismatch(std::size_t ar, std::size_t ac, std::size_t br, std::size_t bc) {
    throw std::invalid_argument("matmul_cuda: inner dimensions differ (A is " + shape_str(ar, ac) +
                                ", B is " + shape_str(br, bc) + ")");
}

}  // namespace

DeviceTensor::DeviceTensor(std::size_t rows, std::size_t cols) : rows_(rows), cols_(cols) {
    void* p = nullptr;
    check(llme_alloc(&p, rows * cols * sizeof(float)));
    data_ = static_cast<float*>(p);
}

DeviceTensor::DeviceTensor(const Tensor& t) : DeviceTensor(t.rows, t.cols) { upload(t); }

DeviceTensor::~DeviceTensor() { llme_free(data_); }

DeviceTensor::DeviceTensor(DeviceTensor&& other) noexcept
    : rows_(std::exchange(other.rows_, 0)),
      cols_(std::exchange(other.cols_, 0)),
      data_(std::exchange(other.data_, nullptr)) {}

DeviceTensor& DeviceTensor::operator=(DeviceTensor&& other) noexcept {
    std::swap(rows_, other.rows_);
    std::swap(cols_, other.cols_);
    std::swap(data_, other.data_);
    return *this;
}

void DeviceTensor::upload(const Tensor& t) {
    if (t.rows != rows_ || t.cols != cols_) *this = DeviceTensor(t.rows, t.cols);
    if (!t.data.empty()) check(llme_copy_to_device(data_, t.data.data(), t.data.size() * sizeof(float)));
}

Tensor DeviceTensor::download() const {
    Tensor t(rows_, cols_);
    if (!t.data.empty()) check(llme_copy_to_host(t.data.data(), data_, t.data.size() * sizeof(float)));
    return t;
}

DeviceQTensor::DeviceQTensor(const QTensor& t) : rows_(t.rows), cols_(t.cols) {
    if (t.data.size() != rows_ * cols_ || t.scale.size() != cols_)
        throw std::invalid_argument("DeviceQTensor: data or scale size doesn't match the shape");
    try {
        void* p = nullptr;
        check(llme_alloc(&p, t.data.size()));
        data_ = static_cast<std::int8_t*>(p);
        check(llme_copy_to_device(data_, t.data.data(), t.data.size()));
        p = nullptr;
        check(llme_alloc(&p, t.scale.size() * sizeof(float)));
        scale_ = static_cast<float*>(p);
        check(llme_copy_to_device(scale_, t.scale.data(), t.scale.size() * sizeof(float)));
    } catch (...) {
        llme_free(data_);
        llme_free(scale_);
        throw;
    }
}

DeviceQTensor::~DeviceQTensor() {
    llme_free(data_);
    llme_free(scale_);
}

DeviceQTensor::DeviceQTensor(DeviceQTensor&& other) noexcept
    : rows_(std::exchange(other.rows_, 0)),
      cols_(std::exchange(other.cols_, 0)),
      data_(std::exchange(other.data_, nullptr)),
      scale_(std::exchange(other.scale_, nullptr)) {}

DeviceQTensor& DeviceQTensor::operator=(DeviceQTensor&& other) noexcept {
    std::swap(rows_, other.rows_);
    std::swap(cols_, other.cols_);
    std::swap(data_, other.data_);
    std::swap(scale_, other.scale_);
    return *this;
}

void matmul_cuda(const DeviceTensor& A, const DeviceTensor& B, DeviceTensor& C, GpuKernel kernel) {
    if (A.cols() != B.rows()) inner_mismatch(A.rows(), A.cols(), B.rows(), B.cols());
    if (C.rows() != A.rows() || C.cols() != B.cols()) C = DeviceTensor(A.rows(), B.cols());
    matmul_cuda(A.rows(), B.cols(), A.cols(), A.data(), B.data(), C.data(), kernel);
}

void matmul_cuda(std::size_t m, std::size_t n, std::size_t k, const float* A, const float* B,
                 float* C, GpuKernel kernel, const MatmulFusion& fusion) {
    check(llme_matmul_f32(m, n, k, A, B, C, kernel_id(kernel), fusion.accumulate ? 1 : 0,
                          fusion.rms_weight, 0, nullptr));
}

void matmul_cuda(std::size_t m, std::size_t n, std::size_t k, const float* A,
                 const std::int8_t* B, const float* scale, float* C, GpuKernel kernel,
                 const MatmulFusion& fusion) {
    check(llme_matmul_q8(m, n, k, A, B, scale, C, kernel_id(kernel), fusion.accumulate ? 1 : 0,
                         fusion.rms_weight, 0, nullptr));
}

std::size_t cuda_scratch_generation() { return llme_scratch_generation(); }

Tensor matmul_cuda(const Tensor& A, const Tensor& B, GpuKernel kernel) {
    const DeviceTensor dA(A), dB(B);
    DeviceTensor dC;
    matmul_cuda(dA, dB, dC, kernel);
    return dC.download();
}

Tensor matmul_cuda(const Tensor& A, const QTensor& B, GpuKernel kernel) {
    if (A.cols != B.rows) inner_mismatch(A.rows, A.cols, B.rows, B.cols);
    const DeviceTensor dA(A);
    const DeviceQTensor dB(B);
    DeviceTensor dC(A.rows, B.cols);
    matmul_cuda(A.rows, B.cols, A.cols, dA.data(), dB.data(), dB.scale(), dC.data(), kernel);
    return dC.download();
}

void cuda_synchronize() { check(llme_synchronize()); }

bool cuda_available() { return llme_device_available() != 0; }

// ---- include/cuda_attention.h over llme_attention* -------------------------------------------

#include "cuda_attention.h"

namespace {

llme_attention_shape c_shape(const AttentionShape& s) {
    llme_attention_shape c;
    c.n_heads = s.n_heads;
    c.n_kv_heads = s.n_kv_heads;
    c.head_size = s.head_size;
    c.seq_len = s.seq_len;
    c.q_stride = s.q_stride;
    c.kv_stride = s.kv_stride;
    c.out_stride = s.out_stride;
    return c;
}

int attention_kernel_id(AttentionKernel k) {
    switch (k) {
        case AttentionKernel::automatic: return LLME_ATTN_AUTOMATIC;
        case AttentionKernel::single_block: return LLME_ATTN_SINGLE_BLOCK;
        case AttentionKernel::split: return LLME_ATTN_SPLIT;
    }
    return -1;
}

}  // namespace

std::size_t attention_scratch_floats(const AttentionShape& s, std::size_t rows,
                                     AttentionKernel kernel) {
    const llme_attention_shape c = c_shape(s);
    return llme_attention_scratch_floats(&c, rows, attention_kernel_id(kernel));
}

void attention_check(const AttentionShape& s, AttentionKernel kernel) {
    const llme_attention_shape c = c_shape(s);
    check(llme_attention_check(&c, attention_kernel_id(kernel)));
}

void attention_cuda(const AttentionShape& s, std::size_t rows, const int* pos_dev, const float* q,
                    const float* key_cache, const float* value_cache, float* out, float* scratch,
                    AttentionKernel kernel) {
    const llme_attention_shape c = c_shape(s);
    check(llme_attention(&c, rows, pos_dev, q, key_cache, value_cache, out, scratch,
                         attention_kernel_id(kernel), nullptr));
}
