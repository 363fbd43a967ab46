#pragma once
// Host matrix types with the same layout as the reference engine's
// src/tensor.h:8-28, for builds of the C++ shim that do not have the
// reference's own header on the include path. A caller that already has the
// reference's tensor.h uses that one instead (put it earlier on the path);
// the layouts are identical, so objects cross the library boundary unchanged.
#include <cstddef>
#include <cstdint>
#include <vector>

// Dense row-major fp32 matrix: element (r, c) at data[r * cols + c].
struct Tensor {
    std::size_t rows;
    std::size_t cols;
    std::vector<float> data;

    Tensor() : rows(0), cols(0) {}
    Tensor(std::size_t r, std::size_t c) : rows(r), cols(c), data(r * c, 0.0f) {}

    float& at(std::size_t r, std::size_t c) { return data[r * cols + c]; }
    float at(std::size_t r, std::size_t c) const { return data[r * cols + c]; }
};

// int8 matrix with one fp32 scale per column: (r, c) stands for
// data[r * cols + c] * scale[c]. Weights are (in x out), a column is one
// output channel.
struct QTensor {
    std::size_t rows = 0;
    std::size_t cols = 0;
    std::vector<std::int8_t> data;
    std::vector<float> scale;  // cols
};
