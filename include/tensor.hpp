// Tensor description shared by the engine and its callers. Same fields and
// enum order as the reference's include/tensor.hpp:14-26 (the engine API is
// a drop-in), backed here by device memory only.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

enum class PrecisionMode { FP32 = 0, FP16 = 1, BF16 = 2 };

struct TensorDescriptor {
    std::vector<size_t> dimensions;  // e.g. {batch, seq_len, d_model}
    std::vector<size_t> strides;     // element strides; empty = row-major contiguous
    PrecisionMode precision;
    void* data;                      // device pointer (arena or caller-owned)
    bool is_on_host;                 // true if `data` is host memory (staged by the caller)
};
