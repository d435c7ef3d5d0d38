// Safetensors weight loader into the device arena (reference
// include/safetensors.hpp:17-49, src/safetensors.cpp). Kept for API parity
// of SubQEngine.load and its error behaviour; the scan never reads weights.
#pragma once

#include <string>
#include <unordered_map>
#include <vector>

#include "arena.hpp"
#include "tensor.hpp"

struct SafetensorMetadata {
    std::string dtype;
    std::vector<size_t> shape;
    size_t data_offset_start;
    size_t data_offset_end;
};

class SafetensorLoader {
public:
    explicit SafetensorLoader(MemoryArena& arena) : arena_(arena) {}
    // False on any malformed file (header length, JSON, offsets, sizes).
    bool load(const std::string& filepath);
    bool has_tensor(const std::string& name) const { return tensors_.count(name) != 0; }
    TensorDescriptor get_tensor(const std::string& name) const;
    const std::unordered_map<std::string, SafetensorMetadata>& metadata() const { return meta_; }

private:
    MemoryArena& arena_;
    std::unordered_map<std::string, SafetensorMetadata> meta_;
    std::unordered_map<std::string, TensorDescriptor> tensors_;
};
