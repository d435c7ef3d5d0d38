// Device memory arena (see include/arena.hpp).
#include "arena.hpp"

#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

namespace {
void check(cudaError_t err, const char* what) {
    if (err != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(err));
}
}  // namespace

MemoryArena::MemoryArena(size_t max_size_bytes) : base_ptr_(nullptr), offset_(0), capacity_(max_size_bytes) {
    void* ptr = nullptr;
    if (capacity_ > 0) {
        check(cudaMalloc(&ptr, capacity_), "cudaMalloc (MemoryArena)");
        cudaError_t err = cudaMemset(ptr, 0, capacity_);
        if (err != cudaSuccess) {
            cudaFree(ptr);
            check(err, "cudaMemset (MemoryArena)");
        }
    }
    base_ptr_ = static_cast<uint8_t*>(ptr);
}

MemoryArena::~MemoryArena() {
    if (base_ptr_) cudaFree(base_ptr_);  // errors ignored: destructors must not throw
    base_ptr_ = nullptr;
}

uint8_t* MemoryArena::allocate(size_t bytes) {
    if (bytes == 0) return base_ptr_ + offset_;
    if (bytes > capacity_) throw std::runtime_error("OOM: Requested allocation exceeds arena capacity.");
    constexpr size_t kAlign = 256;
    if (bytes > SIZE_MAX - (kAlign - 1))
        throw std::runtime_error("OOM: Integer overflow computing aligned allocation size.");
    const size_t aligned = (bytes + kAlign - 1) & ~(kAlign - 1);
    if (capacity_ < aligned || offset_ > capacity_ - aligned)
        throw std::runtime_error("OOM: MemoryArena capacity exceeded during allocation.");
    uint8_t* ptr = base_ptr_ + offset_;
    offset_ += aligned;
    return ptr;
}

void MemoryArena::reset_head() { offset_ = 0; }

void MemoryArena::zero_all() {
    if (capacity_) check(cudaMemset(base_ptr_, 0, capacity_), "cudaMemset (MemoryArena)");
}

size_t MemoryArena::get_offset() const { return offset_; }

void MemoryArena::set_offset(size_t saved_offset) {
    if (saved_offset > capacity_) throw std::runtime_error("OOM: Invalid offset restoration.");
    offset_ = saved_offset;
}

size_t MemoryArena::get_used_bytes() const { return offset_; }

size_t MemoryArena::get_total_bytes() const { return capacity_; }
