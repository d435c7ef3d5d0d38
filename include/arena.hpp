// Device memory arena: one cudaMalloc at construction, 256-byte aligned bump
// allocation, checkpoint/rewind. Interface and error text follow the
// reference's include/arena.hpp:20-75 and src/arena.cpp:10-83 so callers and
// tests see the same behaviour ("OOM: ..." std::runtime_error).
#pragma once

#include <cstddef>
#include <cstdint>

class MemoryArena {
public:
    explicit MemoryArena(size_t max_size_bytes);
    ~MemoryArena();

    MemoryArena(const MemoryArena&) = delete;
    MemoryArena& operator=(const MemoryArena&) = delete;
    MemoryArena(MemoryArena&&) = delete;
    MemoryArena& operator=(MemoryArena&&) = delete;

    // 256-byte aligned block; throws std::runtime_error("OOM: ...") when full.
    uint8_t* allocate(size_t bytes);
    void reset_head();
    void zero_all();
    size_t get_offset() const;
    void set_offset(size_t saved_offset);
    size_t get_used_bytes() const;
    size_t get_total_bytes() const;
    uint8_t* base() const { return base_ptr_; }

private:
    uint8_t* base_ptr_;
    size_t offset_;
    size_t capacity_;
};
