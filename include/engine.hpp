// C++ engine over the C ABI (reference include/engine.hpp:13-22,
// src/engine.cpp:10-26). Device-resident: the arena holds the carried
// float32 state and every scratch buffer; no call allocates device memory.
// Errors surface as std::runtime_error / std::invalid_argument with the
// reference's messages.
#pragma once

#include <cstddef>

#include "arena.hpp"
#include "attention.hpp"
#include "kernels.hpp"

class Engine {
public:
    explicit Engine(MemoryArena& arena);

    // Unnormalised engine scan S = gamma S + phi(k) v^T, O = phi(q) S on
    // device pointers; ctx.S is the carried state (updated in place).
    void forward(AttentionContext& ctx, void* stream = nullptr);

    // Full-control forward/backward over the C ABI; the workspace is taken
    // from the arena above its current head and released on return.
    void forward(subq_fwd_args args);
    void backward(subq_bwd_args args);

    // d loss / d gamma of the unnormalised engine scan (reference
    // SubQEngine.backward_raw): gradients into dQ/dK/dV (device, caller-owned).
    float backward_engine(const void* dO, const void* Q, const void* K, const void* V, void* dQ,
                          void* dK, void* dV, size_t batch, size_t seq_len, size_t d_model,
                          float decay_factor, const float* S0, void* stream);

    // Synchronises `stream` and raises std::runtime_error when the device
    // status word records that a bounded device-side wait gave up
    // (SUBQ_ERR_TIMEOUT) or that a backward was handed another call's forward
    // state (SUBQ_ERR_STATE) since the last check: the outputs of the calls in
    // between are not valid. The status word is read and cleared.
    void check_device(void* stream = nullptr);

    MemoryArena& arena() { return arena_; }

private:
    MemoryArena& arena_;
};
