// Engine-level attention context (reference include/attention.hpp:14-33).
// The reference's free functions run_attention_forward / run_attention_backward
// are replaced by Engine::forward / Engine::backward over the C ABI in
// kernels.hpp; the context keeps its fields so CLI-style callers that carry
// ctx.S across frames (reference src/main.cpp:264-315) keep working.
#pragma once

#include "tensor.hpp"

struct AttentionContext {
    TensorDescriptor Q;  // [B, N, D] query (device)
    TensorDescriptor K;  // [B, N, D] key (device)
    TensorDescriptor V;  // [B, N, D] value (device)
    TensorDescriptor O;  // [B, N, D] output (device)
    TensorDescriptor S;  // [B, D, D] float32 recurrent state, read and updated in place
    float decay_factor = 0.99f;
};
