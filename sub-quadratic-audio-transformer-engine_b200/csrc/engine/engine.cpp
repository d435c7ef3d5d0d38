// C++ engine over the C ABI (see include/engine.hpp).
#include "engine.hpp"

#include <cuda_runtime.h>

#include <cmath>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

void throw_status(int rc) {
    const std::string msg = subq_last_error();
    if (rc == SUBQ_ERR_ALIAS || rc == SUBQ_ERR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}

void check_cuda(cudaError_t err, const char* what) {
    if (err != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(err));
}

int dtype_of(PrecisionMode p) {
    switch (p) {
        case PrecisionMode::FP16: return SUBQ_FP16;
        case PrecisionMode::BF16: return SUBQ_BF16;
        default: return SUBQ_FP32;
    }
}

subq_tensor4 contiguous3(void* data, size_t n, size_t d) {
    subq_tensor4 t;
    t.data = data;
    t.stride_b = (int64_t)(n * d);
    t.stride_h = 0;
    t.stride_n = (int64_t)d;
    return t;
}

// Restores the arena head on scope exit (workspace is call-scoped).
struct ArenaMark {
    MemoryArena& a;
    size_t off;
    explicit ArenaMark(MemoryArena& arena) : a(arena), off(arena.get_offset()) {}
    ~ArenaMark() { a.set_offset(off); }
};

}  // namespace

Engine::Engine(MemoryArena& arena) : arena_(arena) {}

void Engine::check_device(void* stream) {
    int st = SUBQ_OK;
    const int rc = subq_device_status(stream, &st);
    if (rc != SUBQ_OK) throw_status(rc);
    if (st == SUBQ_ERR_TIMEOUT)
        throw std::runtime_error("a bounded device-side wait of a tensor-core kernel gave up (SUBQ_ERR_TIMEOUT); "
                                 "the outputs since the last check are not valid");
    if (st != SUBQ_OK)
        throw std::runtime_error("device status " + std::to_string(st) +
                                 ": a backward was given the forward state of another call; its gradients are "
                                 "not valid");
}

void Engine::forward(AttentionContext& ctx, void* stream) {
    if (ctx.Q.dimensions.size() != 3) throw std::invalid_argument("Q must be [batch, seq_len, d_model]");
    const size_t B = ctx.Q.dimensions[0], N = ctx.Q.dimensions[1], D = ctx.Q.dimensions[2];
    if (!(ctx.decay_factor >= 0.f)) throw std::invalid_argument("decay_factor must be a number >= 0");
    subq_fwd_args a{};
    a.desc.batch = (int64_t)B;
    a.desc.heads = 1;
    a.desc.seq_len = (int64_t)N;
    a.desc.head_dim = (int64_t)D;
    a.desc.value_dim = (int64_t)D;
    a.desc.dtype = dtype_of(ctx.Q.precision);
    a.desc.normalize = 0;
    a.desc.scale = 1.f;
    a.desc.clamp_min = 1e-5f;
    a.desc.decay_mode = ctx.decay_factor == 1.f ? SUBQ_DECAY_NONE : SUBQ_DECAY_SCALAR;
    a.desc.log_gamma_scalar = std::log(ctx.decay_factor);
    a.desc.flush_subnormal = 1;
    a.desc.path = SUBQ_PATH_AUTO;
    a.q = contiguous3(ctx.Q.data, N, D);
    a.k = contiguous3(ctx.K.data, N, D);
    a.v = contiguous3(ctx.V.data, N, D);
    a.o = contiguous3(ctx.O.data, N, D);
    a.state_in = static_cast<const float*>(ctx.S.data);
    a.state_out = static_cast<float*>(ctx.S.data);
    a.stream = stream;
    forward(a);
}

void Engine::forward(subq_fwd_args a) {
    ArenaMark mark(arena_);
    size_t need = subq_fwd_workspace_bytes(&a);
    // The automatic path's chunked kernels need a workspace of about 0.8 KB
    // per token at head_dim 64 (34 KB at 256); when the arena cannot hold it,
    // the call runs on the exact path, which needs none.
    const size_t room = arena_.get_total_bytes() - arena_.get_offset();
    if (a.desc.path == SUBQ_PATH_AUTO && need + 256 > room) {
        a.desc.path = SUBQ_PATH_EXACT;
        need = subq_fwd_workspace_bytes(&a);
    }
    if (need) {
        a.workspace = arena_.allocate(need);
        a.workspace_bytes = need;
    }
    const int rc = subq_fwd(&a);
    if (rc != SUBQ_OK) throw_status(rc);
}

void Engine::backward(subq_bwd_args a) {
    ArenaMark mark(arena_);
    const size_t need = subq_bwd_workspace_bytes(&a);
    if (need) {
        a.workspace = arena_.allocate(need);
        a.workspace_bytes = need;
    }
    const int rc = subq_bwd(&a);
    if (rc != SUBQ_OK) throw_status(rc);
}

float Engine::backward_engine(const void* dO, const void* Q, const void* K, const void* V, void* dQ,
                              void* dK, void* dV, size_t B, size_t N, size_t D, float decay_factor,
                              const float* S0, void* stream) {
    // The reference converts gamma to the logit w and back (python/bindings.cpp:289-292,
    // src/kernels/attention_backward.cpp:58-59); the same rounding is kept.
    const float g_c = std::fmax(std::fmin(decay_factor, 1.0f - 1e-6f), 1e-6f);
    const float w = std::log(g_c / (1.0f - g_c));
    const float gamma = 1.0f / (1.0f + std::exp(-w));
    ArenaMark mark(arena_);
    float* dlg = reinterpret_cast<float*>(arena_.allocate(sizeof(float) * B * N));
    subq_bwd_args a{};
    a.desc.batch = (int64_t)B;
    a.desc.heads = 1;
    a.desc.seq_len = (int64_t)N;
    a.desc.head_dim = (int64_t)D;
    a.desc.value_dim = (int64_t)D;
    a.desc.dtype = SUBQ_FP32;
    a.desc.normalize = 0;
    a.desc.scale = 1.f;
    a.desc.clamp_min = 1e-5f;
    a.desc.decay_mode = SUBQ_DECAY_SCALAR;
    a.desc.log_gamma_scalar = std::log(gamma);
    a.desc.flush_subnormal = 1;
    a.q = contiguous3(const_cast<void*>(Q), N, D);
    a.k = contiguous3(const_cast<void*>(K), N, D);
    a.v = contiguous3(const_cast<void*>(V), N, D);
    a.dout = contiguous3(const_cast<void*>(dO), N, D);
    a.dq = contiguous3(dQ, N, D);
    a.dk = contiguous3(dK, N, D);
    a.dv = contiguous3(dV, N, D);
    a.state_in = S0;
    a.dlog_gamma = dlg;
    a.stream = stream;
    backward(a);
    std::vector<float> host(B * N);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (!host.empty()) {
        check_cuda(cudaMemcpyAsync(host.data(), dlg, sizeof(float) * host.size(), cudaMemcpyDeviceToHost, st),
                   "cudaMemcpyAsync (d_gamma)");
    }
    check_device(stream);  // synchronises the stream
    double acc = 0.0;
    for (float x : host) acc += x;
    return (float)(acc / gamma);
}
