// Shared device-side definitions of the linear-attention scan kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.hpp"

namespace subq {

// Everything a kernel needs about one call, by value in kernel parameters.
struct ScanParams {
    int B, H, N, d, e;
    int normalize;
    float scale, clamp_min;
    int decay_mode;
    float lg_scalar;
    const float* log_gamma;
    const uint8_t* mask;
    int64_t mask_sb;
    int flush;
    // tensors: [B,H,N,*] with element strides
    const void* q; int64_t q_sb, q_sh, q_sn;
    const void* k; int64_t k_sb, k_sh, k_sn;
    const void* v; int64_t v_sb, v_sh, v_sn;
    void* o;       int64_t o_sb, o_sh, o_sn;      // forward output / dq in the backward
    const void* g; int64_t g_sb, g_sh, g_sn;      // upstream gradient (backward)
    void* dk;      int64_t dk_sb, dk_sh, dk_sn;
    void* dv;      int64_t dv_sb, dv_sh, dv_sn;
    const float* S_in; const float* z_in;
    float* S_out; float* z_out;
    float* dlg;                                    // [B,H,N] or null
    float* ws;                                     // float workspace
    // [B*H] per-sequence flags: the tensor-core kernels with per-token decay set
    // fallback[b*H + h] when a chunk of the sequence leaves their decay range;
    // the exact kernels, given the array, then compute only the flagged
    // sequences (null: every sequence).
    int* fallback;
    // K/V group size (GQA): query head h reads K/V head h / kvg; 1 = one K/V
    // head per query head. dk, dv are then written per query head (the caller
    // sums each group).
    int kvg;
    // 1: reverse time (token t sees itself and the later tokens; the
    // backward direction of the bidirectional scan), tensor-core path only
    int reverse;
    // Segment-start states of the tensor-core scans: a 256-byte header (int 0:
    // the segment count G it was written with; 0 = not written) and then, per
    // sequence and segment, the fp32 state [S | z] (64 rows of 65). The
    // forward writes them (seg_out); the backward reads them (seg_in) when
    // their G is its own, in place of recomputing them.
    float* seg_out;
    const float* seg_in;
    // The forward's output o (backward only, with seg_in): the one-pass
    // backward forms the normaliser's adjoint from dO . o.
    const void* fo; int64_t fo_sb, fo_sh, fo_sn;
};

// phi(x) = ELU(x) + 1 and its derivative (reference python/subq_audio/autograd.py:15-28).
__device__ __forceinline__ float phi_f(float x) { return x > 0.f ? x + 1.f : expf(x); }
__device__ __forceinline__ float phi_prime_f(float x) { return x > 0.f ? 1.f : expf(x); }

__device__ __forceinline__ double phi_f(double x) { return x > 0.0 ? x + 1.0 : exp(x); }
__device__ __forceinline__ double phi_prime_f(double x) { return x > 0.0 ? 1.0 : exp(x); }
__device__ __forceinline__ float exp_a(float x) { return expf(x); }
__device__ __forceinline__ double exp_a(double x) { return exp(x); }

template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<double>(double x) { return (float)x; }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ double from_f<double>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Element conversions in the accumulate type A (float, or double for SUBQ_FP64).
template <typename A, typename T> __device__ __forceinline__ A load_a(T x) { return (A)to_f<T>(x); }
template <> __device__ __forceinline__ double load_a<double, double>(double x) { return x; }
template <typename T, typename A> __device__ __forceinline__ T store_a(A x) { return from_f<T>((float)x); }
template <> __device__ __forceinline__ double store_a<double, double>(double x) { return x; }

__device__ __forceinline__ float token_mask(const ScanParams& p, int b, int t) {
    return p.mask ? (p.mask[(int64_t)b * p.mask_sb + t] ? 1.f : 0.f) : 1.f;
}

// log(gamma_t) of a live token (masked tokens use 0 at the call sites).
__device__ __forceinline__ float token_log_gamma(const ScanParams& p, int b, int h, int t) {
    switch (p.decay_mode) {
        case SUBQ_DECAY_SCALAR: return p.lg_scalar;
        case SUBQ_DECAY_PER_HEAD: return p.log_gamma[h];
        case SUBQ_DECAY_PER_TOKEN: return p.log_gamma[((int64_t)b * p.H + h) * p.N + t];
        default: return 0.f;
    }
}

// Token in memory at processing position u (reverse time walks the sequence
// from its end; the recurrence itself is the same).
__device__ __forceinline__ int tok_at(const ScanParams& p, int u) { return p.reverse ? p.N - 1 - u : u; }

template <typename A>
__device__ __forceinline__ A flush_small(A s, int flush) {
    return (flush && fabs(s) < (A)1.17549435e-38f) ? (A)0 : s;
}

}  // namespace subq
