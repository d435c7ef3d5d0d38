// Per-head RMSNorm of the scan's output, forward and backward: the epilogue
// of the reference's SubQLinearAttention (python/subq_audio/autograd.py:706-710
// builds nn.RMSNorm(head_dim, eps=1e-5); :763-767 applies it, then :769
// transposes [B, H, L, D] to [B, L, H*D] with a copy):
//   y = x * rsqrt(mean_D(x^2) + eps) * w
// Each row is one (token, head) of D values. The forward writes y through
// strides, so the [B, L, H*D] layout the output projection wants comes out
// directly (no transpose copy). The backward recomputes rsqrt from x:
//   xh = x r,  g = dy w,  dx = r (g - xh mean_D(g xh)),  dw = sum_rows dy xh
// with dw reduced per CTA into the workspace and then over the CTAs in a
// fixed order (bitwise reproducible). HBM-bound: the forward moves 2 D
// elements per row, the backward 3. Rows are walked in (b, n, h) order, the
// memory order of a scan output written in the projections' [B, L, H, D]
// order, so consecutive rows are consecutive memory.
//
// Thread mapping: D / 8 threads per row, 8 elements (16 bytes for 16-bit
// types) per thread; the row sums are butterfly shuffles inside those lanes.
// D is 8, 16, 32, 64, 128 or 256; rows are 16-byte aligned (host checks).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.hpp"
#include "scan_launch.h"

namespace subq {
namespace {

constexpr int kThreads = 256;

template <typename T> struct Vec8;
template <> struct Vec8<float> {
    __device__ static void load(const float* p, float* f) {
        const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    }
    __device__ static void store(float* p, const float* f) {
        reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
        reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
    }
};
template <> struct Vec8<__nv_bfloat16> {
    __device__ static void load(const __nv_bfloat16* p, float* f) {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 v = __bfloat1622float2(h[i]);
            f[2 * i] = v.x;
            f[2 * i + 1] = v.y;
        }
    }
    __device__ static void store(__nv_bfloat16* p, const float* f) {
        uint4 u;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
        *reinterpret_cast<uint4*>(p) = u;
    }
};
template <> struct Vec8<__half> {
    __device__ static void load(const __half* p, float* f) {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 v = __half22float2(h[i]);
            f[2 * i] = v.x;
            f[2 * i + 1] = v.y;
        }
    }
    __device__ static void store(__half* p, const float* f) {
        uint4 u;
        __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
        *reinterpret_cast<uint4*>(p) = u;
    }
};

// Sum over the TPR lanes of a row (TPR consecutive lanes, a power of two <= 32).
template <int TPR>
__device__ __forceinline__ float row_sum(float v) {
#pragma unroll
    for (int o = TPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Row r of the (b, n, h) walk -> element offset under strides (sb, sh, sn);
// r * D for a tensor dense in that order (bit `t` of p.dense).
__device__ __forceinline__ int64_t row_off(const RmsParams& p, int64_t r, int64_t sb, int64_t sh, int64_t sn,
                                           int t) {
    if (p.dense & (1 << t)) return r * p.D;
    const int h = (int)(r % p.H);
    const int64_t bn = r / p.H;
    const int n = (int)(bn % p.N);
    const int b = (int)(bn / p.N);
    return b * sb + h * sh + n * sn;
}

template <typename T, int TPR>
__global__ void __launch_bounds__(kThreads) rms_fwd_kernel(RmsParams p) {
    constexpr int D = TPR * 8, RPB = kThreads / TPR;  // rows per block step
    const int li = threadIdx.x % TPR;
    float w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = p.w ? p.w[li * 8 + i] : 1.f;
    const int64_t rows = (int64_t)p.B * p.N * p.H;
    const T* x = static_cast<const T*>(p.x);
    T* y = static_cast<T*>(p.y);
    // the loop bound is the same for the whole warp (its rows are consecutive)
    for (int64_t r0 = (int64_t)blockIdx.x * RPB + (threadIdx.x & ~31) / TPR; r0 < rows;
         r0 += (int64_t)gridDim.x * RPB) {
        const int64_t r = r0 + (threadIdx.x & 31) / TPR;
        const bool live = r < rows;
        float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (live) Vec8<T>::load(x + row_off(p, r, p.x_sb, p.x_sh, p.x_sn, 0) + li * 8, f);
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) ss = fmaf(f[i], f[i], ss);
        ss = row_sum<TPR>(ss);
        const float rs = rsqrtf(ss * (1.f / D) + p.eps);
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = f[i] * rs * w[i];
        if (live) Vec8<T>::store(y + row_off(p, r, p.y_sb, p.y_sh, p.y_sn, 1) + li * 8, f);
    }
}

// Backward; each CTA leaves its dw partial sums in part[blockIdx.x][D].
template <typename T, int TPR>
__global__ void __launch_bounds__(kThreads) rms_bwd_kernel(RmsParams p) {
    constexpr int D = TPR * 8, RPB = kThreads / TPR;
    const int li = threadIdx.x % TPR;
    float w[8], dw[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        w[i] = p.w ? p.w[li * 8 + i] : 1.f;
        dw[i] = 0.f;
    }
    const int64_t rows = (int64_t)p.B * p.N * p.H;
    const T* x = static_cast<const T*>(p.x);
    const T* dy = static_cast<const T*>(p.dy);
    T* dx = static_cast<T*>(p.dx);
    for (int64_t r0 = (int64_t)blockIdx.x * RPB + (threadIdx.x & ~31) / TPR; r0 < rows;
         r0 += (int64_t)gridDim.x * RPB) {
        const int64_t r = r0 + (threadIdx.x & 31) / TPR;
        const bool live = r < rows;
        float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        float g[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (live) {
            Vec8<T>::load(x + row_off(p, r, p.x_sb, p.x_sh, p.x_sn, 0) + li * 8, f);
            Vec8<T>::load(dy + row_off(p, r, p.dy_sb, p.dy_sh, p.dy_sn, 2) + li * 8, g);
        }
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) ss = fmaf(f[i], f[i], ss);
        ss = row_sum<TPR>(ss);
        const float rs = rsqrtf(ss * (1.f / D) + p.eps);
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float xh = f[i] * rs;
            dw[i] = fmaf(g[i], xh, dw[i]);
            f[i] = xh;
            g[i] *= w[i];
            dot = fmaf(g[i], xh, dot);
        }
        dot = row_sum<TPR>(dot) * (1.f / D);
#pragma unroll
        for (int i = 0; i < 8; ++i) g[i] = rs * (g[i] - f[i] * dot);
        if (live) Vec8<T>::store(dx + row_off(p, r, p.dx_sb, p.dx_sh, p.dx_sn, 3) + li * 8, g);
    }
    // dw over the CTA: thread group li of each row slot, summed in slot order
    __shared__ float red[kThreads * 8];
#pragma unroll
    for (int i = 0; i < 8; ++i) red[threadIdx.x * 8 + i] = dw[i];
    __syncthreads();
    if (p.part && threadIdx.x < D) {
        const int c = threadIdx.x, g0 = c / 8, e0 = c % 8;
        float s = 0.f;
        for (int k = 0; k < RPB; ++k) s += red[(k * TPR + g0) * 8 + e0];
        p.part[(int64_t)blockIdx.x * D + c] = s;
    }
}

// dw[c] = sum over the nb CTA partials, in CTA order: 1024 threads, 1024 / D
// strided partial sums per column, then those in order.
__global__ void __launch_bounds__(1024) rms_dw_kernel(const float* part, int nb, int D, float* dw) {
    __shared__ float red[1024];
    const int c = threadIdx.x % D, k = threadIdx.x / D, K = blockDim.x / D;
    float s = 0.f;
#pragma unroll 8
    for (int b = k; b < nb; b += K) s += part[(int64_t)b * D + c];
    red[threadIdx.x] = s;
    __syncthreads();
    if (threadIdx.x < D) {
        float t = 0.f;
        for (int j = 0; j < K; ++j) t += red[j * D + c];
        dw[c] = t;
    }
}

template <typename T>
cudaError_t fwd_t(const RmsParams& p, int blocks, cudaStream_t st) {
    switch (p.D) {
        case 8: rms_fwd_kernel<T, 1><<<blocks, kThreads, 0, st>>>(p); break;
        case 16: rms_fwd_kernel<T, 2><<<blocks, kThreads, 0, st>>>(p); break;
        case 32: rms_fwd_kernel<T, 4><<<blocks, kThreads, 0, st>>>(p); break;
        case 64: rms_fwd_kernel<T, 8><<<blocks, kThreads, 0, st>>>(p); break;
        case 128: rms_fwd_kernel<T, 16><<<blocks, kThreads, 0, st>>>(p); break;
        case 256: rms_fwd_kernel<T, 32><<<blocks, kThreads, 0, st>>>(p); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

template <typename T>
cudaError_t bwd_t(const RmsParams& p, int blocks, cudaStream_t st) {
    switch (p.D) {
        case 8: rms_bwd_kernel<T, 1><<<blocks, kThreads, 0, st>>>(p); break;
        case 16: rms_bwd_kernel<T, 2><<<blocks, kThreads, 0, st>>>(p); break;
        case 32: rms_bwd_kernel<T, 4><<<blocks, kThreads, 0, st>>>(p); break;
        case 64: rms_bwd_kernel<T, 8><<<blocks, kThreads, 0, st>>>(p); break;
        case 128: rms_bwd_kernel<T, 16><<<blocks, kThreads, 0, st>>>(p); break;
        case 256: rms_bwd_kernel<T, 32><<<blocks, kThreads, 0, st>>>(p); break;
        default: return cudaErrorInvalidValue;
    }
    cudaError_t err = cudaGetLastError();
    if (err == cudaSuccess && p.dw) {
        rms_dw_kernel<<<1, 1024, 0, st>>>(p.part, blocks, p.D, p.dw);
        err = cudaGetLastError();
    }
    return err;
}

}  // namespace

bool rms_supported_dim(int D) { return D == 8 || D == 16 || D == 32 || D == 64 || D == 128 || D == 256; }

int rms_blocks(const RmsParams& p) {
    const int64_t rows = (int64_t)p.B * p.N * p.H;
    const int64_t rpb = kThreads / (p.D / 8);
    const int64_t need = (rows + rpb - 1) / rpb;
    return (int)(need < kRmsMaxBlocks ? (need > 0 ? need : 1) : kRmsMaxBlocks);
}

cudaError_t launch_rms_fwd(const RmsParams& p, int dtype, cudaStream_t st) {
    const int blocks = rms_blocks(p);
    switch (dtype) {
        case SUBQ_FP32: return fwd_t<float>(p, blocks, st);
        case SUBQ_FP16: return fwd_t<__half>(p, blocks, st);
        case SUBQ_BF16: return fwd_t<__nv_bfloat16>(p, blocks, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_rms_bwd(const RmsParams& p, int dtype, cudaStream_t st) {
    const int blocks = rms_blocks(p);
    switch (dtype) {
        case SUBQ_FP32: return bwd_t<float>(p, blocks, st);
        case SUBQ_FP16: return bwd_t<__half>(p, blocks, st);
        case SUBQ_BF16: return bwd_t<__nv_bfloat16>(p, blocks, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace subq
