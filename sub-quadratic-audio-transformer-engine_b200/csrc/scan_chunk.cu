// Chunk-parallel scan on the CUDA cores, in float32, for the long calls the
// tensor-core kernels do not take (float32 inputs such as the C++ engine's,
// or d, e other than 64; d <= 256). The recurrent kernel (scan_simt.cu) steps
// token by token; here the 64 tokens of a chunk are processed together.
//
// Per chunk, with L_t the inclusive sum of log(gamma) over the chunk's tokens
// up to t (a masked token decays by 1), q~ = scale phi(q), k~ = m phi(k),
// v~ = m v, and [S | z] the state before the chunk:
//   A[t][tau] = (q~_t . k~_tau) exp(L_t - L_tau)   for tau <= t, else 0
//   num_t = sum_tau A[t][tau] v~_tau + exp(L_t) q~_t S
//   den_t = sum_tau A[t][tau] m_tau  + exp(L_t) q~_t . z          (normalised form)
//   out_t = m_t num_t / max(den_t, clamp)  (normalised)  or  m_t num_t
//   S <- exp(L_C) S + sum_tau exp(L_C - L_tau) k~_tau v~_tau^T,  z likewise with m_tau
// which is the recurrence of the reference (src/kernels/attention_forward.cpp:42-58,
// python/subq_audio/autograd.py:108-169 and :292-376) regrouped by chunk.
//
// chunk_scores_kernel (one CTA per chunk, every chunk at once) writes a block
// per chunk into the workspace: A (row stride 65), L (float64: differences of
// two prefix sums keep their precision), and q~, k~ in padded rows.
// chunk_scan_kernel then walks the chunks of one sequence for kET value
// columns per CTA, pulling each block into shared memory with 16-byte
// cp.async copies. L is summed in float64 and log(gamma) is clamped at -1e4
// (exp of it is 0 in float32 either way), so that a gamma of 0 gives weights
// of 0, not NaN. With the subnormal flush on, the state is flushed at chunk
// ends (the recurrence flushes it after every token; the two differ only in
// state entries below FLT_MIN).
//
// state_out may alias state_in: each CTA reads its own columns of S before
// its first barrier and only that CTA writes them. norm_in is read by every
// scan CTA, so the scores kernel copies it into the workspace first, and
// norm_out (written by the CTA of columns 0..3) may alias it too.
#include "scan_common.cuh"
#include "scan_launch.h"

namespace subq {
namespace {

constexpr int kCh = 64;      // tokens per chunk
constexpr int kET = 4;       // value columns per scan CTA
constexpr int kVW = kET + 1; // staged value row: the columns, then m
constexpr int kCThreads = 256;
constexpr int kALd = kCh + 1;  // row stride of A (bank-conflict-free row reads)

// Row stride (floats) of q~, k~ and of the transposed state tile: d rounded
// up to 32, plus 4, so that the 16-byte loads of 8 rows hit distinct banks.
__host__ __device__ inline int row_stride(int d) { return (d + 31) / 32 * 32 + 4; }

// The per-chunk block: A [64][65] f32 | L [64] f64 | q~ [64][DP] f32 | k~ [64][DP] f32.
// Every part starts on a 16-byte boundary.
constexpr size_t kABytes = sizeof(float) * kCh * kALd;  // 16640
constexpr size_t kLBytes = sizeof(double) * kCh;        // 512
__host__ __device__ inline size_t block_bytes(int d) {
    return kABytes + kLBytes + 2 * sizeof(float) * kCh * row_stride(d);
}
// After the blocks of every sequence: the initial normaliser z_in, [B*H][d].
__host__ __device__ inline float* z_copy(const ScanParams& p, int nCh) {
    return reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(p.ws) +
                                    (size_t)p.B * p.H * nCh * block_bytes(p.d));
}

// log(gamma) of token t as the chunk sums take it: 0 past the end or masked,
// clamped below at -1e4 (NaN passes through).
__device__ __forceinline__ double chunk_lg(const ScanParams& p, int b, int h, int t) {
    if (p.decay_mode == SUBQ_DECAY_NONE || t >= p.N || token_mask(p, b, t) == 0.f) return 0.0;
    const float lg = token_log_gamma(p, b, h, t);
    return lg < -1e4f ? -1e4 : (double)lg;
}

// One CTA per chunk: q~, k~ staged (and written out), L by a warp scan, then
// A with thread (ty, tx) forming A[ty + 16 a][tx + 16 c] for a, c < 4.
template <typename T>
__global__ void __launch_bounds__(kCThreads) chunk_scores_kernel(ScanParams p, int nCh) {
    const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int d = p.d, DP = row_stride(d);
    extern __shared__ __align__(16) float smc[];
    float* qs = smc;
    float* ks = qs + kCh * DP;
    double* Ls = reinterpret_cast<double*>(ks + kCh * DP);
    const int t0 = c * kCh;
    unsigned char* blk = reinterpret_cast<unsigned char*>(p.ws) + ((int64_t)(b * p.H + h) * nCh + c) * block_bytes(d);
    float* out_a = reinterpret_cast<float*>(blk);
    double* out_l = reinterpret_cast<double*>(blk + kABytes);
    float* out_q = reinterpret_cast<float*>(blk + kABytes + kLBytes);
    float* out_k = out_q + kCh * DP;

    if (c == 0 && p.normalize) {
        const int64_t bh = (int64_t)b * p.H + h;
        float* zc = z_copy(p, nCh) + bh * d;
        for (int i = threadIdx.x; i < d; i += blockDim.x) zc[i] = p.z_in ? p.z_in[bh * d + i] : 0.f;
    }
    const T* qb = (const T*)p.q + b * p.q_sb + h * p.q_sh;
    const T* kb = (const T*)p.k + b * p.k_sb + (h / p.kvg) * p.k_sh;
    for (int x = threadIdx.x; x < kCh * DP; x += blockDim.x) {
        const int tt = x / DP, i = x - tt * DP;
        const int t = t0 + tt;
        float qv = 0.f, kv = 0.f;
        if (i < d && t < p.N) {
            qv = phi_f(to_f<T>(qb[(int64_t)t * p.q_sn + i])) * p.scale;
            kv = phi_f(to_f<T>(kb[(int64_t)t * p.k_sn + i])) * token_mask(p, b, t);
        }
        qs[x] = qv;
        ks[x] = kv;
        out_q[x] = qv;
        out_k[x] = kv;
    }
    if (threadIdx.x < 32) {  // inclusive prefix of log(gamma): lane l owns tokens 2l, 2l + 1
        const int l = threadIdx.x;
        const double a0 = chunk_lg(p, b, h, t0 + 2 * l), a1 = chunk_lg(p, b, h, t0 + 2 * l + 1);
        double s = a0 + a1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const double y = __shfl_up_sync(0xffffffffu, s, o);
            if (l >= o) s += y;
        }
        double pre = __shfl_up_sync(0xffffffffu, s, 1);
        if (l == 0) pre = 0.0;
        Ls[2 * l] = pre + a0;
        Ls[2 * l + 1] = s;
        out_l[2 * l] = pre + a0;
        out_l[2 * l + 1] = s;
    }
    __syncthreads();
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) acc[a][cc] = 0.f;
    const int dv = (d + 3) & ~3;
    for (int i = 0; i < dv; i += 4) {
        float4 q4[4], k4[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) q4[a] = *reinterpret_cast<const float4*>(qs + (ty + 16 * a) * DP + i);
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) k4[cc] = *reinterpret_cast<const float4*>(ks + (tx + 16 * cc) * DP + i);
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc)
                acc[a][cc] = fmaf(q4[a].w, k4[cc].w, fmaf(q4[a].z, k4[cc].z,
                             fmaf(q4[a].y, k4[cc].y, fmaf(q4[a].x, k4[cc].x, acc[a][cc]))));
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int t = ty + 16 * a;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
            const int tau = tx + 16 * cc;
            float w = 0.f;
            if (tau <= t) w = acc[a][cc] * expf((float)(Ls[t] - Ls[tau]));
            out_a[t * kALd + tau] = w;
        }
    }
    if (threadIdx.x < kCh) out_a[threadIdx.x * kALd + kCh] = 0.f;  // the pad column
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
}

// The scan over the chunks of sequence (b, h) for value columns
// [kET blockIdx.x, + kET) and the normaliser (in every CTA). Thread
// (tq, jq) = (tid / 4, tid % 4) forms the output of token tq, column jq;
// thread ir < d holds row ir of the state tile [S | z] in registers and
// publishes it, transposed, in St for the next chunk's outputs.
template <typename T>
__global__ void __launch_bounds__(kCThreads) chunk_scan_kernel(ScanParams p, int nCh) {
    const int tile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int d = p.d, DP = row_stride(d), dv = (d + 3) & ~3;
    const int j0 = tile * kET;
    const int ncols = min(kET, p.e - j0);
    const int64_t bh = (int64_t)b * p.H + h;
    const size_t BB = block_bytes(d);
    extern __shared__ __align__(16) float smc[];
    const float* As = smc;                                                   // [64][65]
    const double* Ld = reinterpret_cast<const double*>(smc + kCh * kALd);    // [64]
    const float* Qs = smc + (kABytes + kLBytes) / sizeof(float);             // [64][DP]
    const float* Ks = Qs + kCh * DP;                                         // [64][DP]
    float* Vs = smc + BB / sizeof(float);                                    // [64][5]
    float* Ws = Vs + kCh * kVW;                                              // [64]
    float* St = Ws + kCh;                                                    // [5][DP]
    const unsigned char* blk0 = reinterpret_cast<const unsigned char*>(p.ws) + bh * nCh * BB;
    const T* vb = (const T*)p.v + b * p.v_sb + (h / p.kvg) * p.v_sh;
    T* ob = (T*)p.o + b * p.o_sb + h * p.o_sh;
    const int tid = threadIdx.x;
    const int tq = tid >> 2, jq = tid & 3;
    const int tmax = (tid >> 5) * 8 + 7;  // the warp's last token: A is 0 past the diagonal
    const int ir = tid;

    float sreg[kVW];
#pragma unroll
    for (int j = 0; j < kVW; ++j) sreg[j] = 0.f;
    if (ir < d) {
        for (int j = 0; j < ncols; ++j) sreg[j] = p.S_in ? p.S_in[(bh * d + ir) * p.e + j0 + j] : 0.f;
        if (p.normalize) sreg[kET] = z_copy(p, nCh)[bh * d + ir];
    }
    if (ir < dv) {
#pragma unroll
        for (int j = 0; j < kVW; ++j) St[j * DP + ir] = sreg[j];
    }
    for (int c = 0; c < nCh; ++c) {
        const int t0 = c * kCh;
        __syncthreads();  // the previous chunk's reads of the shared tiles are done
        const unsigned char* src = blk0 + c * BB;
        for (size_t x = tid; x < BB / 16; x += kCThreads)
            cp_async16(reinterpret_cast<unsigned char*>(smc) + 16 * x, src + 16 * x);
        for (int x = tid; x < kCh * kVW; x += kCThreads) {
            const int tt = x / kVW, j = x - tt * kVW;
            const int t = t0 + tt;
            float val = 0.f;
            if (t < p.N) {
                const float m = token_mask(p, b, t);
                if (j < ncols) val = to_f<T>(vb[(int64_t)t * p.v_sn + j0 + j]) * m;
                else if (j == kET) val = m;
            }
            Vs[x] = val;
        }
        cp_async_wait_all();
        __syncthreads();
        if (tid < kCh) Ws[tid] = expf((float)(Ld[kCh - 1] - Ld[tid]));
        const int t = t0 + tq;
        if (t < p.N && jq < ncols) {
            float num = 0.f, den = 0.f;
            const float* ar = As + tq * kALd;
            for (int tau = 0; tau <= tmax; ++tau) {
                const float a = ar[tau];
                num = fmaf(a, Vs[tau * kVW + jq], num);
                den = fmaf(a, Vs[tau * kVW + kET], den);
            }
            float qS = 0.f, qz = 0.f;
            const float* qr = Qs + tq * DP;
            const float* sc = St + jq * DP;
            const float* zc = St + kET * DP;
            for (int i = 0; i < dv; i += 4) {
                const float4 q4 = *reinterpret_cast<const float4*>(qr + i);
                const float4 s4 = *reinterpret_cast<const float4*>(sc + i);
                qS = fmaf(q4.w, s4.w, fmaf(q4.z, s4.z, fmaf(q4.y, s4.y, fmaf(q4.x, s4.x, qS))));
                if (p.normalize) {
                    const float4 z4 = *reinterpret_cast<const float4*>(zc + i);
                    qz = fmaf(q4.w, z4.w, fmaf(q4.z, z4.z, fmaf(q4.y, z4.y, fmaf(q4.x, z4.x, qz))));
                }
            }
            const float el = expf((float)Ld[tq]);
            num = fmaf(el, qS, num);
            den = fmaf(el, qz, den);
            const float m = Vs[tq * kVW + kET];
            const float out = p.normalize ? num / fmaxf(den, p.clamp_min) * m : num * m;
            ob[(int64_t)t * p.o_sn + j0 + jq] = from_f<T>(out);
        }
        __syncthreads();  // every read of St is done; Ws is written
        if (ir < d) {
            const float lc = expf((float)Ld[kCh - 1]);
#pragma unroll
            for (int j = 0; j < kVW; ++j) sreg[j] *= lc;
            for (int tau = 0; tau < kCh; ++tau) {
                const float kw = Ks[tau * DP + ir] * Ws[tau];
                const float* vr = Vs + tau * kVW;
#pragma unroll
                for (int j = 0; j < kVW; ++j) sreg[j] = fmaf(kw, vr[j], sreg[j]);
            }
#pragma unroll
            for (int j = 0; j < kVW; ++j) {
                sreg[j] = flush_small<float>(sreg[j], p.flush);
                St[j * DP + ir] = sreg[j];
            }
        }
    }
    if (ir < d) {
        if (p.S_out)
            for (int j = 0; j < ncols; ++j) p.S_out[(bh * d + ir) * p.e + j0 + j] = sreg[j];
        if (p.normalize && p.z_out && tile == 0) p.z_out[bh * d + ir] = sreg[kET];
    }
}

size_t scores_smem(int d) { return sizeof(float) * 2 * kCh * row_stride(d) + sizeof(double) * kCh; }
size_t scan_smem(int d) { return block_bytes(d) + sizeof(float) * (kCh * kVW + kCh + kVW * row_stride(d)); }

template <typename T>
cudaError_t launch_chunk_t(const ScanParams& p, cudaStream_t st) {
    const int nCh = (p.N + kCh - 1) / kCh;
    auto k1 = chunk_scores_kernel<T>;
    auto k2 = chunk_scan_kernel<T>;
    cudaError_t err = cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)scores_smem(p.d));
    if (err == cudaSuccess)
        err = cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)scan_smem(p.d));
    if (err != cudaSuccess) return err;
    k1<<<dim3(nCh, p.H, p.B), kCThreads, scores_smem(p.d), st>>>(p, nCh);
    k2<<<dim3((p.e + kET - 1) / kET, p.H, p.B), kCThreads, scan_smem(p.d), st>>>(p, nCh);
    return cudaGetLastError();
}

}  // namespace

bool chunk_fwd_usable(const ScanParams& p, int dtype) {
    if (dtype != SUBQ_FP32 && dtype != SUBQ_FP16 && dtype != SUBQ_BF16) return false;
    if (p.reverse || p.fallback || p.d < 1 || p.d > 256 || p.e < 1) return false;
    // a growing scalar state (gamma > 1) keeps the token-by-token recurrence
    if (p.decay_mode == SUBQ_DECAY_SCALAR && !(p.lg_scalar <= 0.f)) return false;
    return scan_smem(p.d) <= 227 * 1024;
}

size_t chunk_fwd_workspace_bytes(const ScanParams& p) {
    const int64_t nCh = (p.N + kCh - 1) / kCh;
    return (size_t)p.B * p.H * nCh * block_bytes(p.d) + ((size_t)p.B * p.H * p.d * sizeof(float) + 15) / 16 * 16;
}

cudaError_t launch_fwd_chunk(const ScanParams& p, int dtype, cudaStream_t st) {
    if (p.N == 0) return launch_fwd_exact(p, dtype, st);  // no chunks: the state passes through
    if (reinterpret_cast<uintptr_t>(p.ws) % 16 != 0) return cudaErrorInvalidValue;
    switch (dtype) {
        case SUBQ_FP32: return launch_chunk_t<float>(p, st);
        case SUBQ_FP16: return launch_chunk_t<__half>(p, st);
        case SUBQ_BF16: return launch_chunk_t<__nv_bfloat16>(p, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace subq
