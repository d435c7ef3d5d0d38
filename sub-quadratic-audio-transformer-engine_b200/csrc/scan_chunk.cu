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
// chunk_scores_kernel (three CTAs per chunk, every chunk at once) writes a block
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

// Three CTAs per chunk (blockIdx.x = 3 chunk + quadrant; y = head, z = batch):
// the causal 64 x 64 block A is
// three 32 x 32 quadrants, (t, tau) in (lo, lo), (hi, lo) and (hi, hi); the
// fourth, (lo, hi), is zero. A CTA stages the 32 rows of q~ and of k~ its
// quadrant needs and forms its 32 x 32 outputs (thread (ty, tx) rows ty, ty + 16
// and columns tx, tx + 16). Quadrant (lo, lo) writes L, the zero quadrant and
// rows 0-31 of q~ and k~; quadrant (hi, hi) writes rows 32-63 of both.
constexpr int kHalf = kCh / 2;
template <typename T>
__global__ void __launch_bounds__(kCThreads) chunk_scores_kernel(ScanParams p, int nCh) {
    const int c = blockIdx.x / 3, quad = blockIdx.x - 3 * c, h = blockIdx.y, b = blockIdx.z;
    const int64_t bh = (int64_t)b * p.H + h;
    const int t_lo = quad == 0 ? 0 : kHalf, tau_lo = quad == 2 ? kHalf : 0;
    const bool write_q = quad != 1, write_k = quad != 1;  // rows t_lo.. of q~, tau_lo.. of k~
    const int d = p.d, DP = row_stride(d);
    extern __shared__ __align__(16) float smc[];
    float* qs = smc;                 // [32][DP]: rows t_lo + r
    float* ks = qs + kHalf * DP;     // [32][DP]: rows tau_lo + r
    double* Ls = reinterpret_cast<double*>(ks + kHalf * DP);  // [64]
    const int t0 = c * kCh;
    unsigned char* blk = reinterpret_cast<unsigned char*>(p.ws) + (bh * nCh + c) * block_bytes(d);
    float* out_a = reinterpret_cast<float*>(blk);
    double* out_l = reinterpret_cast<double*>(blk + kABytes);
    float* out_q = reinterpret_cast<float*>(blk + kABytes + kLBytes);
    float* out_k = out_q + kCh * DP;

    if (c == 0 && quad == 0 && p.normalize) {
        float* zc = z_copy(p, nCh) + bh * d;
        for (int i = threadIdx.x; i < d; i += blockDim.x) zc[i] = p.z_in ? p.z_in[bh * d + i] : 0.f;
    }
    const T* qb = (const T*)p.q + b * p.q_sb + h * p.q_sh;
    const T* kb = (const T*)p.k + b * p.k_sb + (h / p.kvg) * p.k_sh;
    // four elements per thread and step, their loads issued before any use
    for (int x0 = threadIdx.x; x0 < kHalf * DP; x0 += 4 * kCThreads) {
        float qr[4], kr[4], mr[4];
        bool inq[4], ink[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int x = x0 + u * kCThreads, rr = x / DP, i = x - rr * DP;
            const int tq = t0 + t_lo + rr, tk = t0 + tau_lo + rr;
            const bool inx = x < kHalf * DP && i < d;
            inq[u] = inx && tq < p.N;
            ink[u] = inx && tk < p.N;
            qr[u] = inq[u] ? to_f<T>(qb[(int64_t)tq * p.q_sn + i]) : 0.f;
            kr[u] = ink[u] ? to_f<T>(kb[(int64_t)tk * p.k_sn + i]) : 0.f;
            mr[u] = ink[u] ? token_mask(p, b, tk) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int x = x0 + u * kCThreads;
            if (x >= kHalf * DP) break;
            const float qf = inq[u] ? phi_f(qr[u]) * p.scale : 0.f;  // padding and tokens past N: 0
            const float kf = ink[u] ? phi_f(kr[u]) * mr[u] : 0.f;
            qs[x] = qf;
            ks[x] = kf;
            if (write_q) out_q[t_lo * DP + x] = qf;
            if (write_k) out_k[tau_lo * DP + x] = kf;
        }
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
        if (quad == 0) {
            out_l[2 * l] = pre + a0;
            out_l[2 * l + 1] = s;
        }
    }
    __syncthreads();
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    const int dv = (d + 3) & ~3;
    for (int i = 0; i < dv; i += 4) {
        float4 q4[2], k4[2];
#pragma unroll
        for (int a = 0; a < 2; ++a) q4[a] = *reinterpret_cast<const float4*>(qs + (ty + 16 * a) * DP + i);
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) k4[cc] = *reinterpret_cast<const float4*>(ks + (tx + 16 * cc) * DP + i);
#pragma unroll
        for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int cc = 0; cc < 2; ++cc)
                acc[a][cc] = fmaf(q4[a].w, k4[cc].w, fmaf(q4[a].z, k4[cc].z,
                             fmaf(q4[a].y, k4[cc].y, fmaf(q4[a].x, k4[cc].x, acc[a][cc]))));
    }
#pragma unroll
    for (int a = 0; a < 2; ++a) {
        const int t = t_lo + ty + 16 * a;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
            const int tau = tau_lo + tx + 16 * cc;
            float w = 0.f;
            if (tau <= t) w = acc[a][cc] * expf((float)(Ls[t] - Ls[tau]));
            out_a[t * kALd + tau] = w;
        }
    }
    if (quad == 0) {  // the zero quadrant (t < 32, tau >= 32) and the pad column of rows 0-31
        for (int x = threadIdx.x; x < kHalf * kHalf; x += kCThreads)
            out_a[(x / kHalf) * kALd + kHalf + (x % kHalf)] = 0.f;
        if (threadIdx.x < kHalf) out_a[threadIdx.x * kALd + kCh] = 0.f;
    } else if (quad == 2 && threadIdx.x < kHalf) {
        out_a[(kHalf + threadIdx.x) * kALd + kCh] = 0.f;  // the pad column of rows 32-63
    }
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

// ------------------------------------------------------------------------
// Chunk-parallel form for calls with few sequences (the sequential walk above
// has only ceil(e / 4) CTAs per sequence): three launches after the scores,
// none of which walks the chunks of a sequence token by token.
//   chunk_state_kernel   U_c = sum_tau exp(L_C - L_tau) k~_tau [v~_tau | m_tau]   (all chunks at once)
//   chunk_prefix_kernel  [S | z] at each chunk's start, in place of U_c: one thread per state
//                        element walks the chunks (S <- exp(L_C) S + U_c); the final state out
//   chunk_out_kernel     out_t = (A v~)_t + exp(L_t) q~_t [S | z]_c                   (all chunks at once)
// U and the chunk-start states share one fp32 buffer [B*H][nCh][d][e + 1]
// after the z copy.
constexpr int kPW = 32;  // value columns per CTA of the state and output kernels

__host__ __device__ inline size_t zcopy_bytes(const ScanParams& p) {
    return ((size_t)p.B * p.H * p.d * sizeof(float) + 15) / 16 * 16;
}
__host__ __device__ inline float* state_buf(const ScanParams& p, int nCh) {
    return z_copy(p, nCh) + zcopy_bytes(p) / sizeof(float);
}

// U_c as an outer-product tile per thread: rows 4 r .. 4 r + 3 and
// 4 (RG + r) .. 4 (RG + r) + 3 (two float4 of k~ along the features; lanes
// read consecutive 16-byte words) times columns 4 q .. 4 q + 3 (one float4 of
// v~), 32 FMAs per three shared-memory loads. A CTA covers every row and
// state_cols(d) columns of [v~ | m].
__host__ __device__ inline int state_rgroups(int d) { return (d + 7) / 8; }
__host__ __device__ inline int state_cols(int d) {
    const int w = 4 * (kCThreads / state_rgroups(d));
    return w < 256 ? w : 256;  // [v~ | m] has at most 257 columns
}

template <typename T>
__global__ void __launch_bounds__(kCThreads) chunk_state_kernel(ScanParams p, int nCh) {
    const int c = blockIdx.x, tile = blockIdx.y, bh = blockIdx.z;
    const int b = bh / p.H, h = bh - b * p.H;
    const int d = p.d, DP = row_stride(d), ES = p.e + 1;
    const int CW = state_cols(d), RG = state_rgroups(d);
    const int j0 = tile * CW, ncol = min(CW, ES - j0);
    extern __shared__ __align__(16) float smc[];
    float* Ks = smc;                 // [64][DP] k~, then scaled by exp(L_C - L_tau)
    float* Vs = Ks + kCh * DP;       // [64][CW] v~ (column e: m)
    float* Ws = Vs + kCh * CW;       // [64] exp(L_C - L_tau)
    const unsigned char* blk = reinterpret_cast<const unsigned char*>(p.ws) + ((int64_t)bh * nCh + c) * block_bytes(d);
    const double* Lg = reinterpret_cast<const double*>(blk + kABytes);
    const unsigned char* ksrc = blk + kABytes + kLBytes + sizeof(float) * kCh * DP;
    for (int x = threadIdx.x; x < kCh * DP / 4; x += kCThreads)
        cp_async16(reinterpret_cast<unsigned char*>(Ks) + 16 * x, ksrc + 16 * x);
    const T* vb = (const T*)p.v + b * p.v_sb + (h / p.kvg) * p.v_sh;
    for (int x = threadIdx.x; x < kCh * CW; x += kCThreads) {
        const int tt = x / CW, jj = x - tt * CW, j = j0 + jj, t = c * kCh + tt;
        float val = 0.f;
        if (t < p.N && jj < ncol) {
            const float m = token_mask(p, b, t);
            val = j < p.e ? to_f<T>(vb[(int64_t)t * p.v_sn + j]) * m : m;
        }
        Vs[x] = val;
    }
    if (threadIdx.x < kCh) Ws[threadIdx.x] = expf((float)(Lg[kCh - 1] - Lg[threadIdx.x]));
    cp_async_wait_all();
    __syncthreads();
    for (int x = threadIdx.x; x < kCh * DP; x += kCThreads) Ks[x] *= Ws[x / DP];  // k~_tau exp(L_C - L_tau)
    __syncthreads();
    const int r = threadIdx.x % RG, q = threadIdx.x / RG;
    if (4 * q >= ncol) return;
    float acc[8][4];
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
        for (int x = 0; x < 4; ++x) acc[a][x] = 0.f;
    for (int tau = 0; tau < kCh; ++tau) {
        const float4 k0 = *reinterpret_cast<const float4*>(Ks + tau * DP + 4 * r);
        const float4 k1 = *reinterpret_cast<const float4*>(Ks + tau * DP + 4 * (RG + r));
        const float4 v4 = *reinterpret_cast<const float4*>(Vs + tau * CW + 4 * q);
        const float kk[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
        const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
        for (int a = 0; a < 8; ++a)
#pragma unroll
            for (int x = 0; x < 4; ++x) acc[a][x] = fmaf(kk[a], vv[x], acc[a][x]);
    }
    float* U = state_buf(p, nCh) + ((int64_t)bh * nCh + c) * d * ES + j0 + 4 * q;
#pragma unroll
    for (int a = 0; a < 8; ++a) {
        const int i = a < 4 ? 4 * r + a : 4 * (RG + r) + a - 4;
        if (i < d) {
#pragma unroll
            for (int x = 0; x < 4; ++x)
                if (4 * q + x < ncol) U[(int64_t)i * ES + x] = acc[a][x];
        }
    }
}

// One thread per element (bh, i, j) of [S | z]: walks the chunks, leaving the
// state at each chunk's start in place of that chunk's U, and writes the final state.
__global__ void __launch_bounds__(kCThreads) chunk_prefix_kernel(ScanParams p, int nCh) {
    const int d = p.d, ES = p.e + 1;
    const int64_t id = (int64_t)blockIdx.x * kCThreads + threadIdx.x;
    if (id >= (int64_t)p.B * p.H * d * ES) return;
    const int64_t bh = id / ((int64_t)d * ES);
    const int rem = (int)(id - bh * d * ES), i = rem / ES, j = rem - i * ES;
    float s = 0.f;
    if (j < p.e) {
        if (p.S_in) s = p.S_in[(bh * d + i) * p.e + j];
    } else if (p.normalize && p.z_in) {
        s = p.z_in[bh * d + i];
    }
    const unsigned char* blk = reinterpret_cast<const unsigned char*>(p.ws) + bh * nCh * block_bytes(d);
    float* U = state_buf(p, nCh) + (bh * nCh * d + i) * ES + j;
    const int64_t cs = (int64_t)d * ES;
    auto lc_of = [&](int c) {
        return expf((float)reinterpret_cast<const double*>(blk + c * block_bytes(d) + kABytes)[kCh - 1]);
    };
    // loads run four chunks ahead of the stores (in program order, so the
    // compiler need not prove that U[c + 4] and U[c] differ)
    constexpr int kAhead = 4;
    float ub[kAhead], lb[kAhead];
#pragma unroll
    for (int a = 0; a < kAhead; ++a) {
        ub[a] = a < nCh ? U[a * cs] : 0.f;
        lb[a] = a < nCh ? lc_of(a) : 0.f;
    }
    for (int c0 = 0; c0 < nCh; c0 += kAhead) {
#pragma unroll
        for (int a = 0; a < kAhead; ++a) {
            const int c = c0 + a;
            if (c >= nCh) break;
            const float u = ub[a], lc = lb[a];
            if (c + kAhead < nCh) {
                ub[a] = U[(c + kAhead) * cs];
                lb[a] = lc_of(c + kAhead);
            }
            U[c * cs] = s;
            s = flush_small<float>(fmaf(lc, s, u), p.flush);
        }
    }
    if (j < p.e) {
        if (p.S_out) p.S_out[(bh * d + i) * p.e + j] = s;
    } else if (p.normalize && p.z_out) {
        p.z_out[bh * d + i] = s;
    }
}

// Outputs of chunk c, value columns [kPW blockIdx.y, + kPW): thread (t, q) =
// (tid / 4, tid % 4) forms token t's columns 8q .. 8q + 7 of the tile.
template <typename T>
__global__ void __launch_bounds__(kCThreads) chunk_out_kernel(ScanParams p, int nCh) {
    const int c = blockIdx.x, tile = blockIdx.y, bh = blockIdx.z;
    const int b = bh / p.H, h = bh - b * p.H;
    const int d = p.d, DP = row_stride(d), ES = p.e + 1, dv = (d + 3) & ~3;
    const int j0 = tile * kPW, ncol = min(kPW, p.e - j0);
    constexpr int kSW = kPW + 4;  // row stride of the state tile
    extern __shared__ __align__(16) float smc[];
    const float* As = smc;                                                  // [64][65]
    const double* Ld = reinterpret_cast<const double*>(smc + kCh * kALd);   // [64]
    const float* Qs = smc + (kABytes + kLBytes) / sizeof(float);            // [64][DP]
    float* Ss = const_cast<float*>(Qs) + kCh * DP;                          // [dv][kSW] S_c tile
    float* Zs = Ss + dv * kSW;                                              // [dv] z_c
    float* Vs = Zs + dv;                                                    // [64][kPW] v~
    float* Ms = Vs + kCh * kPW;                                             // [64] m
    const unsigned char* blk = reinterpret_cast<const unsigned char*>(p.ws) + ((int64_t)bh * nCh + c) * block_bytes(d);
    const size_t head = kABytes + kLBytes + sizeof(float) * kCh * DP;  // A, L, q~
    for (size_t x = threadIdx.x; x < head / 16; x += kCThreads)
        cp_async16(reinterpret_cast<unsigned char*>(smc) + 16 * x, blk + 16 * x);
    const float* Sg = state_buf(p, nCh) + ((int64_t)bh * nCh + c) * d * ES;
    for (int x = threadIdx.x; x < dv * kPW; x += kCThreads) {
        const int i = x / kPW, jj = x - i * kPW;
        Ss[i * kSW + jj] = (i < d && jj < ncol) ? Sg[(int64_t)i * ES + j0 + jj] : 0.f;
    }
    for (int i = threadIdx.x; i < dv; i += kCThreads) Zs[i] = (i < d && p.normalize) ? Sg[(int64_t)i * ES + p.e] : 0.f;
    const T* vb = (const T*)p.v + b * p.v_sb + (h / p.kvg) * p.v_sh;
    for (int x = threadIdx.x; x < kCh * kPW; x += kCThreads) {
        const int tt = x / kPW, jj = x - tt * kPW, t = c * kCh + tt;
        Vs[x] = (t < p.N && jj < ncol) ? to_f<T>(vb[(int64_t)t * p.v_sn + j0 + jj]) * token_mask(p, b, t) : 0.f;
    }
    if (threadIdx.x < kCh) {
        const int t = c * kCh + threadIdx.x;
        Ms[threadIdx.x] = t < p.N ? token_mask(p, b, t) : 0.f;
    }
    cp_async_wait_all();
    __syncthreads();
    const int tq = threadIdx.x >> 2, q = threadIdx.x & 3;
    const int t = c * kCh + tq;
    if (t >= p.N || 8 * q >= ncol) return;
    const int tmax = (threadIdx.x >> 5) * 8 + 7;  // the warp's last token: A is 0 past the diagonal
    float num[8], qs[8], den = 0.f, qz = 0.f;
#pragma unroll
    for (int x = 0; x < 8; ++x) num[x] = qs[x] = 0.f;
    const float* ar = As + tq * kALd;
    for (int tau = 0; tau <= tmax; ++tau) {
        const float a = ar[tau];
        const float4 v0 = *reinterpret_cast<const float4*>(Vs + tau * kPW + 8 * q);
        const float4 v1 = *reinterpret_cast<const float4*>(Vs + tau * kPW + 8 * q + 4);
        num[0] = fmaf(a, v0.x, num[0]); num[1] = fmaf(a, v0.y, num[1]);
        num[2] = fmaf(a, v0.z, num[2]); num[3] = fmaf(a, v0.w, num[3]);
        num[4] = fmaf(a, v1.x, num[4]); num[5] = fmaf(a, v1.y, num[5]);
        num[6] = fmaf(a, v1.z, num[6]); num[7] = fmaf(a, v1.w, num[7]);
        den = fmaf(a, Ms[tau], den);
    }
    const float* qr = Qs + tq * DP;
    for (int i = 0; i < dv; ++i) {
        const float qv = qr[i];
        const float4 s0 = *reinterpret_cast<const float4*>(Ss + i * kSW + 8 * q);
        const float4 s1 = *reinterpret_cast<const float4*>(Ss + i * kSW + 8 * q + 4);
        qs[0] = fmaf(qv, s0.x, qs[0]); qs[1] = fmaf(qv, s0.y, qs[1]);
        qs[2] = fmaf(qv, s0.z, qs[2]); qs[3] = fmaf(qv, s0.w, qs[3]);
        qs[4] = fmaf(qv, s1.x, qs[4]); qs[5] = fmaf(qv, s1.y, qs[5]);
        qs[6] = fmaf(qv, s1.z, qs[6]); qs[7] = fmaf(qv, s1.w, qs[7]);
        qz = fmaf(qv, Zs[i], qz);
    }
    const float el = expf((float)Ld[tq]);
    const float m = Ms[tq];
    den = fmaf(el, qz, den);
    const float inv = p.normalize ? m / fmaxf(den, p.clamp_min) : m;
    T* orow = (T*)p.o + b * p.o_sb + h * p.o_sh + (int64_t)t * p.o_sn + j0 + 8 * q;
#pragma unroll
    for (int x = 0; x < 8; ++x)
        if (8 * q + x < ncol) orow[x] = from_f<T>(fmaf(el, qs[x], num[x]) * inv);
}

size_t state_smem(int d) { return sizeof(float) * (kCh * row_stride(d) + kCh * state_cols(d) + kCh); }
size_t out_smem(int d) {
    const int dv = (d + 3) & ~3;
    return kABytes + kLBytes + sizeof(float) * (kCh * row_stride(d) + dv * (kPW + 4) + dv + kCh * kPW + kCh);
}

// The parallel form when the sequential walk would fill less than two waves.
bool chunk_parallel(const ScanParams& p) { return (int64_t)((p.e + kET - 1) / kET) * p.B * p.H < 2 * 148; }

size_t scores_smem(int d) { return sizeof(float) * 2 * kHalf * row_stride(d) + sizeof(double) * kCh; }
size_t scan_smem(int d) { return block_bytes(d) + sizeof(float) * (kCh * kVW + kCh + kVW * row_stride(d)); }

template <typename T>
cudaError_t launch_chunk_t(const ScanParams& p, cudaStream_t st, int* launches) {
    const int nCh = (p.N + kCh - 1) / kCh;
    auto k1 = chunk_scores_kernel<T>;
    cudaError_t err = cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)scores_smem(p.d));
    if (err != cudaSuccess) return err;
    k1<<<dim3(3 * nCh, p.H, p.B), kCThreads, scores_smem(p.d), st>>>(p, nCh);
    if (!chunk_parallel(p)) {
        auto k2 = chunk_scan_kernel<T>;
        err = cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)scan_smem(p.d));
        if (err != cudaSuccess) return err;
        k2<<<dim3((p.e + kET - 1) / kET, p.H, p.B), kCThreads, scan_smem(p.d), st>>>(p, nCh);
        *launches = 2;
        return cudaGetLastError();
    }
    auto ks = chunk_state_kernel<T>;
    auto ko = chunk_out_kernel<T>;
    err = cudaFuncSetAttribute(ks, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)state_smem(p.d));
    if (err == cudaSuccess) err = cudaFuncSetAttribute(ko, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)out_smem(p.d));
    if (err != cudaSuccess) return err;
    const int BH = p.B * p.H;
    ks<<<dim3(nCh, (p.e + 1 + state_cols(p.d) - 1) / state_cols(p.d), BH), kCThreads, state_smem(p.d), st>>>(p, nCh);
    const int64_t elems = (int64_t)BH * p.d * (p.e + 1);
    chunk_prefix_kernel<<<(unsigned)((elems + kCThreads - 1) / kCThreads), kCThreads, 0, st>>>(p, nCh);
    ko<<<dim3(nCh, (p.e + kPW - 1) / kPW, BH), kCThreads, out_smem(p.d), st>>>(p, nCh);
    *launches = 4;
    return cudaGetLastError();
}

}  // namespace

bool chunk_fwd_usable(const ScanParams& p, int dtype) {
    if (dtype != SUBQ_FP32 && dtype != SUBQ_FP16 && dtype != SUBQ_BF16) return false;
    if (p.reverse || p.fallback || p.d < 1 || p.d > 256 || p.e < 1) return false;
    // a growing scalar state (gamma > 1) keeps the token-by-token recurrence
    if (p.decay_mode == SUBQ_DECAY_SCALAR && !(p.lg_scalar <= 0.f)) return false;
    return scan_smem(p.d) <= 227 * 1024 && out_smem(p.d) <= 227 * 1024;
}

size_t chunk_fwd_workspace_bytes(const ScanParams& p) {
    const int64_t nCh = (p.N + kCh - 1) / kCh;
    size_t bytes = (size_t)p.B * p.H * nCh * block_bytes(p.d) + zcopy_bytes(p);
    if (chunk_parallel(p)) bytes += (size_t)p.B * p.H * nCh * p.d * (p.e + 1) * sizeof(float);
    return bytes;
}

cudaError_t launch_fwd_chunk(const ScanParams& p, int dtype, cudaStream_t st, int* launches) {
    *launches = 1;
    if (p.N == 0) return launch_fwd_exact(p, dtype, st);  // no chunks: the state passes through
    if (reinterpret_cast<uintptr_t>(p.ws) % 16 != 0) return cudaErrorInvalidValue;
    switch (dtype) {
        case SUBQ_FP32: return launch_chunk_t<float>(p, st, launches);
        case SUBQ_FP16: return launch_chunk_t<__half>(p, st, launches);
        case SUBQ_BF16: return launch_chunk_t<__nv_bfloat16>(p, st, launches);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace subq
