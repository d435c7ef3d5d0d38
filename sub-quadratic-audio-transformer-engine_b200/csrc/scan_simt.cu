// Exact float32 path of the scan: a per-token sequential recurrence with the
// d x e state spread over the threads of a CTA.
//
// This family serves the float32 engine semantics (the reference's C++
// engine, src/kernels/attention_forward.cpp:13-63 and :97-170, and its CPU
// backward src/kernels/attention_backward.cpp:44-241) at float32 accuracy,
// and every shape the tensor-core path does not cover (d or e other than 64,
// tiny test shapes). Accumulation order per state element is the reference's
// sequential one, so float32 results stay within ~1e-6 of a float64 scan.
#include <float.h>

#include <algorithm>

#include "scan_common.cuh"
#include "scan_launch.h"

namespace subq {

namespace {

constexpr int kR = 8;    // threads cooperating on one state column
constexpr int kCT = 32;  // tokens staged in shared memory per step

// ---------------------------------------------------------------------------
// Forward. grid = (ceil(e / ET), H, B); block = (ET + normalize) * kR threads
// rounded up to whole warps. Thread (col, r) owns rows r, r + kR, ... of
// column j0 + col of S (col == ncols is the running denominator z).
// ---------------------------------------------------------------------------
template <typename T, typename A, int RPT>
__global__ void __launch_bounds__(288) scan_fwd_exact_kernel(ScanParams p, int ET) {
    const int tile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    if (p.fallback && !p.fallback[b * p.H + h]) return;  // only the sequences flagged for this path
    const int d = p.d;
    const int j0 = tile * ET;
    const int ncols = min(ET, p.e - j0);
    const int col = threadIdx.x / kR;
    const int r = threadIdx.x % kR;
    const bool is_z = p.normalize && col == ncols;
    const bool active = col < ncols || is_z;
    const int VW = ET + 1;  // staged value row width

    extern __shared__ __align__(16) unsigned char smem_raw[];
    A* sm = reinterpret_cast<A*>(smem_raw);
    A* qs = sm;                // [kCT][d]  scale * phi(q)
    A* ks = qs + kCT * d;      // [kCT][d]  m * phi(k)
    A* vs = ks + kCT * d;      // [kCT][VW] m * v, then m in slot ncols
    A* os = vs + kCT * VW;     // [kCT][VW] results
    A* gs = os + kCT * VW;     // [kCT]     gamma
    A* ms = gs + kCT;          // [kCT]     mask

    const int64_t bh = (int64_t)b * p.H + h;
    const T* qb = (const T*)p.q + b * p.q_sb + h * p.q_sh;
    const T* kb = (const T*)p.k + b * p.k_sb + (h / p.kvg) * p.k_sh;
    const T* vb = (const T*)p.v + b * p.v_sb + (h / p.kvg) * p.v_sh;
    T* ob = (T*)p.o + b * p.o_sb + h * p.o_sh;

    A s[RPT];
#pragma unroll
    for (int x = 0; x < RPT; ++x) {
        const int i = r + x * kR;
        A v0 = 0;
        if (active && i < d) {
            if (is_z) {
                if (p.z_in) v0 = p.z_in[bh * d + i];
            } else if (p.S_in) {
                v0 = p.S_in[(bh * d + i) * p.e + j0 + col];
            }
        }
        s[x] = v0;
    }

    for (int t0 = 0; t0 < p.N; t0 += kCT) {
        const int nt = min(kCT, p.N - t0);
        __syncthreads();  // the previous step's results have been written out
        for (int x = threadIdx.x; x < nt * d; x += blockDim.x) {
            const int tt = x / d, i = x - tt * d;
            const int t = tok_at(p, t0 + tt);
            const A m = token_mask(p, b, t);
            qs[x] = phi_f(load_a<A>(qb[(int64_t)t * p.q_sn + i])) * (A)p.scale;
            ks[x] = phi_f(load_a<A>(kb[(int64_t)t * p.k_sn + i])) * m;
        }
        for (int x = threadIdx.x; x < nt * VW; x += blockDim.x) {
            const int tt = x / VW, c = x - tt * VW;
            const int t = tok_at(p, t0 + tt);
            const A m = token_mask(p, b, t);
            A val = 0;
            if (c < ncols) val = load_a<A>(vb[(int64_t)t * p.v_sn + j0 + c]) * m;
            else if (c == ncols) val = m;
            vs[x] = val;
        }
        for (int tt = threadIdx.x; tt < nt; tt += blockDim.x) {
            const int t = tok_at(p, t0 + tt);
            const A m = token_mask(p, b, t);
            gs[tt] = m > 0 ? exp_a((A)token_log_gamma(p, b, h, t)) : (A)1;
            ms[tt] = m;
        }
        __syncthreads();
        for (int tt = 0; tt < nt; ++tt) {
            const A g = gs[tt];
            const A vj = active ? vs[tt * VW + col] : (A)0;
            const A* qrow = qs + tt * d;
            const A* krow = ks + tt * d;
            A acc = 0;
#pragma unroll
            for (int x = 0; x < RPT; ++x) {
                const int i = r + x * kR;
                if (i < d) {
                    const A sv = flush_small<A>(fma(g, s[x], krow[i] * vj), p.flush);
                    s[x] = sv;
                    acc = fma(qrow[i], sv, acc);
                }
            }
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            acc += __shfl_xor_sync(0xffffffffu, acc, 4);
            if (r == 0 && active) os[tt * VW + col] = acc;
        }
        __syncthreads();
        for (int x = threadIdx.x; x < nt * ncols; x += blockDim.x) {
            const int tt = x / ncols, c = x - tt * ncols;
            const A num = os[tt * VW + c];
            const A m = ms[tt];
            const A out = p.normalize ? num / fmax(os[tt * VW + ncols], (A)p.clamp_min) * m : num * m;
            ob[(int64_t)tok_at(p, t0 + tt) * p.o_sn + j0 + c] = store_a<T, A>(out);
        }
    }
    // Final state. Every CTA read its initial state before its first barrier,
    // and only the owner of an element writes it, so state_out may alias state_in.
#pragma unroll
    for (int x = 0; x < RPT; ++x) {
        const int i = r + x * kR;
        if (active && i < d) {
            if (is_z) {
                if (p.z_out) p.z_out[bh * d + i] = (float)s[x];
            } else if (p.S_out) {
                p.S_out[(bh * d + i) * p.e + j0 + col] = (float)s[x];
            }
        }
    }
}

// Sum over the block, result returned to every thread. `red` holds 33 floats.
template <typename A>
__device__ __forceinline__ A block_sum(A v, A* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        A w = lane < (int)(blockDim.x >> 5) ? red[lane] : (A)0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
        if (lane == 0) red[32] = w;
    }
    __syncthreads();
    const A total = red[32];
    __syncthreads();  // red may be reused right after
    return total;
}

// ---------------------------------------------------------------------------
// Backward. One CTA per (h, b); the augmented state S' = [S | z] (d x ep) and
// later the adjoint G live in shared memory with an odd row stride.
//   pass F (t ascending):  S'_t, o'_t = q~_t S'_t, dO'_t (quotient rule),
//                          dq~_t = S'_t dO'_t  -> dq, and q~_t . dq~_t
//   pass R (t descending): G_t = gamma_{t+1} G_{t+1} + q~_t dO'_t^T,
//                          dk~_t = G_t v'_t -> dk, dv_t = G_t^T k_t -> dv,
//                          d log(gamma_t) = sum_{t' >= t} (q~.dq~ - k.dk~)_{t'}
// The workspace keeps three floats per token between the passes.
// ---------------------------------------------------------------------------
template <typename T, typename A>
__global__ void __launch_bounds__(256) scan_bwd_exact_kernel(ScanParams p) {
    const int h = blockIdx.x, b = blockIdx.y;
    if (p.fallback && !p.fallback[b * p.H + h]) return;  // only the sequences flagged for this path
    const int d = p.d, e = p.e;
    const int ep = e + (p.normalize ? 1 : 0);
    const int LD = ep | 1;
    const int64_t bh = (int64_t)b * p.H + h;

    extern __shared__ __align__(16) unsigned char smem_raw[];
    A* Sm = reinterpret_cast<A*>(smem_raw);  // [d][LD]
    A* qv = Sm + d * LD;     // [d]  q~
    A* kv = qv + d;          // [d]  m phi(k)
    A* vv = kv + d;          // [LD] v'
    A* gv = vv + LD;         // [LD] dO' (pass F: raw dO first)
    A* ov = gv + LD;         // [LD] o'
    A* red = ov + LD;        // [33]

    const T* qb = (const T*)p.q + b * p.q_sb + h * p.q_sh;
    const T* kb = (const T*)p.k + b * p.k_sb + (h / p.kvg) * p.k_sh;
    const T* vb = (const T*)p.v + b * p.v_sb + (h / p.kvg) * p.v_sh;
    const T* gb = (const T*)p.g + b * p.g_sb + h * p.g_sh;
    T* dqb = (T*)p.o + b * p.o_sb + h * p.o_sh;
    T* dkb = (T*)p.dk + b * p.dk_sb + h * p.dk_sh;
    T* dvb = (T*)p.dv + b * p.dv_sb + h * p.dv_sh;
    A* wzc = reinterpret_cast<A*>(p.ws) + bh * p.N * 3;  // clamped denominator
    A* wcz = wzc + p.N;                                  // dO'_z (the denominator's adjoint)
    A* wqp = wcz + p.N;                                  // q~ . dq~

    for (int x = threadIdx.x; x < d * ep; x += blockDim.x) {
        const int i = x / ep, j = x - i * ep;
        A v0 = 0;
        if (j < e) { if (p.S_in) v0 = p.S_in[(bh * d + i) * e + j]; }
        else if (p.z_in) v0 = p.z_in[bh * d + i];
        Sm[i * LD + j] = v0;
    }

    // ---------------- pass F ----------------
    for (int u = 0; u < p.N; ++u) {
        const int t = tok_at(p, u);
        const A m = token_mask(p, b, t);
        const A g = m > 0 ? exp_a((A)token_log_gamma(p, b, h, t)) : (A)1;
        for (int i = threadIdx.x; i < d; i += blockDim.x) {
            qv[i] = phi_f(load_a<A>(qb[(int64_t)t * p.q_sn + i])) * (A)p.scale;
            kv[i] = phi_f(load_a<A>(kb[(int64_t)t * p.k_sn + i])) * m;
        }
        for (int j = threadIdx.x; j < ep; j += blockDim.x) {
            vv[j] = j < e ? load_a<A>(vb[(int64_t)t * p.v_sn + j]) * m : m;
            gv[j] = j < e ? load_a<A>(gb[(int64_t)t * p.g_sn + j]) * m : (A)0;
        }
        __syncthreads();
        for (int x = threadIdx.x; x < d * ep; x += blockDim.x) {
            const int i = x / ep, j = x - i * ep;
            Sm[i * LD + j] = flush_small<A>(fma(g, Sm[i * LD + j], kv[i] * vv[j]), p.flush);
        }
        __syncthreads();
        for (int j = threadIdx.x; j < ep; j += blockDim.x) {
            A acc = 0;
            for (int i = 0; i < d; ++i) acc = fma(qv[i], Sm[i * LD + j], acc);
            ov[j] = acc;
        }
        __syncthreads();
        A zc = 1, cz = 0;
        if (p.normalize) {
            zc = fmax(ov[e], (A)p.clamp_min);
            A part = 0;
            for (int j = threadIdx.x; j < e; j += blockDim.x) part = fma(gv[j], ov[j], part);
            const A dot = block_sum<A>(part, red);
            cz = -dot / (zc * zc);
            for (int j = threadIdx.x; j < e; j += blockDim.x) gv[j] = gv[j] / zc;
            if (threadIdx.x == 0) gv[e] = cz;
            __syncthreads();
        }
        A qpart = 0;
        for (int i = threadIdx.x; i < d; i += blockDim.x) {
            A acc = 0;
            for (int j = 0; j < ep; ++j) acc = fma(Sm[i * LD + j], gv[j], acc);
            qpart = fma(qv[i], acc, qpart);
            const A qraw = load_a<A>(qb[(int64_t)t * p.q_sn + i]);
            dqb[(int64_t)t * p.o_sn + i] = store_a<T, A>(acc * (A)p.scale * phi_prime_f(qraw) * m);
        }
        const A qtot = block_sum<A>(qpart, red);
        if (threadIdx.x == 0) {
            wzc[t] = zc;
            wcz[t] = cz;
            wqp[t] = qtot;
        }
        __syncthreads();
    }

    // ---------------- pass R ----------------
    for (int x = threadIdx.x; x < d * LD; x += blockDim.x) Sm[x] = 0;
    A g_next = 1, run = 0;
    for (int u = p.N - 1; u >= 0; --u) {
        const int t = tok_at(p, u);
        const A m = token_mask(p, b, t);
        const A g = m > 0 ? exp_a((A)token_log_gamma(p, b, h, t)) : (A)1;
        const A zc = wzc[t];
        for (int i = threadIdx.x; i < d; i += blockDim.x) {
            qv[i] = phi_f(load_a<A>(qb[(int64_t)t * p.q_sn + i])) * (A)p.scale;
            kv[i] = phi_f(load_a<A>(kb[(int64_t)t * p.k_sn + i])) * m;
        }
        for (int j = threadIdx.x; j < ep; j += blockDim.x) {
            vv[j] = j < e ? load_a<A>(vb[(int64_t)t * p.v_sn + j]) * m : m;
            gv[j] = j < e ? load_a<A>(gb[(int64_t)t * p.g_sn + j]) * m / zc : wcz[t];
        }
        __syncthreads();
        for (int x = threadIdx.x; x < d * ep; x += blockDim.x) {
            const int i = x / ep, j = x - i * ep;
            Sm[i * LD + j] = fma(g_next, Sm[i * LD + j], qv[i] * gv[j]);
        }
        __syncthreads();
        A kpart = 0;
        for (int i = threadIdx.x; i < d; i += blockDim.x) {
            A acc = 0;
            for (int j = 0; j < ep; ++j) acc = fma(Sm[i * LD + j], vv[j], acc);
            kpart = fma(kv[i], acc, kpart);
            const A kraw = load_a<A>(kb[(int64_t)t * p.k_sn + i]);
            dkb[(int64_t)t * p.dk_sn + i] = store_a<T, A>(acc * phi_prime_f(kraw) * m);
        }
        for (int j = threadIdx.x; j < e; j += blockDim.x) {
            A acc = 0;
            for (int i = 0; i < d; ++i) acc = fma(Sm[i * LD + j], kv[i], acc);
            dvb[(int64_t)t * p.dv_sn + j] = store_a<T, A>(acc * m);
        }
        const A ktot = block_sum<A>(kpart, red);
        run += wqp[t] - ktot;
        if (p.dlg && threadIdx.x == 0) p.dlg[bh * p.N + t] = m > 0 ? (float)run : 0.f;
        g_next = g;
        __syncthreads();
    }
}

template <typename T>
__global__ void feature_map_kernel(T* x, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        x[i] = store_a<T, float>(phi_f(to_f<T>(x[i])));
}

template <typename T, typename A, int RPT>
cudaError_t launch_fwd_rpt(const ScanParams& p, cudaStream_t st) {
    const int ET = p.e < 32 ? p.e : 32;
    const int threads = (((ET + (p.normalize ? 1 : 0)) * kR) + 31) / 32 * 32;
    const int VW = ET + 1;
    const size_t smem = sizeof(A) * (2 * kCT * p.d + 2 * kCT * VW + 2 * kCT);
    auto kern = scan_fwd_exact_kernel<T, A, RPT>;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    dim3 grid((p.e + ET - 1) / ET, p.H, p.B);
    kern<<<grid, threads, smem, st>>>(p, ET);
    return cudaGetLastError();
}

template <typename T, typename A>
cudaError_t launch_fwd_t(const ScanParams& p, cudaStream_t st) {
    const int rpt = (p.d + kR - 1) / kR;
    if (rpt <= 1) return launch_fwd_rpt<T, A, 1>(p, st);
    if (rpt <= 2) return launch_fwd_rpt<T, A, 2>(p, st);
    if (rpt <= 4) return launch_fwd_rpt<T, A, 4>(p, st);
    if (rpt <= 8) return launch_fwd_rpt<T, A, 8>(p, st);
    if (rpt <= 16) return launch_fwd_rpt<T, A, 16>(p, st);
    return launch_fwd_rpt<T, A, 32>(p, st);
}

template <typename T, typename A>
cudaError_t launch_bwd_t(const ScanParams& p, cudaStream_t st) {
    const size_t smem = exact_bwd_smem_bytes(p.d, p.e, p.normalize, sizeof(A));
    auto kern = scan_bwd_exact_kernel<T, A>;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    dim3 grid(p.H, p.B);
    kern<<<grid, 256, smem, st>>>(p);
    return cudaGetLastError();
}

}  // namespace

size_t exact_bwd_smem_bytes(int d, int e, int normalize, size_t acc_bytes) {
    const int ep = e + (normalize ? 1 : 0);
    const int LD = ep | 1;
    return acc_bytes * ((size_t)d * LD + 2 * d + 3 * LD + 33);
}

cudaError_t launch_fwd_exact(const ScanParams& p, int dtype, cudaStream_t st) {
    switch (dtype) {
        case SUBQ_FP32: return launch_fwd_t<float, float>(p, st);
        case SUBQ_FP16: return launch_fwd_t<__half, float>(p, st);
        case SUBQ_FP64: return launch_fwd_t<double, double>(p, st);
        default: return launch_fwd_t<__nv_bfloat16, float>(p, st);
    }
}

cudaError_t launch_bwd_exact(const ScanParams& p, int dtype, cudaStream_t st) {
    switch (dtype) {
        case SUBQ_FP32: return launch_bwd_t<float, float>(p, st);
        case SUBQ_FP16: return launch_bwd_t<__half, float>(p, st);
        case SUBQ_FP64: return launch_bwd_t<double, double>(p, st);
        default: return launch_bwd_t<__nv_bfloat16, float>(p, st);
    }
}

// Grouped K/V: dst[b, hk, n, :] = sum over the group's query heads of
// src[b, hk * G + g, n, :] (src contiguous [B, Hkv * G, N, e]; dst strided),
// accumulated in A. The reduction autograd applies to the reference's
// repeat_interleave of K and V (python/subq_audio/autograd.py:746-748).
template <typename T, typename A>
__global__ void __launch_bounds__(256) group_sum_kernel(const T* src, T* dst, int B, int Hkv, int G, int N, int e,
                                                        int64_t dsb, int64_t dsh, int64_t dsn) {
    const int64_t total = (int64_t)B * Hkv * N * e;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % e);
        int64_t r = i / e;
        const int n = (int)(r % N);
        r /= N;
        const int hk = (int)(r % Hkv);
        const int b = (int)(r / Hkv);
        const T* s = src + (((int64_t)b * Hkv * G + (int64_t)hk * G) * N + n) * e + c;
        A acc = 0;
        for (int g = 0; g < G; ++g) acc += load_a<A>(s[(int64_t)g * N * e]);
        dst[b * dsb + hk * dsh + (int64_t)n * dsn + c] = store_a<T, A>(acc);
    }
}

template <typename T, typename A>
cudaError_t launch_group_sum_t(const void* src, void* dst, int B, int Hkv, int G, int N, int e, int64_t dsb,
                               int64_t dsh, int64_t dsn, cudaStream_t st) {
    const int64_t total = (int64_t)B * Hkv * N * e;
    if (total == 0) return cudaSuccess;
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
    group_sum_kernel<T, A><<<blocks, 256, 0, st>>>((const T*)src, (T*)dst, B, Hkv, G, N, e, dsb, dsh, dsn);
    return cudaGetLastError();
}

cudaError_t launch_group_sum(const void* src, void* dst, int dtype, int B, int Hkv, int G, int N, int e,
                             int64_t dsb, int64_t dsh, int64_t dsn, cudaStream_t st) {
    switch (dtype) {
        case SUBQ_FP32: return launch_group_sum_t<float, float>(src, dst, B, Hkv, G, N, e, dsb, dsh, dsn, st);
        case SUBQ_FP16: return launch_group_sum_t<__half, float>(src, dst, B, Hkv, G, N, e, dsb, dsh, dsn, st);
        case SUBQ_FP64: return launch_group_sum_t<double, double>(src, dst, B, Hkv, G, N, e, dsb, dsh, dsn, st);
        default: return launch_group_sum_t<__nv_bfloat16, float>(src, dst, B, Hkv, G, N, e, dsb, dsh, dsn, st);
    }
}

cudaError_t launch_feature_map(void* x, int64_t n, int dtype, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const int threads = 256;
    int64_t blocks = (n + threads - 1) / threads;
    if (blocks > 148 * 16) blocks = 148 * 16;
    switch (dtype) {
        case SUBQ_FP32: feature_map_kernel<float><<<(int)blocks, threads, 0, st>>>((float*)x, n); break;
        case SUBQ_FP16: feature_map_kernel<__half><<<(int)blocks, threads, 0, st>>>((__half*)x, n); break;
        default: feature_map_kernel<__nv_bfloat16><<<(int)blocks, threads, 0, st>>>((__nv_bfloat16*)x, n); break;
    }
    return cudaGetLastError();
}

}  // namespace subq
