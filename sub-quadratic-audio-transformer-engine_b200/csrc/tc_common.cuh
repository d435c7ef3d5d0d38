// Shared pieces of the tensor-core scan kernels (forward and backward):
// tile geometry, 16-bit element helpers, the feature map, bounded waits,
// swizzled-tile row helpers and the host-side launch plumbing.
#pragma once

#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <string.h>

#include "scan_common.cuh"
#include "scan_launch.h"
#include "tc_ptx.cuh"

namespace subq {
namespace tcs {

constexpr int kC = 128;                  // tokens per chunk (MMA M)
constexpr int kD = 64;                   // head_dim = value_dim on this path
constexpr int kThreads = 256;            // 8 warps: row = 32 * (warp % 4) + lane, column half = warp / 4
constexpr uint32_t kTile = kC * kD * 2;  // one 128 x 64 16-bit tile, 128-byte swizzle (16 KB)
constexpr uint32_t kMTile = kC * 16 * 2; // one 128 x 16 16-bit tile, 32-byte swizzle (4 KB)
constexpr uint32_t kSpinLimit = 1u << 22;

template <bool kFp16>
struct Elem;
template <>
struct Elem<false> {
    using T = __nv_bfloat16;
    using T2 = __nv_bfloat162;
    static __device__ __forceinline__ float2 to2(T2 x) { return __bfloat1622float2(x); }
    static __device__ __forceinline__ T2 from2(float a, float b) { return __floats2bfloat162_rn(a, b); }
};
template <>
struct Elem<true> {
    using T = __half;
    using T2 = __half2;
    static __device__ __forceinline__ float2 to2(T2 x) { return __half22float2(x); }
    static __device__ __forceinline__ T2 from2(float a, float b) { return __floats2half2_rn(a, b); }
};

// NaN-propagating min / max (fminf / fmaxf would return the other operand).
__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float min_nan(float a, float b) {
    float r;
    asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// phi(x) = ELU(x) + 1 = max(x, 0) + exp(min(x, 0)), with the fast exponential
// intrinsic. The branch-free form (exp(0) = 1 exactly) keeps straight-line
// code, so the element updates of a row interleave instead of serialising
// behind one exponential each; NaN propagates as in ELU.
__device__ __forceinline__ float phi_fast(float x) { return max_nan(x, 0.f) + __expf(min_nan(x, 0.f)); }

// phi on a packed pair of 16-bit values, computed in the pair's own format:
// max(x, 0) + 2^(min(x, 0) * log2(e)). The log2(e) factor is applied as two
// parts representable in the format (bf16: 1.4375 + 0.0051880; fp16:
// 1.4423828 + 0.00031233) fused into one rounding, so the exponent carries no
// systematic constant error.
template <bool kFp16>
__device__ __forceinline__ uint32_t phi2(uint32_t x);
template <>
__device__ __forceinline__ uint32_t phi2<false>(uint32_t x) {
    constexpr uint32_t kHi = 0x3FB83FB8u;  // 1.4375 (bf16 pair)
    constexpr uint32_t kLo = 0x3BAA3BAAu;  // 0.0051880 (bf16 pair); kHi + kLo = log2(e) to 2^-16
    uint32_t neg, pos, t, e, r;
    asm("min.NaN.bf16x2 %0, %1, %2;" : "=r"(neg) : "r"(x), "r"(0u));
    asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(pos) : "r"(x), "r"(0u));
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(t) : "r"(neg), "r"(kLo));
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(t) : "r"(neg), "r"(kHi), "r"(t));
    asm("ex2.approx.ftz.bf16x2 %0, %1;" : "=r"(e) : "r"(t));
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(pos), "r"(e));
    return r;
}
template <>
__device__ __forceinline__ uint32_t phi2<true>(uint32_t x) {
    constexpr uint32_t kHi = 0x3DC53DC5u;  // 1.4423828 (fp16 pair)
    constexpr uint32_t kLo = 0x0D1E0D1Eu;  // 0.00031233 (fp16 pair); kHi + kLo = log2(e) to 1e-7
    uint32_t neg, pos, t, e, r;
    asm("min.NaN.f16x2 %0, %1, %2;" : "=r"(neg) : "r"(x), "r"(0u));
    asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(pos) : "r"(x), "r"(0u));
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(t) : "r"(neg), "r"(kLo));
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(t) : "r"(neg), "r"(kHi), "r"(t));
    asm("ex2.approx.f16x2 %0, %1;" : "=r"(e) : "r"(t));
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(pos), "r"(e));
    return r;
}

// Number of leading 128-token chunks of sequence b up to and including the one
// that holds its last live token (0 for a fully masked sequence; all chunks
// without a mask). The chunks after it contribute nothing to any state and
// their outputs are zero, so the scans skip them. Every thread of the CTA
// calls this (it synchronises the block); `scratch` is one int of shared memory.
__device__ __forceinline__ int live_chunks(const ScanParams& p, int b, int nC, int* scratch) {
    if (!p.mask) return nC;
    if (threadIdx.x == 0) *scratch = -1;
    __syncthreads();
    const uint8_t* row = p.mask + (int64_t)b * p.mask_sb;
    int last = -1;
    int t0 = 0;
    if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {  // 16 tokens per load
        const int nv = p.N >> 4;
        const uint4* rv = reinterpret_cast<const uint4*>(row);
        for (int i = threadIdx.x; i < nv; i += blockDim.x) {
            const uint4 w = rv[i];
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (ws[k]) last = max(last, i * 16 + k * 4 + (31 - __clz(ws[k])) / 8);
        }
        t0 = nv << 4;
    }
    for (int t = t0 + (int)threadIdx.x; t < p.N; t += blockDim.x)
        if (row[t]) last = max(last, t);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
    if ((threadIdx.x & 31) == 0 && last >= 0) atomicMax(scratch, last);
    __syncthreads();
    const int l = *scratch;
    return l < 0 ? 0 : l / kC + 1;
}

// Work split of the segment sums. Segment s of a sequence is the chunk range
// [s cps, (s + 1) cps) of its live chunks; CTA g of the cluster needs the sum of
// phi~(K)^T [V | 1] over segments 0..g-1. The chunks [0, Ptot) before the last
// segment are summed once, by all G CTAs together: CTA r takes [a, b) (an even
// share). A share is shorter than a segment, so it crosses at most one segment
// boundary x and yields two partial sums: [a, min(b, x)) of segment seg and
// [x, b) of segment seg + 1 (empty when b <= x).
struct PrefixShare {
    int a, b, x, seg;
};
__device__ __forceinline__ PrefixShare prefix_share(int r, int G, int nL, int cps) {
    PrefixShare s;
    const int total = min(nL, (G - 1) * cps);
    s.a = (int)((int64_t)r * total / G);
    s.b = (int)((int64_t)(r + 1) * total / G);
    s.seg = cps > 0 ? s.a / cps : 0;
    s.x = (s.seg + 1) * cps;
    return s;
}

// Exchange layout of a 64 x 64 float32 partial sum read by the other CTAs of
// a cluster over DSMEM: element (row, 32 hf + x) at x * 128 + 64 hf + row, so
// that the 16 rows a warp reads for one x are 64 contiguous bytes (one
// coalesced remote access per load instruction instead of 16 scattered ones).
__device__ __forceinline__ int xch(int row, int hf, int x) { return x * 128 + hf * 64 + row; }

// Exponents of the weights of an ordered list of exchange pieces under decay:
// lane i holds lam_i, the log2 decay across piece i (0 past the list). Returns
// in lane i the sum of lam over the pieces after i (after = true) or before i
// (after = false), and in `total` the sum over all of them.
__device__ __forceinline__ float piece_exponent(float lam, int lane, bool after, float& total) {
    float t = lam;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float y = after ? __shfl_down_sync(0xffffffffu, t, o) : __shfl_up_sync(0xffffffffu, t, o);
        if (after ? (lane + o < 32) : (lane >= o)) t += y;
    }
    total = __shfl_sync(0xffffffffu, t, after ? 0 : 31);
    return t - lam;
}

// v (this thread's 32 values of exchange row `row`, column half hf) and z (the
// normaliser column, `with_z` threads) += sum_i w_i X_i over `np` pieces of
// other CTAs' exchange buffers, piece i at px(pr[i], pb[i]) and pz(pr[i],
// pb[i]) with its weight in lane i of `wl`. The two lane halves of the warp
// read alternate pieces (their remote loads overlap) and the halves' sums are
// combined, so every lane ends with the row's total; callers start half 1
// (lanes 16-31) from zero.
template <typename PX, typename PZ>
__device__ __forceinline__ void gather_pieces(int np, const int* pr, const int* pb, float wl, int row, int hf,
                                              int lane, PX px, PZ pz, bool with_z, float* v, float& z) {
    const int half = lane >> 4;
    for (int i = 0; i < np; i += 2) {
        const int my = i + half;
        const float w = __shfl_sync(0xffffffffu, wl, my & 31);
        if (my < np) {
            const float* rx = px(pr[my], pb[my]) + xch(row, hf, 0);
#pragma unroll
            for (int x = 0; x < 32; ++x) v[x] = fmaf(w, rx[x * 128], v[x]);
            if (with_z) z = fmaf(w, pz(pr[my], pb[my])[row], z);
        }
    }
#pragma unroll
    for (int x = 0; x < 32; ++x) v[x] += __shfl_xor_sync(0xffffffffu, v[x], 16);
    z += __shfl_xor_sync(0xffffffffu, z, 16);
}

// Bounded mbarrier wait; on expiry records SUBQ_ERR_TIMEOUT in *status (the
// library's device status word) and returns false.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, int* status) {
    for (uint32_t i = 0; i < kSpinLimit; ++i)
        if (tc::mbar_try_wait(bar, parity)) return true;
    atomicCAS(status, 0, (int)SUBQ_ERR_TIMEOUT);
    return false;
}

// f(j, v[8]) over the 16-byte chunks j in [j0, j0 + nj) of row r of a 128-byte
// swizzled tile, in place. All chunks are loaded before the first store, so
// the loads and the nj * 8 element updates overlap instead of running as one
// dependent chain per chunk.
template <bool kFp16, typename F>
__device__ __forceinline__ void chunks_transform(uint8_t* tile, int r, int j0, int nj, F&& f) {
    using E = Elem<kFp16>;
    uint4 raw[8];
#pragma unroll
    for (int jj = 0; jj < nj; ++jj) raw[jj] = *reinterpret_cast<const uint4*>(tile + tc::sw128_chunk(r, j0 + jj));
#pragma unroll
    for (int jj = 0; jj < nj; ++jj) {
        typename E::T2* h = reinterpret_cast<typename E::T2*>(&raw[jj]);
        float v[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f2 = E::to2(h[i]);
            v[2 * i] = f2.x;
            v[2 * i + 1] = f2.y;
        }
        f(j0 + jj, v);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = E::from2(v[2 * i], v[2 * i + 1]);
    }
#pragma unroll
    for (int jj = 0; jj < nj; ++jj) *reinterpret_cast<uint4*>(tile + tc::sw128_chunk(r, j0 + jj)) = raw[jj];
}

// Row r of a 128-byte swizzled tile, chunks [j0, j0 + nj), in place:
// phi of every element (live = true) or zeros (a masked token).
template <bool kFp16>
__device__ __forceinline__ void chunks_phi(uint8_t* tile, int r, int j0, int nj, bool live) {
    uint4 raw[8];
    if (live) {
#pragma unroll
        for (int jj = 0; jj < nj; ++jj) raw[jj] = *reinterpret_cast<const uint4*>(tile + tc::sw128_chunk(r, j0 + jj));
#pragma unroll
        for (int jj = 0; jj < nj; ++jj) {
            raw[jj].x = phi2<kFp16>(raw[jj].x);
            raw[jj].y = phi2<kFp16>(raw[jj].y);
            raw[jj].z = phi2<kFp16>(raw[jj].z);
            raw[jj].w = phi2<kFp16>(raw[jj].w);
        }
    } else {
#pragma unroll
        for (int jj = 0; jj < nj; ++jj) raw[jj] = make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int jj = 0; jj < nj; ++jj) *reinterpret_cast<uint4*>(tile + tc::sw128_chunk(r, j0 + jj)) = raw[jj];
}

// ------------------------------------------------------------ per-token decay
// Within a 128-token chunk with inclusive log-decay prefix b_t (b_t = sum of
// log gamma over tokens 0..t of the chunk; masked tokens and tokens past the
// end carry log gamma = 0, reference python/subq_audio/autograd.py:336-341 and
// :130-134), the decay between key tau and query t >= tau is exp(b_t - b_tau).
// The kernels factor it through the chunk midpoint m = 63:
//   q' = phi(q) exp(b_t - b_m),   k' = m phi(k) exp(b_m - b_tau),
// so q' k'^T = (phi(q) phi(k)^T) exp(b_t - b_tau) exactly and the causal mask,
// the tensor-core products and the epilogues keep their form; the inter-chunk
// terms take the scalars exp(b_m) (query side) and exp(b_end - b_m) (state
// side). Both factors stay within 2^kDecaySpan when each half of the chunk
// decays by at most 2^-kDecaySpan; a chunk outside that range marks its
// sequence for the exact path (the `fallback` flags), which then recomputes
// the whole sequence.
constexpr float kDecaySpan = 80.f;  // log2 units per half chunk
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float exp2_fast(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// log2 decay of token t (0 when masked or past the end).
__device__ __forceinline__ float decay_log2_at(const ScanParams& p, int b, int h, int t, float m) {
    if (t >= p.N || m == 0.f) return 0.f;
    return token_log_gamma(p, b, h, t) * kLog2e;
}
// log(gamma_t) as loaded (0 past the sequence's end), for a caller that applies
// the mask and the log2 factor where it uses the value: nothing tests or scales
// the loaded value at the load, so no instruction waits for it there.
__device__ __forceinline__ float decay_log_raw(const ScanParams& p, int b, int h, int t) {
    return t < p.N ? token_log_gamma(p, b, h, t) : 0.f;
}
// The mask byte of token t of sequence b as loaded (1 without a mask, 0 past the end).
__device__ __forceinline__ int mask_raw_at(const ScanParams& p, int b, int t) {
    int v = t < p.N ? 1 : 0;
    if (p.mask && t < p.N) v = __ldg(p.mask + (int64_t)b * p.mask_sb + t);
    return v;
}

// Inclusive scan of the chunk's log2 decay over the 128 threads of a 4-warp
// group (thread r holds token r's value a). Returns B_r; b63 and b127 receive
// B_63 and B_127, summed in the same order as the row values so that row 63
// and row 127 reproduce them exactly. `wt` is 4 floats of shared memory; the
// caller separates successive calls with a barrier of the same group.
__device__ __forceinline__ float decay_scan128(float a, int r, float* wt, int bar_id, float& b63, float& b127) {
    const int lane = r & 31, w = r >> 5;
    float x = a;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) wt[w] = x;
    tc::bar_sync(bar_id, 128);
    const float w0 = wt[0], w1 = wt[1], w2 = wt[2];
    const float p01 = w0 + w1, p012 = p01 + w2;
    b63 = p01;
    b127 = p012 + wt[3];
    const float pre = w == 0 ? 0.f : w == 1 ? w0 : w == 2 ? p01 : p012;
    return w == 0 ? x : x + pre;
}

// Reverse-time counterpart: the tokens are processed from row 127 down to
// row 0, so the prefix in processing order is B'_r = sum over rows r' >= r.
// bmid = B'_64 (the midpoint in processing order) and bend = B'_0 are summed
// in the same order as rows 64 and 0 reproduce them.
__device__ __forceinline__ float decay_scan128_rev(float a, int r, float* wt, int bar_id, float& bmid, float& bend) {
    const int lane = r & 31, w = r >> 5;
    float x = a;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_down_sync(0xffffffffu, x, o);
        if (lane + o < 32) x += y;
    }
    if (lane == 0) wt[w] = x;
    tc::bar_sync(bar_id, 128);
    const float w1 = wt[1], w2 = wt[2], w3 = wt[3];
    const float s23 = w2 + w3, s123 = w1 + s23;
    bmid = s23;
    bend = wt[0] + s123;
    const float pre = w == 3 ? 0.f : w == 2 ? w3 : w == 1 ? s23 : s123;
    return w == 3 ? x : x + pre;
}

// Whether both halves of a chunk stay within the factorisation's range (NaN
// decay passes and propagates like the reference's).
__device__ __forceinline__ bool decay_in_range(float b63, float b127) {
    return !(fabsf(b63) > kDecaySpan) && !(fabsf(b127 - b63) > kDecaySpan);
}

// Row r of a 128-byte swizzled tile, in place: f * phi of every element (live)
// or zeros (a masked token); f is applied in float32 to the feature map's
// 16-bit result.
template <bool kFp16>
__device__ __forceinline__ void chunks_phi_scaled(uint8_t* tile, int r, bool live, float f) {
    using E = Elem<kFp16>;
    uint4 raw[8];
    if (live) {
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) raw[jj] = *reinterpret_cast<const uint4*>(tile + tc::sw128_chunk(r, jj));
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
            uint32_t* w = reinterpret_cast<uint32_t*>(&raw[jj]);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                uint32_t ph = phi2<kFp16>(w[i]);
                const float2 v = E::to2(*reinterpret_cast<typename E::T2*>(&ph));
                typename E::T2 o = E::from2(v.x * f, v.y * f);
                w[i] = *reinterpret_cast<uint32_t*>(&o);
            }
        }
    } else {
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) raw[jj] = make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) *reinterpret_cast<uint4*>(tile + tc::sw128_chunk(r, jj)) = raw[jj];
}

template <bool kFp16>
__device__ __forceinline__ void store_chunk(uint8_t* tile, int r, int j, const float* v) {
    using E = Elem<kFp16>;
    uint4 raw;
    typename E::T2* h = reinterpret_cast<typename E::T2*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = E::from2(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(tile + tc::sw128_chunk(r, j)) = raw;
}

template <bool kFp16>
__device__ __forceinline__ void load_chunks(const uint8_t* tile, int r, int j0, int nj, float* out) {
    using E = Elem<kFp16>;
#pragma unroll
    for (int jj = 0; jj < nj; ++jj) {
        const uint4 raw = *reinterpret_cast<const uint4*>(tile + tc::sw128_chunk(r, j0 + jj));
        const typename E::T2* h = reinterpret_cast<const typename E::T2*>(&raw);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f2 = E::to2(h[i]);
            out[8 * jj + 2 * i] = f2.x;
            out[8 * jj + 2 * i + 1] = f2.y;
        }
    }
}

__device__ __forceinline__ void zero_chunks(uint8_t* tile, int r, int j0, int nj) {
#pragma unroll
    for (int jj = 0; jj < nj; ++jj) *reinterpret_cast<uint4*>(tile + tc::sw128_chunk(r, j0 + jj)) = make_uint4(0, 0, 0, 0);
}

// Row r of a 128 x 16 tile with a 32-byte swizzle (16-byte chunk j of row r
// lands at chunk j ^ ((r >> 2) & 1)): value x in column 0, zeros elsewhere.
template <bool kFp16>
__device__ __forceinline__ void mtile_row(uint8_t* tile, int r, float x) {
    using E = Elem<kFp16>;
    uint4 c0 = make_uint4(0, 0, 0, 0);
    typename E::T2* h = reinterpret_cast<typename E::T2*>(&c0);
    h[0] = E::from2(x, 0.f);
    const int sw = (r >> 2) & 1;
    *reinterpret_cast<uint4*>(tile + r * 32 + (sw << 4)) = c0;
    *reinterpret_cast<uint4*>(tile + r * 32 + ((sw ^ 1) << 4)) = make_uint4(0, 0, 0, 0);
}

// Row r of the same 128 x 16 tile with values x0, x1 in columns 0 and 1.
template <bool kFp16>
__device__ __forceinline__ void mtile_row2(uint8_t* tile, int r, float x0, float x1) {
    using E = Elem<kFp16>;
    uint4 c0 = make_uint4(0, 0, 0, 0);
    typename E::T2* h = reinterpret_cast<typename E::T2*>(&c0);
    h[0] = E::from2(x0, x1);
    const int sw = (r >> 2) & 1;
    *reinterpret_cast<uint4*>(tile + r * 32 + (sw << 4)) = c0;
    *reinterpret_cast<uint4*>(tile + r * 32 + ((sw ^ 1) << 4)) = make_uint4(0, 0, 0, 0);
}

// Row r of a 128 x 64 tile (128-byte swizzle) with x in column 0 and zeros in
// columns 1-15: the extra 16 columns of an N = 80 MN-major operand whose first
// 64 columns are another atom (columns 16-63 are never read).
template <bool kFp16>
__device__ __forceinline__ void atom_col0(uint8_t* tile, int r, float x) {
    using E = Elem<kFp16>;
    uint4 c0 = make_uint4(0, 0, 0, 0);
    typename E::T2* h = reinterpret_cast<typename E::T2*>(&c0);
    h[0] = E::from2(x, 0.f);
    *reinterpret_cast<uint4*>(tile + tc::sw128_chunk(r, 0)) = c0;
    *reinterpret_cast<uint4*>(tile + tc::sw128_chunk(r, 1)) = make_uint4(0, 0, 0, 0);
}

// 32-byte-swizzled MN-major operand (N = 16): SBO = 256 B between 8-row groups.
__device__ __forceinline__ uint64_t sdesc_sw32(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((512u >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((256u >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)6 << 61;
    return d;
}

__device__ __forceinline__ float tmem_ld1(uint32_t taddr) {
    uint32_t r;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    return __uint_as_float(r);
}

// ------------------------------------------------ forward -> backward handover
// The tensor-core forward fills the caller's segment_states buffer with what
// the backward of the same inputs would otherwise recompute:
//   header, 64 ints:  [0] segment count G of the forward's cluster split
//                     [1] kHandMagic  [2] B*H  [3] N  [4] flags (kHand*)
//                     [5] arrival count of the forward's CTAs (prefix pass)
//                     [6] kHandMagic once the live-chunk prefix is written
//   segment states:   per (sequence, segment) the fp32 [S | z] at the
//                     segment's start, 64 rows of 65
//   live chunks:      nL[B*H] and their exclusive prefix off[B*H + 1]
//   chunk states:     per (sequence, chunk in processing order) the bf16
//                     state operand S_c the forward's MMA read (a 64 x 64
//                     128-byte-swizzled tile, 8 KB) and z_c (64 fp32)
//   normalisers:      per token the clamped denominator Zc (fp32, [B*H, N])
// The chunk states and normalisers are written by the undecayed kernels only
// (kHandChunks); the one-pass backward needs them and the forward's output.
constexpr int kHandMagic = 0x53514834;  // "SQH4"
constexpr int kHandReverse = 1, kHandNormalize = 2, kHandDecay = 4, kHandChunks = 8;
constexpr uint32_t kSAtom = kD * kD * 2;            // bf16 64 x 64 state operand
constexpr size_t kChunkSlot = kSAtom + kD * 4 + 0;  // + z_c (64 fp32) = 8448 bytes

struct HandLayout {
    size_t seg, nl, off, chunks, zc, total;
    __host__ __device__ static size_t a256(size_t x) { return (x + 255) / 256 * 256; }
    __host__ __device__ HandLayout(int BH, int N, int G, bool chunk_data) {
        const size_t nC = (size_t)(N + kC - 1) / kC;
        seg = 256;
        nl = seg + a256((size_t)BH * G * kD * (kD + 1) * sizeof(float));
        off = nl + a256((size_t)BH * sizeof(int));
        chunks = off + a256((size_t)(BH + 1) * sizeof(int));
        zc = chunks + (chunk_data ? (size_t)BH * nC * kChunkSlot : 0);
        total = zc + (chunk_data ? a256((size_t)BH * N * sizeof(float)) : 0);
    }
};

__host__ __device__ inline int hand_flags(int reverse, int normalize, int decay_mode, bool chunks) {
    return (reverse ? kHandReverse : 0) | (normalize ? kHandNormalize : 0) | (decay_mode ? kHandDecay : 0) |
           (chunks ? kHandChunks : 0);
}

// Exclusive prefix of n ints (src) into dst[0..n], dst[n] = the total, by one
// block; `scratch` is 33 ints of shared memory. Loads bypass L1 (the values
// were written by other CTAs of the same launch).
__device__ __forceinline__ void block_prefix(const int* src, int* dst, int n, int* scratch) {
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, w = tid >> 5, nw = (nt + 31) >> 5;
    int carry = 0;
    for (int base = 0; base < n; base += nt) {
        const int i = base + tid;
        const int x = i < n ? __ldcg(src + i) : 0;
        int y = x;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, y, o);
            if (lane >= o) y += t;
        }
        if (lane == 31) scratch[w] = y;
        __syncthreads();
        if (tid == 0) {
            int acc = 0;
            for (int k = 0; k < nw; ++k) {
                const int t = scratch[k];
                scratch[k] = acc;
                acc += t;
            }
            scratch[32] = acc;
        }
        __syncthreads();
        if (i < n) dst[i] = carry + scratch[w] + y - x;
        carry += scratch[32];
        __syncthreads();
    }
    if (tid == 0) dst[n] = carry;
}

// Grid-wide work plan of the one-pass backward: the live chunks of all
// sequences, in sequence order, cut into R equal ranges; CTA r takes the
// positions [w0(r), w0(r + 1)). A range runs over pieces: the part of one
// sequence that falls in it.
struct Plan {
    const int* off;  // [BH + 1] live chunks before each sequence
    int BH, R;
    int64_t T;
    __device__ int64_t w0(int r) const { return (int64_t)r * T / R; }
    // the sequence holding position w < T (never an empty one)
    __device__ int seq_at(int64_t w) const {
        int lo = 0, hi = BH - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (__ldg(off + mid) <= w) lo = mid;
            else hi = mid - 1;
        }
        return lo;
    }
};

// Walks the chunks of one CTA's range: pieces in sequence order, the chunks
// of a piece from its last one down (processing order within the sequence).
struct Cursor {
    int s, a, e, j;  // piece: sequence s, chunks [a, e); j chunks of it done
    int64_t w, w1;   // piece start and range end (positions)
    __device__ void begin(const Plan& pl, int r) {
        w = pl.w0(r);
        w1 = pl.w0(r + 1);
        if (w < w1) piece(pl);
    }
    __device__ void piece(const Plan& pl) {
        s = pl.seq_at(w);
        const int o0 = __ldg(pl.off + s), o1 = __ldg(pl.off + s + 1);
        a = (int)(w - o0);
        e = (int)(min(w1, (int64_t)o1) - o0);
        j = 0;
    }
    __device__ int chunk() const { return e - 1 - j; }
    __device__ bool first() const { return j == 0; }
    __device__ void next(const Plan& pl) {
        if (a + ++j >= e) {
            w = __ldg(pl.off + s) + e;
            if (w < w1) piece(pl);
        }
    }
};

// Launch plumbing (scan_tc.cu).
struct Maps;
bool make_map(CUtensorMap* m, const void* base, int dtype, int N, int H, int B, int64_t sn, int64_t sh, int64_t sb);
int pick_segments(const ScanParams& p, const void* kern, int threads, size_t smem);
int* status_ptr();  // device address of the status word (current device)
int fwd_segment_count(const ScanParams& p);
int bwd1_grid(const ScanParams& p);  // CTAs of the one-pass backward
cudaError_t launch_cluster(const void* kern, int G, int BH, int threads, size_t smem, cudaStream_t st, void** args);

}  // namespace tcs
}  // namespace subq
