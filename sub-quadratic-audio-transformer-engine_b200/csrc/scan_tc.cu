// Tensor-core path of the scan for d = e = 64 with 16-bit inputs (bf16/fp16):
// chunked (128 tokens per chunk), tcgen05 MMAs with fp32 accumulation in
// TMEM, TMA tile loads/stores, and a cluster of CTAs per (batch, head)
// sequence that splits the sequence into segments and exchanges segment
// states through distributed shared memory.
//
// Per chunk c of one segment (t, tau index tokens of the chunk):
//   P      = phi(Q) phi(K)^T                       tcgen05, 128x128x64 -> TMEM
//   P     <- P * [tau <= t]; Z_t = sum_tau P + phi(q_t).z   (registers, fp32)
//   O      = phi(Q) S_c + P V                      tcgen05, 128x64x64 + 128x64x128
//   S_c+1  = S_c + phi(K)^T V                      tcgen05, 64x64x128 (TMEM-resident)
//   z_c+1  = z_c + colsum(phi(K))                  CUDA cores, fp32
//   out_t  = O_t / max(Z_t, clamp) (normalised) or O_t
// phi(Q) is scaled; phi(K) rows are multiplied by the token mask, which
// removes masked keys from P, S and z. The state S stays fp32 in TMEM across
// chunks; a bf16 copy in shared memory is the MMA operand of the next chunk.
//
// Segment prefix: CTA g of the cluster first accumulates its segment's
// sum phi(K)^T V and colsum(phi(K)) (phase 1), publishes them in its shared
// memory, and after a cluster barrier adds those of CTAs 0..g-1 (read through
// DSMEM) to the incoming state. Phase 2 then re-reads K and V (mostly from L2).
//
// Reference algorithm: python/subq_audio/autograd.py:108-169 (chunked scan,
// intra/inter split) and :292-376 (normaliser, clamp, mask); the recurrence
// is the one of src/kernels/attention_forward.cpp:42-58.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "scan_common.cuh"
#include "scan_launch.h"
#include "tc_ptx.cuh"

namespace cg = cooperative_groups;

namespace subq {

__device__ int g_tc_status;  // first error code raised by a bounded device wait

namespace {

constexpr int kC = 128;        // tokens per chunk
constexpr int kD = 64;         // head_dim = value_dim on this path
constexpr int kThreads = 128;  // one thread per chunk row / TMEM lane
constexpr int kStages = 2;     // TMA ring depth
constexpr uint32_t kTile = kC * kD * 2;  // one 128 x 64 16-bit tile (16 KB)
constexpr uint32_t kSpinLimit = 1u << 25;

struct FwdSmem {
    static constexpr uint32_t q = 0;
    static constexpr uint32_t k = q + kStages * kTile;
    static constexpr uint32_t v = k + kStages * kTile;
    static constexpr uint32_t p = v + kStages * kTile;  // P (two 64-column blocks); exchange buffer in phase 1
    static constexpr uint32_t sb = p + 2 * kTile;       // bf16 copy of S (MN-major B operand), 8 KB
    static constexpr uint32_t zc = sb + kD * kD * 2;    // running z (fp32 [64])
    static constexpr uint32_t zp = zc + kD * 4;         // column-sum partials (fp32 [2][64])
    static constexpr uint32_t bars = zp + 2 * kD * 4;   // mbarriers: tma[kStages], mma
    static constexpr uint32_t tslot = bars + 8 * (kStages + 1);
    static constexpr uint32_t total = tslot + 16;
};
static_assert(FwdSmem::p % 1024 == 0 && FwdSmem::sb % 1024 == 0, "tiles must be 1024-byte aligned");

// TMEM columns (fp32): P [0,128), O [128,192), S [192,256) (M = 64 layout).
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColP = 0, kColO = 128, kColS = 192;

struct TcFwdParams {
    CUtensorMap tm_q, tm_k, tm_v, tm_o;
    ScanParams p;
    int G;    // CTAs (segments) per sequence = cluster size
    int cps;  // chunks per segment
};

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

__device__ __forceinline__ float phi_fast(float x) { return x > 0.f ? x + 1.f : __expf(x); }

// Bounded mbarrier wait; on expiry records SUBQ_ERR_TIMEOUT and returns false.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < kSpinLimit; ++i)
        if (tc::mbar_try_wait(bar, parity)) return true;
    atomicCAS(&g_tc_status, 0, (int)SUBQ_ERR_TIMEOUT);
    return false;
}

// Applies f to the 64 values of row r of a swizzled 128 x 64 tile, in place,
// chunk by chunk; f(j, v[8]) gets the logical chunk index and 8 fp32 values.
template <bool kFp16, typename F>
__device__ __forceinline__ void row_transform(uint8_t* tile, int r, F&& f) {
    using E = Elem<kFp16>;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint4* ptr = reinterpret_cast<uint4*>(tile + tc::sw128_chunk(r, j));
        uint4 raw = *ptr;
        typename E::T2* h = reinterpret_cast<typename E::T2*>(&raw);
        float v[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 f2 = E::to2(h[i]);
            v[2 * i] = f2.x;
            v[2 * i + 1] = f2.y;
        }
        f(j, v);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = E::from2(v[2 * i], v[2 * i + 1]);
        *ptr = raw;
    }
}

// Writes 8 fp32 values as one 16-byte chunk j of row r of a swizzled tile.
template <bool kFp16>
__device__ __forceinline__ void store_chunk(uint8_t* tile, int r, int j, const float* v) {
    using E = Elem<kFp16>;
    uint4 raw;
    typename E::T2* h = reinterpret_cast<typename E::T2*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = E::from2(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(tile + tc::sw128_chunk(r, j)) = raw;
}

// Column sums of a swizzled 128 x 64 tile: thread t sums column t % 64 over
// rows [64 * (t / 64), +64) and leaves the partial in zp[t / 64][t % 64].
template <bool kFp16>
__device__ __forceinline__ void tile_colsum(const uint8_t* tile, float* zp, int tid) {
    using E = Elem<kFp16>;
    const int col = tid & 63, half = tid >> 6;
    float acc = 0.f;
    for (int r = half * 64; r < half * 64 + 64; ++r) {
        const typename E::T* e = reinterpret_cast<const typename E::T*>(tile + tc::sw128_off(r, col));
        acc += (float)(*e);
    }
    zp[half * 64 + col] = acc;
}

template <bool kFp16, bool kNorm>
__global__ void __launch_bounds__(kThreads, 1) fwd_tc_kernel(const __grid_constant__ TcFwdParams P) {
    using E = Elem<kFp16>;
    const ScanParams& p = P.p;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    cg::cluster_group cluster = cg::this_cluster();

    const int g = (int)cluster.block_rank();
    const int bh = blockIdx.y;
    const int b = bh / p.H, h = bh - b * p.H;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nC = (p.N + kC - 1) / kC;
    const int c_begin = min(nC, g * P.cps);
    const int c_end = min(nC, c_begin + P.cps);

    uint64_t* tma_bar = reinterpret_cast<uint64_t*>(sm + FwdSmem::bars);
    uint64_t* mma_bar = tma_bar + kStages;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + FwdSmem::tslot);
    float* zc = reinterpret_cast<float*>(sm + FwdSmem::zc);
    float* zp = reinterpret_cast<float*>(sm + FwdSmem::zp);
    uint8_t* Pt = sm + FwdSmem::p;
    uint8_t* Sb = sm + FwdSmem::sb;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) tc::mbar_init(&tma_bar[s], 1);
        tc::mbar_init(mma_bar, 1);
        tc::fence_mbar_init();
        tc::prefetch_tmap(&P.tm_q);
        tc::prefetch_tmap(&P.tm_k);
        tc::prefetch_tmap(&P.tm_v);
        tc::prefetch_tmap(&P.tm_o);
    }
    if (warp == 0) tc::tmem_alloc(tslot, kTmemCols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const uint32_t tP = tmem + kColP, tO = tmem + kColO, tS = tmem + kColS;

    bool ok = true;  // uniform across the CTA: every wait result is combined by __syncthreads_and
    uint32_t tma_phase[kStages] = {0, 0};
    int pending[kStages] = {0, 0};  // TMA loads issued and not yet waited for (thread 0's view)
    uint32_t mma_phase = 0;

    constexpr uint32_t idP = tc::idesc_f16<kFp16>(128, 128, false, false);  // phi(Q) phi(K)^T
    constexpr uint32_t idO = tc::idesc_f16<kFp16>(128, 64, false, true);    // X[K-major] * Y[MN-major]
    constexpr uint32_t idS = tc::idesc_f16<kFp16>(64, 64, true, true);      // phi(K)^T V
    const uint32_t sbase = tc::smem_u32(sm);

    auto issue = [&](int chunk, int s, bool with_q) {
        const int t0 = chunk * kC;
        pending[s] = 1;
        tc::mbar_arrive_expect_tx(&tma_bar[s], (with_q ? 3u : 2u) * kTile);
        if (with_q) tc::tma_load_4d(sm + FwdSmem::q + s * kTile, &P.tm_q, 0, t0, h, b, &tma_bar[s]);
        tc::tma_load_4d(sm + FwdSmem::k + s * kTile, &P.tm_k, 0, t0, h, b, &tma_bar[s]);
        tc::tma_load_4d(sm + FwdSmem::v + s * kTile, &P.tm_v, 0, t0, h, b, &tma_bar[s]);
    };
    auto row_mask = [&](int chunk, int r) -> float {
        const int t = chunk * kC + r;
        if (t >= p.N) return 0.f;
        return p.mask ? (p.mask[(int64_t)b * p.mask_sb + t] ? 1.f : 0.f) : 1.f;
    };
    // S += phi(K)^T V over one chunk (8 K-steps of 16 tokens).
    auto mma_state = [&](int s, bool first) {
        const uint32_t ka = sbase + FwdSmem::k + s * kTile, va = sbase + FwdSmem::v + s * kTile;
        for (int kk = 0; kk < 8; ++kk) {
            const uint64_t ad = tc::sdesc_sw128(ka + kk * 2048, kTile, 1024);
            const uint64_t bd = tc::sdesc_sw128(va + kk * 2048, kTile, 1024);
            tc::mma_f16(tS, ad, bd, idS, (first && kk == 0) ? 0u : 1u);
        }
    };

    // ------------------------------------------------------------ phase 1
    const bool need_agg = (g < P.G - 1);
    float* Xs = reinterpret_cast<float*>(Pt);            // [64][64] fp32 segment sum of phi(K)^T V
    float* Xz = reinterpret_cast<float*>(Pt + kD * kD * 4);  // [64] segment sum of phi(K)
    if (need_agg) {
        float zacc = 0.f;
        const int n = c_end - c_begin;
        if (tid == 0 && n > 0) issue(c_begin, 0, false);
        for (int i = 0; i < n && ok; ++i) {
            const int c = c_begin + i, s = i % kStages;
            if (tid == 0 && i + 1 < n) issue(c + 1, (i + 1) % kStages, false);
            ok = __syncthreads_and(wait_bar(&tma_bar[s], tma_phase[s]));
            tma_phase[s] ^= 1u;
            pending[s] = 0;
            if (!ok) break;
            uint8_t* kt = sm + FwdSmem::k + s * kTile;
            const float m = row_mask(c, tid);
            row_transform<kFp16>(kt, tid, [&](int, float* v) {
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = phi_fast(v[u]) * m;
            });
            tc::fence_proxy_async();
            __syncthreads();
            if (tid == 0) {
                tc::tc_fence_after();
                mma_state(s, i == 0);
                tc::mma_commit(mma_bar);
            }
            if (kNorm) {
                tile_colsum<kFp16>(kt, zp, tid);
                zacc += zp[tid];
            }
            ok = __syncthreads_and(wait_bar(mma_bar, mma_phase));
            mma_phase ^= 1u;
            tc::tc_fence_after();
        }
        // Publish the segment sums (zero for an empty segment).
        float row[64];
        if (n > 0 && ok) {
            tc::tmem_ld32(tS + lane_off + 0, row);
            tc::tmem_ld32(tS + lane_off + 32, row + 32);
        } else {
#pragma unroll
            for (int j = 0; j < 64; ++j) row[j] = 0.f;
        }
        if (lane < 16) {
            const int r = warp * 16 + lane;
#pragma unroll
            for (int j = 0; j < 64; ++j) Xs[r * 64 + j] = row[j];
        }
        zp[tid] = zacc;
        __syncthreads();
        if (tid < 64) Xz[tid] = kNorm ? zp[tid] + zp[tid + 64] : 0.f;
    }
    tc::tc_fence_before();
    cluster.sync();
    tc::tc_fence_after();

    // ------------------------------------------------------ segment prefix
    {
        float row[64];
        const int r = warp * 16 + lane;  // state row held by lanes 0..15 of each warp
        const int64_t sbase_g = ((int64_t)bh * kD + r) * kD;
#pragma unroll
        for (int j = 0; j < 64; ++j) row[j] = 0.f;
        if (lane < 16) {
            if (p.S_in) {
                for (int j = 0; j < 64; ++j) row[j] = p.S_in[sbase_g + j];
            }
            for (int src = 0; src < g; ++src) {
                const float* rx = cluster.map_shared_rank(Xs, src);
                for (int j = 0; j < 64; ++j) row[j] += rx[r * 64 + j];
            }
            // bf16 copy: MN-major B operand, row = state row (K), 64 columns (N)
#pragma unroll
            for (int j = 0; j < 8; ++j) store_chunk<kFp16>(Sb, r, j, row + 8 * j);
        }
        tc::tmem_st32(tS + lane_off + 0, row);
        tc::tmem_st32(tS + lane_off + 32, row + 32);
        if (kNorm && tid < 64) {
            float z = p.z_in ? p.z_in[(int64_t)bh * kD + tid] : 0.f;
            for (int src = 0; src < g; ++src) z += cluster.map_shared_rank(Xz, src)[tid];
            zc[tid] = z;
        }
    }
    tc::fence_proxy_async();
    tc::tc_fence_before();
    cluster.sync();  // every remote read of the exchange buffers is done
    tc::tc_fence_after();

    // ------------------------------------------------------------ phase 2
    {
        const int n = c_end - c_begin;
        if (tid == 0 && n > 0) issue(c_begin, 0, true);
        for (int i = 0; i < n && ok; ++i) {
            const int c = c_begin + i, s = i % kStages;
            if (tid == 0 && i + 1 < n) {
                tc::bulk_wait_read0();  // the output staged in that stage's Q tile has been read
                issue(c + 1, (i + 1) % kStages, true);
            }
            ok = __syncthreads_and(wait_bar(&tma_bar[s], tma_phase[s]));
            tma_phase[s] ^= 1u;
            pending[s] = 0;
            if (!ok) break;
            uint8_t* qt = sm + FwdSmem::q + s * kTile;
            uint8_t* kt = sm + FwdSmem::k + s * kTile;
            const float m = row_mask(c, tid);
            float zq = 0.f;  // scale phi(q_t) . z_c
            row_transform<kFp16>(qt, tid, [&](int j, float* v) {
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    v[u] = phi_fast(v[u]) * p.scale;
                    if (kNorm) zq = fmaf(v[u], zc[8 * j + u], zq);
                }
            });
            row_transform<kFp16>(kt, tid, [&](int, float* v) {
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = phi_fast(v[u]) * m;
            });
            tc::fence_proxy_async();
            tc::tc_fence_before();
            __syncthreads();
            const uint32_t qa = sbase + FwdSmem::q + s * kTile, ka = sbase + FwdSmem::k + s * kTile;
            const uint32_t va = sbase + FwdSmem::v + s * kTile;
            if (tid == 0) {
                tc::tc_fence_after();
                for (int kk = 0; kk < 4; ++kk) {  // P = phi(Q) phi(K)^T
                    tc::mma_f16(tP, tc::sdesc_sw128(qa + kk * 32, 16, 1024), tc::sdesc_sw128(ka + kk * 32, 16, 1024),
                                idP, kk > 0);
                }
                for (int kk = 0; kk < 4; ++kk) {  // O = phi(Q) S_c
                    tc::mma_f16(tO, tc::sdesc_sw128(qa + kk * 32, 16, 1024),
                                tc::sdesc_sw128(sbase + FwdSmem::sb + kk * 2048, 8192, 1024), idO, kk > 0);
                }
                tc::mma_commit(mma_bar);
            }
            if (kNorm) tile_colsum<kFp16>(kt, zp, tid);
            ok = __syncthreads_and(wait_bar(mma_bar, mma_phase));
            mma_phase ^= 1u;
            tc::tc_fence_after();
            if (!ok) break;
            // Causal mask on P, row sums (intra-chunk normaliser), bf16 P to shared memory.
            float zt = zq;
            for (int blk = 0; blk < 4; ++blk) {
                float v[32];
                tc::tmem_ld32(tP + lane_off + blk * 32, v);
#pragma unroll
                for (int u = 0; u < 32; ++u) {
                    const int tau = blk * 32 + u;
                    v[u] = (tau <= tid) ? v[u] : 0.f;
                    zt += v[u];
                }
                uint8_t* pblk = Pt + (blk >> 1) * kTile;
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) store_chunk<kFp16>(pblk, tid, (blk & 1) * 4 + q4, v + 8 * q4);
            }
            tc::fence_proxy_async();
            tc::tc_fence_before();
            __syncthreads();
            if (tid == 0) {
                tc::tc_fence_after();
                for (int kk = 0; kk < 8; ++kk) {  // O += P V
                    const uint32_t pa = sbase + FwdSmem::p + (kk >> 2) * kTile + (kk & 3) * 32;
                    tc::mma_f16(tO, tc::sdesc_sw128(pa, 16, 1024), tc::sdesc_sw128(va + kk * 2048, kTile, 1024),
                                idO, 1u);
                }
                mma_state(s, false);  // S += phi(K)^T V
                tc::mma_commit(mma_bar);
            }
            if (kNorm && tid < 64) zc[tid] += zp[tid] + zp[tid + 64];
            ok = __syncthreads_and(wait_bar(mma_bar, mma_phase));
            mma_phase ^= 1u;
            tc::tc_fence_after();
            if (!ok) break;
            // Epilogue: normalise, stage the output tile in this stage's Q tile.
            {
                float o[64];
                tc::tmem_ld32(tO + lane_off + 0, o);
                tc::tmem_ld32(tO + lane_off + 32, o + 32);
                const float inv = kNorm ? m / fmaxf(zt, p.clamp_min) : m;
#pragma unroll
                for (int j = 0; j < 64; ++j) o[j] *= inv;
#pragma unroll
                for (int j = 0; j < 8; ++j) store_chunk<kFp16>(qt, tid, j, o + 8 * j);
            }
            // Refresh the bf16 state operand for the next chunk.
            {
                float srow[64];
                tc::tmem_ld32(tS + lane_off + 0, srow);
                tc::tmem_ld32(tS + lane_off + 32, srow + 32);
                if (lane < 16) {
                    const int r = warp * 16 + lane;
#pragma unroll
                    for (int j = 0; j < 8; ++j) store_chunk<kFp16>(Sb, r, j, srow + 8 * j);
                }
            }
            tc::fence_proxy_async();
            tc::tc_fence_before();
            __syncthreads();
            if (tid == 0) {
                tc::tma_store_4d(&P.tm_o, qt, 0, c * kC, h, b);
                tc::bulk_commit();
            }
        }
    }

    // Final state (the last segment holds the whole sequence's state).
    if (g == P.G - 1 && ok && (p.S_out || p.z_out)) {
        float srow[64];
        tc::tmem_ld32(tS + lane_off + 0, srow);
        tc::tmem_ld32(tS + lane_off + 32, srow + 32);
        if (lane < 16 && p.S_out) {
            const int r = warp * 16 + lane;
            for (int j = 0; j < 64; ++j) p.S_out[((int64_t)bh * kD + r) * kD + j] = srow[j];
        }
        if (p.z_out && tid < 64) p.z_out[(int64_t)bh * kD + tid] = kNorm ? zc[tid] : 0.f;
    }
    if (tid == 0) {
        // Loads still in flight after an error are drained (bounded) before exit.
        for (int s = 0; s < kStages; ++s)
            if (pending[s]) wait_bar(&tma_bar[s], tma_phase[s]);
        tc::bulk_wait0();
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, kTmemCols);
}

// ===================================================================
// Backward. One cluster of G CTAs per (batch, head) sequence; CTA g owns
// segment g. With q~ = scale phi(q), k~ = m phi(k), Zc_t = max(Z_t, clamp):
//   o^_t = m_t dO_t / Zc_t,   c_t = -(m_t dO_t . num_t) / Zc_t^2   (quotient rule)
//   dA   = (O^ V^T + c m^T) * [tau <= t]                 (per chunk, 128 x 128)
//   dQ~  = dA K~ + O^ S_c^T + c z_c^T                    (S_c, z_c: prefix state)
//   dK~  = dA^T Q~ + V dS_c^T + m dz_c^T                 (dS_c, dz_c: suffix adjoint)
//   dV   = (P * [tau <= t])^T O^ + K~ dS_c
//   dS_c-1 = dS_c + Q~^T O^,  dz_c-1 = dz_c + Q~^T c
// then dq = dQ~ scale phi'(q), dk = dK~ phi'(k) m, dv = dV m, with
// phi'(x) = min(phi(x), 1). Phases:
//   A  segment sums of K~^T V and colsum K~ (g < G-1) -> DSMEM -> S_c, z_c prefix
//   B  chunks ascending: recompute num and Z, build O^ and c, emit dq, store
//      (Zc_t, c_t) per token in the workspace, accumulate the segment's
//      Q~^T O^ and Q~^T c
//   -> DSMEM -> dS, dz suffix of the segment
//   C  chunks descending: rebuild O^ from dO and (Zc, c), emit dk and dv.
// Reference: python/subq_audio/autograd.py:441-544 (quotient rule :497-499,
// adjoint scan :172-289) and src/kernels/attention_backward.cpp:165-229.
// ===================================================================
struct BwdSmem {
    static constexpr uint32_t stage = 4 * kTile;  // q, k, v, dO
    static constexpr uint32_t q = 0, k = kTile, v = 2 * kTile, g = 3 * kTile;
    static constexpr uint32_t p = kStages * stage;     // P, 2 blocks (also the exchange buffer)
    static constexpr uint32_t da = p + 2 * kTile;      // dA, 2 blocks
    static constexpr uint32_t ob = da + 2 * kTile;     // O^ tile [t][e]
    static constexpr uint32_t sb = ob + kTile;         // bf16 S_c (phase B) / dS_c (phase C)
    static constexpr uint32_t zc = sb + kD * kD * 2;   // z_c (B) / dz_c (C), fp32 [64]
    static constexpr uint32_t zp = zc + kD * 4;        // partial column sums [2][64]
    static constexpr uint32_t cb = zp + 2 * kD * 4;    // c_t [128]
    static constexpr uint32_t mb = cb + kC * 4;        // m_t [128]
    static constexpr uint32_t bars = mb + kC * 4;
    static constexpr uint32_t tslot = bars + 8 * (kStages + 1);
    static constexpr uint32_t total = tslot + 16;
};
static_assert(BwdSmem::p % 1024 == 0 && BwdSmem::da % 1024 == 0 && BwdSmem::ob % 1024 == 0 &&
                  BwdSmem::sb % 1024 == 0,
              "tiles must be 1024-byte aligned");

// TMEM columns: P [0,128), dA [128,256), X1 [256,320), X2 [320,384),
// S [384,448) and dS [448,512) (both M = 64 layout).
constexpr uint32_t kBwdTmemCols = 512;
constexpr uint32_t kBP = 0, kBdA = 128, kBX1 = 256, kBX2 = 320, kBS = 384, kBdS = 448;

struct TcBwdParams {
    CUtensorMap tm_q, tm_k, tm_v, tm_g, tm_dq, tm_dk, tm_dv;
    ScanParams p;
    int G;
    int cps;
};

// Weighted column sums of a swizzled 128 x 64 tile: zp[half][col] = sum_r tile[r][col] * w[r].
template <bool kFp16>
__device__ __forceinline__ void tile_colsum_w(const uint8_t* tile, const float* w, float* zp, int tid) {
    using E = Elem<kFp16>;
    const int col = tid & 63, half = tid >> 6;
    float acc = 0.f;
    for (int r = half * 64; r < half * 64 + 64; ++r) {
        const typename E::T* e = reinterpret_cast<const typename E::T*>(tile + tc::sw128_off(r, col));
        acc = fmaf((float)(*e), w[r], acc);
    }
    zp[half * 64 + col] = acc;
}

// Reads the 64 values of row r of a swizzled tile into fp32.
template <bool kFp16>
__device__ __forceinline__ void load_row(const uint8_t* tile, int r, float* out) {
    using E = Elem<kFp16>;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint4 raw = *reinterpret_cast<const uint4*>(tile + tc::sw128_chunk(r, j));
        const typename E::T2* h = reinterpret_cast<const typename E::T2*>(&raw);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 f2 = E::to2(h[i]);
            out[8 * j + 2 * i] = f2.x;
            out[8 * j + 2 * i + 1] = f2.y;
        }
    }
}

template <bool kFp16, bool kNorm>
__global__ void __launch_bounds__(kThreads, 1) bwd_tc_kernel(const __grid_constant__ TcBwdParams P) {
    const ScanParams& p = P.p;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    cg::cluster_group cluster = cg::this_cluster();

    const int g = (int)cluster.block_rank();
    const int bh = blockIdx.y;
    const int b = bh / p.H, h = bh - b * p.H;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nC = (p.N + kC - 1) / kC;
    const int c_begin = min(nC, g * P.cps);
    const int c_end = min(nC, c_begin + P.cps);
    const int n = c_end - c_begin;

    uint64_t* tma_bar = reinterpret_cast<uint64_t*>(sm + BwdSmem::bars);
    uint64_t* mma_bar = tma_bar + kStages;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + BwdSmem::tslot);
    float* zc = reinterpret_cast<float*>(sm + BwdSmem::zc);
    float* zp = reinterpret_cast<float*>(sm + BwdSmem::zp);
    float* cb = reinterpret_cast<float*>(sm + BwdSmem::cb);
    float* mb = reinterpret_cast<float*>(sm + BwdSmem::mb);
    uint8_t* Pt = sm + BwdSmem::p;
    uint8_t* dAt = sm + BwdSmem::da;
    uint8_t* Ot = sm + BwdSmem::ob;
    uint8_t* Sb = sm + BwdSmem::sb;
    float2* wsz = reinterpret_cast<float2*>(p.ws) + (int64_t)bh * p.N;  // (Zc_t, c_t) per token

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) tc::mbar_init(&tma_bar[s], 1);
        tc::mbar_init(mma_bar, 1);
        tc::fence_mbar_init();
    }
    if (warp == 0) tc::tmem_alloc(tslot, kBwdTmemCols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const uint32_t tP = tmem + kBP, tdA = tmem + kBdA, tX1 = tmem + kBX1, tX2 = tmem + kBX2;
    const uint32_t tS = tmem + kBS, tdS = tmem + kBdS;
    const uint32_t sbase = tc::smem_u32(sm);

    bool ok = true;
    uint32_t tma_phase[kStages] = {0, 0};
    int pending[kStages] = {0, 0};
    uint32_t mma_phase = 0;

    constexpr uint32_t id128_KK = tc::idesc_f16<kFp16>(128, 128, false, false);
    constexpr uint32_t id64_KM = tc::idesc_f16<kFp16>(128, 64, false, true);
    constexpr uint32_t id64_KK = tc::idesc_f16<kFp16>(128, 64, false, false);
    constexpr uint32_t id64_MM = tc::idesc_f16<kFp16>(128, 64, true, true);
    constexpr uint32_t idS_MM = tc::idesc_f16<kFp16>(64, 64, true, true);

    auto stage_addr = [&](int s, uint32_t which) { return sbase + s * BwdSmem::stage + which; };
    auto stage_ptr = [&](int s, uint32_t which) { return sm + s * BwdSmem::stage + which; };
    auto issue = [&](int chunk, int s, bool full) {
        const int t0 = chunk * kC;
        pending[s] = 1;
        tc::mbar_arrive_expect_tx(&tma_bar[s], (full ? 4u : 2u) * kTile);
        if (full) {
            tc::tma_load_4d(stage_ptr(s, BwdSmem::q), &P.tm_q, 0, t0, h, b, &tma_bar[s]);
            tc::tma_load_4d(stage_ptr(s, BwdSmem::g), &P.tm_g, 0, t0, h, b, &tma_bar[s]);
        }
        tc::tma_load_4d(stage_ptr(s, BwdSmem::k), &P.tm_k, 0, t0, h, b, &tma_bar[s]);
        tc::tma_load_4d(stage_ptr(s, BwdSmem::v), &P.tm_v, 0, t0, h, b, &tma_bar[s]);
    };
    auto row_mask = [&](int chunk, int r) -> float {
        const int t = chunk * kC + r;
        if (t >= p.N) return 0.f;
        return p.mask ? (p.mask[(int64_t)b * p.mask_sb + t] ? 1.f : 0.f) : 1.f;
    };
    auto wait_mma = [&]() {
        ok = __syncthreads_and(wait_bar(mma_bar, mma_phase)) && ok;
        mma_phase ^= 1u;
        tc::tc_fence_after();
    };
    auto sync_for_mma = [&]() {
        tc::fence_proxy_async();
        tc::tc_fence_before();
        __syncthreads();
    };
    // acc (+)= X^T Y over 128 tokens: X, Y are [128][64] tiles read MN-major (M=64 layout).
    auto mma_xty = [&](uint32_t dst, uint32_t xa, uint32_t ya, bool first) {
        for (int kk = 0; kk < 8; ++kk)
            tc::mma_f16(dst, tc::sdesc_sw128(xa + kk * 2048, kTile, 1024), tc::sdesc_sw128(ya + kk * 2048, kTile, 1024),
                        idS_MM, (first && kk == 0) ? 0u : 1u);
    };
    // Causal-masked 128 x 128 tile from TMEM to bf16 shared memory (two 64-column blocks),
    // optionally adding c_t m_tau and returning the row sum.
    auto tile_out = [&](uint32_t tsrc, uint8_t* dst, bool add_cm, float ct) -> float {
        float rs = 0.f;
        for (int blk = 0; blk < 4; ++blk) {
            float v[32];
            tc::tmem_ld32(tsrc + lane_off + blk * 32, v);
#pragma unroll
            for (int u = 0; u < 32; ++u) {
                const int tau = blk * 32 + u;
                float x = add_cm ? fmaf(ct, mb[tau], v[u]) : v[u];
                x = (tau <= tid) ? x : 0.f;
                rs += x;
                v[u] = x;
            }
            uint8_t* pb = dst + (blk >> 1) * kTile;
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) store_chunk<kFp16>(pb, tid, (blk & 1) * 4 + q4, v + 8 * q4);
        }
        return rs;
    };
    // M = 64 state (TMEM) -> bf16 shared-memory copy (row = state row).
    auto refresh_state_copy = [&](uint32_t tsrc) {
        float srow[64];
        tc::tmem_ld32(tsrc + lane_off + 0, srow);
        tc::tmem_ld32(tsrc + lane_off + 32, srow + 32);
        if (lane < 16) {
            const int r = warp * 16 + lane;
#pragma unroll
            for (int j = 0; j < 8; ++j) store_chunk<kFp16>(Sb, r, j, srow + 8 * j);
        }
    };
    // Writes a 64 x 64 fp32 state into TMEM (M = 64 layout) and its bf16 copy.
    auto load_state = [&](uint32_t tdst, float* row) {
        if (lane < 16) {
            const int r = warp * 16 + lane;
#pragma unroll
            for (int j = 0; j < 8; ++j) store_chunk<kFp16>(Sb, r, j, row + 8 * j);
        }
        tc::tmem_st32(tdst + lane_off + 0, row);
        tc::tmem_st32(tdst + lane_off + 32, row + 32);
    };

    float* Xs = reinterpret_cast<float*>(Pt);
    float* Xz = reinterpret_cast<float*>(Pt + kD * kD * 4);

    // ------------------------------------------------------------ phase A
    if (g < P.G - 1) {
        float zacc = 0.f;
        if (tid == 0 && n > 0) issue(c_begin, 0, false);
        for (int i = 0; i < n && ok; ++i) {
            const int c = c_begin + i, s = i % kStages;
            if (tid == 0 && i + 1 < n) issue(c + 1, (i + 1) % kStages, false);
            ok = __syncthreads_and(wait_bar(&tma_bar[s], tma_phase[s]));
            tma_phase[s] ^= 1u;
            pending[s] = 0;
            if (!ok) break;
            uint8_t* kt = stage_ptr(s, BwdSmem::k);
            const float m = row_mask(c, tid);
            row_transform<kFp16>(kt, tid, [&](int, float* v) {
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = phi_fast(v[u]) * m;
            });
            sync_for_mma();
            if (tid == 0) {
                tc::tc_fence_after();
                mma_xty(tS, stage_addr(s, BwdSmem::k), stage_addr(s, BwdSmem::v), i == 0);
                tc::mma_commit(mma_bar);
            }
            if (kNorm) {
                tile_colsum<kFp16>(kt, zp, tid);
                zacc += zp[tid];
            }
            wait_mma();
        }
        float row[64];
        if (n > 0 && ok) {
            tc::tmem_ld32(tS + lane_off + 0, row);
            tc::tmem_ld32(tS + lane_off + 32, row + 32);
        } else {
#pragma unroll
            for (int j = 0; j < 64; ++j) row[j] = 0.f;
        }
        if (lane < 16) {
            const int r = warp * 16 + lane;
#pragma unroll
            for (int j = 0; j < 64; ++j) Xs[r * 64 + j] = row[j];
        }
        zp[tid] = zacc;
        __syncthreads();
        if (tid < 64) Xz[tid] = kNorm ? zp[tid] + zp[tid + 64] : 0.f;
    }
    tc::tc_fence_before();
    cluster.sync();
    tc::tc_fence_after();
    {
        float row[64];
        const int r = warp * 16 + lane;
#pragma unroll
        for (int j = 0; j < 64; ++j) row[j] = 0.f;
        if (lane < 16) {
            if (p.S_in)
                for (int j = 0; j < 64; ++j) row[j] = p.S_in[((int64_t)bh * kD + r) * kD + j];
            for (int src = 0; src < g; ++src) {
                const float* rx = cluster.map_shared_rank(Xs, src);
                for (int j = 0; j < 64; ++j) row[j] += rx[r * 64 + j];
            }
        }
        load_state(tS, row);
        if (kNorm && tid < 64) {
            float z = p.z_in ? p.z_in[(int64_t)bh * kD + tid] : 0.f;
            for (int src = 0; src < g; ++src) z += cluster.map_shared_rank(Xz, src)[tid];
            zc[tid] = z;
        }
    }
    tc::fence_proxy_async();
    tc::tc_fence_before();
    cluster.sync();
    tc::tc_fence_after();

    // ------------------------------------------------------------ phase B
    float dzacc = 0.f;  // this thread's column partial of Q~^T c over the segment
    if (tid == 0 && n > 0) issue(c_begin, 0, true);
    for (int i = 0; i < n && ok; ++i) {
        const int c = c_begin + i, s = i % kStages;
        if (tid == 0 && i + 1 < n) {
            tc::bulk_wait_read0();
            issue(c + 1, (i + 1) % kStages, true);
        }
        ok = __syncthreads_and(wait_bar(&tma_bar[s], tma_phase[s]));
        tma_phase[s] ^= 1u;
        pending[s] = 0;
        if (!ok) break;
        uint8_t* qt = stage_ptr(s, BwdSmem::q);
        uint8_t* kt = stage_ptr(s, BwdSmem::k);
        const float m = row_mask(c, tid);
        mb[tid] = m;
        float zq = 0.f;
        row_transform<kFp16>(qt, tid, [&](int j, float* v) {
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                v[u] = phi_fast(v[u]) * p.scale;
                if (kNorm) zq = fmaf(v[u], zc[8 * j + u], zq);
            }
        });
        row_transform<kFp16>(kt, tid, [&](int, float* v) {
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = phi_fast(v[u]) * m;
        });
        sync_for_mma();
        const uint32_t qa = stage_addr(s, BwdSmem::q), ka = stage_addr(s, BwdSmem::k);
        const uint32_t va = stage_addr(s, BwdSmem::v);
        if (tid == 0) {
            tc::tc_fence_after();
            for (int kk = 0; kk < 4; ++kk)  // P = Q~ K~^T
                tc::mma_f16(tP, tc::sdesc_sw128(qa + kk * 32, 16, 1024), tc::sdesc_sw128(ka + kk * 32, 16, 1024),
                            id128_KK, kk > 0);
            for (int kk = 0; kk < 4; ++kk)  // num = Q~ S_c
                tc::mma_f16(tX1, tc::sdesc_sw128(qa + kk * 32, 16, 1024),
                            tc::sdesc_sw128(sbase + BwdSmem::sb + kk * 2048, 8192, 1024), id64_KM, kk > 0);
            tc::mma_commit(mma_bar);
        }
        wait_mma();
        if (!ok) break;
        const float Zt = tile_out(tP, Pt, false, 0.f) + zq;
        sync_for_mma();
        if (tid == 0) {
            tc::tc_fence_after();
            for (int kk = 0; kk < 8; ++kk) {  // num += P V
                const uint32_t pa = sbase + BwdSmem::p + (kk >> 2) * kTile + (kk & 3) * 32;
                tc::mma_f16(tX1, tc::sdesc_sw128(pa, 16, 1024), tc::sdesc_sw128(va + kk * 2048, kTile, 1024), id64_KM,
                            1u);
            }
            tc::mma_commit(mma_bar);
        }
        wait_mma();
        if (!ok) break;
        // O^ and c (quotient rule); (Zc, c) go to the workspace for phase C.
        float ct = 0.f;
        {
            float num[64], go[64];
            tc::tmem_ld32(tX1 + lane_off + 0, num);
            tc::tmem_ld32(tX1 + lane_off + 32, num + 32);
            load_row<kFp16>(stage_ptr(s, BwdSmem::g), tid, go);
            const float zcl = kNorm ? fmaxf(Zt, p.clamp_min) : 1.f;
            const float inv = m / zcl;
            float dot = 0.f;
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                dot = fmaf(go[j] * m, num[j], dot);
                go[j] *= inv;
            }
            ct = kNorm ? -dot / (zcl * zcl) : 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) store_chunk<kFp16>(Ot, tid, j, go + 8 * j);
            if (c * kC + tid < p.N) wsz[c * kC + tid] = make_float2(zcl, ct);
        }
        cb[tid] = ct;
        sync_for_mma();
        if (tid == 0) {
            tc::tc_fence_after();
            for (int kk = 0; kk < 4; ++kk)  // dA = O^ V^T
                tc::mma_f16(tdA, tc::sdesc_sw128(sbase + BwdSmem::ob + kk * 32, 16, 1024),
                            tc::sdesc_sw128(va + kk * 32, 16, 1024), id128_KK, kk > 0);
            mma_xty(tdS, qa, sbase + BwdSmem::ob, i == 0);  // segment sum of Q~^T O^
            mma_xty(tS, ka, va, false);                      // S_c+1 = S_c + K~^T V
            tc::mma_commit(mma_bar);
        }
        if (kNorm) tile_colsum_w<kFp16>(qt, cb, zp, tid);  // this chunk's Q~^T c
        wait_mma();
        if (!ok) break;
        tile_out(tdA, dAt, kNorm, ct);
        sync_for_mma();
        if (tid == 0) {
            tc::tc_fence_after();
            for (int kk = 0; kk < 8; ++kk) {  // dQ~ = dA K~
                const uint32_t aa = sbase + BwdSmem::da + (kk >> 2) * kTile + (kk & 3) * 32;
                tc::mma_f16(tX2, tc::sdesc_sw128(aa, 16, 1024), tc::sdesc_sw128(ka + kk * 2048, kTile, 1024), id64_KM,
                            kk > 0);
            }
            for (int kk = 0; kk < 4; ++kk)  // dQ~ += O^ S_c^T
                tc::mma_f16(tX2, tc::sdesc_sw128(sbase + BwdSmem::ob + kk * 32, 16, 1024),
                            tc::sdesc_sw128(sbase + BwdSmem::sb + kk * 32, 16, 1024), id64_KK, 1u);
            tc::mma_commit(mma_bar);
        }
        wait_mma();
        if (!ok) break;
        {
            float dq[64], qr[64];
            tc::tmem_ld32(tX2 + lane_off + 0, dq);
            tc::tmem_ld32(tX2 + lane_off + 32, dq + 32);
            load_row<kFp16>(qt, tid, qr);
            const float inv_scale = 1.f / p.scale;
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                float x = kNorm ? fmaf(ct, zc[j], dq[j]) : dq[j];
                x *= p.scale * fminf(qr[j] * inv_scale, 1.f) * m;
                dq[j] = x;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) store_chunk<kFp16>(qt, tid, j, dq + 8 * j);
        }
        if (kNorm) dzacc += zp[tid];
        __syncthreads();
        // z_c+1 = z_c + colsum(K~): recompute the K~ column sums (zp was reused above).
        if (kNorm) {
            tile_colsum<kFp16>(kt, zp, tid);
            __syncthreads();
            if (tid < 64) zc[tid] += zp[tid] + zp[tid + 64];
        }
        refresh_state_copy(tS);
        sync_for_mma();
        if (tid == 0) {
            tc::tma_store_4d(&P.tm_dq, qt, 0, c * kC, h, b);
            tc::bulk_commit();
        }
    }

    // --------------------------------------------- suffix exchange (dS, dz)
    {
        float row[64];
        if (n > 0 && ok) {
            tc::tmem_ld32(tdS + lane_off + 0, row);
            tc::tmem_ld32(tdS + lane_off + 32, row + 32);
        } else {
#pragma unroll
            for (int j = 0; j < 64; ++j) row[j] = 0.f;
        }
        if (tid == 0) tc::bulk_wait_read0();
        tc::tc_fence_before();
        __syncthreads();
        if (lane < 16) {
            const int r = warp * 16 + lane;
#pragma unroll
            for (int j = 0; j < 64; ++j) Xs[r * 64 + j] = row[j];
        }
        zp[tid] = dzacc;
        __syncthreads();
        if (tid < 64) Xz[tid] = kNorm ? zp[tid] + zp[tid + 64] : 0.f;
    }
    cluster.sync();
    tc::tc_fence_after();
    {
        float row[64];
        const int r = warp * 16 + lane;
#pragma unroll
        for (int j = 0; j < 64; ++j) row[j] = 0.f;
        if (lane < 16) {
            for (int src = g + 1; src < P.G; ++src) {
                const float* rx = cluster.map_shared_rank(Xs, src);
                for (int j = 0; j < 64; ++j) row[j] += rx[r * 64 + j];
            }
        }
        float dz = 0.f;
        if (kNorm && tid < 64)
            for (int src = g + 1; src < P.G; ++src) dz += cluster.map_shared_rank(Xz, src)[tid];
        tc::tc_fence_before();
        cluster.sync();  // remote reads finished before the buffers are reused
        tc::tc_fence_after();
        load_state(tdS, row);
        if (tid < 64) zc[tid] = dz;
    }
    tc::fence_proxy_async();
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();

    // ------------------------------------------------------------ phase C
    if (tid == 0 && n > 0) issue(c_end - 1, 0, true);
    for (int i = 0; i < n && ok; ++i) {
        const int c = c_end - 1 - i, s = i % kStages;
        if (tid == 0 && i + 1 < n) {
            tc::bulk_wait_read0();
            issue(c - 1, (i + 1) % kStages, true);
        }
        ok = __syncthreads_and(wait_bar(&tma_bar[s], tma_phase[s]));
        tma_phase[s] ^= 1u;
        pending[s] = 0;
        if (!ok) break;
        uint8_t* qt = stage_ptr(s, BwdSmem::q);
        uint8_t* kt = stage_ptr(s, BwdSmem::k);
        uint8_t* vt = stage_ptr(s, BwdSmem::v);
        const float m = row_mask(c, tid);
        mb[tid] = m;
        float2 zcc = make_float2(1.f, 0.f);
        if (c * kC + tid < p.N) zcc = wsz[c * kC + tid];
        const float ct = zcc.y;
        cb[tid] = ct;
        row_transform<kFp16>(qt, tid, [&](int, float* v) {
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = phi_fast(v[u]) * p.scale;
        });
        row_transform<kFp16>(kt, tid, [&](int, float* v) {
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = phi_fast(v[u]) * m;
        });
        {
            float go[64];
            load_row<kFp16>(stage_ptr(s, BwdSmem::g), tid, go);
            const float inv = m / zcc.x;
#pragma unroll
            for (int j = 0; j < 64; ++j) go[j] *= inv;
#pragma unroll
            for (int j = 0; j < 8; ++j) store_chunk<kFp16>(Ot, tid, j, go + 8 * j);
        }
        sync_for_mma();
        const uint32_t qa = stage_addr(s, BwdSmem::q), ka = stage_addr(s, BwdSmem::k);
        const uint32_t va = stage_addr(s, BwdSmem::v);
        if (tid == 0) {
            tc::tc_fence_after();
            for (int kk = 0; kk < 4; ++kk) {
                tc::mma_f16(tP, tc::sdesc_sw128(qa + kk * 32, 16, 1024), tc::sdesc_sw128(ka + kk * 32, 16, 1024),
                            id128_KK, kk > 0);
                tc::mma_f16(tdA, tc::sdesc_sw128(sbase + BwdSmem::ob + kk * 32, 16, 1024),
                            tc::sdesc_sw128(va + kk * 32, 16, 1024), id128_KK, kk > 0);
            }
            tc::mma_commit(mma_bar);
        }
        wait_mma();
        if (!ok) break;
        tile_out(tP, Pt, false, 0.f);
        tile_out(tdA, dAt, kNorm, ct);
        sync_for_mma();
        if (tid == 0) {
            tc::tc_fence_after();
            for (int kk = 0; kk < 8; ++kk) {  // dK~ = dA^T Q~ ; dV = P^T O^  (A read MN-major, M = 128)
                tc::mma_f16(tX1, tc::sdesc_sw128(sbase + BwdSmem::da + kk * 2048, kTile, 1024),
                            tc::sdesc_sw128(qa + kk * 2048, kTile, 1024), id64_MM, kk > 0);
                tc::mma_f16(tX2, tc::sdesc_sw128(sbase + BwdSmem::p + kk * 2048, kTile, 1024),
                            tc::sdesc_sw128(sbase + BwdSmem::ob + kk * 2048, kTile, 1024), id64_MM, kk > 0);
            }
            for (int kk = 0; kk < 4; ++kk) {
                // dK~ += V dS_c^T
                tc::mma_f16(tX1, tc::sdesc_sw128(va + kk * 32, 16, 1024),
                            tc::sdesc_sw128(sbase + BwdSmem::sb + kk * 32, 16, 1024), id64_KK, 1u);
                // dV += K~ dS_c
                tc::mma_f16(tX2, tc::sdesc_sw128(ka + kk * 32, 16, 1024),
                            tc::sdesc_sw128(sbase + BwdSmem::sb + kk * 2048, 8192, 1024), id64_KM, 1u);
            }
            mma_xty(tdS, qa, sbase + BwdSmem::ob, false);  // dS_c-1 = dS_c + Q~^T O^
            tc::mma_commit(mma_bar);
        }
        if (kNorm) tile_colsum_w<kFp16>(qt, cb, zp, tid);
        wait_mma();
        if (!ok) break;
        {
            float acc[64], kr[64];
            tc::tmem_ld32(tX1 + lane_off + 0, acc);
            tc::tmem_ld32(tX1 + lane_off + 32, acc + 32);
            load_row<kFp16>(kt, tid, kr);
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                float x = kNorm ? fmaf(m, zc[j], acc[j]) : acc[j];
                acc[j] = x * fminf(kr[j], 1.f) * m;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) store_chunk<kFp16>(kt, tid, j, acc + 8 * j);
            tc::tmem_ld32(tX2 + lane_off + 0, acc);
            tc::tmem_ld32(tX2 + lane_off + 32, acc + 32);
#pragma unroll
            for (int j = 0; j < 64; ++j) acc[j] *= m;
#pragma unroll
            for (int j = 0; j < 8; ++j) store_chunk<kFp16>(vt, tid, j, acc + 8 * j);
        }
        __syncthreads();
        if (kNorm && tid < 64) zc[tid] += zp[tid] + zp[tid + 64];
        refresh_state_copy(tdS);
        sync_for_mma();
        if (tid == 0) {
            tc::tma_store_4d(&P.tm_dk, kt, 0, c * kC, h, b);
            tc::tma_store_4d(&P.tm_dv, vt, 0, c * kC, h, b);
            tc::bulk_commit();
        }
    }

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s)
            if (pending[s]) wait_bar(&tma_bar[s], tma_phase[s]);
        tc::bulk_wait0();
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, kBwdTmemCols);
}

// ------------------------------------------------------------------- host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

// [B, H, N, 64] 16-bit tensor, box 64 x 128 tokens, 128-byte swizzle.
bool make_map(CUtensorMap* m, const void* base, int dtype, int N, int H, int B, int64_t sn, int64_t sh,
              int64_t sb) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    if (H == 1) sh = sn * (int64_t)(N > 0 ? N : 1);
    if (B == 1) sb = sh * H;
    cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)N, (cuuint64_t)H, (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)sn * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
    cuuint32_t box[4] = {(cuuint32_t)kD, (cuuint32_t)kC, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(m, dtype == SUBQ_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                     const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool strides_ok(int64_t sb, int64_t sh, int64_t sn, const void* ptr) {
    return (reinterpret_cast<uintptr_t>(ptr) % 16 == 0) && sn % 8 == 0 && sh % 8 == 0 && sb % 8 == 0 && sn >= kD &&
           sn * 2 < ((int64_t)1 << 40) && sh * 2 < ((int64_t)1 << 40) && sb * 2 < ((int64_t)1 << 40);
}

int num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

int pick_segments(const ScanParams& p) {
    const int nC = (p.N + kC - 1) / kC;
    const int bh = p.B * p.H;
    int G = 1;
    while (G < 8 && bh * G * 2 <= num_sms() && G * 2 <= nC) G *= 2;
    return G;
}

template <bool kFp16, bool kNorm>
cudaError_t launch_fwd_impl(const ScanParams& p, cudaStream_t st) {
    TcFwdParams P;
    memset(&P, 0, sizeof(P));
    P.p = p;
    if (!make_map(&P.tm_q, p.q, kFp16 ? SUBQ_FP16 : SUBQ_BF16, p.N, p.H, p.B, p.q_sn, p.q_sh, p.q_sb) ||
        !make_map(&P.tm_k, p.k, kFp16 ? SUBQ_FP16 : SUBQ_BF16, p.N, p.H, p.B, p.k_sn, p.k_sh, p.k_sb) ||
        !make_map(&P.tm_v, p.v, kFp16 ? SUBQ_FP16 : SUBQ_BF16, p.N, p.H, p.B, p.v_sn, p.v_sh, p.v_sb) ||
        !make_map(&P.tm_o, p.o, kFp16 ? SUBQ_FP16 : SUBQ_BF16, p.N, p.H, p.B, p.o_sn, p.o_sh, p.o_sb))
        return cudaErrorInvalidValue;
    const int nC = (p.N + kC - 1) / kC;
    P.G = pick_segments(p);
    P.cps = (nC + P.G - 1) / P.G;
    auto kern = fwd_tc_kernel<kFp16, kNorm>;
    const size_t smem = FwdSmem::total + 1024;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(P.G, p.B * p.H, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = P.G;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, P);
}

template <bool kFp16, bool kNorm>
cudaError_t launch_bwd_impl(const ScanParams& p, cudaStream_t st) {
    TcBwdParams P;
    memset(&P, 0, sizeof(P));
    P.p = p;
    const int dt = kFp16 ? SUBQ_FP16 : SUBQ_BF16;
    if (!make_map(&P.tm_q, p.q, dt, p.N, p.H, p.B, p.q_sn, p.q_sh, p.q_sb) ||
        !make_map(&P.tm_k, p.k, dt, p.N, p.H, p.B, p.k_sn, p.k_sh, p.k_sb) ||
        !make_map(&P.tm_v, p.v, dt, p.N, p.H, p.B, p.v_sn, p.v_sh, p.v_sb) ||
        !make_map(&P.tm_g, p.g, dt, p.N, p.H, p.B, p.g_sn, p.g_sh, p.g_sb) ||
        !make_map(&P.tm_dq, p.o, dt, p.N, p.H, p.B, p.o_sn, p.o_sh, p.o_sb) ||
        !make_map(&P.tm_dk, p.dk, dt, p.N, p.H, p.B, p.dk_sn, p.dk_sh, p.dk_sb) ||
        !make_map(&P.tm_dv, p.dv, dt, p.N, p.H, p.B, p.dv_sn, p.dv_sh, p.dv_sb))
        return cudaErrorInvalidValue;
    const int nC = (p.N + kC - 1) / kC;
    P.G = pick_segments(p);
    P.cps = (nC + P.G - 1) / P.G;
    auto kern = bwd_tc_kernel<kFp16, kNorm>;
    const size_t smem = BwdSmem::total + 1024;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(P.G, p.B * p.H, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = P.G;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, P);
}

}  // namespace

bool tc_bwd_supported(const ScanParams& p, int) { return p.dlg == nullptr; }

bool tc_supported(const ScanParams& p, int dtype) {
    if (dtype != SUBQ_BF16 && dtype != SUBQ_FP16) return false;
    if (p.d != kD || p.e != kD || p.N < 1) return false;
    if (p.decay_mode != SUBQ_DECAY_NONE || p.flush) return false;
    if (p.B * p.H > 65535) return false;
    return strides_ok(p.q_sb, p.q_sh, p.q_sn, p.q) && strides_ok(p.k_sb, p.k_sh, p.k_sn, p.k) &&
           strides_ok(p.v_sb, p.v_sh, p.v_sn, p.v) && strides_ok(p.o_sb, p.o_sh, p.o_sn, p.o) && encode_fn() != nullptr;
}

size_t tc_fwd_workspace_bytes(const ScanParams&) { return 0; }

// (Zc_t, c_t) per token, written by phase B and read back by phase C.
size_t tc_bwd_workspace_bytes(const ScanParams& p) {
    return ((size_t)p.B * p.H * (size_t)p.N * sizeof(float2) + 255) / 256 * 256;
}

cudaError_t launch_fwd_tc(const ScanParams& p, int dtype, cudaStream_t st, int* launches) {
    *launches = 1;
    const bool fp16 = dtype == SUBQ_FP16;
    if (fp16) return p.normalize ? launch_fwd_impl<true, true>(p, st) : launch_fwd_impl<true, false>(p, st);
    return p.normalize ? launch_fwd_impl<false, true>(p, st) : launch_fwd_impl<false, false>(p, st);
}

cudaError_t launch_bwd_tc(const ScanParams& p, int dtype, cudaStream_t st, int* launches) {
    *launches = 1;
    const bool fp16 = dtype == SUBQ_FP16;
    if (fp16) return p.normalize ? launch_bwd_impl<true, true>(p, st) : launch_bwd_impl<true, false>(p, st);
    return p.normalize ? launch_bwd_impl<false, true>(p, st) : launch_bwd_impl<false, false>(p, st);
}

cudaError_t tc_read_status(cudaStream_t st, int* status) {
    int v = 0;
    cudaError_t err = cudaMemcpyFromSymbolAsync(&v, g_tc_status, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
    if (err == cudaSuccess) err = cudaStreamSynchronize(st);
    if (err == cudaSuccess && v != 0) {
        const int zero = 0;
        err = cudaMemcpyToSymbolAsync(g_tc_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
        if (err == cudaSuccess) err = cudaStreamSynchronize(st);
    }
    *status = v;
    return err;
}

}  // namespace subq
