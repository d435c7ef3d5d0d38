// Tensor-core forward scan (d = e = 64, bf16/fp16 inputs, fp32 accumulation).
//
// One cluster of G CTAs per (batch, head) sequence; CTA g owns segment g
// (a run of 128-token chunks). Per chunk (t, tau index the chunk's tokens):
//   P       = phi~(Q) phi~(K)^T                 tcgen05 128x128x64   -> TMEM
//   P      <- P [tau <= t];  Z_t = sum_tau P + phi~(q_t) . z_c         (registers)
//   O       = phi~(Q) S_c + P V                 tcgen05 128x64x64 + 128x64x128
//   S_c+1   = S_c + phi~(K)^T V                 tcgen05 64x64x128, TMEM-resident fp32
//   z_c+1   = z_c + phi~(K)^T m                 tcgen05 64x16x128 against a mask column
//   out_t   = O_t / max(Z_t, clamp)  (normalised)  or  O_t
// with phi~(q) = scale phi(q), phi~(k) = m phi(k) (masked keys drop out of P,
// S and z). The bf16 copy of S in shared memory is the next chunk's operand.
//
// Segment prefix: CTA g first sums phi~(K)^T V and phi~(K)^T m over its own
// segment (phase 1), publishes them in shared memory, and after a cluster
// barrier adds those of CTAs 0..g-1 (read over DSMEM) to the incoming state;
// phase 2 re-reads K and V, mostly from L2.
//
// Threads: 256. TMEM lane / chunk row = 32 * (warp % 4) + lane; the two warps
// of a TMEM quadrant split each row's columns (half = warp / 4).
//
// Reference algorithm: python/subq_audio/autograd.py:108-169 (chunked scan),
// :292-376 (normaliser, clamp, mask); recurrence of
// src/kernels/attention_forward.cpp:42-58.
#include "tc_common.cuh"

namespace cg = cooperative_groups;

namespace subq {
namespace tcs {
namespace {

constexpr int kStages = 3;

struct FwdLayout {
    static constexpr uint32_t stage = 3 * kTile;  // q, k, v
    static constexpr uint32_t q = 0, k = kTile, v = 2 * kTile;
    static constexpr uint32_t p = kStages * stage;  // P (two 64-column blocks); exchange buffer between phases
    static constexpr uint32_t sb = p + 2 * kTile;   // bf16 S_c (MN-major B operand)
    static constexpr uint32_t mt = sb + kD * kD * 2;  // mask column tile (128 x 16, 32-byte swizzle)
    static constexpr uint32_t zc = mt + kMTile;     // z_c fp32 [64]
    static constexpr uint32_t zq = zc + 256;        // partial phi~(q).z_c [2][128]
    static constexpr uint32_t rs = zq + 1024;       // partial row sums of P [2][128]
    static constexpr uint32_t bars = rs + 1024;     // tma[kStages], mma
    static constexpr uint32_t tslot = bars + 8 * (kStages + 1);
    static constexpr uint32_t total = tslot + 16;
};
static_assert(FwdLayout::p % 1024 == 0 && FwdLayout::sb % 1024 == 0 && FwdLayout::mt % 1024 == 0, "alignment");
static_assert(FwdLayout::total + 1024 <= 232448, "shared memory");

// TMEM (fp32 columns): P [0,128), O [128,192), S [192,256) (M=64), z' [256,288) (M=64, column 0 = z).
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t cP = 0, cO = 128, cS = 192, cZ = 256;

struct FwdParams {
    CUtensorMap tm_q, tm_k, tm_v, tm_o;
    ScanParams p;
    int G;
    int cps;
    int* status;
};

template <bool kFp16, bool kNorm>
__global__ void __launch_bounds__(kThreads, 1) fwd_kernel(const __grid_constant__ FwdParams P) {
    const ScanParams& p = P.p;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    cg::cluster_group cluster = cg::this_cluster();

    const int g = (int)cluster.block_rank();
    const int bh = blockIdx.y;
    const int b = bh / p.H, h = bh - b * p.H;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quad = warp & 3, hf = warp >> 2;
    const int row = quad * 32 + lane;   // chunk row == TMEM lane
    const int srow = quad * 16 + lane;  // state row held by lanes < 16 (M = 64 layout)
    const int nC = (p.N + kC - 1) / kC;
    const int c_begin = min(nC, g * P.cps);
    const int n = min(nC, c_begin + P.cps) - c_begin;

    uint64_t* tma_bar = reinterpret_cast<uint64_t*>(sm + FwdLayout::bars);
    uint64_t* mma_bar = tma_bar + kStages;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + FwdLayout::tslot);
    float* zc = reinterpret_cast<float*>(sm + FwdLayout::zc);
    float* zqs = reinterpret_cast<float*>(sm + FwdLayout::zq);
    float* rss = reinterpret_cast<float*>(sm + FwdLayout::rs);
    uint8_t* Pt = sm + FwdLayout::p;
    uint8_t* Sb = sm + FwdLayout::sb;
    uint8_t* Mt = sm + FwdLayout::mt;
    float* Xs = reinterpret_cast<float*>(Pt);                // [64][64] segment sum phi~(K)^T V
    float* Xz = reinterpret_cast<float*>(Pt + kD * kD * 4);  // [64] segment sum phi~(K)^T m

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
    const uint32_t loff = (uint32_t)(quad * 32) << 16;
    const uint32_t tP = tmem + cP, tO = tmem + cO, tS = tmem + cS, tZ = tmem + cZ;
    const uint32_t sbase = tc::smem_u32(sm);

    bool ok = true;
    uint32_t tma_phase[kStages];
    int pending[kStages];
    for (int s = 0; s < kStages; ++s) {
        tma_phase[s] = 0;
        pending[s] = 0;
    }
    uint32_t mma_phase = 0;

    constexpr uint32_t idP = tc::idesc_f16<kFp16>(128, 128, false, false);
    constexpr uint32_t idO = tc::idesc_f16<kFp16>(128, 64, false, true);
    constexpr uint32_t idS = tc::idesc_f16<kFp16>(64, 64, true, true);
    constexpr uint32_t idZ = tc::idesc_f16<kFp16>(64, 16, true, true);

    auto issue = [&](int chunk, int s, bool with_q) {
        const int t0 = chunk * kC;
        pending[s] = 1;
        uint8_t* base = sm + s * FwdLayout::stage;
        tc::mbar_arrive_expect_tx(&tma_bar[s], (with_q ? 3u : 2u) * kTile);
        if (with_q) tc::tma_load_4d(base + FwdLayout::q, &P.tm_q, 0, t0, h, b, &tma_bar[s]);
        tc::tma_load_4d(base + FwdLayout::k, &P.tm_k, 0, t0, h, b, &tma_bar[s]);
        tc::tma_load_4d(base + FwdLayout::v, &P.tm_v, 0, t0, h, b, &tma_bar[s]);
    };
    auto row_mask = [&](int chunk) -> float {
        const int t = chunk * kC + row;
        if (t >= p.N) return 0.f;
        return p.mask ? (p.mask[(int64_t)b * p.mask_sb + t] ? 1.f : 0.f) : 1.f;
    };
    auto wait_tma = [&](int s) {
        ok = __syncthreads_and(wait_bar(&tma_bar[s], tma_phase[s], P.status)) && ok;
        tma_phase[s] ^= 1u;
        pending[s] = 0;
    };
    auto wait_mma = [&]() {
        ok = __syncthreads_and(wait_bar(mma_bar, mma_phase, P.status)) && ok;
        mma_phase ^= 1u;
        tc::tc_fence_after();
    };
    auto publish = [&]() {  // generic-proxy smem writes -> MMA, TMEM reads done -> next MMA
        tc::fence_proxy_async();
        tc::tc_fence_before();
        __syncthreads();
    };
    // S (+)= phi~(K)^T V and z' (+)= phi~(K)^T m over one chunk.
    auto mma_state = [&](int s, bool first) {
        const uint32_t ka = sbase + s * FwdLayout::stage + FwdLayout::k;
        const uint32_t va = sbase + s * FwdLayout::stage + FwdLayout::v;
        const uint32_t ma = sbase + FwdLayout::mt;
        for (int kk = 0; kk < 8; ++kk) {
            const uint64_t ad = tc::sdesc_sw128(ka + kk * 2048, kTile, 1024);
            tc::mma_f16(tS, ad, tc::sdesc_sw128(va + kk * 2048, kTile, 1024), idS, (first && kk == 0) ? 0u : 1u);
            if (kNorm) tc::mma_f16(tZ, ad, sdesc_sw32(ma + kk * 512), idZ, (first && kk == 0) ? 0u : 1u);
        }
    };
    auto transform_k = [&](uint8_t* kt, float m) {
        chunks_transform<kFp16>(kt, row, hf * 4, 4, [&](int, float* v) {
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = phi_fast(v[u]) * m;
        });
        if (kNorm && hf == 0) mtile_row<kFp16>(Mt, row, m);
    };

    // ------------------------------------------------------------ phase 1
    if (g < P.G - 1) {
        if (tid == 0)
            for (int j = 0; j < kStages - 1 && j < n; ++j) issue(c_begin + j, j, false);
        for (int i = 0; i < n && ok; ++i) {
            const int s = i % kStages;
            if (tid == 0 && i + kStages - 1 < n) issue(c_begin + i + kStages - 1, (i + kStages - 1) % kStages, false);
            wait_tma(s);
            if (!ok) break;
            transform_k(sm + s * FwdLayout::stage + FwdLayout::k, row_mask(c_begin + i));
            publish();
            if (tid == 0) {
                tc::tc_fence_after();
                mma_state(s, i == 0);
                tc::mma_commit(mma_bar);
            }
            wait_mma();
        }
        float v[32];
        if (n > 0 && ok) {
            tc::tmem_ld32(tS + loff + hf * 32, v);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.f;
        }
        if (lane < 16) {
#pragma unroll
            for (int j = 0; j < 32; ++j) Xs[srow * 64 + hf * 32 + j] = v[j];
        }
        if (hf == 0) {
            const float zv = (kNorm && n > 0 && ok) ? tmem_ld1(tZ + loff) : 0.f;
            if (lane < 16) Xz[srow] = zv;
        }
    }
    tc::tc_fence_before();
    cluster.sync();
    tc::tc_fence_after();

    // ------------------------------------------------------ segment prefix
    {
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
        if (lane < 16) {
            if (p.S_in) {
                const float* src = p.S_in + ((int64_t)bh * kD + srow) * kD + hf * 32;
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = src[j];
            }
            for (int r = 0; r < g; ++r) {
                const float* rx = cluster.map_shared_rank(Xs, r) + srow * 64 + hf * 32;
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += rx[j];
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) store_chunk<kFp16>(Sb, srow, hf * 4 + j, v + 8 * j);
        }
        tc::tmem_st32(tS + loff + hf * 32, v);
        if (kNorm && tid < 64) {
            float z = p.z_in ? p.z_in[(int64_t)bh * kD + tid] : 0.f;
            for (int r = 0; r < g; ++r) z += cluster.map_shared_rank(Xz, r)[tid];
            zc[tid] = z;
        }
    }
    __syncthreads();
    if (kNorm && hf == 0) {  // z' column 0 <- z_c (the accumulator of the mask-column MMA)
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
        if (lane < 16) v[0] = zc[srow];
        tc::tmem_st32(tZ + loff, v);
    }
    tc::fence_proxy_async();
    tc::tc_fence_before();
    cluster.sync();  // every remote read of the exchange buffers is done
    tc::tc_fence_after();

    // ------------------------------------------------------------ phase 2
    if (tid == 0)
        for (int j = 0; j < kStages - 1 && j < n; ++j) issue(c_begin + j, j, true);
    for (int i = 0; i < n && ok; ++i) {
        const int c = c_begin + i, s = i % kStages;
        if (tid == 0 && i + kStages - 1 < n) {
            tc::bulk_wait_read0();  // outputs staged in that stage's Q tile have been read
            issue(c + kStages - 1, (i + kStages - 1) % kStages, true);
        }
        wait_tma(s);
        if (!ok) break;
        uint8_t* qt = sm + s * FwdLayout::stage + FwdLayout::q;
        uint8_t* kt = sm + s * FwdLayout::stage + FwdLayout::k;
        const uint32_t qa = sbase + s * FwdLayout::stage + FwdLayout::q;
        const uint32_t ka = sbase + s * FwdLayout::stage + FwdLayout::k;
        const uint32_t va = sbase + s * FwdLayout::stage + FwdLayout::v;
        const float m = row_mask(c);
        float zq = 0.f;
        chunks_transform<kFp16>(qt, row, hf * 4, 4, [&](int j, float* v) {
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                v[u] = phi_fast(v[u]) * p.scale;
                if (kNorm) zq = fmaf(v[u], zc[8 * j + u], zq);
            }
        });
        if (kNorm) zqs[hf * 128 + row] = zq;
        transform_k(kt, m);
        publish();
        if (tid == 0) {
            tc::tc_fence_after();
            for (int kk = 0; kk < 4; ++kk)  // P = phi~(Q) phi~(K)^T
                tc::mma_f16(tP, tc::sdesc_sw128(qa + kk * 32, 16, 1024), tc::sdesc_sw128(ka + kk * 32, 16, 1024), idP,
                            kk > 0);
            for (int kk = 0; kk < 4; ++kk)  // O = phi~(Q) S_c
                tc::mma_f16(tO, tc::sdesc_sw128(qa + kk * 32, 16, 1024),
                            tc::sdesc_sw128(sbase + FwdLayout::sb + kk * 2048, 8192, 1024), idO, kk > 0);
            tc::mma_commit(mma_bar);
        }
        wait_mma();
        if (!ok) break;
        // P columns [64 hf, 64 hf + 64): causal mask on the diagonal block only; the
        // block right of the diagonal (rows < 64, half 1) is all zero.
        {
            uint8_t* pb = Pt + hf * kTile;
            float rs = 0.f;
            if (hf == 1 && quad < 2) {
                zero_chunks(pb, row, 0, 8);
            } else {
                const bool diag = (hf == (quad >> 1));
#pragma unroll
                for (int half32 = 0; half32 < 2; ++half32) {
                    float v[32];
                    tc::tmem_ld32(tP + loff + hf * 64 + half32 * 32, v);
#pragma unroll
                    for (int u = 0; u < 32; ++u) {
                        const int tau = hf * 64 + half32 * 32 + u;
                        if (diag && tau > row) v[u] = 0.f;
                        rs += v[u];
                    }
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) store_chunk<kFp16>(pb, row, half32 * 4 + q4, v + 8 * q4);
                }
            }
            if (kNorm) rss[hf * 128 + row] = rs;
        }
        publish();
        if (tid == 0) {
            tc::tc_fence_after();
            for (int kk = 0; kk < 8; ++kk) {  // O += P V
                const uint32_t pa = sbase + FwdLayout::p + (kk >> 2) * kTile + (kk & 3) * 32;
                tc::mma_f16(tO, tc::sdesc_sw128(pa, 16, 1024), tc::sdesc_sw128(va + kk * 2048, kTile, 1024), idO, 1u);
            }
            mma_state(s, false);  // S_c+1, z_c+1
            tc::mma_commit(mma_bar);
        }
        wait_mma();
        if (!ok) break;
        {
            float o[32];
            tc::tmem_ld32(tO + loff + hf * 32, o);
            float inv = m;
            if (kNorm) inv = m / fmaxf(rss[row] + rss[128 + row] + zqs[row] + zqs[128 + row], p.clamp_min);
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] *= inv;
#pragma unroll
            for (int j = 0; j < 4; ++j) store_chunk<kFp16>(qt, row, hf * 4 + j, o + 8 * j);
        }
        {
            float v[32];
            tc::tmem_ld32(tS + loff + hf * 32, v);
            if (lane < 16) {
#pragma unroll
                for (int j = 0; j < 4; ++j) store_chunk<kFp16>(Sb, srow, hf * 4 + j, v + 8 * j);
            }
            if (kNorm && hf == 0) {
                const float zv = tmem_ld1(tZ + loff);
                if (lane < 16) zc[srow] = zv;
            }
        }
        publish();
        if (tid == 0) {
            tc::tma_store_4d(&P.tm_o, qt, 0, c * kC, h, b);
            tc::bulk_commit();
        }
    }

    if (g == P.G - 1 && ok) {
        float v[32];
        tc::tmem_ld32(tS + loff + hf * 32, v);
        if (lane < 16 && p.S_out) {
            float* dst = p.S_out + ((int64_t)bh * kD + srow) * kD + hf * 32;
#pragma unroll
            for (int j = 0; j < 32; ++j) dst[j] = v[j];
        }
        if (p.z_out && tid < 64) p.z_out[(int64_t)bh * kD + tid] = kNorm ? zc[tid] : 0.f;
    }
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s)
            if (pending[s]) wait_bar(&tma_bar[s], tma_phase[s], P.status);
        tc::bulk_wait0();
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, kTmemCols);
}

template <bool kFp16, bool kNorm>
cudaError_t launch(const ScanParams& p, cudaStream_t st) {
    FwdParams P;
    memset(&P, 0, sizeof(P));
    P.p = p;
    const int dt = kFp16 ? SUBQ_FP16 : SUBQ_BF16;
    if (!make_map(&P.tm_q, p.q, dt, p.N, p.H, p.B, p.q_sn, p.q_sh, p.q_sb) ||
        !make_map(&P.tm_k, p.k, dt, p.N, p.H, p.B, p.k_sn, p.k_sh, p.k_sb) ||
        !make_map(&P.tm_v, p.v, dt, p.N, p.H, p.B, p.v_sn, p.v_sh, p.v_sb) ||
        !make_map(&P.tm_o, p.o, dt, p.N, p.H, p.B, p.o_sn, p.o_sh, p.o_sb))
        return cudaErrorInvalidValue;
    const int nC = (p.N + kC - 1) / kC;
    P.status = status_ptr();
    if (!P.status) return cudaErrorInvalidDevice;
    P.G = pick_segments(p);
    P.cps = (nC + P.G - 1) / P.G;
    const void* kern = reinterpret_cast<const void*>(&fwd_kernel<kFp16, kNorm>);
    void* args[] = {&P};
    return launch_cluster(kern, P.G, p.B * p.H, FwdLayout::total + 1024, st, args);
}

}  // namespace

cudaError_t launch_fwd_v2(const ScanParams& p, int dtype, cudaStream_t st) {
    if (dtype == SUBQ_FP16) return p.normalize ? launch<true, true>(p, st) : launch<true, false>(p, st);
    return p.normalize ? launch<false, true>(p, st) : launch<false, false>(p, st);
}

}  // namespace tcs
}  // namespace subq
