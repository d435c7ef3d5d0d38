// Tensor-core backward scan (d = e = 64, bf16/fp16 inputs, fp32 accumulation).
//
// One cluster of G CTAs per (batch, head) sequence; CTA g owns segment g.
// With q~ = scale phi(q), k~ = m phi(k), Zc_t = max(Z_t, clamp) and the
// quotient rule of the normaliser,
//   o^_t = m_t dO_t / Zc_t,      c_t = -(m_t dO_t . num_t) / Zc_t^2
// the gradients per 128-token chunk are
//   dA   = (O^ V^T + c m^T) [tau <= t]
//   dQ~  = dA K~ + O^ S_c^T + c z_c^T                (S_c, z_c: prefix state)
//   dK~  = dA^T Q~ + V dS_c^T + m dz_c^T             (dS_c, dz_c: suffix adjoint)
//   dV   = (P [tau <= t])^T O^ + K~ dS_c
//   dS_c-1 = dS_c + Q~^T O^,   dz_c-1 = dz_c + Q~^T c
// and dq = dQ~ scale phi'(q), dk = dK~ phi'(k) m, dv = dV m with
// phi'(x) = min(phi(x), 1). The normaliser terms z and dz run on the tensor
// core against a two-column tile [m | c].
//
// Phases of a CTA:
//   A  segment sums of K~^T V and K~^T m (CTAs g < G-1)   -> DSMEM -> S_c, z_c
//   B  chunks ascending: recompute num and Z, form O^ and c, emit dq, keep
//      (Zc_t, c_t) in the workspace, sum Q~^T O^ and Q~^T c over the segment
//                                                          -> DSMEM -> dS, dz
//   C  chunks descending: rebuild O^ from dO and (Zc, c), emit dk and dv.
//
// Reference: python/subq_audio/autograd.py:441-544 (quotient rule :497-499,
// chunked adjoint :172-289); src/kernels/attention_backward.cpp:165-229.
#include "tc_common.cuh"

namespace cg = cooperative_groups;

namespace subq {
namespace tcs {
namespace {

constexpr int kStages = 2;

struct BwdLayout {
    static constexpr uint32_t stage = 4 * kTile;  // q, k, v, dO
    static constexpr uint32_t q = 0, k = kTile, v = 2 * kTile, g = 3 * kTile;
    static constexpr uint32_t p = kStages * stage;     // P (2 blocks); exchange buffer between phases
    static constexpr uint32_t da = p + 2 * kTile;      // dA (2 blocks)
    static constexpr uint32_t ob = da + 2 * kTile;     // O^ [t][e]
    static constexpr uint32_t sb = ob + kTile;         // bf16 S_c (phase B) or dS_c (phase C)
    static constexpr uint32_t mc = sb + kD * kD * 2;   // [m | c] column tile (128 x 16)
    static constexpr uint32_t zc = mc + kMTile;        // z_c or dz_c, fp32 [2][64] (double buffer)
    static constexpr uint32_t zq = zc + 512;           // partial q~.z [2][128]
    static constexpr uint32_t rs = zq + 1024;          // partial row sums / dot products [2][128]
    static constexpr uint32_t mb = rs + 1024;          // m_t [128]
    static constexpr uint32_t bars = mb + 512;
    static constexpr uint32_t tslot = bars + 8 * (kStages + 1);
    static constexpr uint32_t total = tslot + 16;
};
static_assert(BwdLayout::p % 1024 == 0 && BwdLayout::da % 1024 == 0 && BwdLayout::ob % 1024 == 0 &&
                  BwdLayout::sb % 1024 == 0 && BwdLayout::mc % 1024 == 0,
              "alignment");
static_assert(BwdLayout::total + 1024 <= 232448, "shared memory");

// TMEM (512 fp32 columns): P [0,128) -- reused for dQ~ / dV [0,64) once P is
// consumed --, dA [128,256), X1 [256,320) (num / dK~), z' [320,352), dz' [352,384),
// S [384,448), dS [448,512). z', dz', S, dS use the M = 64 layout.
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t cP = 0, cdA = 128, cX1 = 256, cZ = 320, cdZ = 352, cS = 384, cdS = 448;

struct BwdParams {
    CUtensorMap tm_q, tm_k, tm_v, tm_g, tm_dq, tm_dk, tm_dv;
    ScanParams p;
    int G;
    int cps;
    int* status;
};

template <bool kFp16, bool kNorm>
__global__ void __launch_bounds__(kThreads, 1) bwd_kernel(const __grid_constant__ BwdParams P) {
    const ScanParams& p = P.p;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    cg::cluster_group cluster = cg::this_cluster();

    const int g = (int)cluster.block_rank();
    const int bh = blockIdx.y;
    const int b = bh / p.H, h = bh - b * p.H;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quad = warp & 3, hf = warp >> 2;
    const int row = quad * 32 + lane;
    const int srow = quad * 16 + lane;
    const int nC = (p.N + kC - 1) / kC;
    const int c_begin = min(nC, g * P.cps);
    const int c_end = min(nC, c_begin + P.cps);
    const int n = c_end - c_begin;

    uint64_t* tma_bar = reinterpret_cast<uint64_t*>(sm + BwdLayout::bars);
    uint64_t* mma_bar = tma_bar + kStages;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + BwdLayout::tslot);
    float* zc = reinterpret_cast<float*>(sm + BwdLayout::zc);  // [2][64]
    float* zqs = reinterpret_cast<float*>(sm + BwdLayout::zq);
    float* rss = reinterpret_cast<float*>(sm + BwdLayout::rs);
    float* mb = reinterpret_cast<float*>(sm + BwdLayout::mb);
    uint8_t* Pt = sm + BwdLayout::p;
    uint8_t* dAt = sm + BwdLayout::da;
    uint8_t* Ot = sm + BwdLayout::ob;
    uint8_t* Sb = sm + BwdLayout::sb;
    uint8_t* MC = sm + BwdLayout::mc;
    float* Xs = reinterpret_cast<float*>(Pt);
    float* Xz = reinterpret_cast<float*>(Pt + kD * kD * 4);
    float2* wsz = reinterpret_cast<float2*>(p.ws) + (int64_t)bh * p.N;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) tc::mbar_init(&tma_bar[s], 1);
        tc::mbar_init(mma_bar, 1);
        tc::fence_mbar_init();
    }
    if (warp == 0) tc::tmem_alloc(tslot, kTmemCols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t loff = (uint32_t)(quad * 32) << 16;
    const uint32_t tP = tmem + cP, tdA = tmem + cdA, tX1 = tmem + cX1, tX2 = tmem + cP;
    const uint32_t tZ = tmem + cZ, tdZ = tmem + cdZ, tS = tmem + cS, tdS = tmem + cdS;
    const uint32_t sbase = tc::smem_u32(sm);

    bool ok = true;
    uint32_t tma_phase[kStages] = {0, 0};
    int pending[kStages] = {0, 0};
    uint32_t mma_phase = 0;

    constexpr uint32_t idKK128 = tc::idesc_f16<kFp16>(128, 128, false, false);
    constexpr uint32_t idKM = tc::idesc_f16<kFp16>(128, 64, false, true);
    constexpr uint32_t idKK = tc::idesc_f16<kFp16>(128, 64, false, false);
    constexpr uint32_t idMM = tc::idesc_f16<kFp16>(128, 64, true, true);
    constexpr uint32_t idS = tc::idesc_f16<kFp16>(64, 64, true, true);
    constexpr uint32_t idZ = tc::idesc_f16<kFp16>(64, 16, true, true);

    auto stp = [&](int s, uint32_t w) { return sm + s * BwdLayout::stage + w; };
    auto sta = [&](int s, uint32_t w) { return sbase + s * BwdLayout::stage + w; };
    auto issue = [&](int chunk, int s, bool full) {
        const int t0 = chunk * kC;
        pending[s] = 1;
        tc::mbar_arrive_expect_tx(&tma_bar[s], (full ? 4u : 2u) * kTile);
        if (full) {
            tc::tma_load_4d(stp(s, BwdLayout::q), &P.tm_q, 0, t0, h, b, &tma_bar[s]);
            tc::tma_load_4d(stp(s, BwdLayout::g), &P.tm_g, 0, t0, h, b, &tma_bar[s]);
        }
        tc::tma_load_4d(stp(s, BwdLayout::k), &P.tm_k, 0, t0, h, b, &tma_bar[s]);
        tc::tma_load_4d(stp(s, BwdLayout::v), &P.tm_v, 0, t0, h, b, &tma_bar[s]);
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
    auto publish = [&]() {
        tc::fence_proxy_async();
        tc::tc_fence_before();
        __syncthreads();
    };
    // acc (+)= X^T Y over 128 tokens (X, Y [128][64] tiles read MN-major; M = 64).
    auto mma_xty = [&](uint32_t dst, uint32_t xa, uint32_t ya, bool first) {
        for (int kk = 0; kk < 8; ++kk)
            tc::mma_f16(dst, tc::sdesc_sw128(xa + kk * 2048, kTile, 1024), tc::sdesc_sw128(ya + kk * 2048, kTile, 1024),
                        idS, (first && kk == 0) ? 0u : 1u);
    };
    // acc (+)= X^T [m | c] (the two-column tile; M = 64, N = 16).
    auto mma_xtm = [&](uint32_t dst, uint32_t xa, bool first) {
        for (int kk = 0; kk < 8; ++kk)
            tc::mma_f16(dst, tc::sdesc_sw128(xa + kk * 2048, kTile, 1024), sdesc_sw32(sbase + BwdLayout::mc + kk * 512),
                        idZ, (first && kk == 0) ? 0u : 1u);
    };
    auto transform_q = [&](uint8_t* qt, const float* z, float* zq_out) {
        float zq = 0.f;
        chunks_transform<kFp16>(qt, row, hf * 4, 4, [&](int j, float* v) {
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                v[u] = phi_fast(v[u]) * p.scale;
                if (kNorm && z) zq = fmaf(v[u], z[8 * j + u], zq);
            }
        });
        if (zq_out) *zq_out = zq;
    };
    auto transform_k = [&](uint8_t* kt, float m) {
        chunks_transform<kFp16>(kt, row, hf * 4, 4, [&](int, float* v) {
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = phi_fast(v[u]) * m;
        });
    };
    // 128 x 128 causal tile (TMEM fp32) -> bf16 shared memory, this thread's column
    // half; optionally adds c_t m_tau; returns the partial row sum.
    auto tile_out = [&](uint32_t tsrc, uint8_t* dst, bool add_cm, float ct) -> float {
        uint8_t* pb = dst + hf * kTile;
        float rs = 0.f;
        if (hf == 1 && quad < 2) {
            zero_chunks(pb, row, 0, 8);
            return 0.f;
        }
        const bool diag = (hf == (quad >> 1));
#pragma unroll
        for (int half32 = 0; half32 < 2; ++half32) {
            float v[32];
            tc::tmem_ld32(tsrc + loff + hf * 64 + half32 * 32, v);
#pragma unroll
            for (int u = 0; u < 32; ++u) {
                const int tau = hf * 64 + half32 * 32 + u;
                float x = add_cm ? fmaf(ct, mb[tau], v[u]) : v[u];
                if (diag && tau > row) x = 0.f;
                rs += x;
                v[u] = x;
            }
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) store_chunk<kFp16>(pb, row, half32 * 4 + q4, v + 8 * q4);
        }
        return rs;
    };
    // M = 64 state (TMEM) -> bf16 copy in Sb (this thread's column half).
    auto refresh_sb = [&](uint32_t tsrc) {
        float v[32];
        tc::tmem_ld32(tsrc + loff + hf * 32, v);
        if (lane < 16) {
#pragma unroll
            for (int j = 0; j < 4; ++j) store_chunk<kFp16>(Sb, srow, hf * 4 + j, v + 8 * j);
        }
    };
    // Column `col` of an M = 64, N = 32 accumulator -> dst[64] (warps of half 0).
    auto read_col = [&](uint32_t tsrc, int col, float* dst) {
        if (hf == 0) {
            const float x = tmem_ld1(tsrc + loff + col);
            if (lane < 16) dst[srow] = x;
        }
    };
    // 64 x 64 fp32 state rows (this thread's half) -> TMEM and Sb.
    auto put_state = [&](uint32_t tdst, float* v) {
        if (lane < 16) {
#pragma unroll
            for (int j = 0; j < 4; ++j) store_chunk<kFp16>(Sb, srow, hf * 4 + j, v + 8 * j);
        }
        tc::tmem_st32(tdst + loff + hf * 32, v);
    };
    // Column `col` of an M = 64, N = 32 accumulator <- src[64], other columns zero.
    auto put_col = [&](uint32_t tdst, int col, const float* src) {
        if (hf == 0) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.f;
            if (lane < 16) v[col] = src[srow];
            tc::tmem_st32(tdst + loff, v);
        }
    };

    // ------------------------------------------------------------ phase A
    if (g < P.G - 1) {
        if (tid == 0 && n > 0) issue(c_begin, 0, false);
        for (int i = 0; i < n && ok; ++i) {
            const int s = i % kStages;
            if (tid == 0 && i + 1 < n) issue(c_begin + i + 1, (i + 1) % kStages, false);
            wait_tma(s);
            if (!ok) break;
            const float m = row_mask(c_begin + i);
            transform_k(stp(s, BwdLayout::k), m);
            if (kNorm && hf == 0) mtile_row2<kFp16>(MC, row, m, 0.f);
            publish();
            if (tid == 0) {
                tc::tc_fence_after();
                mma_xty(tS, sta(s, BwdLayout::k), sta(s, BwdLayout::v), i == 0);
                if (kNorm) mma_xtm(tZ, sta(s, BwdLayout::k), i == 0);
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
        }
        put_state(tS, v);
        if (kNorm && tid < 64) {
            float z = p.z_in ? p.z_in[(int64_t)bh * kD + tid] : 0.f;
            for (int r = 0; r < g; ++r) z += cluster.map_shared_rank(Xz, r)[tid];
            zc[tid] = z;
        }
    }
    __syncthreads();
    if (kNorm) put_col(tZ, 0, zc);
    tc::fence_proxy_async();
    tc::tc_fence_before();
    cluster.sync();
    tc::tc_fence_after();

    // ------------------------------------------------------------ phase B
    if (tid == 0 && n > 0) issue(c_begin, 0, true);
    for (int i = 0; i < n && ok; ++i) {
        const int c = c_begin + i, s = i % kStages;
        float* zcur = zc + (i & 1) * 64;        // z_c
        float* znext = zc + ((i + 1) & 1) * 64;  // z_c+1
        if (tid == 0 && i + 1 < n) {
            tc::bulk_wait_read0();
            issue(c + 1, (i + 1) % kStages, true);
        }
        wait_tma(s);
        if (!ok) break;
        uint8_t* qt = stp(s, BwdLayout::q);
        uint8_t* kt = stp(s, BwdLayout::k);
        const uint32_t qa = sta(s, BwdLayout::q), ka = sta(s, BwdLayout::k), va = sta(s, BwdLayout::v);
        const float m = row_mask(c);
        float zq = 0.f;
        transform_q(qt, zcur, &zq);
        transform_k(kt, m);
        if (kNorm) zqs[hf * 128 + row] = zq;
        if (hf == 0) mb[row] = m;
        publish();
        if (tid == 0) {
            tc::tc_fence_after();
            for (int kk = 0; kk < 4; ++kk)  // P = Q~ K~^T
                tc::mma_f16(tP, tc::sdesc_sw128(qa + kk * 32, 16, 1024), tc::sdesc_sw128(ka + kk * 32, 16, 1024),
                            idKK128, kk > 0);
            for (int kk = 0; kk < 4; ++kk)  // num = Q~ S_c
                tc::mma_f16(tX1, tc::sdesc_sw128(qa + kk * 32, 16, 1024),
                            tc::sdesc_sw128(sbase + BwdLayout::sb + kk * 2048, 8192, 1024), idKM, kk > 0);
            tc::mma_commit(mma_bar);
        }
        wait_mma();
        if (!ok) break;
        {
            const float rs = tile_out(tP, Pt, false, 0.f);
            if (kNorm) rss[hf * 128 + row] = rs;
        }
        publish();
        if (tid == 0) {
            tc::tc_fence_after();
            for (int kk = 0; kk < 8; ++kk) {  // num += P V
                const uint32_t pa = sbase + BwdLayout::p + (kk >> 2) * kTile + (kk & 3) * 32;
                tc::mma_f16(tX1, tc::sdesc_sw128(pa, 16, 1024), tc::sdesc_sw128(va + kk * 2048, kTile, 1024), idKM, 1u);
            }
            tc::mma_commit(mma_bar);
        }
        wait_mma();
        if (!ok) break;
        // O^ and c from the recomputed numerator and denominator.
        float num[32], go[32];
        tc::tmem_ld32(tX1 + loff + hf * 32, num);
        load_chunks<kFp16>(stp(s, BwdLayout::g), row, hf * 4, 4, go);
        float zcl = 1.f;
        if (kNorm) zcl = fmaxf(rss[row] + rss[128 + row] + zqs[row] + zqs[128 + row], p.clamp_min);
        float dot = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) dot = fmaf(go[j], num[j], dot);
        __syncthreads();  // everyone has read rss / zqs
        if (kNorm) rss[hf * 128 + row] = dot * m;
        __syncthreads();
        const float ct = kNorm ? -(rss[row] + rss[128 + row]) / (zcl * zcl) : 0.f;
        {
            const float inv = m / zcl;
#pragma unroll
            for (int j = 0; j < 32; ++j) go[j] *= inv;
#pragma unroll
            for (int j = 0; j < 4; ++j) store_chunk<kFp16>(Ot, row, hf * 4 + j, go + 8 * j);
        }
        if (hf == 0) {
            if (kNorm) mtile_row2<kFp16>(MC, row, m, ct);
            if (c * kC + row < p.N) wsz[c * kC + row] = make_float2(zcl, ct);
        }
        publish();
        if (tid == 0) {
            tc::tc_fence_after();
            for (int kk = 0; kk < 4; ++kk)  // dA = O^ V^T
                tc::mma_f16(tdA, tc::sdesc_sw128(sbase + BwdLayout::ob + kk * 32, 16, 1024),
                            tc::sdesc_sw128(va + kk * 32, 16, 1024), idKK128, kk > 0);
            mma_xty(tdS, qa, sbase + BwdLayout::ob, i == 0);  // segment sum of Q~^T O^
            mma_xty(tS, ka, va, false);                        // S_c+1
            if (kNorm) {
                mma_xtm(tdZ, qa, i == 0);  // column 1: segment sum of Q~^T c
                mma_xtm(tZ, ka, false);    // column 0: z_c+1
            }
            tc::mma_commit(mma_bar);
        }
        wait_mma();
        if (!ok) break;
        tile_out(tdA, dAt, kNorm, ct);
        publish();
        if (tid == 0) {
            tc::tc_fence_after();
            for (int kk = 0; kk < 8; ++kk) {  // dQ~ = dA K~
                const uint32_t aa = sbase + BwdLayout::da + (kk >> 2) * kTile + (kk & 3) * 32;
                tc::mma_f16(tX2, tc::sdesc_sw128(aa, 16, 1024), tc::sdesc_sw128(ka + kk * 2048, kTile, 1024), idKM,
                            kk > 0);
            }
            for (int kk = 0; kk < 4; ++kk)  // dQ~ += O^ S_c^T
                tc::mma_f16(tX2, tc::sdesc_sw128(sbase + BwdLayout::ob + kk * 32, 16, 1024),
                            tc::sdesc_sw128(sbase + BwdLayout::sb + kk * 32, 16, 1024), idKK, 1u);
            tc::mma_commit(mma_bar);
        }
        wait_mma();
        if (!ok) break;
        {
            float dq[32], qv[32];
            tc::tmem_ld32(tX2 + loff + hf * 32, dq);
            load_chunks<kFp16>(qt, row, hf * 4, 4, qv);
            const float inv_scale = 1.f / p.scale;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const float x = kNorm ? fmaf(ct, zcur[hf * 32 + j], dq[j]) : dq[j];
                dq[j] = x * p.scale * fminf(qv[j] * inv_scale, 1.f) * m;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) store_chunk<kFp16>(qt, row, hf * 4 + j, dq + 8 * j);
        }
        refresh_sb(tS);
        if (kNorm) read_col(tZ, 0, znext);
        publish();
        if (tid == 0) {
            tc::tma_store_4d(&P.tm_dq, qt, 0, c * kC, h, b);
            tc::bulk_commit();
        }
    }

    // --------------------------------------------- suffix exchange (dS, dz)
    {
        float v[32];
        if (n > 0 && ok) {
            tc::tmem_ld32(tdS + loff + hf * 32, v);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.f;
        }
        float dzv = 0.f;
        if (hf == 0) {
            const float x = (kNorm && n > 0 && ok) ? tmem_ld1(tdZ + loff + 1) : 0.f;
            dzv = x;
        }
        if (tid == 0) tc::bulk_wait_read0();
        tc::tc_fence_before();
        __syncthreads();
        if (lane < 16) {
#pragma unroll
            for (int j = 0; j < 32; ++j) Xs[srow * 64 + hf * 32 + j] = v[j];
            if (hf == 0) Xz[srow] = dzv;
        }
    }
    cluster.sync();
    tc::tc_fence_after();
    {
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
        if (lane < 16) {
            for (int r = g + 1; r < P.G; ++r) {
                const float* rx = cluster.map_shared_rank(Xs, r) + srow * 64 + hf * 32;
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += rx[j];
            }
        }
        float dz = 0.f;
        if (kNorm && tid < 64)
            for (int r = g + 1; r < P.G; ++r) dz += cluster.map_shared_rank(Xz, r)[tid];
        tc::tc_fence_before();
        cluster.sync();  // remote reads done before the buffers are reused
        tc::tc_fence_after();
        put_state(tdS, v);
        if (tid < 64) zc[tid] = dz;
    }
    __syncthreads();
    if (kNorm) put_col(tdZ, 1, zc);
    tc::fence_proxy_async();
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();

    // ------------------------------------------------------------ phase C
    if (tid == 0 && n > 0) issue(c_end - 1, 0, true);
    for (int i = 0; i < n && ok; ++i) {
        const int c = c_end - 1 - i, s = i % kStages;
        float* dzcur = zc + (i & 1) * 64;         // dz_c
        float* dznext = zc + ((i + 1) & 1) * 64;  // dz_c-1
        if (tid == 0 && i + 1 < n) {
            tc::bulk_wait_read0();
            issue(c - 1, (i + 1) % kStages, true);
        }
        wait_tma(s);
        if (!ok) break;
        uint8_t* qt = stp(s, BwdLayout::q);
        uint8_t* kt = stp(s, BwdLayout::k);
        uint8_t* vt = stp(s, BwdLayout::v);
        const uint32_t qa = sta(s, BwdLayout::q), ka = sta(s, BwdLayout::k), va = sta(s, BwdLayout::v);
        const float m = row_mask(c);
        float2 zcc = make_float2(1.f, 0.f);
        if (c * kC + row < p.N) zcc = wsz[c * kC + row];
        const float ct = zcc.y;
        transform_q(qt, nullptr, nullptr);
        transform_k(kt, m);
        {
            float go[32];
            load_chunks<kFp16>(stp(s, BwdLayout::g), row, hf * 4, 4, go);
            const float inv = m / zcc.x;
#pragma unroll
            for (int j = 0; j < 32; ++j) go[j] *= inv;
#pragma unroll
            for (int j = 0; j < 4; ++j) store_chunk<kFp16>(Ot, row, hf * 4 + j, go + 8 * j);
        }
        if (hf == 0) {
            mb[row] = m;
            if (kNorm) mtile_row2<kFp16>(MC, row, m, ct);
        }
        publish();
        if (tid == 0) {
            tc::tc_fence_after();
            for (int kk = 0; kk < 4; ++kk) {
                tc::mma_f16(tP, tc::sdesc_sw128(qa + kk * 32, 16, 1024), tc::sdesc_sw128(ka + kk * 32, 16, 1024),
                            idKK128, kk > 0);
                tc::mma_f16(tdA, tc::sdesc_sw128(sbase + BwdLayout::ob + kk * 32, 16, 1024),
                            tc::sdesc_sw128(va + kk * 32, 16, 1024), idKK128, kk > 0);
            }
            tc::mma_commit(mma_bar);
        }
        wait_mma();
        if (!ok) break;
        tile_out(tP, Pt, false, 0.f);
        tile_out(tdA, dAt, kNorm, ct);
        publish();
        if (tid == 0) {
            tc::tc_fence_after();
            for (int kk = 0; kk < 8; ++kk) {
                // dK~ = dA^T Q~ ; dV = P^T O^   (A read MN-major across both 64-token blocks)
                tc::mma_f16(tX1, tc::sdesc_sw128(sbase + BwdLayout::da + kk * 2048, kTile, 1024),
                            tc::sdesc_sw128(qa + kk * 2048, kTile, 1024), idMM, kk > 0);
                tc::mma_f16(tX2, tc::sdesc_sw128(sbase + BwdLayout::p + kk * 2048, kTile, 1024),
                            tc::sdesc_sw128(sbase + BwdLayout::ob + kk * 2048, kTile, 1024), idMM, kk > 0);
            }
            for (int kk = 0; kk < 4; ++kk) {
                tc::mma_f16(tX1, tc::sdesc_sw128(va + kk * 32, 16, 1024),  // dK~ += V dS_c^T
                            tc::sdesc_sw128(sbase + BwdLayout::sb + kk * 32, 16, 1024), idKK, 1u);
                tc::mma_f16(tX2, tc::sdesc_sw128(ka + kk * 32, 16, 1024),  // dV += K~ dS_c
                            tc::sdesc_sw128(sbase + BwdLayout::sb + kk * 2048, 8192, 1024), idKM, 1u);
            }
            mma_xty(tdS, qa, sbase + BwdLayout::ob, false);  // dS_c-1
            if (kNorm) mma_xtm(tdZ, qa, false);              // dz_c-1 (column 1)
            tc::mma_commit(mma_bar);
        }
        wait_mma();
        if (!ok) break;
        {
            float acc[32], kv[32];
            tc::tmem_ld32(tX1 + loff + hf * 32, acc);
            load_chunks<kFp16>(kt, row, hf * 4, 4, kv);
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const float x = kNorm ? fmaf(m, dzcur[hf * 32 + j], acc[j]) : acc[j];
                acc[j] = x * fminf(kv[j], 1.f) * m;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) store_chunk<kFp16>(kt, row, hf * 4 + j, acc + 8 * j);
            tc::tmem_ld32(tX2 + loff + hf * 32, acc);
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] *= m;
#pragma unroll
            for (int j = 0; j < 4; ++j) store_chunk<kFp16>(vt, row, hf * 4 + j, acc + 8 * j);
        }
        refresh_sb(tdS);
        if (kNorm) read_col(tdZ, 1, dznext);
        publish();
        if (tid == 0) {
            tc::tma_store_4d(&P.tm_dk, kt, 0, c * kC, h, b);
            tc::tma_store_4d(&P.tm_dv, vt, 0, c * kC, h, b);
            tc::bulk_commit();
        }
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
    BwdParams P;
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
    P.status = status_ptr();
    if (!P.status) return cudaErrorInvalidDevice;
    P.G = pick_segments(p);
    P.cps = (nC + P.G - 1) / P.G;
    const void* kern = reinterpret_cast<const void*>(&bwd_kernel<kFp16, kNorm>);
    void* args[] = {&P};
    return launch_cluster(kern, P.G, p.B * p.H, kThreads, BwdLayout::total + 1024, st, args);
}

}  // namespace

cudaError_t launch_bwd_v2(const ScanParams& p, int dtype, cudaStream_t st) {
    if (dtype == SUBQ_FP16) return p.normalize ? launch<true, true>(p, st) : launch<true, false>(p, st);
    return p.normalize ? launch<false, true>(p, st) : launch<false, false>(p, st);
}

}  // namespace tcs
}  // namespace subq
