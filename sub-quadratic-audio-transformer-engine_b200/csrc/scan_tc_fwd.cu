// Tensor-core forward scan (d = e = 64, bf16/fp16 inputs, fp32 accumulation),
// warp-specialised and pipelined across chunks.
//
// One cluster of G CTAs per (batch, head) sequence; CTA g owns segment g
// (a run of 128-token chunks). Per chunk (t, tau index the chunk's tokens):
//   [S|z]' = [S|z] + phi~(K)^T [V | 1]           tcgen05 64x80x128, TMEM-resident fp32
//   P      = phi~(Q) phi~(K)^T                   tcgen05 128x128x64 -> TMEM P[b]
//   P     <- bf16(P [tau <= t])                  (compute warps, in TMEM)
//   [O|Z]  = phi~(Q) [S_c | z_c]                 tcgen05 128x80x64  -> TMEM O'[b]
//   [O|Z] += P [V | 1]                           tcgen05 128x80x128, A = P from TMEM
//   out_t  = s O_t / max(s Z_t, clamp)  (normalised)  or  s O_t
// with phi~(q) = phi(q), phi~(k) = m phi(k) and s = scale (applied in the fp32
// epilogue, so the 16-bit operands carry no rounded scale): masked keys drop
// out of P, S and z (z = phi~(K)^T 1). The normaliser rides along as 16 extra
// output columns (a ones column beside V), so Z_t = q~_t . z_c + the causal
// row sum of P comes out of the tensor core. The feature map runs on packed
// 16-bit pairs in shared memory.
//
// The state MMA of chunk c is issued first; while the chunk's other MMAs run,
// the compute warps convert [S|z]_c+1 into a bf16 copy (double-buffered in
// shared memory), which is the B operand of chunk c+1.
//
// Roles (448 threads): warps 0-7 compute (TMEM lane = 32 (warp % 4) + lane,
// column half = warp / 4); warps 8-11 transform (feature map in shared
// memory); warp 12 TMA producer; warp 13 MMA issuer. P and O' are
// double-buffered in TMEM: while the tensor core runs chunk c's O MMAs, the
// compute warps mask P of chunk c+1.
//
// Segment prefix: CTA g first sums phi~(K)^T [V | 1] over its own segment
// (phase 1), publishes the sums in shared memory, and after a cluster barrier
// adds those of CTAs 0..g-1 (read over DSMEM) to the incoming state.
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
constexpr int kFwdThreads = 448;
constexpr int kComputeThreads = 256, kTransformThreads = 128;
constexpr int kBarCompute = 1, kBarTransform = 2;  // named barrier ids
constexpr int kBarQuad = 3;  // 3..6: the two compute warps of TMEM lane quadrant q (64 threads)
constexpr int kWarpProducer = 12, kWarpMma = 13;
constexpr int kNX = 80;  // state / output MMA width: 64 value columns + 16 normaliser columns

struct L {
    static constexpr uint32_t stage = 3 * kTile;  // q, k, v
    static constexpr uint32_t q = 0, k = kTile, v = 2 * kTile;
    static constexpr uint32_t ones = kStages * stage;  // 128 x 64 atom, column 0 = 1 (the "| 1" of [V | 1])
    static constexpr uint32_t sbuf = 2 * kD * kD * 2;  // one bf16 [S_c | z_c]: two 64 x 64 atoms (MN-major B)
    static constexpr uint32_t sb = ones + kTile;       // two of them: chunk c reads sb[c % 2]
    static constexpr uint32_t os = sb + 2 * sbuf;      // output staging; before phase 2 the first
                                                       // partial segment sum [64][64] fp32 (the
                                                       // second one uses sb[0])
    static constexpr uint32_t xz = os + kTile;         // their normaliser parts [2][64] fp32
    static constexpr uint32_t bars = xz + 512;
    static constexpr uint32_t tslot = bars + 8 * 24;
    // per-token decay: B_63, B_127 (log2 decay prefix at the chunk midpoint and
    // end) of each stage's chunk, the feature-map group's scan totals, and the
    // log2 decay totals of the two partial segment sums (read over DSMEM)
    static constexpr uint32_t dec = tslot + 16;
    static constexpr uint32_t wt = dec + 8 * kStages;
    static constexpr uint32_t lam = wt + 16;
    static constexpr uint32_t total = lam + 8;
};
static_assert(kD * kD * 4 <= kTile, "exchange fits the staging tile");
static_assert(L::stage % 1024 == 0 && L::ones % 1024 == 0 && L::sb % 1024 == 0 && L::os % 1024 == 0,
              "alignment");
static_assert(L::total + 1024 <= 232448, "shared memory");

enum {
    B_FULL = 0,                    // [kStages] TMA -> transform
    B_TDONE = B_FULL + kStages,    // [kStages] transform -> MMA
    B_EMPTY = B_TDONE + kStages,   // [kStages] MMA -> producer
    B_PFULL = B_EMPTY + kStages,   // [2] MMA -> compute (P ready)
    B_PSDONE = B_PFULL + 2,        // [2] compute -> MMA (P consumed, bf16 P written)
    B_OFULL = B_PSDONE + 2,        // [2] MMA -> compute (O' ready)
    B_ODONE = B_OFULL + 2,         // [2] compute -> MMA (O' consumed)
    B_SFULL = B_ODONE + 2,         // MMA -> compute (state updated)
    B_SBDONE = B_SFULL + 1,        // compute -> MMA (state read, bf16 copy written)
    B_UFULL = B_SBDONE + 1,        // [2] decay, phase 1: MMA -> compute (chunk sum ready)
    B_UDONE = B_UFULL + 2,         // [2] decay, phase 1: compute -> MMA (chunk sum read)
    B_COUNT = B_UDONE + 2
};
static_assert(B_COUNT <= 24, "barrier slots");

// TMEM (512 fp32 columns): P0 [0,128) P1 [128,256) O'0 [256,336) O'1 [336,416)
// S' [416,496) (M = 64 layout; column 64 of S' is z, column 64 of O' is Zi).
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t cP = 0, cO = 256, cS = 416;

struct FwdParams {
    CUtensorMap tm_q, tm_k, tm_v, tm_o;
    ScanParams p;
    int G;
    int cps;
    int* status;
    // handover to the backward (null when not written): header, live-chunk
    // counts and prefix, per-chunk state operands and per-token normalisers
    int* hdr;
    int* nl;
    int* off;
    uint8_t* chunks;
    float* zc;
};

template <bool kFp16, bool kNorm, bool kDecay, bool kRev>
__global__ void __launch_bounds__(kFwdThreads, 1) fwd_kernel(const __grid_constant__ FwdParams P) {
    const ScanParams& p = P.p;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    cg::cluster_group cluster = cg::this_cluster();

    const int g = (int)cluster.block_rank();
    const int bh = blockIdx.y;
    const int b = bh / p.H, h = bh - b * p.H;
    const int hk = h / p.kvg;  // K/V head (grouped K/V: shared by kvg query heads)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nC = (p.N + kC - 1) / kC;

    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::bars);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + L::tslot);
    float* Xs1 = reinterpret_cast<float*>(sm + L::os);  // [64][64] partial sums phi~(K)^T V
    float* Xs2 = reinterpret_cast<float*>(sm + L::sb);
    float* Xz = reinterpret_cast<float*>(sm + L::xz);   // [2][64] partial sums phi~(K)^T 1
    float* dec = reinterpret_cast<float*>(sm + L::dec);
    float* Lam = reinterpret_cast<float*>(sm + L::lam);
    const uint32_t sbase = tc::smem_u32(sm);

    if (tid == 0) {
        // with decay a stage is released by the tensor core (its operands read)
        // and by the compute warps (its decay scalars read)
        // the compute warps signal P, O' and the state operand consumed one arrival
        // per warp (8), each after its own TMEM or shared-memory work
        for (int i = 0; i < B_COUNT; ++i) {
            const bool per_warp = (i >= B_PSDONE && i < B_PSDONE + 2) || (i >= B_ODONE && i < B_ODONE + 2) ||
                                  i == B_SBDONE;
            tc::mbar_init(&bars[i], per_warp ? 8 : (kDecay && i >= B_EMPTY && i < B_EMPTY + kStages) ? 2 : 1);
        }
        tc::fence_mbar_init();
    }
    if (warp == kWarpMma) tc::tmem_alloc(tslot, kTmemCols);
    if (warp >= 8 && warp < 12) {  // the constant ones column (chunks 0-1 of each row; others never read)
        const int r = tid - 256;
        float one[8] = {1.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        store_chunk<kFp16>(sm + L::ones, r, 0, one);
        zero_chunks(sm + L::ones, r, 1, 1);
        tc::fence_proxy_async();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tslot;
    // The segments split the live chunks (up to the sequence's last live token);
    // the chunks after them are zero-filled at the end.
    const int nL = live_chunks(p, b, nC, reinterpret_cast<int*>(tslot + 1));
    if (P.nl && g == 0) {
        // live-chunk counts of the handover; the last CTA to record its count
        // writes their prefix (the backward's work plan)
        if (tid == 0) {
            P.nl[bh] = nL;
            __threadfence();
            tslot[2] = atomicAdd(P.hdr + 5, 1) == p.B * p.H - 1 ? 1u : 0u;
        }
        __syncthreads();
        if (tslot[2]) {
            __threadfence();
            block_prefix(P.nl, P.off, p.B * p.H, reinterpret_cast<int*>(sm + L::xz));
            if (tid == 0) P.hdr[6] = kHandMagic;  // the plan is complete
        }
        __syncthreads();
    }
    if (P.hdr && bh == 0 && g == 0 && tid == 0) {
        P.hdr[1] = kHandMagic;
        P.hdr[2] = p.B * p.H;
        P.hdr[3] = p.N;
        P.hdr[4] = hand_flags(kRev, kNorm, kDecay ? 1 : 0, P.chunks != nullptr);
    }
    const int cps = (nL + P.G - 1) / P.G;
    const int c_begin = min(nL, g * cps);
    const int n = min(nL, c_begin + cps) - c_begin;
    const PrefixShare share = prefix_share(g, P.G, nL, cps);
    const int n1 = share.b - share.a;  // phase-1 chunks: this CTA's share of the segment sums
    // handover slot of chunk c (processing order) of this sequence: the bf16
    // state operand, then z_c
    auto chunk_slot = [&](int c) { return P.chunks + ((size_t)bh * nC + c) * kChunkSlot; };

    constexpr uint32_t idP = tc::idesc_f16<kFp16>(128, 128, false, false);
    constexpr uint32_t idOX = tc::idesc_f16<kFp16>(128, kNX, false, true);  // phi~(Q) [S | z]
    constexpr uint32_t idO = tc::idesc_f16<kFp16>(128, 64, false, true);    // P V
    constexpr uint32_t idSX = tc::idesc_f16<kFp16>(64, kNX, true, true);    // phi~(K)^T [V | 1]

    // Chunks are numbered in processing order; reverse time processes the live
    // chunks from the last one down (act maps to the chunk's place in memory),
    // and each chunk's rows from 127 down (the mask and decay scan follow).
    auto act = [&](int c) { return kRev ? nL - 1 - c : c; };
    // [S|z] (+)= phi~(K)^T [V | 1] over the chunk in stage s (8 K-steps of 16 tokens),
    // into the M = 64 accumulator at TMEM column `col`.
    auto mma_state = [&](int s, bool first, uint32_t col = cS) {
        const uint32_t ka = sbase + s * L::stage + L::k, va = sbase + s * L::stage + L::v;
        const uint32_t lbo = L::ones - (s * L::stage + L::v);  // V atom -> ones atom
        const uint32_t n80 = kNorm ? idSX : tc::idesc_f16<kFp16>(64, 64, true, true);
        const uint64_t da = tc::sdesc_sw128(ka, kTile, 1024), db = tc::sdesc_sw128(va, lbo, 1024);
        // 8 K-steps of 16 tokens, each 2048 bytes on (a descriptor step of 128)
        tc::mma_f16_x8(tmem + col, da, 128, db, 128, n80, first ? 0u : 1u);
    };

    // Chunk of pipeline slot j: phase-1 slots (j < n1) visit the share in an
    // order rotated per sequence, so that the clusters do not all read the
    // same offset of their sequences at the same time (the sums do not depend
    // on the order); phase-2 slots run the segment in order.
    const int rot = (!kDecay && n1 > 0) ? (bh * 7) % n1 : 0;  // decayed sums run in order
    auto chunk_of = [&](int j) {
        if (j >= n1) return c_begin + (j - n1);
        const int r = j + rot;
        return share.a + (r >= n1 ? r - n1 : r);
    };

    bool ok = true;

    auto produce = [&](int jlo, int jhi) {
        for (int j = jlo; j < jhi && ok; ++j) {
            const bool ph2 = j >= n1;
            const int chunk = chunk_of(j);
            const int s = j % kStages, u = j / kStages;
            if (u >= 1) ok = wait_bar(&bars[B_EMPTY + s], (u - 1) & 1, P.status);
            if (!ok) break;
            uint8_t* base = sm + s * L::stage;
            tc::mbar_arrive_expect_tx(&bars[B_FULL + s], (ph2 ? 3u : 2u) * kTile);
            if (ph2) tc::tma_load_4d(base + L::q, &P.tm_q, 0, act(chunk) * kC, h, b, &bars[B_FULL + s]);
            tc::tma_load_4d(base + L::k, &P.tm_k, 0, act(chunk) * kC, hk, b, &bars[B_FULL + s]);
            tc::tma_load_4d(base + L::v, &P.tm_v, 0, act(chunk) * kC, hk, b, &bars[B_FULL + s]);
        }
    };
    auto transform = [&](int jlo, int jhi) {
        const int r = tid - 256;
        // (mask byte and log(gamma) loaded a chunk ahead, raw: they are tested and
        // scaled after the wait, so the loads overlap it)
        int mr_next = jlo < jhi ? mask_raw_at(p, b, act(chunk_of(jlo)) * kC + r) : 0;
        float lg_next = (kDecay && jlo < jhi) ? decay_log_raw(p, b, h, act(chunk_of(jlo)) * kC + r) : 0.f;
        for (int j = jlo; j < jhi && ok; ++j) {
            const bool ph2 = j >= n1;
            const int s = j % kStages, u = j / kStages;
            const int mr = mr_next;
            const float lg = lg_next;
            if (j + 1 < jhi) {  // in flight during the wait
                mr_next = mask_raw_at(p, b, act(chunk_of(j + 1)) * kC + r);
                if (kDecay) lg_next = decay_log_raw(p, b, h, act(chunk_of(j + 1)) * kC + r);
            }
            ok = tc::bar_and(kBarTransform, kTransformThreads, wait_bar(&bars[B_FULL + s], u & 1, P.status)) && ok;
            if (!ok) break;
            const float m = mr != 0 ? 1.f : 0.f;
            const float a = (kDecay && m != 0.f) ? lg * kLog2e : 0.f;
            uint8_t* base = sm + s * L::stage;
            if constexpr (kDecay) {
                float b63, b127;
                float* wt = reinterpret_cast<float*>(sm + L::wt);
                const float br = kRev ? decay_scan128_rev(a, r, wt, kBarTransform, b63, b127)
                                      : decay_scan128(a, r, wt, kBarTransform, b63, b127);
                if (r == 0) {
                    dec[2 * s] = b63;
                    dec[2 * s + 1] = b127;
                    if (!decay_in_range(b63, b127)) p.fallback[bh] = 1;
                }
                if (ph2) chunks_phi_scaled<kFp16>(base + L::q, r, true, exp2_fast(br - b63));
                chunks_phi_scaled<kFp16>(base + L::k, r, m != 0.f, exp2_fast(b63 - br));
            } else {
                if (ph2) chunks_phi<kFp16>(base + L::q, r, 0, 8, true);  // scale is applied in the epilogue
                chunks_phi<kFp16>(base + L::k, r, 0, 8, m != 0.f);
            }
            tc::fence_proxy_async();
            tc::bar_sync(kBarTransform, kTransformThreads);
            if (r == 0) tc::mbar_arrive(&bars[B_TDONE + s]);
        }
    };

    // ------------------------------------------------------------ phase 1
    if (warp == kWarpProducer) {
        if (lane == 0) {
            tc::prefetch_tmap(&P.tm_q);
            tc::prefetch_tmap(&P.tm_k);
            tc::prefetch_tmap(&P.tm_v);
            tc::prefetch_tmap(&P.tm_o);
            produce(0, n1 + min(n, kStages));  // later phase-2 stages are freed only after the barriers
        }
        __syncwarp();
    } else if (warp >= 8 && warp < 12) {
        transform(0, n1);
    } else if (warp == kWarpMma) {
        // (the whole warp runs the MMA role, converged; one elected lane issues)
        if (kDecay) {
            // decayed sums: each chunk's phi~(K')^T [V | 1] into one of two
            // buffers in the O' columns; the compute warps chain them
            for (int j = 0; j < n1 && ok; ++j) {
                const int s = j % kStages, u = j / kStages;
                ok = wait_bar(&bars[B_TDONE + s], u & 1, P.status);
                if (ok && j >= 2) ok = wait_bar(&bars[B_UDONE + (j & 1)], ((j >> 1) - 1) & 1, P.status);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) break;
                tc::tc_fence_after();
                mma_state(s, true, cO + (j & 1) * kNX);
                tc::mma_commit_w(&bars[B_EMPTY + s]);
                tc::mma_commit_w(&bars[B_UFULL + (j & 1)]);
            }
        } else {
            // the share's two partial sums accumulate in S' (before the segment
            // boundary) and in the still unused P columns (after it)
            bool first1 = true, first2 = true;
            for (int j = 0; j < n1 && ok; ++j) {
                const int s = j % kStages, u = j / kStages;
                ok = __all_sync(0xffffffffu, wait_bar(&bars[B_TDONE + s], u & 1, P.status));
                if (!ok) break;
                tc::tc_fence_after();
                if (chunk_of(j) < share.x) {
                    mma_state(s, first1, cS);
                    first1 = false;
                } else {
                    mma_state(s, first2, cP);
                    first2 = false;
                }
                tc::mma_commit_w(&bars[B_EMPTY + s]);
            }
            if (n1 > 0 && ok) tc::mma_commit_w(&bars[B_SFULL]);
        }
        __syncwarp();
    }
    uint32_t sfull_count = 0;
    if (kDecay && warp < 8) {
        // Horner over the share in chunk order: X = exp(b_end) X + exp(b_end - b_m) U'
        // per piece, and the piece's log2 decay total
        const int quad = warp & 3, hf = warp >> 2, srow = quad * 16 + lane;
        const uint32_t loff = (uint32_t)(quad * 32) << 16;
        float X[32], xz = 0.f, lam0 = 0.f, lam1 = 0.f;
#pragma unroll
        for (int x = 0; x < 32; ++x) X[x] = 0.f;
        int piece = 0;
        auto flush = [&](int pc) {
            float* dst = pc == 0 ? Xs1 : Xs2;
            if (lane < 16) {
#pragma unroll
                for (int x = 0; x < 32; ++x) dst[xch(srow, hf, x)] = X[x];
                if (hf == 0) Xz[pc * 64 + srow] = xz;
            }
        };
        for (int j = 0; j < n1 && ok; ++j) {
            const int s = j % kStages;
            if (piece == 0 && chunk_of(j) >= share.x) {
                if (j > 0) flush(0);
#pragma unroll
                for (int x = 0; x < 32; ++x) X[x] = 0.f;
                xz = 0.f;
                piece = 1;
            }
            ok = tc::bar_and(kBarCompute, kComputeThreads,
                             wait_bar(&bars[B_UFULL + (j & 1)], (j >> 1) & 1, P.status) &&
                                 wait_bar(&bars[B_TDONE + s], (j / kStages) & 1, P.status)) && ok;
            if (!ok) break;
            tc::tc_fence_after();
            const float b63 = dec[2 * s], b127 = dec[2 * s + 1];
            const float ld = exp2_fast(b127), mu = exp2_fast(b127 - b63);
            float uu[32];
            tc::tmem_ld32(tmem + cO + (j & 1) * kNX + loff + hf * 32, uu);
#pragma unroll
            for (int x = 0; x < 32; ++x) X[x] = fmaf(ld, X[x], mu * uu[x]);
            if (kNorm && hf == 0) xz = fmaf(ld, xz, mu * tmem_ld1(tmem + cO + (j & 1) * kNX + loff + 64));
            if (piece) lam1 += b127;
            else lam0 += b127;
            tc::tc_fence_before();
            tc::bar_sync(kBarCompute, kComputeThreads);
            if (tid == 0) {
                tc::mbar_arrive(&bars[B_UDONE + (j & 1)]);
                tc::mbar_arrive(&bars[B_EMPTY + s]);
            }
        }
        if (n1 > 0) flush(piece);
        if (tid == 0) {
            Lam[0] = lam0;
            Lam[1] = lam1;
        }
    } else if (warp < 8) {
        const int quad = warp & 3, hf = warp >> 2, srow = quad * 16 + lane;
        const uint32_t loff = (uint32_t)(quad * 32) << 16;
        if (n1 > 0) {
            ok = tc::bar_and(kBarCompute, kComputeThreads, wait_bar(&bars[B_SFULL], 0, P.status)) && ok;
            sfull_count = 1;
            tc::tc_fence_after();
        }
        const bool have1 = ok && min(share.b, share.x) > share.a, have2 = ok && share.b > share.x;
#pragma unroll
        for (int piece = 0; piece < 2; ++piece) {
            const bool have = piece == 0 ? have1 : have2;
            const uint32_t col = piece == 0 ? cS : cP;
            float* X = piece == 0 ? Xs1 : Xs2;
            float v[32];
            if (have) {
                tc::tmem_ld32(tmem + col + loff + hf * 32, v);
            } else {
#pragma unroll
                for (int x = 0; x < 32; ++x) v[x] = 0.f;
            }
            if (lane < 16) {
#pragma unroll
                for (int x = 0; x < 32; ++x) X[xch(srow, hf, x)] = v[x];
            }
            if (hf == 0) {
                const float zv = (kNorm && have) ? tmem_ld1(tmem + col + loff + 64) : 0.f;
                if (lane < 16) Xz[piece * 64 + srow] = zv;
            }
        }
    }
    tc::tc_fence_before();
    cluster.sync();
    tc::tc_fence_after();

    // ------------------------------------------------------ segment prefix
    // S_in plus every partial sum of a segment before this CTA's, read over DSMEM
    // (decayed: S_in decays over all the pieces and each piece over the ones after
    // it, the Horner chain written as one weighted sum)
    float v[32], z = 0.f;
#pragma unroll
    for (int x = 0; x < 32; ++x) v[x] = 0.f;
    if (warp < 8) {
        const int quad = warp & 3, hf = warp >> 2, row = quad * 16 + (lane & 15);
        int pr[16], pb[16], np = 0;  // the pieces of the segments before this one, in order
        for (int r = 0; r < P.G; ++r) {
            const PrefixShare sr = prefix_share(r, P.G, nL, cps);
            if (min(sr.b, sr.x) > sr.a && sr.seg < g) pr[np] = r, pb[np++] = 0;
            if (sr.b > sr.x && sr.seg + 1 < g) pr[np] = r, pb[np++] = 1;
        }
        float wl = 1.f, w_in = 1.f;
        if (kDecay) {
            const float lam = lane < np ? cluster.map_shared_rank(Lam, pr[lane])[pb[lane]] : 0.f;
            float total;
            wl = exp2_fast(piece_exponent(lam, lane, true, total));
            w_in = exp2_fast(total);
        }
        if (lane < 16) {
            if (p.S_in) {
                const float* src = p.S_in + ((int64_t)bh * kD + row) * kD + hf * 32;
#pragma unroll
                for (int x = 0; x < 32; ++x) v[x] = w_in * src[x];
            }
            if (kNorm && hf == 0) z = p.z_in ? w_in * p.z_in[(int64_t)bh * kD + row] : 0.f;
        }
        gather_pieces(
            np, pr, pb, wl, row, hf, lane,
            [&](int r, int pc) { return cluster.map_shared_rank(pc == 0 ? Xs1 : Xs2, r); },
            [&](int r, int pc) { return cluster.map_shared_rank(Xz, r) + pc * 64; }, kNorm && hf == 0, v, z);
        if (lane >= 16) {  // lanes 16-31 keep zeros (the M = 64 state rows live in lanes 0-15)
#pragma unroll
            for (int x = 0; x < 32; ++x) v[x] = 0.f;
            z = 0.f;
        }
    }
    tc::tc_fence_before();
    cluster.sync();  // remote reads done before the exchange buffers are reused
    tc::tc_fence_after();
    if (warp < 8) {
        const int quad = warp & 3, hf = warp >> 2, srow = quad * 16 + lane;
        const uint32_t loff = (uint32_t)(quad * 32) << 16;
        // the segment's start state for the backward of the same call (lanes
        // 0-15 hold rows srow), and the header with the segment count
        if (p.seg_out && lane < 16) {
            float* dst = p.seg_out + 64 + ((int64_t)(bh * P.G + g) * kD + srow) * (kD + 1);
#pragma unroll
            for (int x = 0; x < 32; ++x) dst[hf * 32 + x] = v[x];
            if (hf == 0) dst[kD] = kNorm ? z : 0.f;
        }
        if (p.seg_out && bh == 0 && g == 0 && tid == 0) *reinterpret_cast<int*>(p.seg_out) = P.G;
        // (with decay the state stays in these registers and the first chunk's
        // operand is written at the start of phase 2, scaled by its exp(b_m))
        if (!kDecay && lane < 16) {
#pragma unroll
            for (int x = 0; x < 4; ++x) store_chunk<kFp16>(sm + L::sb, srow, hf * 4 + x, v + 8 * x);
        }
        if (!kDecay) tc::tmem_st32(tmem + cS + loff + hf * 32, v);
        if (hf == 0) {
            if (lane < 16) {
                float zc8[8] = {z, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                if (!kDecay) store_chunk<kFp16>(sm + L::sb + kD * kD * 2, srow, 0, zc8);
                // columns 1-15 of the z atom are read as zeros (N = 80) in both buffers
                zero_chunks(sm + L::sb + kD * kD * 2, srow, 1, 1);
                zero_chunks(sm + L::sb + L::sbuf + kD * kD * 2, srow, 1, 1);
            }
            if (!kDecay) {
                float w[32];
#pragma unroll
                for (int x = 0; x < 32; ++x) w[x] = 0.f;
                w[0] = (lane < 16) ? z : 0.f;
                tc::tmem_st32(tmem + cS + loff + 64, w);
            }
            if (P.chunks && n > 0 && lane < 16)
                reinterpret_cast<float*>(chunk_slot(c_begin) + kSAtom)[srow] = kNorm ? z : 0.f;
        }
        tc::fence_proxy_async();
    }
    tc::tc_fence_before();
    __syncthreads();  // prefix state in place
    tc::tc_fence_after();
    if (P.chunks && n > 0 && tid == 0) {  // the first chunk's state operand to the handover
        tc::bulk_store(chunk_slot(c_begin), sm + L::sb, kSAtom);
        tc::bulk_commit();
    }

    // ============================================================ phase 2
    if (warp == kWarpProducer) {
        if (lane == 0) produce(n1 + min(n, kStages), n1 + n);
        __syncwarp();
    } else if (warp >= 8 && warp < 12) {
        transform(n1, n1 + n);
    } else if (warp == kWarpMma) {
        {  // warp-converged; one elected lane issues each MMA
            auto issue_p = [&](int i) -> bool {  // P[i % 2] = phi~(Q) phi~(K)^T
                const int j = n1 + i, s = j % kStages, u = j / kStages, bf = i & 1;
                if (!__all_sync(0xffffffffu, wait_bar(&bars[B_TDONE + s], u & 1, P.status))) return false;
                if (i >= 2 && !__all_sync(0xffffffffu, wait_bar(&bars[B_PSDONE + bf], ((i >> 1) - 1) & 1, P.status)))
                    return false;
                tc::tc_fence_after();
                const uint64_t dq = tc::sdesc_sw128(sbase + s * L::stage + L::q, 16, 1024);
                const uint64_t dk = tc::sdesc_sw128(sbase + s * L::stage + L::k, 16, 1024);
                // 4 K-steps of 16 features, each 32 bytes on (a descriptor step of 2)
                tc::mma_f16_x4(tmem + cP + bf * 128, dq, 2, dk, 2, idP, 0u);
                tc::mma_commit_w(&bars[B_PFULL + bf]);
                return true;
            };
            if (n > 0) ok = issue_p(0);
            for (int i = 0; i < n && ok; ++i) {
                const int j = n1 + i, s = j % kStages, bf = i & 1, pu = i >> 1;
                // [S|z]_c+1 first: the compute warps turn it into the next chunk's
                // bf16 operand while this chunk's other MMAs run. It may start once
                // the previous refresh has read S' (and written sb[i % 2]).
                if (i >= 1) ok = __all_sync(0xffffffffu, wait_bar(&bars[B_SBDONE], (i - 1) & 1, P.status));
                if (!ok) break;
                tc::tc_fence_after();
                mma_state(s, kDecay);  // with decay: this chunk's sum alone, chained in registers
                tc::mma_commit_w(&bars[B_SFULL]);
                if (i + 1 < n) ok = issue_p(i + 1);
                if (ok) ok = wait_bar(&bars[B_PSDONE + bf], pu & 1, P.status);
                if (ok && i >= 2) ok = wait_bar(&bars[B_ODONE + bf], (pu - 1) & 1, P.status);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) break;
                tc::tc_fence_after();
                const uint32_t tOb = tmem + cO + bf * kNX;
                const uint64_t dq = tc::sdesc_sw128(sbase + s * L::stage + L::q, 16, 1024);
                const uint64_t dsb = tc::sdesc_sw128(sbase + L::sb + (i & 1) * L::sbuf, kD * kD * 2, 1024);
                tc::mma_f16_x4(tOb, dq, 2, dsb, 128, kNorm ? idOX : idO, 0u);  // [O | Zi] = phi~(Q) [S_c | z_c]
                // [O | Zi] += P [V | 1]: bf16 P read from TMEM (8 columns per 16 tokens);
                // the ones column adds the causal row sums to the normaliser
                const uint32_t lbo = kNorm ? L::ones - (s * L::stage + L::v) : kTile;
                const uint64_t dv = tc::sdesc_sw128(sbase + s * L::stage + L::v, lbo, 1024);
                tc::mma_f16_ts_x8(tOb, tmem + cP + bf * 128, 8, dv, 128, kNorm ? idOX : idO, 1u);
                tc::mma_commit_w(&bars[B_OFULL + bf]);
                tc::mma_commit_w(&bars[B_EMPTY + s]);
            }
        }
        __syncwarp();
    } else if (warp < 8) {
        const int quad = warp & 3, hf = warp >> 2;
        const int row = quad * 32 + lane, srow = quad * 16 + lane;
        const uint32_t loff = (uint32_t)(quad * 32) << 16;
        // P of chunk i: causal mask on the diagonal block and the bf16 copy packed
        // back into the first 64 TMEM columns of P[b] (the A operand of O += P V).
        auto mask_p = [&](int i) -> bool {
            const int bf = i & 1;
            if (!tc::bar_and(kBarCompute, kComputeThreads, wait_bar(&bars[B_PFULL + bf], (i >> 1) & 1, P.status)))
                return false;
            tc::tc_fence_after();
            using E = Elem<kFp16>;
            uint32_t packed[32];
            // causal: keep tau <= t (the block right of the diagonal blocks is zero);
            // reverse: keep tau >= t (the block left of them is zero)
            if (kRev ? (hf == 0 && quad >= 2) : (hf == 1 && quad < 2)) {
#pragma unroll
                for (int x = 0; x < 32; ++x) packed[x] = 0u;
            } else if (kDecay) {  // 32 columns at a time: the decayed state occupies 33 registers
                const bool diag = (hf == (quad >> 1));
#pragma unroll
                for (int part = 0; part < 2; ++part) {
                    float v[32];
                    tc::tmem_ld32(tmem + cP + bf * 128 + loff + hf * 64 + part * 32, v);
#pragma unroll
                    for (int x = 0; x < 32; ++x)
                        if (diag && (kRev ? (hf * 64 + part * 32 + x) < row : (hf * 64 + part * 32 + x) > row)) v[x] = 0.f;
#pragma unroll
                    for (int x = 0; x < 16; ++x) {
                        typename E::T2 h2 = E::from2(v[2 * x], v[2 * x + 1]);
                        packed[part * 16 + x] = *reinterpret_cast<uint32_t*>(&h2);
                    }
                }
            } else {
                const bool diag = (hf == (quad >> 1));
                float v[64];
                tc::tmem_ld32(tmem + cP + bf * 128 + loff + hf * 64, v);
                tc::tmem_ld32(tmem + cP + bf * 128 + loff + hf * 64 + 32, v + 32);
#pragma unroll
                for (int x = 0; x < 64; ++x)
                    if (diag && (kRev ? (hf * 64 + x) < row : (hf * 64 + x) > row)) v[x] = 0.f;
#pragma unroll
                for (int x = 0; x < 32; ++x) {
                    typename E::T2 h2 = E::from2(v[2 * x], v[2 * x + 1]);
                    packed[x] = *reinterpret_cast<uint32_t*>(&h2);
                }
            }
            // the packed half of warp (quad, 1) lands in columns that warp (quad, 0)
            // reads as fp32: the two warps of a lane quadrant meet first
            tc::tc_fence_before();
            tc::bar_sync(kBarQuad + quad, 64);
            tc::tc_fence_after();
            tc::tmem_st32_raw(tmem + cP + bf * 128 + loff + hf * 32, packed);
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bars[B_PSDONE + bf]);
            return true;
        };
        // decay: bf16 f [S | z] (registers v, z) into the operand buffer `dst`
        auto write_operand = [&](uint8_t* dst, float f) {
            if (lane < 16) {
                float w[8];
#pragma unroll
                for (int x = 0; x < 4; ++x) {
#pragma unroll
                    for (int y = 0; y < 8; ++y) w[y] = f * v[8 * x + y];
                    store_chunk<kFp16>(dst, srow, hf * 4 + x, w);
                }
                if (kNorm && hf == 0) {
                    float zc8[8] = {f * z, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                    store_chunk<kFp16>(dst + kD * kD * 2, srow, 0, zc8);
                }
            }
        };
        if (kDecay && n > 0) {  // the first chunk's operand exp(b_m) [S | z]_in
            const int s0 = n1 % kStages;
            ok = tc::bar_and(kBarCompute, kComputeThreads,
                             wait_bar(&bars[B_TDONE + s0], (n1 / kStages) & 1, P.status)) && ok;
            if (ok) write_operand(sm + L::sb, exp2_fast(dec[2 * s0]));
            tc::fence_proxy_async();
        }
        if (n > 0 && ok) ok = mask_p(0);
        // the output rows' mask values, loaded one chunk ahead (off the epilogue's path)
        int mr_next = n > 0 ? mask_raw_at(p, b, act(c_begin) * kC + row) : 0;  // (raw: tested where used)
        for (int i = 0; i < n && ok; ++i) {
            const int c = c_begin + i, bf = i & 1, pu = i >> 1;
            const int mr_row = mr_next;
            if (i + 1 < n) mr_next = mask_raw_at(p, b, act(c + 1) * kC + row);
            // state refresh: bf16 [S | z]_c+1 into sb[(i + 1) % 2], the next chunk's operand
            ok = tc::bar_and(kBarCompute, kComputeThreads,
                             wait_bar(&bars[B_SFULL], sfull_count & 1, P.status)) && ok;
            ++sfull_count;
            if (!ok) break;
            tc::tc_fence_after();
            if constexpr (kDecay) {
                // [S|z]_c+1 = exp(b_end) [S|z]_c + exp(b_end - b_m) U'_c in registers; the
                // operand of chunk c+1 carries its own exp(b_m). The decay scalars of
                // both chunks are final once their feature maps are (TDONE), and their
                // stages stay until this warp group releases them.
                const int j = n1 + i, s = j % kStages, s1 = (j + 1) % kStages;
                ok = tc::bar_and(kBarCompute, kComputeThreads,
                                 wait_bar(&bars[B_TDONE + s], (j / kStages) & 1, P.status) &&
                                     (i + 1 >= n ||
                                      wait_bar(&bars[B_TDONE + s1], ((j + 1) / kStages) & 1, P.status))) && ok;
                if (!ok) break;
                const float b63 = dec[2 * s], b127 = dec[2 * s + 1];
                const float ld = exp2_fast(b127), mu = exp2_fast(b127 - b63);
                float uu[32];
                tc::tmem_ld32(tmem + cS + loff + hf * 32, uu);
#pragma unroll
                for (int x = 0; x < 32; ++x) v[x] = fmaf(ld, v[x], mu * uu[x]);
                if (kNorm && hf == 0) z = fmaf(ld, z, mu * tmem_ld1(tmem + cS + loff + 64));
                if (i + 1 < n) write_operand(sm + L::sb + ((i + 1) & 1) * L::sbuf, exp2_fast(dec[2 * s1]));
                tc::fence_proxy_async();
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&bars[B_SBDONE]);
                tc::bar_sync(kBarCompute, kComputeThreads);  // every read of the stage's decay scalars
                if (tid == 0) tc::mbar_arrive(&bars[B_EMPTY + s]);
            } else {
            {
                uint8_t* sbn = sm + L::sb + ((i + 1) & 1) * L::sbuf;
                float v[32];
                tc::tmem_ld32(tmem + cS + loff + hf * 32, v);
                if (lane < 16) {
#pragma unroll
                    for (int x = 0; x < 4; ++x) store_chunk<kFp16>(sbn, srow, hf * 4 + x, v + 8 * x);
                }
                if (kNorm && hf == 0) {
                    const float zv = tmem_ld1(tmem + cS + loff + 64);
                    if (lane < 16) {
                        float zc8[8] = {zv, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                        store_chunk<kFp16>(sbn + kD * kD * 2, srow, 0, zc8);
                        if (P.chunks && i + 1 < n) reinterpret_cast<float*>(chunk_slot(c + 1) + kSAtom)[srow] = zv;
                    }
                }
            }
            tc::fence_proxy_async();
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bars[B_SBDONE]);
            if (P.chunks && i + 1 < n) {  // the next chunk's state operand to the handover
                tc::bar_sync(kBarCompute, kComputeThreads);
                if (tid == 0) {
                    tc::bulk_store(chunk_slot(c + 1), sm + L::sb + ((i + 1) & 1) * L::sbuf, kSAtom);
                    tc::bulk_commit();
                }
            }
            }
            if (i + 1 < n) {
                ok = mask_p(i + 1);
                if (!ok) break;
            }
            // output of chunk i
            ok = tc::bar_and(kBarCompute, kComputeThreads, wait_bar(&bars[B_OFULL + bf], pu & 1, P.status)) && ok;
            if (!ok) break;
            tc::tc_fence_after();
            float o[32];
            tc::tmem_ld32(tmem + cO + bf * kNX + loff + hf * 32, o);
            float zi = 0.f;
            if (kNorm) zi = tmem_ld1(tmem + cO + bf * kNX + loff + 64);
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bars[B_ODONE + bf]);  // this warp has read O'[bf]
            if (tid == 0) tc::bulk_wait_read0();  // the previous chunk's output has left the staging tile
            tc::bar_sync(kBarCompute, kComputeThreads);
            {
                // O' and its normaliser column carry phi(q) unscaled: o = s O' / max(s Z', clamp)
                float inv = (mr_row != 0 ? 1.f : 0.f) * p.scale;
                if (kNorm) {
                    const float zc = max_nan(p.scale * zi, p.clamp_min);
                    inv = inv / zc;
                    if (P.zc && hf == 0 && act(c) * kC + row < p.N) P.zc[(int64_t)bh * p.N + act(c) * kC + row] = zc;
                }
#pragma unroll
                for (int x = 0; x < 32; ++x) o[x] *= inv;
#pragma unroll
                for (int x = 0; x < 4; ++x) store_chunk<kFp16>(sm + L::os, row, hf * 4 + x, o + 8 * x);
            }
            tc::fence_proxy_async();
            tc::bar_sync(kBarCompute, kComputeThreads);
            if (tid == 0) {
                tc::tma_store_4d(&P.tm_o, sm + L::os, 0, act(c) * kC, h, b);
                tc::bulk_commit();
            }
        }
        if (g == P.G - 1 && ok) {  // final state of the whole sequence
            float fs[32];
            if (kDecay) {
#pragma unroll
                for (int x = 0; x < 32; ++x) fs[x] = v[x];
            } else {
                tc::tmem_ld32(tmem + cS + loff + hf * 32, fs);
            }
            if (lane < 16 && p.S_out) {
                float* dst = p.S_out + ((int64_t)bh * kD + srow) * kD + hf * 32;
#pragma unroll
                for (int x = 0; x < 32; ++x) dst[x] = fs[x];
            }
            if (p.z_out && hf == 0) {
                const float zv = !kNorm ? 0.f : kDecay ? z : tmem_ld1(tmem + cS + loff + 64);
                if (lane < 16) p.z_out[(int64_t)bh * kD + srow] = zv;
            }
        }
        // zero outputs of the chunks past the last live token (round-robin over the cluster)
        if (nL + g < nC) {
            if (tid == 0) tc::bulk_wait_read0();  // the staging tile has been read
            tc::bar_sync(kBarCompute, kComputeThreads);
            zero_chunks(sm + L::os, row, hf * 4, 4);
            tc::fence_proxy_async();
            tc::bar_sync(kBarCompute, kComputeThreads);
            if (tid == 0) {
                for (int d = nL + g; d < nC; d += P.G) tc::tma_store_4d(&P.tm_o, sm + L::os, 0, d * kC, h, b);
                tc::bulk_commit();
            }
        }
        if (tid == 0) tc::bulk_wait0();
    }

    tc::tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma) tc::tmem_dealloc(tmem, kTmemCols);
}

template <bool kFp16, bool kNorm, bool kDecay, bool kRev = false>
cudaError_t launch(const ScanParams& p, cudaStream_t st) {
    FwdParams P;
    memset(&P, 0, sizeof(P));
    P.p = p;
    const int dt = kFp16 ? SUBQ_FP16 : SUBQ_BF16;
    if (!make_map(&P.tm_q, p.q, dt, p.N, p.H, p.B, p.q_sn, p.q_sh, p.q_sb) ||
        !make_map(&P.tm_k, p.k, dt, p.N, p.H / p.kvg, p.B, p.k_sn, p.k_sh, p.k_sb) ||
        !make_map(&P.tm_v, p.v, dt, p.N, p.H / p.kvg, p.B, p.v_sn, p.v_sh, p.v_sb) ||
        !make_map(&P.tm_o, p.o, dt, p.N, p.H, p.B, p.o_sn, p.o_sh, p.o_sb))
        return cudaErrorInvalidValue;
    const int nC = (p.N + kC - 1) / kC;
    P.status = status_ptr();
    if (!P.status) return cudaErrorInvalidDevice;
    const void* kern = reinterpret_cast<const void*>(&fwd_kernel<kFp16, kNorm, kDecay, kRev>);
    P.G = pick_segments(p, kern, kFwdThreads, L::total + 1024);
    P.cps = (nC + P.G - 1) / P.G;
    if (p.seg_out) {
        const HandLayout hl(p.B * p.H, p.N, P.G, !kDecay);
        char* base = reinterpret_cast<char*>(p.seg_out);
        P.hdr = reinterpret_cast<int*>(base);
        P.nl = reinterpret_cast<int*>(base + hl.nl);
        P.off = reinterpret_cast<int*>(base + hl.off);
        if (!kDecay) {
            P.chunks = reinterpret_cast<uint8_t*>(base + hl.chunks);
            if (kNorm) P.zc = reinterpret_cast<float*>(base + hl.zc);
        }
    }
    void* args[] = {&P};
    return launch_cluster(kern, P.G, p.B * p.H, kFwdThreads, L::total + 1024, st, args);
}

}  // namespace

// Segment count the forward launches with (every instantiation has the same
// block size and shared memory, so one of them answers for all).
int fwd_segment_count(const ScanParams& p) {
    const void* kern = reinterpret_cast<const void*>(&fwd_kernel<false, true, false, false>);
    return pick_segments(p, kern, kFwdThreads, L::total + 1024);
}

cudaError_t launch_fwd_v2(const ScanParams& p, int dtype, cudaStream_t st) {
    if (p.reverse) {  // reverse time: normalised form only
        if (!p.normalize) return cudaErrorInvalidValue;
        if (p.decay_mode != SUBQ_DECAY_NONE) {
            if (dtype != SUBQ_BF16 || !p.fallback) return cudaErrorInvalidValue;
            return launch<false, true, true, true>(p, st);
        }
        return dtype == SUBQ_FP16 ? launch<true, true, false, true>(p, st) : launch<false, true, false, true>(p, st);
    }
    if (p.decay_mode != SUBQ_DECAY_NONE) {  // bf16 only (the factorised decay needs its exponent range)
        if (dtype != SUBQ_BF16 || !p.fallback) return cudaErrorInvalidValue;
        return p.normalize ? launch<false, true, true>(p, st) : launch<false, false, true>(p, st);
    }
    if (dtype == SUBQ_FP16) return p.normalize ? launch<true, true, false>(p, st) : launch<true, false, false>(p, st);
    return p.normalize ? launch<false, true, false>(p, st) : launch<false, false, false>(p, st);
}

}  // namespace tcs
}  // namespace subq
