// Tensor-core backward scan (d = e = 64, bf16/fp16 inputs, fp32 accumulation),
// warp-specialised and pipelined across chunks.
//
// One cluster of G CTAs per (batch, head) sequence; CTA g owns segment g.
// With q^ = phi(q), k^ = m phi(k) (raw features; s = scale is applied in the
// fp32 epilogues), the forward's num_t = s (q^_t S_c + sum_{tau<=t} P_t,tau v_tau)
// and Z_t = s (q^_t z_c + sum_{tau<=t} P_t,tau) with P = q^ k^T, the quotient
// rule of the normaliser gives, per 128-token chunk,
//   o^_t = m_t dO_t / Zc_t,      c_t = -(m_t dO_t . num_t) / Zc_t^2,   Zc = max(Z, clamp)
//   dA   = ([o^ | c] [V | 1]^T) [tau <= t]
//   dQ~  = dA K^ + [o^ | c] [S_c | z_c]^T                    dq = s dQ~ phi'(q)
//   dK~  = s (dA^T q^ + [V | 1] [dS^ | dz^]^T)              dk = dK~ phi'(k) m
//   dV   = s ((P [tau <= t])^T o^ + K^ dS^)                 dv = dV m
// with S_c, z_c the prefix state of the chunk and dS^, dz^ = sum over later
// tokens of q^^T [o^ | c] (the raw suffix adjoint). phi'(x) = min(phi(x), 1).
// Every normaliser term rides on the tensor core as 16 extra columns: a ones
// atom beside V, a c atom beside o^, a z atom beside S.
//
// Phases of a CTA (chunk order within the segment):
//   A  segment sums of K^^T [V | 1] (CTAs g < G-1)              -> DSMEM -> S_c, z_c
//   B  ascending: recompute [num | Z], form o^ and c, emit dq, keep (Zc_t, c_t)
//      in the workspace, sum q^^T [o^ | c] over the segment     -> DSMEM -> suffix
//   C  descending: rebuild o^ from dO and (Zc, c); P^T = K^ q^^T and
//      dA^T = [V | 1] [o^ | c]^T directly in the key-major orientation, so that
//      dK and dV are tensor-core products with A read from TMEM; emit dk, dv.
//
// Roles (448 threads): warps 0-7 compute (TMEM lane = 32 (warp % 4) + lane,
// column half = warp / 4), warps 8-11 feature map (packed 16-bit, in shared
// memory), warp 12 TMA producer, warp 13 MMA issuer. The prefix state S_c
// (phase B) and the suffix adjoint dS^ (phase C) accumulate in TMEM; their bf16
// copies, the B operands of the next chunk, are double-buffered in shared
// memory and refreshed while the chunk's other MMAs run. P and dA are masked
// and packed to bf16 in place in TMEM and consumed from there (A operand).
//
// Reference: python/subq_audio/autograd.py:441-544 (quotient rule :497-499,
// chunked adjoint :172-289); src/kernels/attention_backward.cpp:165-229.
#include "tc_common.cuh"

namespace cg = cooperative_groups;

namespace subq {
namespace tcs {
namespace {

constexpr int kStages = 2;
constexpr int kBwdThreads = 448;
constexpr int kComputeThreads = 256, kTransformThreads = 128;
constexpr int kBarCompute = 1, kBarTransform = 2;
constexpr int kWarpProducer = 12, kWarpMma = 13;
constexpr int kNX = 80;  // 64 value columns + 16 normaliser columns

struct BL {
    static constexpr uint32_t stage = 4 * kTile;  // q, k, v, dO
    static constexpr uint32_t q = 0, k = kTile, v = 2 * kTile, g = 3 * kTile;
    static constexpr uint32_t ones = kStages * stage;  // 128 x 64 atom, column 0 = 1
    static constexpr uint32_t ob = ones + kTile;       // o^ [t][e]; between phases the fp32 exchange
    static constexpr uint32_t ca = ob + kTile;         // c atom: column 0 = c_t
    static constexpr uint32_t sbuf = 2 * kD * kD * 2;  // bf16 [S | z] (or [dS | dz]): S atom + z atom
    static constexpr uint32_t sb = ca + kTile;         // two of them
    static constexpr uint32_t xz = sb + 2 * sbuf;      // [2][64] fp32 exchange of z / dz
    static constexpr uint32_t dx = xz + 512;           // [2][128] fp32 partial dot products
    static constexpr uint32_t bars = dx + 1024;
    static constexpr uint32_t tslot = bars + 8 * 32;
    // per-token decay: per stage the chunk's log2 decay prefix B_t of every row
    // and (B_63, B_127) at [128], [129]; the feature-map group's scan totals;
    // misc: [0,2) the partial sums' log2 decay totals, [2] the segment's log2
    // decay total, [3] its d log(gamma) total, [4,8) quad totals of the
    // d log(gamma) suffix scan (all read over DSMEM where exchanged)
    static constexpr uint32_t decs = 132 * 4;
    static constexpr uint32_t dec = tslot + 16;
    static constexpr uint32_t wt = dec + kStages * decs;
    static constexpr uint32_t misc = wt + 16;
    static constexpr uint32_t total = misc + 32;
};
static_assert(kD * kD * 4 <= kTile, "exchange fits the o^ tile");
static_assert(BL::ones % 1024 == 0 && BL::ob % 1024 == 0 && BL::ca % 1024 == 0 && BL::sb % 1024 == 0,
              "alignment");
static_assert(BL::total + 1024 <= 232448, "shared memory");

enum {
    B_FULL = 0,                 // [kStages] TMA -> feature map
    B_TDONE = B_FULL + kStages, // [kStages] feature map -> MMA
    B_EMPTY = B_TDONE + kStages,// [kStages] consumers -> producer
    B_AFULL = B_EMPTY + kStages,// phase A sums done
    // phase B
    B_SFULL, B_SBDONE, B_PFULL, B_PSDONE, B_NZFULL, B_OCDONE, B_DAFULL, B_DADONE, B_DQFULL, B_DQDONE,
    // phase C
    B_COCDONE, B_CPFULL, B_CPDONE, B_DSFULL, B_DSBDONE, B_KVFULL, B_KVDONE,
    // decay, phase A: per-chunk sums, double-buffered
    B_UFULL, B_UDONE = B_UFULL + 2,
    B_COUNT = B_UDONE + 2
};
static_assert(B_COUNT <= 32, "barrier slots");

// TMEM (512 fp32 columns).
//   phase B: P [0,128) | dA [128,256) | [N|Z], later dQ [256,336) | S [336,416) | dS^ sum [416,496)
//   phase C: P^T [0,128) | dA^T [128,256) | dK [256,320) | dV [320,384) | dS^ [416,496)
// S and dS^ use the M = 64 layout (column 64 = z / dz).
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t cP = 0, cDA = 128, cNZ = 256, cS = 336, cDS = 416;
constexpr uint32_t cPT = 0, cDAT = 128, cDK = 256, cDV = 320;

struct BwdParams {
    CUtensorMap tm_q, tm_k, tm_v, tm_g, tm_dq, tm_dk, tm_dv;
    ScanParams p;
    int G;
    int cps;
    int* status;
};

template <bool kFp16, bool kNorm, bool kDecay, bool kRev>
__global__ void __launch_bounds__(kBwdThreads, 1) bwd_kernel(const __grid_constant__ BwdParams P) {
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

    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + BL::bars);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + BL::tslot);
    // exchange buffers between phases: [64][64] fp32 partial sums in the o^ tile
    // (and a second one in sb[0]), their normaliser parts [2][64] in xz
    float* Xs = reinterpret_cast<float*>(sm + BL::ob);
    float* Xs2 = reinterpret_cast<float*>(sm + BL::sb);
    float* Xz = reinterpret_cast<float*>(sm + BL::xz);
    float* dxs = reinterpret_cast<float*>(sm + BL::dx);
    const uint32_t sbase = tc::smem_u32(sm);
    float2* wsz = reinterpret_cast<float2*>(p.ws) + (int64_t)bh * p.N;
    // decay: s q~ . dQ~ per token (the query part of d log(gamma)), after the (Zc, c) pairs
    float* wgq = p.ws + 2 * (int64_t)p.B * p.H * p.N + (int64_t)bh * p.N;
    float* dec = reinterpret_cast<float*>(sm + BL::dec);
    float* misc = reinterpret_cast<float*>(sm + BL::misc);
    const bool want_dlg = kDecay && p.dlg != nullptr;

    if (tid == 0) {
        for (int i = 0; i < B_COUNT; ++i) tc::mbar_init(&bars[i], 1);
        tc::fence_mbar_init();
    }
    if (warp == kWarpMma) tc::tmem_alloc(tslot, kTmemCols);
    if (warp >= 8 && warp < 12) {
        // constant ones atom; zero the columns 1-15 that the 16-wide normaliser
        // K-steps / N-atoms read in the c atom and both z atoms
        const int r = tid - 256;
        float one[8] = {1.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        store_chunk<kFp16>(sm + BL::ones, r, 0, one);
        zero_chunks(sm + BL::ones, r, 1, 1);
        zero_chunks(sm + BL::ca, r, 0, 2);
        if (r < kD) {
            zero_chunks(sm + BL::sb + kD * kD * 2, r, 0, 2);
            zero_chunks(sm + BL::sb + BL::sbuf + kD * kD * 2, r, 0, 2);
        }
        tc::fence_proxy_async();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tslot;
    // The segments split the live chunks (up to the sequence's last live token);
    // the gradients of the chunks after them are zero-filled at the end.
    const int nL = live_chunks(p, b, nC, reinterpret_cast<int*>(tslot + 1));
    const int cps = (nL + P.G - 1) / P.G;
    const int c_begin = min(nL, g * cps);
    const int n = min(nL, c_begin + cps) - c_begin;
    const PrefixShare share = prefix_share(g, P.G, nL, cps);
    // The forward of the same call may hand over the segment-start states
    // (written with the same segment count): phase A and the prefix exchange
    // are then skipped.
    // (the header stamps this call's shape and flags: a buffer from another call is ignored)
    const int* hdr = reinterpret_cast<const int*>(p.seg_in);
    const bool use_seg = hdr != nullptr && hdr[0] == P.G && hdr[1] == kHandMagic && hdr[2] == p.B * p.H &&
                         hdr[3] == p.N && (hdr[4] & ~kHandChunks) == hand_flags(kRev, kNorm, kDecay ? 1 : 0, false);
    const int nA = use_seg ? 0 : share.b - share.a;  // phase-A chunks: this CTA's share of the segment sums
    // pipeline slots: [0, nA) phase A, [nA, nA + n) phase B, [nA + n, nA + 2n) phase C
    const int nslots = nA + 2 * n;

    // instruction descriptors
    constexpr uint32_t idPP = tc::idesc_f16<kFp16>(128, 128, false, false);  // K-major x K-major, N = 128
    constexpr uint32_t idNZ = tc::idesc_f16<kFp16>(128, kNorm ? kNX : 64, false, true);
    constexpr uint32_t idKK64 = tc::idesc_f16<kFp16>(128, 64, false, false);
    constexpr uint32_t idKM64 = tc::idesc_f16<kFp16>(128, 64, false, true);
    constexpr uint32_t idST = tc::idesc_f16<kFp16>(64, kNorm ? kNX : 64, true, true);  // X^T [Y | 1]

    // Chunks are numbered in processing order; reverse time processes the live
    // chunks from the last one down (act maps to the chunk's place in memory),
    // and each chunk's rows from 127 down (masks, decay scan and the d log(gamma)
    // scan follow). Every global index below is the token's place in memory.
    auto act = [&](int c) { return kRev ? nL - 1 - c : c; };
    auto row_mask_at = [&](int chunk, int r) -> float {
        const int t = act(chunk) * kC + r;
        if (t >= p.N) return 0.f;
        return p.mask ? (p.mask[(int64_t)b * p.mask_sb + t] ? 1.f : 0.f) : 1.f;
    };
    // chunk of pipeline slot j (phase A visits its share rotated per sequence)
    const int rot = (!kDecay && nA > 0) ? (bh * 7) % nA : 0;  // decayed sums run in order
    auto chunk_of = [&](int j) {
        if (j < nA) {
            const int r = j + rot;
            return share.a + (r >= nA ? r - nA : r);
        }
        if (j < nA + n) return c_begin + (j - nA);
        return c_begin + n - 1 - (j - nA - n);
    };
    auto slot_addr = [&](int j, uint32_t w) { return sbase + (j % kStages) * BL::stage + w; };
    auto slot_ptr = [&](int j, uint32_t w) { return sm + (j % kStages) * BL::stage + w; };
    // acc (+)= X^T [Y | extra] over 128 tokens, X and Y [128][64] tiles read MN-major (M = 64)
    auto mma_xt = [&](uint32_t dst, uint32_t xa, uint32_t ya, uint32_t extra, bool first) {
        const uint32_t lbo = kNorm ? extra - ya : kTile;
        for (int kk = 0; kk < 8; ++kk)
            tc::mma_f16(dst, (tc::sdesc_sw128(xa, kTile, 1024) + kk * 128), (tc::sdesc_sw128(ya, lbo, 1024) + kk * 128),
                        idST, (first && kk == 0) ? 0u : 1u);
    };

    bool ok = true;

    // ---------------------------------------------------------------- roles
    auto produce = [&](int jlo, int jhi) {
        for (int j = jlo; j < jhi && ok; ++j) {
            const int s = j % kStages, u = j / kStages;
            if (u >= 1) ok = wait_bar(&bars[B_EMPTY + s], (u - 1) & 1, P.status);
            if (!ok) break;
            const bool full = j >= nA;
            const int chunk = chunk_of(j);
            uint8_t* base = sm + s * BL::stage;
            tc::mbar_arrive_expect_tx(&bars[B_FULL + s], (full ? 4u : 2u) * kTile);
            if (full) {
                tc::tma_load_4d(base + BL::q, &P.tm_q, 0, act(chunk) * kC, h, b, &bars[B_FULL + s]);
                tc::tma_load_4d(base + BL::g, &P.tm_g, 0, act(chunk) * kC, h, b, &bars[B_FULL + s]);
            }
            tc::tma_load_4d(base + BL::k, &P.tm_k, 0, act(chunk) * kC, hk, b, &bars[B_FULL + s]);
            tc::tma_load_4d(base + BL::v, &P.tm_v, 0, act(chunk) * kC, hk, b, &bars[B_FULL + s]);
        }
    };
    auto transform = [&](int jlo, int jhi) {
        const int r = tid - 256;
        // (mask byte and log(gamma) loaded a chunk ahead, raw: they are tested and
        // scaled after the wait, so the loads overlap it)
        int mr_next = jlo < jhi ? mask_raw_at(p, b, act(chunk_of(jlo)) * kC + r) : 0;
        float lg_next = (kDecay && jlo < jhi) ? decay_log_raw(p, b, h, act(chunk_of(jlo)) * kC + r) : 0.f;
        for (int j = jlo; j < jhi && ok; ++j) {
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
            uint8_t* base = sm + s * BL::stage;
            if constexpr (kDecay) {
                float b63, b127;
                float* wt = reinterpret_cast<float*>(sm + BL::wt);
                const float br = kRev ? decay_scan128_rev(a, r, wt, kBarTransform, b63, b127)
                                      : decay_scan128(a, r, wt, kBarTransform, b63, b127);
                float* dc = dec + s * (BL::decs / 4);
                dc[r] = br;
                if (r == 0) {
                    dc[128] = b63;
                    dc[129] = b127;
                    if (!decay_in_range(b63, b127)) p.fallback[bh] = 1;
                }
                if (j >= nA) chunks_phi_scaled<kFp16>(base + BL::q, r, true, exp2_fast(br - b63));
                chunks_phi_scaled<kFp16>(base + BL::k, r, m != 0.f, exp2_fast(b63 - br));
            } else {
                if (j >= nA) chunks_phi<kFp16>(base + BL::q, r, 0, 8, true);
                chunks_phi<kFp16>(base + BL::k, r, 0, 8, m != 0.f);
            }
            tc::fence_proxy_async();
            tc::bar_sync(kBarTransform, kTransformThreads);
            if (r == 0) tc::mbar_arrive(&bars[B_TDONE + s]);
        }
    };

    // compute-warp geometry
    const int quad = warp & 3, hf = (warp >> 2) & 1;
    const int row = quad * 32 + lane, srow = quad * 16 + lane;
    const uint32_t loff = (uint32_t)(quad * 32) << 16;
    using E = Elem<kFp16>;

    // 128 x 128 fp32 tile in TMEM -> causal-masked bf16 packed into its first 64
    // columns (this thread's half of its row), after every thread's fp32 reads.
    // keep_upper: keep col >= row (key-major tiles), else col <= row (query-major).
    auto mask_to_bf16 = [&](uint32_t tcol, bool keep_upper) {
        keep_upper = keep_upper != kRev;  // reverse time: the other triangle
        uint32_t packed[32];
        const bool zero = keep_upper ? (hf == 0 && quad >= 2) : (hf == 1 && quad < 2);
        if (zero) {
#pragma unroll
            for (int x = 0; x < 32; ++x) packed[x] = 0u;
        } else if (kDecay) {  // 32 columns at a time: the decayed state occupies 33 registers
            const bool diag = (hf == (quad >> 1));
#pragma unroll
            for (int part = 0; part < 2; ++part) {
                uint32_t r[32];
                tc::tmem_ld32_issue(tmem + tcol + loff + hf * 64 + part * 32, r);
                tc::tmem_wait_ld();
                tc::tmem_regs_ready<32>(r);
#pragma unroll
                for (int x = 0; x < 16; ++x) {
                    float a = __uint_as_float(r[2 * x]), bb = __uint_as_float(r[2 * x + 1]);
                    if (diag) {
                        const int col = hf * 64 + part * 32 + 2 * x;
                        if (keep_upper ? (col < row) : (col > row)) a = 0.f;
                        if (keep_upper ? (col + 1 < row) : (col + 1 > row)) bb = 0.f;
                    }
                    typename E::T2 h2 = E::from2(a, bb);
                    packed[part * 16 + x] = *reinterpret_cast<uint32_t*>(&h2);
                }
            }
        } else {
            const bool diag = (hf == (quad >> 1));
            uint32_t r[64];
            tc::tmem_ld32_issue(tmem + tcol + loff + hf * 64, r);
            tc::tmem_ld32_issue(tmem + tcol + loff + hf * 64 + 32, r + 32);
            tc::tmem_wait_ld();
            tc::tmem_regs_ready<64>(r);
#pragma unroll
            for (int x = 0; x < 32; ++x) {
                float a = __uint_as_float(r[2 * x]), bb = __uint_as_float(r[2 * x + 1]);
                if (diag) {
                    const int col = hf * 64 + 2 * x;
                    if (keep_upper ? (col < row) : (col > row)) a = 0.f;
                    if (keep_upper ? (col + 1 < row) : (col + 1 > row)) bb = 0.f;
                }
                typename E::T2 h2 = E::from2(a, bb);
                packed[x] = *reinterpret_cast<uint32_t*>(&h2);
            }
        }
        tc::tc_fence_before();
        tc::bar_sync(kBarCompute, kComputeThreads);
        tc::tc_fence_after();
        tc::tmem_st32_raw(tmem + tcol + loff + hf * 32, packed);
    };
    // M = 64 accumulator [X | x] (TMEM, 80 columns) -> bf16 S atom + z atom of `dst`
    auto refresh = [&](uint32_t tcol, uint8_t* dst) {
        float v[32];
        tc::tmem_ld32(tmem + tcol + loff + hf * 32, v);
        if (lane < 16) {
#pragma unroll
            for (int x = 0; x < 4; ++x) store_chunk<kFp16>(dst, srow, hf * 4 + x, v + 8 * x);
        }
        if (kNorm && hf == 0) {
            const float zv = tmem_ld1(tmem + tcol + loff + 64);
            if (lane < 16) {
                float z8[8] = {zv, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                store_chunk<kFp16>(dst + kD * kD * 2, srow, 0, z8);
            }
        }
    };
    // end of a compute step: shared-memory writes visible to the tensor core,
    // TMEM accesses ordered, then one arrive on `bar`
    auto publish = [&](uint64_t* bar) {
        tc::fence_proxy_async();
        tc::tc_fence_before();
        tc::bar_sync(kBarCompute, kComputeThreads);
        if (tid == 0) tc::mbar_arrive(bar);
    };
    auto cwait = [&](uint64_t* bar, uint32_t parity) -> bool {
        ok = tc::bar_and(kBarCompute, kComputeThreads, wait_bar(bar, parity, P.status)) && ok;
        if (ok) tc::tc_fence_after();
        return ok;
    };
    // exchange helpers (compute warps): own M = 64 accumulator -> X / Xz[piece]
    auto publish_sums = [&](uint32_t tcol, bool have, float* X, int piece) {
        float v[32];
        if (have) {
            tc::tmem_ld32(tmem + tcol + loff + hf * 32, v);
        } else {
#pragma unroll
            for (int x = 0; x < 32; ++x) v[x] = 0.f;
        }
        if (lane < 16) {
#pragma unroll
            for (int x = 0; x < 32; ++x) X[xch(srow, hf, x)] = v[x];
        }
        if (hf == 0) {
            const float zv = (kNorm && have) ? tmem_ld1(tmem + tcol + loff + 64) : 0.f;
            if (lane < 16) Xz[piece * 64 + srow] = zv;
        }
    };
    // Exchange gathers (compute warps): every lane ends with the sum for row
    // quad * 16 + (lane & 15); lanes 16-31 are then cleared (the M = 64 rows
    // live in lanes 0-15, and with decay lanes 16-31 start the adjoint sum at 0).
    auto clear_upper = [&](float* v, float& z) {
        if (lane >= 16) {
#pragma unroll
            for (int x = 0; x < 32; ++x) v[x] = 0.f;
            z = 0.f;
        }
    };
    // S_in plus the partial segment sums of the segments before this CTA's
    // (decayed: S_in decays over all the pieces and each piece over the ones
    // after it, the Horner chain written as one weighted sum)
    auto gather_prefix = [&](float* v, float& z) {
        const int row = quad * 16 + (lane & 15);
#pragma unroll
        for (int x = 0; x < 32; ++x) v[x] = 0.f;
        z = 0.f;
        int pr[16], pb[16], np = 0;
        for (int r = 0; r < P.G; ++r) {
            const PrefixShare sr = prefix_share(r, P.G, nL, cps);
            if (min(sr.b, sr.x) > sr.a && sr.seg < g) pr[np] = r, pb[np++] = 0;
            if (sr.b > sr.x && sr.seg + 1 < g) pr[np] = r, pb[np++] = 1;
        }
        float wl = 1.f, w_in = 1.f;
        if (kDecay) {
            const float lam = lane < np ? cluster.map_shared_rank(misc, pr[lane])[pb[lane]] : 0.f;
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
            [&](int r, int pc) { return cluster.map_shared_rank(pc == 0 ? Xs : Xs2, r); },
            [&](int r, int pc) { return cluster.map_shared_rank(Xz, r) + pc * 64; }, kNorm && hf == 0, v, z);
        clear_upper(v, z);
    };
    // the adjoint at this segment's end: the later segments' sums X_r (each at
    // its segment's start); decayed, X_r takes the decay of the segments
    // between (G = X_g+1 + exp(Lambda_g+1) (X_g+2 + ...), as one weighted sum)
    auto gather_suffix = [&](float* v, float& z) {
        const int row = quad * 16 + (lane & 15);
#pragma unroll
        for (int x = 0; x < 32; ++x) v[x] = 0.f;
        z = 0.f;
        int pr[8], pb[8], np = 0;
        for (int r = g + 1; r < P.G; ++r) pr[np] = r, pb[np++] = 0;
        float wl = 1.f;
        if (kDecay) {
            const float lam = lane < np ? cluster.map_shared_rank(misc, pr[lane])[2] : 0.f;
            float total;
            wl = exp2_fast(piece_exponent(lam, lane, false, total));
        }
        gather_pieces(
            np, pr, pb, wl, row, hf, lane, [&](int r, int) { return cluster.map_shared_rank(Xs, r); },
            [&](int r, int) { return cluster.map_shared_rank(Xz, r); }, kNorm && hf == 0, v, z);
        clear_upper(v, z);
    };
    // registers -> TMEM accumulator (M = 64 layout) and bf16 copy in `dst`
    auto install_state = [&](uint32_t tcol, uint8_t* dst, const float* v, float z) {
        if (lane < 16) {
#pragma unroll
            for (int x = 0; x < 4; ++x) store_chunk<kFp16>(dst, srow, hf * 4 + x, v + 8 * x);
        }
        tc::tmem_st32(tmem + tcol + loff + hf * 32, v);
        if (hf == 0) {
            if (lane < 16) {
                float z8[8] = {z, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                store_chunk<kFp16>(dst + kD * kD * 2, srow, 0, z8);
                zero_chunks(dst + kD * kD * 2, srow, 1, 1);
            }
            float w[32];
#pragma unroll
            for (int x = 0; x < 32; ++x) w[x] = 0.f;
            w[0] = (lane < 16) ? z : 0.f;
            tc::tmem_st32(tmem + tcol + loff + 64, w);
        }
    };

    // decay: bf16 f [X | x] from registers (rows in lanes 0-15) into the operand
    // buffer `dst` (the z atom's columns 8-15 zeroed alongside)
    auto write_operand = [&](uint8_t* dst, float f, const float* v, float z) {
        if (lane < 16) {
            float w[8];
#pragma unroll
            for (int x = 0; x < 4; ++x) {
#pragma unroll
                for (int y = 0; y < 8; ++y) w[y] = f * v[8 * x + y];
                store_chunk<kFp16>(dst, srow, hf * 4 + x, w);
            }
            if (kNorm && hf == 0) {
                float z8[8] = {f * z, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                store_chunk<kFp16>(dst + kD * kD * 2, srow, 0, z8);
                zero_chunks(dst + kD * kD * 2, srow, 1, 1);
            }
        }
    };
    // ============================================================ phase A
    if (warp == kWarpProducer) {
        if (lane == 0) {
            for (int m = 0; m < 7; ++m)
                tc::prefetch_tmap(m == 0 ? &P.tm_q : m == 1 ? &P.tm_k : m == 2 ? &P.tm_v : m == 3 ? &P.tm_g
                                  : m == 4 ? &P.tm_dq : m == 5 ? &P.tm_dk : &P.tm_dv);
            produce(0, min(nslots, nA + kStages));
        }
        __syncwarp();
    } else if (warp >= 8 && warp < 12) {
        transform(0, nA);
    } else if (warp == kWarpMma) {
        if (kDecay && lane == 0) {
            // decayed sums: each chunk's k'^T [V | 1] into one of two buffers (the
            // NZ and S columns); the compute warps chain them and release the stage
            for (int j = 0; j < nA && ok; ++j) {
                const int s = j % kStages, u = j / kStages;
                ok = wait_bar(&bars[B_TDONE + s], u & 1, P.status);
                if (ok && j >= 2) ok = wait_bar(&bars[B_UDONE + (j & 1)], ((j >> 1) - 1) & 1, P.status);
                if (!ok) break;
                tc::tc_fence_after();
                mma_xt(tmem + ((j & 1) ? cS : cNZ), slot_addr(j, BL::k), slot_addr(j, BL::v), sbase + BL::ones, true);
                tc::mma_commit(&bars[B_UFULL + (j & 1)]);
            }
        } else if (lane == 0) {
            // the share's two partial sums accumulate in S (before the segment
            // boundary) and in the still unused P columns (after it)
            bool first1 = true, first2 = true;
            for (int j = 0; j < nA && ok; ++j) {
                const int s = j % kStages, u = j / kStages;
                ok = wait_bar(&bars[B_TDONE + s], u & 1, P.status);
                if (!ok) break;
                tc::tc_fence_after();
                const bool second = chunk_of(j) >= share.x;
                mma_xt(tmem + (second ? cP : cS), slot_addr(j, BL::k), slot_addr(j, BL::v), sbase + BL::ones,
                       second ? first2 : first1);
                (second ? first2 : first1) = false;
                tc::mma_commit(&bars[B_EMPTY + s]);
            }
            if (nA > 0 && ok) tc::mma_commit(&bars[B_AFULL]);
        }
        __syncwarp();
    } else if (kDecay && warp < 8) {
        // Horner over the share in chunk order, per piece: X = exp(b_end) X + exp(b_end - b_m) U'
        float X[32], xz = 0.f, lam0 = 0.f, lam1 = 0.f;
#pragma unroll
        for (int x = 0; x < 32; ++x) X[x] = 0.f;
        int piece = 0;
        auto flush = [&](int pc) {
            float* dst = pc == 0 ? Xs : Xs2;
            if (lane < 16) {
#pragma unroll
                for (int x = 0; x < 32; ++x) dst[xch(srow, hf, x)] = X[x];
                if (hf == 0) Xz[pc * 64 + srow] = xz;
            }
        };
        for (int j = 0; j < nA && ok; ++j) {
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
            const float* dc = dec + s * (BL::decs / 4);
            const float b63 = dc[128], b127 = dc[129];
            const float ld = exp2_fast(b127), mu = exp2_fast(b127 - b63);
            const uint32_t ucol = (j & 1) ? cS : cNZ;
            float uu[32];
            tc::tmem_ld32(tmem + ucol + loff + hf * 32, uu);
#pragma unroll
            for (int x = 0; x < 32; ++x) X[x] = fmaf(ld, X[x], mu * uu[x]);
            if (kNorm && hf == 0) xz = fmaf(ld, xz, mu * tmem_ld1(tmem + ucol + loff + 64));
            if (piece) lam1 += b127;
            else lam0 += b127;
            tc::tc_fence_before();
            tc::bar_sync(kBarCompute, kComputeThreads);
            if (tid == 0) {
                tc::mbar_arrive(&bars[B_UDONE + (j & 1)]);
                tc::mbar_arrive(&bars[B_EMPTY + s]);
            }
        }
        if (nA > 0) flush(piece);
        if (tid == 0) {
            misc[0] = lam0;
            misc[1] = lam1;
        }
    } else if (warp < 8) {
        if (nA > 0) cwait(&bars[B_AFULL], 0);
        publish_sums(cS, ok && min(share.b, share.x) > share.a, Xs, 0);
        publish_sums(cP, ok && share.b > share.x, Xs2, 1);
    }
    tc::tc_fence_before();
    cluster.sync();
    tc::tc_fence_after();
    float carry[32], carry_z = 0.f;  // prefix (phase B) / suffix (phase C) state rows, compute warps
    float lf = 0.f;                  // decay: log2 decay total of the segment's chunks (phase B)
    if (warp < 8) {
        if (use_seg) {  // this segment's start state from the forward (rows in lanes 0-15)
#pragma unroll
            for (int x = 0; x < 32; ++x) carry[x] = 0.f;
            carry_z = 0.f;
            if (lane < 16) {
                const float* src = p.seg_in + 64 + ((int64_t)(bh * P.G + g) * kD + srow) * (kD + 1);
#pragma unroll
                for (int x = 0; x < 32; ++x) carry[x] = src[hf * 32 + x];
                if (kNorm && hf == 0) carry_z = src[kD];
            }
        } else {
            gather_prefix(carry, carry_z);
        }
    }
    tc::tc_fence_before();
    cluster.sync();  // remote reads done before the exchange tile is reused
    tc::tc_fence_after();
    if (warp < 8 && !kDecay) {  // (with decay the state stays in registers, lanes 0-15)
        install_state(cS, sm + BL::sb, carry, carry_z);
        tc::fence_proxy_async();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();

    // ============================================================ phase B
    if (warp == kWarpProducer) {
        if (lane == 0) produce(min(nslots, nA + kStages), min(nslots, nA + n + kStages));
        __syncwarp();
    } else if (warp >= 8 && warp < 12) {
        transform(nA, nA + n);
    } else if (warp == kWarpMma) {
        if (lane == 0) {
            auto issue_p = [&](int i, bool ready = false) -> bool {  // P = q^ k^^T
                const int j = nA + i;
                if (!ready && !wait_bar(&bars[B_TDONE + j % kStages], (j / kStages) & 1, P.status)) return false;
                tc::tc_fence_after();
                const uint32_t qa = slot_addr(j, BL::q), ka = slot_addr(j, BL::k);
                for (int kk = 0; kk < 4; ++kk)
                    tc::mma_f16(tmem + cP, (tc::sdesc_sw128(qa, 16, 1024) + kk * 2),
                                (tc::sdesc_sw128(ka, 16, 1024) + kk * 2), idPP, kk > 0);
                tc::mma_commit(&bars[B_PFULL]);
                return true;
            };
            if (n > 0) ok = issue_p(0);
            for (int i = 0; i < n && ok; ++i) {
                const int j = nA + i;
                const uint32_t qa = slot_addr(j, BL::q), ka = slot_addr(j, BL::k), va = slot_addr(j, BL::v);
                const uint32_t sba = sbase + BL::sb + (i & 1) * BL::sbuf;
                const uint32_t lbo_v1 = kNorm ? (sbase + BL::ones) - va : kTile;
                // [S|z]_c+1 = [S|z]_c + k^^T [V | 1]
                if (i >= 1) ok = wait_bar(&bars[B_SBDONE], (i - 1) & 1, P.status);
                if (!ok) break;
                tc::tc_fence_after();
                mma_xt(tmem + cS, ka, va, sbase + BL::ones, kDecay);  // decay: this chunk's sum alone
                tc::mma_commit(&bars[B_SFULL]);
                // [N | Z] = q^ [S_c | z_c] + bf16(P) [V | 1]   (into the NZ / dQ columns)
                ok = wait_bar(&bars[B_PSDONE], i & 1, P.status);
                if (ok && i >= 1) ok = wait_bar(&bars[B_DQDONE], (i - 1) & 1, P.status);
                if (!ok) break;
                tc::tc_fence_after();
                for (int kk = 0; kk < 4; ++kk)
                    tc::mma_f16(tmem + cNZ, (tc::sdesc_sw128(qa, 16, 1024) + kk * 2),
                                (tc::sdesc_sw128(sba, kD * kD * 2, 1024) + kk * 128), idNZ, kk > 0);
                for (int kk = 0; kk < 8; ++kk)
                    tc::mma_f16_ts(tmem + cNZ, tmem + cP + kk * 8, (tc::sdesc_sw128(va, lbo_v1, 1024) + kk * 128),
                                   idNZ, 1u);
                tc::mma_commit(&bars[B_NZFULL]);
                // P of the next chunk now when its feature map is already done (the
                // NZ MMAs above have taken their bf16 P), else after dQ~
                const int jn = j + 1;
                const bool p_early = i + 1 < n && tc::mbar_test_wait(&bars[B_TDONE + jn % kStages], (jn / kStages) & 1);
                if (p_early) issue_p(i + 1, true);
                // dA = [o^ | c] [V | 1]^T ; dS^ sum += q^^T [o^ | c]
                ok = wait_bar(&bars[B_OCDONE], i & 1, P.status);
                if (!ok) break;
                tc::tc_fence_after();
                for (int kk = 0; kk < 4; ++kk)
                    tc::mma_f16(tmem + cDA, (tc::sdesc_sw128(sbase + BL::ob, 16, 1024) + kk * 2),
                                (tc::sdesc_sw128(va, 16, 1024) + kk * 2), idPP, kk > 0);
                if (kNorm)
                    tc::mma_f16(tmem + cDA, tc::sdesc_sw128(sbase + BL::ca, 16, 1024),
                                tc::sdesc_sw128(sbase + BL::ones, 16, 1024), idPP, 1u);
                tc::mma_commit(&bars[B_DAFULL]);
                mma_xt(tmem + cDS, qa, sbase + BL::ob, sbase + BL::ca, kDecay || i == 0);
                // dQ~ = [o^ | c] [S_c | z_c]^T (issued while the compute warps mask dA)
                //     + bf16(dA) K^                (into the NZ / dQ columns)
                for (int kk = 0; kk < 4; ++kk)
                    tc::mma_f16(tmem + cNZ, (tc::sdesc_sw128(sbase + BL::ob, 16, 1024) + kk * 2),
                                (tc::sdesc_sw128(sba, 16, 1024) + kk * 2), idKK64, kk > 0);
                if (kNorm)
                    tc::mma_f16(tmem + cNZ, tc::sdesc_sw128(sbase + BL::ca, 16, 1024),
                                tc::sdesc_sw128(sba + kD * kD * 2, 16, 1024), idKK64, 1u);
                ok = wait_bar(&bars[B_DADONE], i & 1, P.status);
                if (!ok) break;
                tc::tc_fence_after();
                for (int kk = 0; kk < 8; ++kk)
                    tc::mma_f16_ts(tmem + cNZ, tmem + cDA + kk * 8, (tc::sdesc_sw128(ka, kTile, 1024) + kk * 128),
                                   idKM64, 1u);
                tc::mma_commit(&bars[B_DQFULL]);
                // P of the next chunk, if not issued above
                if (i + 1 < n && !p_early) ok = issue_p(i + 1);
            }
        }
        __syncwarp();
    } else if (warp < 8) {
        // decay: lanes 0-15 carry the prefix state [S | z] (rows srow), lanes 16-31
        // the segment's adjoint sum X = sum_c exp(B_c - B_seg) exp(b_m) q'^T [o^ | c]
        // (rows srow - 16); lf = log2 decay of the segment's chunks so far
        if (kDecay && n > 0) {  // the first chunk's operand exp(b_m) [S | z]_in
            const int s0 = nA % kStages;
            if (cwait(&bars[B_TDONE + s0], (nA / kStages) & 1))
                write_operand(sm + BL::sb, exp2_fast(dec[s0 * (BL::decs / 4) + 128]), carry, carry_z);
        }
        if (n > 0) {
            cwait(&bars[B_PFULL], 0);
            if (ok) {
                mask_to_bf16(cP, false);
                publish(&bars[B_PSDONE]);
            }
        }
        float m_cur = n > 0 ? row_mask_at(c_begin, row) : 0.f;
        for (int i = 0; i < n && ok; ++i) {
            const int j = nA + i, c = c_begin + i;
            const float m = m_cur;
            if (i + 1 < n) m_cur = row_mask_at(c + 1, row);  // in flight during this chunk
            // (1) state refresh: bf16 [S | z]_c+1 into sb[(i + 1) % 2]; the previous
            // chunk's dq store has left its dO tile, so that slot is released
            if (!cwait(&bars[B_SFULL], i & 1)) break;
            if constexpr (kDecay) {
                // [S|z]_c+1 = exp(b_end) [S|z]_c + exp(b_end - b_m) U'_c (the chunk's decay
                // values are final once its feature map is; its stage stays until
                // released by this warp group). The operand of chunk c+1, which carries
                // that chunk's exp(b_m), is written when its P is masked (step 5): with
                // two stages, chunk c+1 may not be loaded before this chunk's
                // predecessor leaves its stage.
                const int s = j % kStages;
                if (!cwait(&bars[B_TDONE + s], (j / kStages) & 1)) break;
                const float* dc = dec + s * (BL::decs / 4);
                const float ld = exp2_fast(dc[129]), mu = exp2_fast(dc[129] - dc[128]);
                float uu[32];
                tc::tmem_ld32(tmem + cS + loff + hf * 32, uu);
                const float uz = (kNorm && hf == 0) ? tmem_ld1(tmem + cS + loff + 64) : 0.f;
                if (lane < 16) {
#pragma unroll
                    for (int x = 0; x < 32; ++x) carry[x] = fmaf(ld, carry[x], mu * uu[x]);
                    carry_z = fmaf(ld, carry_z, mu * uz);
                }
            } else {
                refresh(cS, sm + BL::sb + ((i + 1) & 1) * BL::sbuf);
            }
            if (tid == 0 && i >= 1) {
                tc::bulk_wait_read0();
                tc::mbar_arrive(&bars[B_EMPTY + (j - 1) % kStages]);
            }
            publish(&bars[B_SBDONE]);
            // (2) o^ and c from [num | Z] and dO (the slot's q^ and dO are complete
            // once its feature map is: TDONE implies FULL)
            if (!cwait(&bars[B_NZFULL], i & 1)) break;
            if (!cwait(&bars[B_TDONE + j % kStages], (j / kStages) & 1)) break;
            float num[32], go[32];
            tc::tmem_ld32(tmem + cNZ + loff + hf * 32, num);
            const float zraw = kNorm ? tmem_ld1(tmem + cNZ + loff + 64) : 0.f;
            load_chunks<kFp16>(slot_ptr(j, BL::g), row, hf * 4, 4, go);
            float dot = 0.f;
#pragma unroll
            for (int x = 0; x < 32; ++x) dot = fmaf(go[x], num[x], dot);
            dxs[hf * 128 + row] = dot;
            tc::bar_sync(kBarCompute, kComputeThreads);
            const float zc = kNorm ? max_nan(p.scale * zraw, p.clamp_min) : 1.f;
            const float inv = m / zc;
            const float ct = kNorm ? -m * p.scale * (dxs[row] + dxs[128 + row]) * inv / zc : 0.f;
#pragma unroll
            for (int x = 0; x < 32; ++x) go[x] *= inv;
#pragma unroll
            for (int x = 0; x < 4; ++x) store_chunk<kFp16>(sm + BL::ob, row, hf * 4 + x, go + 8 * x);
            if (hf == 0) {
                if (kNorm) {
                    float c8[8] = {ct, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                    store_chunk<kFp16>(sm + BL::ca, row, 0, c8);
                }
                if (act(c) * kC + row < p.N) wsz[act(c) * kC + row] = make_float2(zc, ct);
            }
            publish(&bars[B_OCDONE]);  // also: every thread has read dxs, [N | Z] and dO
            // (3) dA: causal mask, bf16 in place
            if (!cwait(&bars[B_DAFULL], i & 1)) break;
            mask_to_bf16(cDA, false);
            publish(&bars[B_DADONE]);
            // (4) dq = s dQ~ phi'(q), written over the slot's (dead) dO tile
            if (!cwait(&bars[B_DQFULL], i & 1)) break;
            {
                float dq[32], qv[32];
                tc::tmem_ld32(tmem + cNZ + loff + hf * 32, dq);
                load_chunks<kFp16>(slot_ptr(j, BL::q), row, hf * 4, 4, qv);
                if constexpr (kDecay) {
                    // q' = phi(q) f_t and dQ~ = f_t x (the accumulator), f_t = exp(b_t - b_m);
                    // s q' . acc is the query part of d log(gamma_t)
                    const float* dc = dec + (j % kStages) * (BL::decs / 4);
                    const float ft = exp2_fast(dc[row] - dc[128]), ift = exp2_fast(dc[128] - dc[row]);
                    float gq = 0.f;
#pragma unroll
                    for (int x = 0; x < 32; ++x) {
                        gq = fmaf(qv[x], dq[x], gq);
                        dq[x] *= p.scale * ft * min_nan(qv[x] * ift, 1.f);
                    }
                    if (want_dlg) dxs[hf * 128 + row] = gq;
                } else {
#pragma unroll
                    for (int x = 0; x < 32; ++x) dq[x] *= p.scale * min_nan(qv[x], 1.f);
                }
                uint8_t* dst = slot_ptr(j, BL::g);
#pragma unroll
                for (int x = 0; x < 4; ++x) store_chunk<kFp16>(dst, row, hf * 4 + x, dq + 8 * x);
                tc::fence_proxy_async();
                tc::tc_fence_before();
                tc::bar_sync(kBarCompute, kComputeThreads);
                if (tid == 0) {
                    tc::mbar_arrive(&bars[B_DQDONE]);  // dQ~ columns read
                    tc::tma_store_4d(&P.tm_dq, dst, 0, act(c) * kC, h, b);
                    tc::bulk_commit();
                }
                if (want_dlg && hf == 0 && act(c) * kC + row < p.N)
                    wgq[act(c) * kC + row] = p.scale * (dxs[row] + dxs[128 + row]);
            }
            if constexpr (kDecay) {
                // X += exp(B_c - B_seg) exp(b_m) W'_c, W'_c = q'^T [o^ | c] of this chunk
                // (TMEM, rows in lanes 0-15, handed to lanes 16-31)
                const float* dc = dec + (j % kStages) * (BL::decs / 4);
                const float sg = exp2_fast(lf + dc[128]);
                lf += dc[129];
                float ww[32];
                tc::tmem_ld32(tmem + cDS + loff + hf * 32, ww);
                float wz = (kNorm && hf == 0) ? tmem_ld1(tmem + cDS + loff + 64) : 0.f;
#pragma unroll
                for (int x = 0; x < 32; ++x) ww[x] = __shfl_sync(0xffffffffu, ww[x], lane & 15);
                wz = __shfl_sync(0xffffffffu, wz, lane & 15);
                if (lane >= 16) {
#pragma unroll
                    for (int x = 0; x < 32; ++x) carry[x] = fmaf(sg, ww[x], carry[x]);
                    carry_z = fmaf(sg, wz, carry_z);
                }
            }
            // (5) P of the next chunk: causal mask, bf16 in place
            if (i + 1 < n) {
                if (!cwait(&bars[B_PFULL], (i + 1) & 1)) break;
                if constexpr (kDecay) {  // and its operand exp(b_m) [S | z]_c+1 (its stage is loaded: P is done)
                    const int s1 = (j + 1) % kStages;
                    if (!cwait(&bars[B_TDONE + s1], ((j + 1) / kStages) & 1)) break;
                    write_operand(sm + BL::sb + ((i + 1) & 1) * BL::sbuf,
                                  exp2_fast(dec[s1 * (BL::decs / 4) + 128]), carry, carry_z);
                }
                mask_to_bf16(cP, false);
                publish(&bars[B_PSDONE]);
            }
        }
        if (tid == 0 && n > 0) {  // release the last slot once its dq has left
            tc::bulk_wait_read0();
            tc::mbar_arrive(&bars[B_EMPTY + (nA + n - 1) % kStages]);
        }
    }

    // ------------------------------------------------ suffix exchange (dS^, dz^)
    if (warp < 8) {
        if constexpr (kDecay) {  // X from lanes 16-31, and the segment's log2 decay total
            if (lane >= 16) {
                const int xr = srow - 16;
#pragma unroll
                for (int x = 0; x < 32; ++x) Xs[xch(xr, hf, x)] = (n > 0 && ok) ? carry[x] : 0.f;
                if (hf == 0) Xz[xr] = (kNorm && n > 0 && ok) ? carry_z : 0.f;
            }
            if (tid == 0) misc[2] = lf;
        } else {
            publish_sums(cDS, n > 0 && ok, Xs, 0);
        }
    }
    tc::tc_fence_before();
    cluster.sync();
    tc::tc_fence_after();
    if (warp < 8) {
        gather_suffix(carry, carry_z);
    }
    tc::tc_fence_before();
    cluster.sync();
    tc::tc_fence_after();
    if (warp < 8 && !kDecay) {  // (with decay the adjoint stays in registers, lanes 0-15)
        install_state(cDS, sm + BL::sb, carry, carry_z);
        tc::fence_proxy_async();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();

    // ============================================================ phase C
    if (warp == kWarpProducer) {
        if (lane == 0) produce(min(nslots, nA + n + kStages), nslots);
        __syncwarp();
    } else if (warp >= 8 && warp < 12) {
        transform(nA + n, nslots);
    } else if (warp == kWarpMma) {
        if (lane == 0) {
            for (int i = 0; i < n && ok; ++i) {
                const int j = nA + n + i;
                const uint32_t qa = slot_addr(j, BL::q), ka = slot_addr(j, BL::k), va = slot_addr(j, BL::v);
                const uint32_t dsa = sbase + BL::sb + (i & 1) * BL::sbuf;  // dS^ of the later chunks
                ok = wait_bar(&bars[B_TDONE + j % kStages], (j / kStages) & 1, P.status);
                if (ok) ok = wait_bar(&bars[B_COCDONE], i & 1, P.status);
                if (!ok) break;
                tc::tc_fence_after();
                // P^T = K^ q^^T ; dA^T = [V | 1] [o^ | c]^T   (key-major rows)
                for (int kk = 0; kk < 4; ++kk) {
                    tc::mma_f16(tmem + cPT, (tc::sdesc_sw128(ka, 16, 1024) + kk * 2),
                                (tc::sdesc_sw128(qa, 16, 1024) + kk * 2), idPP, kk > 0);
                    tc::mma_f16(tmem + cDAT, (tc::sdesc_sw128(va, 16, 1024) + kk * 2),
                                (tc::sdesc_sw128(sbase + BL::ob, 16, 1024) + kk * 2), idPP, kk > 0);
                }
                if (kNorm)
                    tc::mma_f16(tmem + cDAT, tc::sdesc_sw128(sbase + BL::ones, 16, 1024),
                                tc::sdesc_sw128(sbase + BL::ca, 16, 1024), idPP, 1u);
                tc::mma_commit(&bars[B_CPFULL]);
                // dS^ += q^^T [o^ | c]   (after the previous refresh has read it)
                if (i >= 1) ok = wait_bar(&bars[B_DSBDONE], (i - 1) & 1, P.status);
                if (!ok) break;
                tc::tc_fence_after();
                mma_xt(tmem + cDS, qa, sbase + BL::ob, sbase + BL::ca, kDecay);
                tc::mma_commit(&bars[B_DSFULL]);
                // dK~ = [V | 1] [dS^ | dz^]^T + bf16(dA^T) q^ ;  dV = K^ dS^ + bf16(P^T) o^.
                // The state terms go first, while the compute warps mask P^T and dA^T.
                if (i >= 1) ok = wait_bar(&bars[B_KVDONE], (i - 1) & 1, P.status);
                if (!ok) break;
                tc::tc_fence_after();
                for (int kk = 0; kk < 4; ++kk) {
                    tc::mma_f16(tmem + cDK, (tc::sdesc_sw128(va, 16, 1024) + kk * 2),
                                (tc::sdesc_sw128(dsa, 16, 1024) + kk * 2), idKK64, kk > 0);
                    tc::mma_f16(tmem + cDV, (tc::sdesc_sw128(ka, 16, 1024) + kk * 2),
                                (tc::sdesc_sw128(dsa, kTile, 1024) + kk * 128), idKM64, kk > 0);
                }
                if (kNorm)
                    tc::mma_f16(tmem + cDK, tc::sdesc_sw128(sbase + BL::ones, 16, 1024),
                                tc::sdesc_sw128(dsa + kD * kD * 2, 16, 1024), idKK64, 1u);
                ok = wait_bar(&bars[B_CPDONE], i & 1, P.status);
                if (!ok) break;
                tc::tc_fence_after();
                for (int kk = 0; kk < 8; ++kk) {
                    tc::mma_f16_ts(tmem + cDK, tmem + cDAT + kk * 8, (tc::sdesc_sw128(qa, kTile, 1024) + kk * 128),
                                   idKM64, 1u);
                    tc::mma_f16_ts(tmem + cDV, tmem + cPT + kk * 8,
                                   (tc::sdesc_sw128(sbase + BL::ob, kTile, 1024) + kk * 128), idKM64, 1u);
                }
                tc::mma_commit(&bars[B_KVFULL]);
            }
        }
        __syncwarp();
    } else if (warp < 8) {
        // mask and (Zc, c) of a chunk's row, fetched one chunk ahead
        auto fetch = [&](int cc, float& m_, float2& z_, float& gq_) {
            const int t = act(cc) * kC + row;
            const bool in = t < p.N;
            m_ = row_mask_at(cc, row);
            z_ = in ? wsz[t] : make_float2(1.f, 0.f);
            if (want_dlg) gq_ = in ? wgq[t] : 0.f;
        };
        float m_cur = 0.f, gq_cur = 0.f;
        float2 zcc_cur = make_float2(1.f, 0.f);
        float dlg_carry = 0.f;  // d log(gamma) summed over this segment's later tokens
        if (kDecay && n > 0) {  // the first (last in time) chunk's operand exp(b_end - b_m) [dS^ | dz^]
            const int s0 = (nA + n) % kStages;
            if (cwait(&bars[B_TDONE + s0], ((nA + n) / kStages) & 1)) {
                const float* dc = dec + s0 * (BL::decs / 4);
                write_operand(sm + BL::sb, exp2_fast(dc[129] - dc[128]), carry, carry_z);
                tc::fence_proxy_async();
            }
        }
        if (n > 0) fetch(c_begin + n - 1, m_cur, zcc_cur, gq_cur);
        for (int i = 0; i < n && ok; ++i) {
            const int j = nA + n + i, c = c_begin + n - 1 - i;
            const float m = m_cur, gq = gq_cur;
            const float2 zcc = zcc_cur;
            if (i + 1 < n) fetch(c - 1, m_cur, zcc_cur, gq_cur);
            // (1) o^ = m dO / Zc and the c atom, from the workspace
            {
                const float inv = m / zcc.x;
                if (!cwait(&bars[B_TDONE + j % kStages], (j / kStages) & 1)) break;  // dO, q^, k^ ready
                if (kDecay && i >= 1) {  // this chunk's operand exp(b_end - b_m) G_c+1
                    const float* dc = dec + (j % kStages) * (BL::decs / 4);
                    write_operand(sm + BL::sb + (i & 1) * BL::sbuf, exp2_fast(dc[129] - dc[128]), carry, carry_z);
                }
                float go[32];
                load_chunks<kFp16>(slot_ptr(j, BL::g), row, hf * 4, 4, go);
#pragma unroll
                for (int x = 0; x < 32; ++x) go[x] *= inv;
                if (tid == 0 && i >= 1) {
                    // the previous chunk's dk / dv stores have left its dO tile and
                    // the o^ tile: that slot is released
                    tc::bulk_wait_read0();
                    tc::mbar_arrive(&bars[B_EMPTY + (j - 1) % kStages]);
                }
                tc::bar_sync(kBarCompute, kComputeThreads);
#pragma unroll
                for (int x = 0; x < 4; ++x) store_chunk<kFp16>(sm + BL::ob, row, hf * 4 + x, go + 8 * x);
                if (kNorm && hf == 0) {
                    float c8[8] = {zcc.y, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                    store_chunk<kFp16>(sm + BL::ca, row, 0, c8);
                }
                publish(&bars[B_COCDONE]);
            }
            // (2) P^T and dA^T: causal mask (keep t >= tau), bf16 in place
            if (!cwait(&bars[B_CPFULL], i & 1)) break;
            mask_to_bf16(cPT, true);
            mask_to_bf16(cDAT, true);
            publish(&bars[B_CPDONE]);
            // (3) suffix refresh: bf16 [dS^ | dz^] into sb[(i + 1) % 2]
            if (!cwait(&bars[B_DSFULL], i & 1)) break;
            if constexpr (kDecay) {
                // G_c = exp(b_m) W'_c + exp(b_end) G_c+1 (the adjoint of the state before
                // chunk c); the operand of chunk c-1, which carries that chunk's
                // exp(b_end - b_m), is written in its step 1
                const float* dc = dec + (j % kStages) * (BL::decs / 4);
                const float fm = exp2_fast(dc[128]), fe = exp2_fast(dc[129]);
                float ww[32];
                tc::tmem_ld32(tmem + cDS + loff + hf * 32, ww);
                const float wz = (kNorm && hf == 0) ? tmem_ld1(tmem + cDS + loff + 64) : 0.f;
                if (lane < 16) {
#pragma unroll
                    for (int x = 0; x < 32; ++x) carry[x] = fmaf(fm, ww[x], fe * carry[x]);
                    carry_z = fmaf(fm, wz, fe * carry_z);
                }
            } else {
                refresh(cDS, sm + BL::sb + ((i + 1) & 1) * BL::sbuf);
            }
            publish(&bars[B_DSBDONE]);
            // (4) dk = s dK~ phi'(k) m over the (dead) dO tile, dv = s dV m over o^
            if (!cwait(&bars[B_KVFULL], i & 1)) break;
            if constexpr (kDecay) {
                // k' = m phi(k) g and dK~ = s g x (the accumulator), g = exp(b_m - b_tau);
                // s k' . acc is the key part of d log(gamma_tau)
                const float* dc = dec + (j % kStages) * (BL::decs / 4);
                const float gt = exp2_fast(dc[128] - dc[row]), igt = exp2_fast(dc[row] - dc[128]);
                const float sm_ = p.scale * m;
                uint8_t* dst = slot_ptr(j, BL::g);
                float gk = 0.f;
                {
                    float dk[32], kv[32];
                    tc::tmem_ld32(tmem + cDK + loff + hf * 32, dk);
                    load_chunks<kFp16>(slot_ptr(j, BL::k), row, hf * 4, 4, kv);
#pragma unroll
                    for (int x = 0; x < 32; ++x) {
                        gk = fmaf(kv[x], dk[x], gk);
                        dk[x] *= sm_ * gt * min_nan(kv[x] * igt, 1.f);
                    }
#pragma unroll
                    for (int x = 0; x < 4; ++x) store_chunk<kFp16>(dst, row, hf * 4 + x, dk + 8 * x);
                }
                {
                    float dv[32];
                    tc::tmem_ld32(tmem + cDV + loff + hf * 32, dv);
#pragma unroll
                    for (int x = 0; x < 32; ++x) dv[x] *= sm_;
#pragma unroll
                    for (int x = 0; x < 4; ++x) store_chunk<kFp16>(sm + BL::ob, row, hf * 4 + x, dv + 8 * x);
                }
                if (want_dlg) dxs[hf * 128 + row] = gk;
                tc::fence_proxy_async();
                tc::tc_fence_before();
                tc::bar_sync(kBarCompute, kComputeThreads);
                if (tid == 0) {
                    tc::mbar_arrive(&bars[B_KVDONE]);  // dK / dV columns read
                    tc::tma_store_4d(&P.tm_dk, dst, 0, act(c) * kC, h, b);
                    tc::tma_store_4d(&P.tm_dv, sm + BL::ob, 0, act(c) * kC, h, b);
                    tc::bulk_commit();
                }
                if (want_dlg) {
                    // g_t = s q~.dQ~ - s k~.dK~; d log(gamma_t) = m_t sum_{t' >= t} g_t'
                    // (reverse scan: lanes within the quad's 32 rows, then the quads, then
                    // the later chunks of the segment; later segments are added at the end)
                    // (reverse time: the rows after t in processing order are the rows
                    // before it in the chunk, so the scan runs the other way)
                    float x = gq - p.scale * (dxs[row] + dxs[128 + row]);
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const float y = kRev ? __shfl_up_sync(0xffffffffu, x, o) : __shfl_down_sync(0xffffffffu, x, o);
                        if (kRev ? lane >= o : lane + o < 32) x += y;
                    }
                    const float qtot = __shfl_sync(0xffffffffu, x, kRev ? 31 : 0);
                    if (hf == 0 && lane == 0) misc[4 + quad] = qtot;
                    tc::bar_sync(kBarCompute, kComputeThreads);
                    float later = dlg_carry;
                    for (int qq = kRev ? 0 : quad + 1; qq < (kRev ? quad : 4); ++qq) later += misc[4 + qq];
                    const int t = act(c) * kC + row;
                    if (hf == 0 && t < p.N) p.dlg[(int64_t)bh * p.N + t] = m * (x + later);
                    dlg_carry += misc[4] + misc[5] + misc[6] + misc[7];
                }
            } else {
                float dk[32], dv[32], kv[32];
                tc::tmem_ld32(tmem + cDK + loff + hf * 32, dk);
                tc::tmem_ld32(tmem + cDV + loff + hf * 32, dv);
                load_chunks<kFp16>(slot_ptr(j, BL::k), row, hf * 4, 4, kv);
                const float sm_ = p.scale * m;
#pragma unroll
                for (int x = 0; x < 32; ++x) {
                    dk[x] *= sm_ * min_nan(kv[x], 1.f);
                    dv[x] *= sm_;
                }
                uint8_t* dst = slot_ptr(j, BL::g);
#pragma unroll
                for (int x = 0; x < 4; ++x) {
                    store_chunk<kFp16>(dst, row, hf * 4 + x, dk + 8 * x);
                    store_chunk<kFp16>(sm + BL::ob, row, hf * 4 + x, dv + 8 * x);
                }
                tc::fence_proxy_async();
                tc::tc_fence_before();
                tc::bar_sync(kBarCompute, kComputeThreads);
                if (tid == 0) {
                    tc::mbar_arrive(&bars[B_KVDONE]);  // dK / dV columns read
                    tc::tma_store_4d(&P.tm_dk, dst, 0, act(c) * kC, h, b);
                    tc::tma_store_4d(&P.tm_dv, sm + BL::ob, 0, act(c) * kC, h, b);
                    tc::bulk_commit();
                }
            }
        }
        // zero gradients of the chunks past the last live token (round-robin over the cluster)
        if (nL + g < nC) {
            if (tid == 0) tc::bulk_wait_read0();  // the o^ tile has been read by the last store
            tc::bar_sync(kBarCompute, kComputeThreads);
            zero_chunks(sm + BL::ob, row, hf * 4, 4);
            tc::fence_proxy_async();
            tc::bar_sync(kBarCompute, kComputeThreads);
            if (tid == 0) {
                for (int d = nL + g; d < nC; d += P.G) {
                    tc::tma_store_4d(&P.tm_dq, sm + BL::ob, 0, d * kC, h, b);
                    tc::tma_store_4d(&P.tm_dk, sm + BL::ob, 0, d * kC, h, b);
                    tc::tma_store_4d(&P.tm_dv, sm + BL::ob, 0, d * kC, h, b);
                }
                tc::bulk_commit();
            }
            if (want_dlg && hf == 0)  // and their d log(gamma) (masked tokens)
                for (int d = nL + g; d < nC; d += P.G)
                    if (d * kC + row < p.N) p.dlg[(int64_t)bh * p.N + d * kC + row] = 0.f;
        }
        if (want_dlg && tid == 0) misc[3] = dlg_carry;
        if (tid == 0) tc::bulk_wait0();
    }

    if (want_dlg) {
        // d log(gamma) of this segment's live tokens takes the sum over the later
        // segments' tokens (their totals, read over DSMEM)
        tc::tc_fence_before();
        cluster.sync();
        float off = 0.f;
        for (int r = g + 1; r < P.G; ++r) off += cluster.map_shared_rank(misc, r)[3];
        cluster.sync();  // remote reads done
        if (warp < 8 && n > 0 && ok && off != 0.f) {
            float* dl = p.dlg + (int64_t)bh * p.N;
            const int c0 = kRev ? nL - c_begin - n : c_begin;  // the segment's chunks in memory
            const int t1 = min(p.N, (c0 + n) * kC);
            for (int t = c0 * kC + tid; t < t1; t += kComputeThreads)
                if (!p.mask || p.mask[(int64_t)b * p.mask_sb + t]) dl[t] += off;
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma) tc::tmem_dealloc(tmem, kTmemCols);
}

template <bool kFp16, bool kNorm, bool kDecay, bool kRev = false>
cudaError_t launch(const ScanParams& p, cudaStream_t st) {
    BwdParams P;
    memset(&P, 0, sizeof(P));
    P.p = p;
    const int dt = kFp16 ? SUBQ_FP16 : SUBQ_BF16;
    if (!make_map(&P.tm_q, p.q, dt, p.N, p.H, p.B, p.q_sn, p.q_sh, p.q_sb) ||
        !make_map(&P.tm_k, p.k, dt, p.N, p.H / p.kvg, p.B, p.k_sn, p.k_sh, p.k_sb) ||
        !make_map(&P.tm_v, p.v, dt, p.N, p.H / p.kvg, p.B, p.v_sn, p.v_sh, p.v_sb) ||
        !make_map(&P.tm_g, p.g, dt, p.N, p.H, p.B, p.g_sn, p.g_sh, p.g_sb) ||
        !make_map(&P.tm_dq, p.o, dt, p.N, p.H, p.B, p.o_sn, p.o_sh, p.o_sb) ||
        !make_map(&P.tm_dk, p.dk, dt, p.N, p.H, p.B, p.dk_sn, p.dk_sh, p.dk_sb) ||
        !make_map(&P.tm_dv, p.dv, dt, p.N, p.H, p.B, p.dv_sn, p.dv_sh, p.dv_sb))
        return cudaErrorInvalidValue;
    const int nC = (p.N + kC - 1) / kC;
    P.status = status_ptr();
    if (!P.status) return cudaErrorInvalidDevice;
    const void* kern = reinterpret_cast<const void*>(&bwd_kernel<kFp16, kNorm, kDecay, kRev>);
    P.G = pick_segments(p, kern, kBwdThreads, BL::total + 1024);
    P.cps = (nC + P.G - 1) / P.G;
    void* args[] = {&P};
    return launch_cluster(kern, P.G, p.B * p.H, kBwdThreads, BL::total + 1024, st, args);
}

}  // namespace

cudaError_t launch_bwd_v2(const ScanParams& p, int dtype, cudaStream_t st) {
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
