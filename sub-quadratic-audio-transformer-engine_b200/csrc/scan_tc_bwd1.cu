// One-pass tensor-core backward (d = e = 64, bf16/fp16, no decay), over a
// grid-wide balanced split of the live chunks, for a backward whose forward
// handed over its per-chunk state operands, per-token normalisers and output.
//
// With q^ = phi(q), k^ = m phi(k), s = scale, the forward's output o and its
// clamped normaliser Zc, the quotient rule of the normalised form gives per
// token o^_t = m_t dO_t / Zc_t and c_t = -(dO_t . o_t) / Zc_t, and per
// 128-token chunk (S_c, z_c the state before the chunk, from the forward;
// dS, dz the adjoint of the state after the chunk, sum over later tokens of
// q^^T [o^ | c]):
//   P^T  = K^ q^^T                      [t >= tau]
//   dA   = o^ V^T + c 1^T               [tau <= t]     (dA^T likewise, key-major)
//   dQ~  = dA K^ + o^ S_c^T + c z_c^T                  dq = s dQ~ phi'(q)
//   dK~  = dA^T q^ + V dS^T + 1 dz^T                   dk = s dK~ phi'(k) m
//   dV   = P^T o^ + K^ dS                              dv = s dV m
//   [dS | dz] += q^^T [o^ | c]
// phi'(x) = min(phi(x), 1). The rank-one terms (c, z_c, dz) are added on the
// CUDA cores (in the mask step and the epilogues); every contraction is a
// tcgen05 MMA. The chunks of a piece run from the last one down, carrying
// [dS | dz] in TMEM; a piece that a later CTA continues starts from the sum of
// the later pieces' q^^T [o^ | c], which adj_kernel (launched first) computes
// for every piece that starts after its sequence's first live chunk.
//
// The mathematics is the reference's analytic backward
// (python/subq_audio/autograd.py:441-544: quotient rule :497-499, chunked
// adjoint :172-289) with the forward's saved quantities in place of its
// recomputation; the unnormalised form (engine) has o^ = m dO and c = 0.
//
// Roles (448 threads): warps 0-7 compute (TMEM lane = 32 (warp % 4) + lane,
// column half = warp / 4), warps 8-11 feature map, warp 12 TMA producer,
// warp 13 MMA issuer.
#include "tc_common.cuh"

#include <algorithm>

namespace subq {
namespace tcs {
namespace {

constexpr int kStages = 2;
constexpr int kThreads1 = 448;
constexpr int kComputeThreads = 256, kTransformThreads = 128;
constexpr int kBarCompute = 1, kBarTransform = 2, kBarPair = 3;  // kBarPair + quad: warps quad, quad + 4
constexpr int kWarpProducer = 12, kWarpMma = 13;
constexpr int kNX = 80;  // 64 value columns + the c atom's 16

struct L1 {
    // stage: q^, k^, v, dO (then o^), S_c, z_c, the c tile (128 x 16) and the z tile (64 x 16)
    static constexpr uint32_t q = 0, k = kTile, v = 2 * kTile, g = 3 * kTile;
    static constexpr uint32_t sat = 4 * kTile;     // S_c (bf16 state operand of the forward)
    static constexpr uint32_t ct = sat + kSAtom;   // c tile: column 0 = c_t (32-byte swizzle)
    static constexpr uint32_t zt = ct + kMTile;    // z tile: row f, column 0 = z_c[f]
    static constexpr uint32_t zv = zt + 2048;      // z_c, 64 fp32 (from the handover)
    static constexpr uint32_t stage = zv + 1024;
    static constexpr uint32_t da = kStages * stage;   // masked bf16 dA^T as dA's MN-major operand [2 atoms]
    static constexpr uint32_t dsb = da + 2 * kTile;   // bf16 dS of the later tokens (64 x 64)
    static constexpr uint32_t dzt = dsb + kSAtom;     // dz tile: row f, column 0 = dz[f]
    static constexpr uint32_t ones = dzt + 2048;      // ones tile: column 0 = 1 (128 x 16)
    static constexpr uint32_t dx = ones + kMTile;     // [2][2][128] fp32 partial dot products (chunk parity, half)
    static constexpr uint32_t inst = dx + 2048;       // [64][65] fp32: the later CTAs' sums for the last piece
    static constexpr uint32_t bars = inst + kD * (kD + 1) * 4;
    static constexpr uint32_t tslot = bars + 8 * 16;
    static constexpr uint32_t total = tslot + 16;
};
static_assert(L1::stage % 1024 == 0 && L1::da % 1024 == 0 && L1::dsb % 1024 == 0 &&
                  L1::ct % 1024 == 0 && L1::ones % 1024 == 0 && L1::zt % 256 == 0 && L1::dzt % 256 == 0,
              "alignment");
static_assert(L1::total + 1024 <= 232448, "shared memory");

enum {
    F_FULL = 0,          // [2] TMA -> feature map, compute
    F_TDONE = 2,         // [2] feature map -> MMA: q^, k^, z tile
    F_OUT = 4,           // [2] compute -> producer: dq, dk, dv staged over the stage's dO, k, v tiles
    F_OC = 6,            // [2] compute -> MMA: o^ (over dO) and the c tile of the stage
    F_MFULL = 8,         // MMA -> feature map: P^T
    F_MDONEP = 9,        // feature map -> MMA: P^T masked (bf16 in place)
    F_MDONEA = 10,       // compute -> MMA: dA^T masked (bf16 in place and in shared memory)
    F_DSFULL = 11,       // MMA -> compute: the chunk's MMAs done ([dS | dz] after it)
    F_EPI = 12,          // compute -> MMA: dV, dK, dQ~ read
    F_DSB = 13,          // compute -> MMA: bf16 dS and the dz tile of the later tokens in place
    F_MFULLA = 14,       // MMA -> compute: dA^T
    F_INST = 15,         // feature map -> compute: the last piece's suffix sums in shared memory
    F_COUNT = 16
};

// TMEM: P^T [0,128) (bf16 in [0,64), then dV in [64,128)), dA^T [128,256)
// (dK in its upper half), dQ~ [256,320), [dS | dz] [320,400) (M = 64 layout,
// column 64 = dz).
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t cPT = 0, cDAT = 128, cDQ = 256, cDS = 320;

struct Bwd1Params {
    CUtensorMap tm_q, tm_k, tm_v, tm_g, tm_dq, tm_dk, tm_dv, tm_fo;
    ScanParams p;
    Plan pl;
    const int* hdr;          // handover header (checked against this call)
    const uint8_t* chunks;   // per-chunk state operands
    const float* zc;         // per-token normalisers
    const float* agg;        // [R][64][65] q^^T [o^ | c] of each CTA's first piece (adj_kernel)
    int nC;
    int flags;               // expected header flags
    int* status;
};

// Whether the handover matches this call (every thread evaluates it).
__device__ __forceinline__ bool hand_ok(const Bwd1Params& P) {
    const int* h = P.hdr;
    if (!(h[1] == kHandMagic && h[6] == kHandMagic && h[2] == P.p.B * P.p.H && h[3] == P.p.N && h[4] == P.flags))
        return false;
    const int64_t T = __ldg(P.pl.off + P.pl.BH);
    return T >= 0 && T <= (int64_t)P.pl.BH * P.nC;
}

// per-chunk geometry from a cursor
struct Where {
    int sq, b, h, hk, nLs, c, mc;
};
__device__ __forceinline__ Where where_of(const ScanParams& p, const Plan& pl, const Cursor& cu, bool rev) {
    Where w;
    w.sq = cu.s;
    w.b = w.sq / p.H;
    w.h = w.sq - w.b * p.H;
    w.hk = w.h / p.kvg;
    w.nLs = __ldg(pl.off + w.sq + 1) - __ldg(pl.off + w.sq);
    w.c = cu.chunk();
    w.mc = rev ? w.nLs - 1 - w.c : w.c;  // the chunk's place in memory
    return w;
}
// The mask byte of row r of a chunk (1 without a mask, 0 past the sequence's
// end). The load is predicated on the position alone and its value is not
// tested here, so a thread waits for it only where it is used (mask_f, after the
// barrier waits), not at the load.
__device__ __forceinline__ int row_mask_raw(const ScanParams& p, const Where& w, int r) {
    const int t = w.mc * kC + r;
    int v = t < p.N ? 1 : 0;
    if (p.mask && t < p.N) v = __ldg(p.mask + (int64_t)w.b * p.mask_sb + t);
    return v;
}
__device__ __forceinline__ float mask_f(int raw) { return raw != 0 ? 1.f : 0.f; }

template <bool kFp16, bool kNorm, bool kRev>
__global__ void __launch_bounds__(kThreads1, 1) bwd1_kernel(const __grid_constant__ Bwd1Params P) {
    const ScanParams& p = P.p;
    Plan pl = P.pl;
    pl.T = __ldg(pl.off + pl.BH);  // live chunks of the call (the forward's prefix)
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r_cta = blockIdx.x;
    if (!hand_ok(P)) {
        if (tid == 0) atomicCAS(P.status, 0, (int)SUBQ_ERR_STATE);
        return;
    }
    Cursor cur0;
    cur0.begin(pl, r_cta);
    const int n = (int)(cur0.w1 - cur0.w);  // chunks of this CTA

    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L1::bars);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + L1::tslot);
    float* dxs = reinterpret_cast<float*>(sm + L1::dx);
    const uint32_t sbase = tc::smem_u32(sm);

    if (tid == 0) {
        // the compute warps' signals take one arrival per warp (8), each after that
        // warp's own shared-memory or TMEM work
        for (int i = 0; i < F_COUNT; ++i) {
            const bool per_warp = i == F_OC || i == F_OC + 1 || i == F_OUT || i == F_OUT + 1 || i == F_MDONEA ||
                                  i == F_DSB || i == F_EPI;
            tc::mbar_init(&bars[i], per_warp ? 8 : 1);
        }
        tc::fence_mbar_init();
    }
    if (warp == kWarpMma) tc::tmem_alloc(tslot, kTmemCols);
    if (warp >= 8 && warp < 12) {  // the ones tile
        mtile_row<kFp16>(sm + L1::ones, tid - 256, 1.f);
        tc::fence_proxy_async();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tslot;

    constexpr uint32_t idPP = tc::idesc_f16<kFp16>(128, 128, false, false);
    constexpr uint32_t idKK64 = tc::idesc_f16<kFp16>(128, 64, false, false);
    constexpr uint32_t idKM64 = tc::idesc_f16<kFp16>(128, 64, false, true);
    constexpr uint32_t idMM64 = tc::idesc_f16<kFp16>(128, 64, true, true);
    constexpr uint32_t idS64 = tc::idesc_f16<kFp16>(64, 64, true, true);
    constexpr uint32_t idZ16 = tc::idesc_f16<kFp16>(64, 16, true, true);
    auto slot_addr = [&](int i, uint32_t off) { return sbase + (i % kStages) * L1::stage + off; };
    auto slot_ptr = [&](int i, uint32_t off) { return sm + (i % kStages) * L1::stage + off; };

    bool ok = true;

    if (warp == kWarpProducer) {
        // ------------------------------------------------------------ TMA
        if (lane == 0) {
            tc::prefetch_tmap(&P.tm_q);
            tc::prefetch_tmap(&P.tm_k);
            tc::prefetch_tmap(&P.tm_v);
            tc::prefetch_tmap(&P.tm_g);
            // The outputs of chunk i leave from its stage's dO, k, v tiles; the
            // stage is loaded again (chunk i + 2) once those stores have read it.
            Where ws[kStages];
            auto store_out = [&](int j) -> bool {
                const int sj = j % kStages;
                if (!wait_bar(&bars[F_OUT + sj], (j / kStages) & 1, P.status)) return false;
                uint8_t* base = sm + sj * L1::stage;
                const Where& w = ws[sj];
                tc::tma_store_4d(&P.tm_dq, base + L1::g, 0, w.mc * kC, w.h, w.b);
                tc::tma_store_4d(&P.tm_dk, base + L1::k, 0, w.mc * kC, w.h, w.b);
                tc::tma_store_4d(&P.tm_dv, base + L1::v, 0, w.mc * kC, w.h, w.b);
                tc::bulk_commit();
                return true;
            };
            Cursor cu = cur0;
            for (int i = 0; i < n && ok; ++i, cu.next(pl)) {
                const int s = i % kStages;
                if (i >= kStages) {
                    ok = store_out(i - kStages);
                    tc::bulk_wait_read0();
                }
                if (!ok) break;
                const Where w = where_of(p, pl, cu, kRev);
                ws[s] = w;
                uint8_t* base = sm + s * L1::stage;
                const uint8_t* slot = P.chunks + ((size_t)w.sq * P.nC + w.c) * kChunkSlot;
                tc::mbar_arrive_expect_tx(&bars[F_FULL + s], 4 * kTile + kSAtom + (kNorm ? 256u : 0u));
                tc::tma_load_4d(base + L1::g, &P.tm_g, 0, w.mc * kC, w.h, w.b, &bars[F_FULL + s]);
                tc::tma_load_4d(base + L1::q, &P.tm_q, 0, w.mc * kC, w.h, w.b, &bars[F_FULL + s]);
                tc::tma_load_4d(base + L1::k, &P.tm_k, 0, w.mc * kC, w.hk, w.b, &bars[F_FULL + s]);
                tc::tma_load_4d(base + L1::v, &P.tm_v, 0, w.mc * kC, w.hk, w.b, &bars[F_FULL + s]);
                tc::bulk_load(base + L1::sat, slot, kSAtom, &bars[F_FULL + s]);
                if (kNorm) tc::bulk_load(base + L1::zv, slot + kSAtom, 256, &bars[F_FULL + s]);
            }
            for (int j = (n > kStages ? n - kStages : 0); j < n && ok; ++j) ok = store_out(j);
            tc::bulk_wait0();
        }
        __syncwarp();
    } else if (warp >= 8 && warp < 12) {
        // ------------------- feature map (row r) and z tile; P^T masked (row r)
        using E = Elem<kFp16>;
        const int r = tid - 256;
        const uint32_t toff = (uint32_t)((warp & 3) * 32) << 16;  // TMEM lanes of this warp
        auto transform = [&](int i, const Cursor& cu) -> bool {
            const int s = i % kStages, u = i / kStages;
            const int mr = row_mask_raw(p, where_of(p, pl, cu, kRev), r);
            ok = tc::bar_and(kBarTransform, kTransformThreads, wait_bar(&bars[F_FULL + s], u & 1, P.status)) && ok;
            if (!ok) return false;
            uint8_t* base = sm + s * L1::stage;
            // q^ then m phi(k) (scale is applied in the epilogue); one copy of the code
#pragma unroll 1
            for (int tt = 0; tt < 2; ++tt) chunks_phi<kFp16>(base + (tt ? L1::k : L1::q), r, 0, 8, tt ? mr != 0 : true);
            if (kNorm && r < kD) mtile_row<kFp16>(base + L1::zt, r, reinterpret_cast<const float*>(base + L1::zv)[r]);
            tc::fence_proxy_async();
            tc::bar_sync(kBarTransform, kTransformThreads);
            if (r == 0) tc::mbar_arrive(&bars[F_TDONE + s]);
            return true;
        };
        // row r (key tau) of P^T: keep queries t >= tau (reverse time: t <= tau),
        // bf16 into the row's first 64 columns. One thread holds the whole row, so
        // it overwrites only columns it has already read.
        auto mask_pt = [&]() {
#pragma unroll 1
            for (int half = 0; half < 2; ++half) {
                const bool dead = kRev ? (half == 1 && r < 64) : (half == 0 && r >= 64);
                const bool diag = half == (r >> 6);
                uint32_t packed[32];
                if (dead) {
#pragma unroll
                    for (int x = 0; x < 32; ++x) packed[x] = 0u;
                } else {
                    uint32_t v[64];
                    tc::tmem_ld32_issue(tmem + cPT + toff + half * 64, v);
                    tc::tmem_ld32_issue(tmem + cPT + toff + half * 64 + 32, v + 32);
                    tc::tmem_wait_ld();
                    tc::tmem_regs_ready<64>(v);
#pragma unroll
                    for (int x = 0; x < 32; ++x) {
                        const int col = half * 64 + 2 * x;
                        float a = __uint_as_float(v[2 * x]), bb = __uint_as_float(v[2 * x + 1]);
                        if (diag) {
                            if (kRev ? (col > r) : (col < r)) a = 0.f;
                            if (kRev ? (col + 1 > r) : (col + 1 < r)) bb = 0.f;
                        }
                        typename E::T2 h2 = E::from2(a, bb);
                        packed[x] = *reinterpret_cast<uint32_t*>(&h2);
                    }
                }
                tc::tmem_st32_raw_nowait(tmem + cPT + toff + half * 32, packed);
            }
            tc::tmem_wait_st();
        };
        // While the first chunk loads: when this CTA's last piece continues in later
        // CTAs, the sum of their first pieces' q^^T [o^ | c] (adj_kernel) is that
        // piece's suffix; it goes to shared memory, in the [64][65] layout of agg.
        {
            float* inst = reinterpret_cast<float*>(sm + L1::inst);
            const int sqL = n > 0 ? pl.seq_at(cur0.w1 - 1) : 0;
            const int o1 = n > 0 ? __ldg(pl.off + sqL + 1) : 0;
            if (n > 0 && cur0.w1 < (int64_t)o1) {
                float acc[33];
#pragma unroll
                for (int x = 0; x < 33; ++x) acc[x] = 0.f;
                int64_t a2 = pl.w0(r_cta + 1);
                for (int r2 = r_cta + 1; r2 < pl.R && a2 < o1; ++r2) {
                    const int64_t a3 = pl.w0(r2 + 1);
                    if (a3 > a2) {  // (an empty range has no first piece)
                        const float* src = P.agg + (size_t)r2 * kD * (kD + 1);
#pragma unroll
                        for (int x = 0; x < 33; ++x) {
                            const int idx = r + x * kTransformThreads;
                            if (idx < kD * (kD + 1)) acc[x] += __ldg(src + idx);
                        }
                    }
                    a2 = a3;
                }
#pragma unroll
                for (int x = 0; x < 33; ++x) {
                    const int idx = r + x * kTransformThreads;
                    if (idx < kD * (kD + 1)) inst[idx] = acc[x];
                }
            }
            tc::bar_sync(kBarTransform, kTransformThreads);
            if (r == 0) tc::mbar_arrive(&bars[F_INST]);
        }
        Cursor cu = cur0;
        // i = -1 only maps chunk 0 (one call site of each step keeps the code small);
        // a CTA without chunks runs no iteration (its cursor holds no piece)
        for (int i = n > 0 ? -1 : 0; i < n && ok; ++i) {
            if (i >= 0) {
                ok = tc::bar_and(kBarTransform, kTransformThreads, wait_bar(&bars[F_MFULL], i & 1, P.status)) && ok;
                if (!ok) break;
                tc::tc_fence_after();
                mask_pt();
                tc::tc_fence_before();
                tc::bar_sync(kBarTransform, kTransformThreads);
                if (r == 0) tc::mbar_arrive(&bars[F_MDONEP]);
                if (i + 1 < n) cu.next(pl);
            }
            if (i + 1 < n && !transform(i + 1, cu)) break;
        }
    } else if (warp == kWarpMma) {
        // ------------------------------------------------------------- MMA
        // (the whole warp runs this, converged; one elected lane issues each MMA)
        {
            const uint32_t dsa = sbase + L1::dsb, oneA = sbase + L1::ones, dza = sbase + L1::dzt;
            const uint32_t daa = sbase + L1::da;
            for (int i = 0; i < n && ok; ++i) {
                const int s = i % kStages, u = i / kStages;
                const uint32_t qa = slot_addr(i, L1::q), ka = slot_addr(i, L1::k), va = slot_addr(i, L1::v);
                const uint32_t oa = slot_addr(i, L1::g), sa = slot_addr(i, L1::sat), ca = slot_addr(i, L1::ct);
                const uint32_t za = slot_addr(i, L1::zt);
                ok = wait_bar(&bars[F_TDONE + s], u & 1, P.status);
                if (ok) ok = wait_bar(&bars[F_OC + s], u & 1, P.status);
                if (ok && i >= 1) ok = wait_bar(&bars[F_EPI], (i - 1) & 1, P.status);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) break;
                tc::tc_fence_after();
                // P^T = K^ q^^T ; dA^T = V o^^T + 1 c^T
                {
                    const uint64_t dk = tc::sdesc_sw128(ka, 16, 1024), dq = tc::sdesc_sw128(qa, 16, 1024);
                    const uint64_t dv = tc::sdesc_sw128(va, 16, 1024), dob = tc::sdesc_sw128(oa, 16, 1024);
                    tc::mma_f16_x4(tmem + cPT, dk, 2, dq, 2, idPP, 0u);
                    tc::mma_commit_w(&bars[F_MFULL]);
                    tc::mma_f16_x4(tmem + cDAT, dv, 2, dob, 2, idPP, 0u);
                    if (kNorm) tc::mma_f16_w(tmem + cDAT, sdesc_sw32(oneA), sdesc_sw32(ca), idPP, 1u);
                }
                tc::mma_commit_w(&bars[F_MFULLA]);
                const uint64_t dkm = tc::sdesc_sw128(ka, kTile, 1024), dqm = tc::sdesc_sw128(qa, kTile, 1024);
                const uint64_t dom = tc::sdesc_sw128(oa, kTile, 1024);
                const uint64_t dob = tc::sdesc_sw128(oa, 16, 1024), dsat = tc::sdesc_sw128(sa, 16, 1024);
                const uint64_t dv = tc::sdesc_sw128(va, 16, 1024), dsk = tc::sdesc_sw128(dsa, 16, 1024);
                const uint64_t dk = tc::sdesc_sw128(ka, 16, 1024), dsm = tc::sdesc_sw128(dsa, kTile, 1024);
                // The products that need no mask run while P^T and dA^T are masked.
                // dQ~ = o^ S_c^T + c z_c^T
                tc::mma_f16_x4(tmem + cDQ, dob, 2, dsat, 2, idKK64, 0u);
                if (kNorm) tc::mma_f16_w(tmem + cDQ, sdesc_sw32(ca), sdesc_sw32(za), idKK64, 1u);
                // [dS | dz] += q^^T [o^ | c]  (M = 64: dS from the o^ tile, dz from the c tile), once
                // the compute warps have copied [dS | dz] of the later tokens (the bf16 operand)
                ok = __all_sync(0xffffffffu, wait_bar(&bars[F_DSB], i & 1, P.status));
                if (!ok) break;
                tc::tc_fence_after();
                {
                    const uint64_t dqt = tc::sdesc_sw128(qa, kTile, 1024);
                    tc::mma_f16_x8(tmem + cDS, dqt, 128, dom, 128, idS64, 1u);
                    // (the c tile's 16-token steps are 512 bytes: 32 in the descriptor)
                    if (kNorm) tc::mma_f16_x8(tmem + cDS + 64, dqt, 128, sdesc_sw32(ca), 32, idZ16, 1u);
                }
                ok = __all_sync(0xffffffffu, wait_bar(&bars[F_MDONEP], i & 1, P.status));
                if (!ok) break;
                tc::tc_fence_after();
                // dV = P^T o^ + K^ dS   (A = bf16 P^T from TMEM, 8 columns per 16 tokens)
                tc::mma_f16_ts_x8(tmem + cPT + 64, tmem + cPT, 8, dom, 128, idKM64, 0u);
                tc::mma_f16_x4(tmem + cPT + 64, dk, 2, dsm, 128, idKM64, 1u);
                ok = wait_bar(&bars[F_MDONEA], i & 1, P.status);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) break;
                tc::tc_fence_after();
                // dK~ = dA^T q^ + V dS^T + 1 dz^T
                tc::mma_f16_ts_x8(tmem + cDAT + 64, tmem + cDAT, 8, dqm, 128, idKM64, 0u);
                tc::mma_f16_x4(tmem + cDAT + 64, dv, 2, dsk, 2, idKK64, 1u);
                if (kNorm) tc::mma_f16_w(tmem + cDAT + 64, sdesc_sw32(oneA), sdesc_sw32(dza), idKK64, 1u);
                // dQ~ += dA K^  (A = masked dA^T in shared memory, read as dA: MN-major over queries)
                {
                    const uint64_t dda = tc::sdesc_sw128(daa, kTile, 1024);
                    tc::mma_f16_x8(tmem + cDQ, dda, 128, dkm, 128, idMM64, 1u);
                }
                tc::mma_commit_w(&bars[F_DSFULL]);
            }
        }
        __syncwarp();
    } else {
        // --------------------------------------------------------- compute
        using E = Elem<kFp16>;
        const int quad = warp & 3, hf = warp >> 2;
        const int row = quad * 32 + lane, srow = quad * 16 + lane;
        const uint32_t loff = (uint32_t)(quad * 32) << 16;
        // this warp's shared-memory writes (to the async proxy) and TMEM accesses
        // are complete: one arrival of the 8 the barrier counts
        auto publish = [&](uint64_t* bar) {
            tc::fence_proxy_async();
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(bar);
        };
        auto cwait = [&](uint64_t* bar, uint32_t parity) -> bool {
            ok = tc::bar_and(kBarCompute, kComputeThreads, wait_bar(bar, parity, P.status)) && ok;
            if (ok) tc::tc_fence_after();
            return ok;
        };
        // [dS | dz] -> bf16 dS (64 x 64) and the dz tile, from registers (rows in lanes 0-15)
        auto put_ds = [&](const float* v, float z) {
            if (lane < 16) {
#pragma unroll
                for (int x = 0; x < 4; ++x) store_chunk<kFp16>(sm + L1::dsb, srow, hf * 4 + x, v + 8 * x);
                if (kNorm && hf == 0) mtile_row<kFp16>(sm + L1::dzt, srow, z);
            }
        };
        // [dS | dz] of the tokens after piece (sq, e): the adjoint sums of the
        // first pieces of the later CTAs that lie in sequence sq (zero when the
        // piece ends its sequence) -> TMEM accumulator and its bf16 operands
        auto install = [&](const Cursor& cu) {
            float v[32], z = 0.f;
#pragma unroll
            for (int x = 0; x < 32; ++x) v[x] = 0.f;
            const int o1 = __ldg(pl.off + cu.s + 1);
            if (cu.w1 < (int64_t)o1) {  // the last piece, continued by later CTAs
                if (!cwait(&bars[F_INST], 0)) return;
                if (lane < 16) {
                    const float* src = reinterpret_cast<const float*>(sm + L1::inst) + srow * (kD + 1);
#pragma unroll
                    for (int x = 0; x < 32; ++x) v[x] = src[hf * 32 + x];
                    if (kNorm) z = src[kD];
                }
            }
            tc::tmem_st32(tmem + cDS + loff + hf * 32, v);
            if (hf == 0) {
                float w[32];
#pragma unroll
                for (int x = 0; x < 32; ++x) w[x] = 0.f;
                w[0] = z;
                tc::tmem_st32(tmem + cDS + loff + 64, w);
            }
            put_ds(v, z);
        };
        auto refresh = [&]() {
            float v[32];
            tc::tmem_ld32(tmem + cDS + loff + hf * 32, v);
            const float z = (kNorm && hf == 0) ? tmem_ld1(tmem + cDS + loff + 64) : 0.f;
            put_ds(v, z);
        };
        // the forward's output (this thread's half row) and normaliser of chunk i
        // (issued together with the mask's load: the mask is applied afterwards)
        auto fetch_o = [&](const Where& w, uint4* ov, float& zc) {
            const int t = w.mc * kC + row;
            zc = 1.f;
            if (kNorm && t < p.N) {
                const uint4* src = reinterpret_cast<const uint4*>(
                    reinterpret_cast<const typename E::T*>(p.fo) + (int64_t)w.b * p.fo_sb + (int64_t)w.h * p.fo_sh +
                    (int64_t)t * p.fo_sn + hf * 32);
#pragma unroll
                for (int j = 0; j < 4; ++j) ov[j] = __ldg(src + j);
                zc = __ldg(P.zc + (int64_t)w.sq * p.N + t);
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) ov[j] = make_uint4(0, 0, 0, 0);
            }
        };
        // o^ = m dO / Zc over the dO tile and c = -(dO . o) / Zc into the c tile (chunk i)
        auto make_oc = [&](int i, const Where& w) -> bool {
            const int s = i % kStages;
            uint4 ov[4];
            float zc;
            fetch_o(w, ov, zc);  // (in flight during the wait)
            const int mr = row_mask_raw(p, w, row);
            if (!cwait(&bars[F_FULL + s], (i / kStages) & 1)) return false;
            const float m = mask_f(mr);
            uint8_t* gt = slot_ptr(i, L1::g);
            float go[32];
            load_chunks<kFp16>(gt, row, hf * 4, 4, go);
            float inv = m;
            if (kNorm) {
                float dot = 0.f;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const typename E::T2* o2 = reinterpret_cast<const typename E::T2*>(&ov[j]);
#pragma unroll
                    for (int y = 0; y < 4; ++y) {
                        const float2 b = E::to2(o2[y]);
                        dot = fmaf(go[8 * j + 2 * y], b.x, fmaf(go[8 * j + 2 * y + 1], b.y, dot));
                    }
                }
                dxs[(i & 1) * 256 + hf * 128 + row] = dot;
                tc::bar_sync(kBarCompute, kComputeThreads);
                const float full = dxs[(i & 1) * 256 + row] + dxs[(i & 1) * 256 + 128 + row];
                if (hf == 0) mtile_row<kFp16>(slot_ptr(i, L1::ct), row, m != 0.f ? -full / zc : 0.f);
                inv = m != 0.f ? m / zc : 0.f;
            } else {
                tc::bar_sync(kBarCompute, kComputeThreads);  // every half row of dO is read
            }
#pragma unroll
            for (int x = 0; x < 32; ++x) go[x] *= inv;
#pragma unroll
            for (int x = 0; x < 4; ++x) store_chunk<kFp16>(gt, row, hf * 4 + x, go + 8 * x);
            publish(&bars[F_OC + s]);
            return true;
        };
        // 128 x 128 fp32 tile (rows = keys, columns = queries) -> masked bf16
        // (keep t >= tau) in its first 64 columns; with `smem`, the same bf16
        // values also into the dA^T tile (two 64-column atoms, 128-byte swizzle)
        auto mask_tile = [&](uint32_t tcol, bool to_smem) {
            const bool keep_upper = !kRev;  // reverse time: the other triangle
            uint32_t packed[32];
            const bool zero = keep_upper ? (hf == 0 && quad >= 2) : (hf == 1 && quad < 2);
            if (zero) {
#pragma unroll
                for (int x = 0; x < 32; ++x) packed[x] = 0u;
            } else {
                const bool diag = (hf == (quad >> 1));
                uint32_t r[64];
                tc::tmem_ld32_issue(tmem + tcol + loff + hf * 64, r);
                tc::tmem_ld32_issue(tmem + tcol + loff + hf * 64 + 32, r + 32);
                tc::tmem_wait_ld();
                tc::tmem_regs_ready<64>(r);
#pragma unroll
                for (int x = 0; x < 32; ++x) {
                    const int col = hf * 64 + 2 * x;
                    float a = __uint_as_float(r[2 * x]), bb = __uint_as_float(r[2 * x + 1]);
                    if (diag) {
                        if (keep_upper ? (col < row) : (col > row)) a = 0.f;
                        if (keep_upper ? (col + 1 < row) : (col + 1 > row)) bb = 0.f;
                    }
                    typename E::T2 h2 = E::from2(a, bb);
                    packed[x] = *reinterpret_cast<uint32_t*>(&h2);
                }
            }
            if (to_smem) {  // row = key tau, this half's 64 queries -> atom hf
                uint8_t* atom = sm + L1::da + hf * kTile;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    *reinterpret_cast<uint4*>(atom + tc::sw128_chunk(row, j)) =
                        make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
            }
            // the other half of these rows (warp w ^ 4) has read its fp32 columns,
            // which this half's bf16 columns overwrite
            tc::tc_fence_before();
            tc::bar_sync(kBarPair + quad, 64);
            tc::tc_fence_after();
            tc::tmem_st32_raw_nowait(tmem + tcol + loff + hf * 32, packed);
        };

        // i = -1 only prepares chunk 0 (o^, c and its [dS | dz] operand): one call
        // site of each step keeps the loop's code small. A CTA without chunks runs
        // no iteration (its cursor holds no piece), and cn never steps past the range.
        Cursor cu = cur0, cn = cur0;  // chunk i and chunk i + 1
        for (int i = n > 0 ? -1 : 0; i < n && ok; ++i) {
            const int s = i % kStages;
            int mr_row = 0;
            if (i >= 0) {
                mr_row = row_mask_raw(p, where_of(p, pl, cu, kRev), row);  // (for the epilogue; loaded early)
                // (1) mask dA^T (also into shared memory for dQ~); the feature-map warps mask P^T
                if (!cwait(&bars[F_MFULLA], i & 1)) break;
                mask_tile(cDAT, true);
                tc::tmem_wait_st();
                publish(&bars[F_MDONEA]);
            }
            // (2) o^, c of the next chunk (the tensor core runs this chunk's products)
            if (i + 1 < n && !make_oc(i + 1, where_of(p, pl, cn, kRev))) break;
            // (3) once the chunk's MMAs are done: [dS | dz] after this chunk, the next
            // chunk's operand (or the next piece's suffix), first, so that the next
            // chunk's [dS | dz] products can run while its masks are made
            if (i >= 0 && !cwait(&bars[F_DSFULL], i & 1)) break;
            if (i + 1 < n) {
                if (cn.first()) install(cn);
                else refresh();
            }
            publish(&bars[F_DSB]);
            tc::tc_fence_after();
            // (4) epilogue; the producer stores the gradients
            if (i >= 0) {
                const float sm_ = p.scale * mask_f(mr_row);
                uint32_t rv[32], rk[32], rq[32];
                tc::tmem_ld32_issue(tmem + cPT + 64 + loff + hf * 32, rv);
                tc::tmem_ld32_issue(tmem + cDAT + 64 + loff + hf * 32, rk);
                tc::tmem_ld32_issue(tmem + cDQ + loff + hf * 32, rq);
                tc::tmem_wait_ld();
                tc::tmem_regs_ready<32>(rv);
                tc::tmem_regs_ready<32>(rk);
                tc::tmem_regs_ready<32>(rq);
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&bars[F_EPI]);  // this warp's accumulator rows are read
                // dv = s m dV over the v tile; dk = s m dK~ phi'(k) over the k^ tile; dq =
                // s dQ~ phi'(q) over the o^ tile (phi' = min(phi, 1)), 8 columns at a time
#pragma unroll
                for (int x = 0; x < 4; ++x) {
                    float o[8], f[8];
#pragma unroll
                    for (int y = 0; y < 8; ++y) o[y] = __uint_as_float(rv[8 * x + y]) * sm_;
                    store_chunk<kFp16>(slot_ptr(i, L1::v), row, hf * 4 + x, o);
                    load_chunks<kFp16>(slot_ptr(i, L1::k), row, hf * 4 + x, 1, f);
#pragma unroll
                    for (int y = 0; y < 8; ++y) o[y] = __uint_as_float(rk[8 * x + y]) * sm_ * min_nan(f[y], 1.f);
                    store_chunk<kFp16>(slot_ptr(i, L1::k), row, hf * 4 + x, o);
                    load_chunks<kFp16>(slot_ptr(i, L1::q), row, hf * 4 + x, 1, f);
#pragma unroll
                    for (int y = 0; y < 8; ++y) o[y] = __uint_as_float(rq[8 * x + y]) * p.scale * min_nan(f[y], 1.f);
                    store_chunk<kFp16>(slot_ptr(i, L1::g), row, hf * 4 + x, o);
                }
                publish(&bars[F_OUT + s]);  // the producer stores them and reloads the stage
            }
            cu = cn;
            if (i + 2 < n) cn.next(pl);
        }
    }

    tc::tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma) tc::tmem_dealloc(tmem, kTmemCols);
}

// Pre-pass of the one-pass backward, on the same grid and plan:
//  * CTA r whose first piece starts after its sequence's first live chunk sums
//    q^^T [o^ | c] over that piece into agg[r] (the adjoint that the earlier
//    CTAs of the sequence start from);
//  * every CTA zeroes dq, dk, dv of its share of the dead chunks (those after
//    each sequence's last live token), with TMA stores of a zero tile.
// Four stages of q^, o^ (over dO) and the forward's output o; once a row's
// o . dO is formed, c_t goes into column 0 of the same row of the o tile, which
// is then the last 16 columns of the N = 80 operand [o^ | c].
constexpr int kAdjStages = 4;
struct LA {
    static constexpr uint32_t q = 0, g = kTile, o = 2 * kTile;
    static constexpr uint32_t stage = 3 * kTile;
    static constexpr uint32_t zt = kAdjStages * stage;  // zero tile
    static constexpr uint32_t dx = zt + kTile;          // [2][256] partial dot products
    static constexpr uint32_t bars = dx + 2048;
    static constexpr uint32_t tslot = bars + 8 * 16;
    static constexpr uint32_t total = tslot + 16;
};
static_assert(LA::stage % 1024 == 0 && LA::zt % 1024 == 0, "alignment");
static_assert(LA::total + 1024 <= 232448, "shared memory");
enum { A_FULL = 0, A_TDONE = kAdjStages, A_EMPTY = 2 * kAdjStages, A_DONE = 3 * kAdjStages, A_COUNT = A_DONE + 1 };
static_assert(A_COUNT <= 16, "barrier slots");

template <bool kFp16, bool kNorm, bool kRev>
__global__ void __launch_bounds__(kThreads1, 1) adj_kernel(const __grid_constant__ Bwd1Params P, float* agg) {
    const ScanParams& p = P.p;
    if (!hand_ok(P)) return;  // (bwd1_kernel reports the mismatch)
    Plan pl = P.pl;
    pl.T = __ldg(pl.off + pl.BH);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r_cta = blockIdx.x;
    Cursor cu0;
    cu0.begin(pl, r_cta);
    const bool need = cu0.w < cu0.w1 && cu0.a > 0;
    const int n = need ? cu0.e - cu0.a : 0;
    const int sq = need ? cu0.s : 0;
    const int b = sq / p.H, h = sq - b * p.H;
    const int nLs = need ? __ldg(pl.off + sq + 1) - __ldg(pl.off + sq) : 0;
    auto mem_chunk = [&](int i) { const int c = cu0.a + i; return kRev ? nLs - 1 - c : c; };

    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + LA::bars);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + LA::tslot);
    const uint32_t sbase = tc::smem_u32(sm);
    if (tid == 0) {  // a stage is ready when both the feature map and o^, c are (two arrivals)
        for (int i = 0; i < A_COUNT; ++i) tc::mbar_init(&bars[i], (i >= A_TDONE && i < A_EMPTY) ? 2 : 1);
        tc::fence_mbar_init();
    }
    if (warp == kWarpMma && need) tc::tmem_alloc(tslot, 128);
    if (warp < 8) zero_chunks(sm + LA::zt, tid & 127, (tid >> 7) * 4, 4);  // the zero tile
    tc::fence_proxy_async();
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = need ? *tslot : 0u;

    // dead chunks: D = B H nC - T in all, this CTA's even share; dead chunks
    // before sequence s number s nC - off[s]; those of s are its memory chunks [nL_s, nC)
    auto zero_dead = [&]() {
        const int BH = p.B * p.H, nC = P.nC;
        const int64_t D = (int64_t)BH * nC - pl.T;
        const int64_t d0 = D * r_cta / gridDim.x, d1 = D * (r_cta + 1) / gridDim.x;
        if (d0 < d1) {
            int lo = 0, hi = BH - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if ((int64_t)mid * nC - __ldg(pl.off + mid) <= d0) lo = mid;
                else hi = mid - 1;
            }
            for (int64_t d = d0; d < d1; ++d) {
                while ((int64_t)(lo + 1) * nC - __ldg(pl.off + lo + 1) <= d) ++lo;
                const int nl = __ldg(pl.off + lo + 1) - __ldg(pl.off + lo);
                const int mc = nl + (int)(d - ((int64_t)lo * nC - __ldg(pl.off + lo)));
                const int bb = lo / p.H, hh = lo - bb * p.H;
                tc::tma_store_4d(&P.tm_dq, sm + LA::zt, 0, mc * kC, hh, bb);
                tc::tma_store_4d(&P.tm_dk, sm + LA::zt, 0, mc * kC, hh, bb);
                tc::tma_store_4d(&P.tm_dv, sm + LA::zt, 0, mc * kC, hh, bb);
            }
            tc::bulk_commit();
        }
    };

    // [dS | dz] += q^^T [o^ | c]: M = 64, N = 80 (the o^ tile, then the c columns LBO bytes on)
    constexpr uint32_t idSX = tc::idesc_f16<kFp16>(64, kNorm ? kNX : 64, true, true);
    bool ok = true;
    if (warp == kWarpProducer) {
        if (lane == 0) {
            for (int i = 0; i < n && ok; ++i) {
                const int s = i % kAdjStages, u = i / kAdjStages;
                if (u >= 1) ok = wait_bar(&bars[A_EMPTY + s], (u - 1) & 1, P.status);
                if (!ok) break;
                uint8_t* base = sm + s * LA::stage;
                tc::mbar_arrive_expect_tx(&bars[A_FULL + s], (kNorm ? 3u : 2u) * kTile);
                tc::tma_load_4d(base + LA::g, &P.tm_g, 0, mem_chunk(i) * kC, h, b, &bars[A_FULL + s]);
                if (kNorm) tc::tma_load_4d(base + LA::o, &P.tm_fo, 0, mem_chunk(i) * kC, h, b, &bars[A_FULL + s]);
                tc::tma_load_4d(base + LA::q, &P.tm_q, 0, mem_chunk(i) * kC, h, b, &bars[A_FULL + s]);
            }
            zero_dead();
            tc::bulk_wait0();  // the zero stores are done with the tile
        }
        __syncwarp();
    } else if (warp >= 8 && warp < 12) {
        // phi(q) of row r
        const int r = tid - 256;
        for (int i = 0; i < n && ok; ++i) {
            const int s = i % kAdjStages, u = i / kAdjStages;
            ok = tc::bar_and(kBarTransform, kTransformThreads, wait_bar(&bars[A_FULL + s], u & 1, P.status)) && ok;
            if (!ok) break;
            chunks_phi<kFp16>(sm + s * LA::stage + LA::q, r, 0, 8, true);
            tc::fence_proxy_async();
            tc::bar_sync(kBarTransform, kTransformThreads);
            if (r == 0) tc::mbar_arrive(&bars[A_TDONE + s]);
        }
    } else if (warp == kWarpMma) {
        {  // warp-converged; one elected lane issues
            for (int i = 0; i < n && ok; ++i) {
                const int s = i % kAdjStages, u = i / kAdjStages;
                ok = __all_sync(0xffffffffu, wait_bar(&bars[A_TDONE + s], u & 1, P.status));
                if (!ok) break;
                tc::tc_fence_after();
                const uint32_t qa = sbase + s * LA::stage + LA::q, oa = sbase + s * LA::stage + LA::g;
                const uint64_t dqt = tc::sdesc_sw128(qa, kTile, 1024);
                const uint64_t dbo = tc::sdesc_sw128(oa, LA::o - LA::g, 1024);
                tc::mma_f16_x8(tmem, dqt, 128, dbo, 128, idSX, i > 0 ? 1u : 0u);
                tc::mma_commit_w(&bars[A_EMPTY + s]);
            }
            if (n > 0 && ok) tc::mma_commit_w(&bars[A_DONE]);
        }
        __syncwarp();
    } else if (warp < 8) {
        // o^ = m dO / Zc (over the dO tile) and c = -(dO . o) / Zc (column 0 of the o
        // tile): two threads per row (row = 32 (warp % 4) + lane, column half = warp / 4)
        using E = Elem<kFp16>;
        const int quad = warp & 3, hf = warp >> 2;
        const int row = quad * 32 + lane, srow = quad * 16 + lane;
        const uint32_t loff = (uint32_t)(quad * 32) << 16;
        float* dxs = reinterpret_cast<float*>(sm + LA::dx);
        // mask and normaliser of a row of chunk i (loaded a chunk ahead); both loads
        // issue at once (the normaliser's does not wait for the mask's)
        // (the mask byte is kept raw until it is used: see row_mask_raw)
        auto row_info = [&](int i, int& mr, float& zc) {
            const int t = mem_chunk(i) * kC + row;
            const bool in = t < p.N;
            mr = in ? 1 : 0;
            if (p.mask && in) mr = __ldg(p.mask + (int64_t)b * p.mask_sb + t);
            zc = (kNorm && in) ? __ldg(P.zc + (int64_t)sq * p.N + t) : 1.f;
        };
        int mr_next = 0;
        float zc_next = 1.f;
        if (n > 0) row_info(0, mr_next, zc_next);
        for (int i = 0; i < n && ok; ++i) {
            const int s = i % kAdjStages, u = i / kAdjStages;
            const int mr = mr_next;
            const float zc = zc_next;
            if (i + 1 < n) row_info(i + 1, mr_next, zc_next);
            ok = tc::bar_and(kBarCompute, kComputeThreads, wait_bar(&bars[A_FULL + s], u & 1, P.status)) && ok;
            if (!ok) break;
            const float m = mask_f(mr);
            uint8_t* gt = sm + s * LA::stage + LA::g;
            float go[32];
            load_chunks<kFp16>(gt, row, hf * 4, 4, go);
            float inv = m;
            if (kNorm) {
                float ov[32];
                load_chunks<kFp16>(sm + s * LA::stage + LA::o, row, hf * 4, 4, ov);
                float dot = 0.f;
#pragma unroll
                for (int x = 0; x < 32; ++x) dot = fmaf(go[x], ov[x], dot);
                dxs[(i & 1) * 256 + hf * 128 + row] = dot;
                tc::bar_sync(kBarCompute, kComputeThreads);  // (every half row of o is read)
                const float full = dxs[(i & 1) * 256 + row] + dxs[(i & 1) * 256 + 128 + row];
                if (hf == 0) atom_col0<kFp16>(sm + s * LA::stage + LA::o, row, m != 0.f ? -full / zc : 0.f);
                inv = m != 0.f ? m / zc : 0.f;
            } else {
                tc::bar_sync(kBarCompute, kComputeThreads);  // every half row of dO is read
            }
#pragma unroll
            for (int x = 0; x < 32; ++x) go[x] *= inv;
#pragma unroll
            for (int x = 0; x < 4; ++x) store_chunk<kFp16>(gt, row, hf * 4 + x, go + 8 * x);
            tc::fence_proxy_async();
            tc::bar_sync(kBarCompute, kComputeThreads);
            if (tid == 0) tc::mbar_arrive(&bars[A_TDONE + s]);
        }
        if (n > 0) {
            ok = tc::bar_and(kBarCompute, kComputeThreads, ok && wait_bar(&bars[A_DONE], 0, P.status));
            if (ok) {
                tc::tc_fence_after();
                float v[32];
                tc::tmem_ld32(tmem + loff + hf * 32, v);
                float* dst = agg + ((size_t)r_cta * kD + srow) * (kD + 1);
                if (lane < 16) {
#pragma unroll
                    for (int x = 0; x < 32; ++x) dst[hf * 32 + x] = v[x];
                }
                if (hf == 0) {
                    const float z = kNorm ? tmem_ld1(tmem + loff + 64) : 0.f;
                    if (lane < 16) dst[kD] = z;
                }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma && need) tc::tmem_dealloc(tmem, 128);
}

template <bool kFp16, bool kNorm, bool kRev>
cudaError_t launch1(const ScanParams& p, cudaStream_t st, int* launches) {
    Bwd1Params P;
    memset(&P, 0, sizeof(P));
    P.p = p;
    const int dt = kFp16 ? SUBQ_FP16 : SUBQ_BF16;
    if (!make_map(&P.tm_q, p.q, dt, p.N, p.H, p.B, p.q_sn, p.q_sh, p.q_sb) ||
        !make_map(&P.tm_k, p.k, dt, p.N, p.H / p.kvg, p.B, p.k_sn, p.k_sh, p.k_sb) ||
        !make_map(&P.tm_v, p.v, dt, p.N, p.H / p.kvg, p.B, p.v_sn, p.v_sh, p.v_sb) ||
        !make_map(&P.tm_g, p.g, dt, p.N, p.H, p.B, p.g_sn, p.g_sh, p.g_sb) ||
        !make_map(&P.tm_dq, p.o, dt, p.N, p.H, p.B, p.o_sn, p.o_sh, p.o_sb) ||
        !make_map(&P.tm_dk, p.dk, dt, p.N, p.H, p.B, p.dk_sn, p.dk_sh, p.dk_sb) ||
        !make_map(&P.tm_dv, p.dv, dt, p.N, p.H, p.B, p.dv_sn, p.dv_sh, p.dv_sb) ||
        !make_map(&P.tm_fo, p.fo, dt, p.N, p.H, p.B, p.fo_sn, p.fo_sh, p.fo_sb))
        return cudaErrorInvalidValue;
    P.status = status_ptr();
    if (!P.status) return cudaErrorInvalidDevice;
    const int BH = p.B * p.H;
    P.nC = (p.N + kC - 1) / kC;
    const int G = fwd_segment_count(p);
    const HandLayout hl(BH, p.N, G, true);
    const char* base = reinterpret_cast<const char*>(p.seg_in);
    P.hdr = reinterpret_cast<const int*>(base);
    P.pl.off = reinterpret_cast<const int*>(base + hl.off);
    P.chunks = reinterpret_cast<const uint8_t*>(base + hl.chunks);
    P.zc = reinterpret_cast<const float*>(base + hl.zc);
    P.flags = hand_flags(kRev, kNorm, 0, true) | 0;
    P.pl.BH = BH;
    P.pl.R = bwd1_grid(p);
    P.pl.T = 0;  // read on the device: off[BH]
    // (the total number of live chunks is known on the device only: the
    // kernels read it from off[B*H])
    float* agg = p.ws;
    P.agg = agg;
    void* args_a[] = {&P, &agg};
    const void* ka = reinterpret_cast<const void*>(&adj_kernel<kFp16, kNorm, kRev>);
    const void* kb = reinterpret_cast<const void*>(&bwd1_kernel<kFp16, kNorm, kRev>);
    cudaError_t err = cudaFuncSetAttribute(ka, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(LA::total + 1024));
    if (err == cudaSuccess)
        err = cudaFuncSetAttribute(kb, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(L1::total + 1024));
    if (err == cudaSuccess)
        err = cudaLaunchKernel(ka, dim3(P.pl.R), dim3(kThreads1), args_a, LA::total + 1024, st);
    void* args_b[] = {&P};
    if (err == cudaSuccess) err = cudaLaunchKernel(kb, dim3(P.pl.R), dim3(kThreads1), args_b, L1::total + 1024, st);
    *launches = 2;
    return err;
}

}  // namespace
}  // namespace tcs
}  // namespace subq

namespace subq {
namespace tcs {

// CTAs of the one-pass backward: one per SM (each holds all of TMEM), at
// most one per chunk of the call.
int bwd1_grid(const ScanParams& p) {
    static int sms[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!sms[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        sms[dev] = n > 0 ? n : 1;
    }
    const int64_t chunks = (int64_t)p.B * p.H * ((p.N + kC - 1) / kC);
    return (int)std::max<int64_t>(1, std::min<int64_t>(sms[dev], chunks));
}

}  // namespace tcs

// The forward's output is read with 16-byte loads: aligned base and strides.
bool bwd1_usable(const ScanParams& p) {
    if (p.decay_mode != SUBQ_DECAY_NONE || !p.seg_in || !p.fo || (p.reverse && !p.normalize)) return false;
    return reinterpret_cast<uintptr_t>(p.fo) % 16 == 0 && p.fo_sb % 8 == 0 && p.fo_sh % 8 == 0 && p.fo_sn % 8 == 0;
}

// Bytes of workspace: the adjoint sums of each CTA's first piece.
size_t bwd1_workspace_bytes(const ScanParams& p) {
    return tcs::HandLayout::a256((size_t)tcs::bwd1_grid(p) * tcs::kD * (tcs::kD + 1) * sizeof(float));
}

cudaError_t launch_bwd1(const ScanParams& p, int dtype, cudaStream_t st, int* launches) {
    if (!bwd1_usable(p)) return cudaErrorInvalidValue;
    const bool f16 = dtype == SUBQ_FP16;
    if (p.reverse) {
        if (!p.normalize) return cudaErrorInvalidValue;
        return f16 ? tcs::launch1<true, true, true>(p, st, launches) : tcs::launch1<false, true, true>(p, st, launches);
    }
    if (p.normalize) return f16 ? tcs::launch1<true, true, false>(p, st, launches) : tcs::launch1<false, true, false>(p, st, launches);
    return f16 ? tcs::launch1<true, false, false>(p, st, launches) : tcs::launch1<false, false, false>(p, st, launches);
}

}  // namespace subq
