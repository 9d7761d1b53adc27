// Causal prefill attention on tcgen05, two instantiations of one kernel:
//  * prefill_core (benchmark configuration 3): already-prepared fp16 queries
//    q [T][24][256] against the fp16 caches [rows][4][256],
//    out [T][24][256] = softmax(q.k / 16 over cache rows [0, position + t]) v,
//    with fp16 probabilities and fp32 accumulation; the semantics of
//    tests/cpu_reference.py:72-88 (scores, softmax, P.V) over a causal block.
//  * prefill_precise (the attention layer's prefill regime, the reference's
//    attention_tiled, src/kernels.cu:459-503, whose scores and probabilities
//    are fp32): queries and probabilities are split into fp16 hi = fp16(x) and
//    lo = fp16(x - hi), and the lo halves extend the MMAs' reduction: the
//    scores are [Q_hi | Q_lo] . [K | K]^T and the output [P_hi | P_lo] . [V ; V],
//    the second half of each product issued as separate K=16 steps on the same
//    shared-memory K or V operand, so the fp32 accumulator of a row holds
//    (hi + lo) . K and scores and probabilities keep ~22 mantissa bits; the
//    output is multiplied by sigmoid(gate).
//
// One CTA per (128 queries, query head), 384 threads:
//  * warp 0: TMA producer. The CTA's query rows once (64 KB per fp16 half, four
//    128B-swizzled 64-dim column chunks each), then the K and V tiles of 128
//    keys as chunks into a ring of slots, in the order the MMA warp consumes
//    them: K0, K1, V0, K2, V1, ..., K(n-1), V(n-2), V(n-1). Plain: a chunk is a
//    whole 64 KB K or V tile (two slots); precise: half a tile, 32 KB (three
//    slots), a K chunk 128 keys x 128 dims, a V chunk 64 keys x 256 dims. The
//    MMA thread's per-chunk wait, fence and commit cost more than its MMAs at
//    16 KB chunks, hence the large ones.
//  * warp 1: MMA issuer. S_j = Q K_j^T as M=128 N=128 K=16 MMAs (16, or 32 in
//    the precise form) into one of two 128-column TMEM buffers, then
//    O += P_(j-1) V_(j-1) as M=128 N=256 MMAs (8, or 16) whose A operand, the
//    fp16 probabilities, is read from TMEM, where the softmax wrote them over
//    their own score tile. A 128-key tile keeps the QK instruction at N=128,
//    where tcgen05 runs at its full rate (N=64 issues at about two thirds of
//    it).
//  * warps 4-11: softmax, two warpgroups; thread = TMEM lane = query row,
//    warpgroup g takes keys [64g, 64g+64) of every tile. The row maximum is
//    agreed through shared memory once per tile, the O rescale is lazy (only
//    when the maximum grew by more than 2^8), and each warpgroup keeps its own
//    row sum. Epilogue: warpgroup g writes O columns [128g, 128g+128).
// TMEM: S buffers [0, 256), O [256, 512). A score buffer's probabilities take
// its columns [0, 64) (fp16 pairs), the precise form's lo halves [64, 128).
// Shared memory: Q 64 KB + a ring of two 64 KB slots, or Q hi + lo 128 KB + three
// 32 KB slots.
#include "common.cuh"
#include "hotpath.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdexcept>
#include <string>

namespace qv {

namespace {
constexpr int PF_NQ = 24, PF_NKV = 4, PF_HD = 256, PF_GROUP = PF_NQ / PF_NKV;
constexpr int PF_QROWS = 128;                  // queries per CTA
constexpr int PF_BN = 128;                     // keys per tile
constexpr int PF_QCHUNK = 16384;               // bytes per 64-dim query chunk [128 rows][128 B]
template <bool PRECISE>
struct PfLayout {
    static constexpr int CPT = PRECISE ? 2 : 1;                     // ring chunks per K or V tile
    static constexpr int CHUNK = 65536 / CPT;                       // bytes per ring slot
    static constexpr int SLOTS = PRECISE ? 3 : 2;                   // ring slots
    static constexpr int SM_Q = 0;                                  // 4 query chunks
    static constexpr int SM_QLO = SM_Q + 4 * PF_QCHUNK;             // precise: the lo halves, 4 chunks
    static constexpr int SM_RING = SM_Q + (PRECISE ? 8 : 4) * PF_QCHUNK;
    static constexpr int SM_XCH = SM_RING + SLOTS * CHUNK;          // [2 buffers][2 warpgroups][128 rows] floats
    static constexpr int SM_BAR = SM_XCH + 2 * 2 * 128 * 4;
    static constexpr int SMEM_BYTES = SM_BAR + 256;
    static_assert(SMEM_BYTES <= 227 * 1024, "prefill kernel exceeds the shared memory of a CTA");
    static_assert((2 * SLOTS + 11) * 8 <= 248, "mbarriers overlap the TMEM address slot");
};
constexpr uint32_t PF_TM_S = 0, PF_TM_O = 256;
constexpr uint32_t PF_TM_PLO = 64;             // lo probabilities within a score buffer
constexpr float PF_SCORE_LOG2 = 0.0625f * 1.4426950408889634f;   // (1/16) * log2(e)
constexpr float PF_RESCALE_THRESHOLD = 8.f;                      // lazy O rescale, log2 units
constexpr float PF_LN2 = 0.6931471805599453f;

struct PfParams {
    float *out;          // [T][24][256]
    float *lse;          // [T][24] natural-log LSE, or null
    const float *q_gate; // [T][24][512], gate = [256:512), or null (no gate)
    int T, position;     // tokens; cache row of token 0
    int kv_rows;         // valid cache rows (>= position + T)
};

__device__ __forceinline__ bool warp_wait_all(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
}

template <bool PRECISE>
__global__ void __launch_bounds__(384, 1)
prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmQlo,
               const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, const PfParams p) {
    using L = PfLayout<PRECISE>;
    constexpr int SLOTS = L::SLOTS, CPT = L::CPT, CHUNK = L::CHUNK;
    constexpr int DPC = PF_HD / CPT, KPC = PF_BN / CPT;          // K dims / V keys per chunk
    extern __shared__ __align__(1024) uint8_t smem[];
    if (smem_addr(smem) & 1023) {           // 128B-swizzle atoms need a 1024-byte aligned base
        if (threadIdx.x == 0) raise_status(STATUS_BAD_ARGUMENT);
        return;
    }
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::SM_BAR);
    uint64_t *full = bars, *empty = bars + SLOTS, *q_full = bars + 2 * SLOTS, *s_full = q_full + 1,
             *p_full = s_full + 2, *p_free = p_full + 2, *xbar = p_free + 2, *lbar = xbar + 2, *mma_done = lbar + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::SM_BAR + 248);      // after the mbarriers
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::SM_BAR + 252);
    float *xch = reinterpret_cast<float *>(smem + L::SM_XCH);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = blockIdx.x, kv_head = head / PF_GROUP;
    const int qtile = gridDim.y - 1 - blockIdx.y;                 // longest query tiles first
    const int tok0 = qtile * PF_QROWS;
    const int last_tok = min(p.T, tok0 + PF_QROWS) - 1;
    const int ntiles = (min(p.kv_rows, p.position + last_tok + 1) + PF_BN - 1) / PF_BN;

    if (threadIdx.x == 0) {
        for (int i = 0; i < SLOTS; ++i) { mbar_init(full + i, 1); mbar_init(empty + i, 1); }
        mbar_init(q_full, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(s_full + i, 1);
            mbar_init(p_full + i, 8);
            mbar_init(p_free + i, 1);
            mbar_init(xbar + i, 8);
        }
        mbar_init(lbar, 8);
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmQ);
        if (PRECISE) prefetch_tmap(&tmQlo);
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
    }
    if (warp == 1) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // L2 prefetch hints for the gate half-rows the epilogue multiplies by
    // (softmax thread = query row; its warpgroup's 128 gate values, 4 lines).
    if (warp >= 4 && p.q_gate && tok0 + (warp & 3) * 32 + lane < p.T) {
        const float *g = p.q_gate + ((size_t)(tok0 + (warp & 3) * 32 + lane) * PF_NQ + head) * 2 * PF_HD + PF_HD +
                         ((warp - 4) >> 2) * 128;
#pragma unroll
        for (int k = 0; k < 4; ++k) prefetch_l2(g + 32 * k);
    }

    // Everything below may read what the previous kernel of the stream wrote.
    grid_dependency_wait();
    if (threadIdx.x == 0) launch_dependents();

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            mbar_expect_tx(q_full, (PRECISE ? 8 : 4) * PF_QCHUNK);
            for (int c = 0; c < 4; ++c) {
                tma_load_2d(smem + L::SM_Q + c * PF_QCHUNK, &tmQ, q_full, head * PF_HD + c * 64, tok0);
                if (PRECISE)
                    tma_load_2d(smem + L::SM_QLO + c * PF_QCHUNK, &tmQlo, q_full, head * PF_HD + c * 64, tok0);
            }
            int seq = 0;
            bool ok = true;
            // Step s of the consumption order: s = 0 -> K0; s = 2i+1 -> K(i+1)
            // (or the last V when i+1 == ntiles); s = 2i+2 -> V(i).
            const int steps = 2 * ntiles;
            for (int s = 0; s < steps && ok; ++s) {
                bool is_k;
                int tile;
                if (s == 0) { is_k = true; tile = 0; }
                else if (s & 1) { tile = (s + 1) / 2; is_k = tile < ntiles; if (!is_k) tile = ntiles - 1; }
                else { is_k = false; tile = s / 2 - 1; }
                for (int c = 0; c < CPT && ok; ++c, ++seq) {
                    const int slot = seq % SLOTS;
                    if (seq >= SLOTS && !mbar_wait(empty + slot, ((seq / SLOTS) - 1) & 1, abort_flag)) { ok = false; break; }
                    uint8_t *dst = smem + L::SM_RING + slot * CHUNK;
                    mbar_expect_tx(full + slot, CHUNK);
                    if (is_k) {                 // dims [DPC c, DPC c + DPC) of the tile's 128 keys
#pragma unroll
                        for (int e = 0; e < DPC / 64; ++e)
                            tma_load_2d(dst + e * 16384, &tmK, full + slot, kv_head * PF_HD + c * DPC + e * 64, tile * PF_BN);
                    } else {                    // keys [KPC c, KPC c + KPC), all 256 dims
#pragma unroll
                        for (int d = 0; d < 4; ++d)
                            tma_load_2d(dst + d * KPC * 128, &tmV, full + slot, kv_head * PF_HD + d * 64, tile * PF_BN + c * KPC);
                    }
                }
            }
            // Drain: every issued load must land before the CTA may exit.
            const long long t0 = clock64();
            while (!mbar_try_wait(q_full, 0) && clock64() - t0 < WAIT_LIMIT_CYCLES) {}
            for (int i = max(0, seq - SLOTS); i < seq; ++i)
                while (!mbar_try_wait(full + i % SLOTS, (i / SLOTS) & 1) && clock64() - t0 < WAIT_LIMIT_CYCLES) {}
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc_qk = idesc_f16(128, PF_BN, false, false);
            constexpr uint32_t idesc_pv = idesc_f16(128, PF_HD, false, true);
            // Operand descriptors: the base ones once, then the 16-byte units of
            // an operand's offset added to the start-address field (shared
            // addresses stay below 256 KB, so the 14-bit field cannot carry).
            const uint64_t qd0 = sw128_desc(smem_addr(smem + L::SM_Q), 16, 1024);
            const uint64_t qld0 = sw128_desc(smem_addr(smem + L::SM_QLO), 16, 1024);
            const uint64_t kd0 = sw128_desc(smem_addr(smem + L::SM_RING), 16, 1024);
            const uint64_t vd0 = sw128_desc(smem_addr(smem + L::SM_RING), KPC * 128, 1024);
            int seq = 0;
            auto take = [&](int &slot) -> bool {
                slot = seq % SLOTS;
                if (!mbar_wait(full + slot, (seq / SLOTS) & 1, abort_flag)) return false;
                tc_fence_after();
                return true;
            };
            auto issue_pv = [&](int i) -> bool {
                const int b = i & 1;
                if (!mbar_wait(p_full + b, (i >> 1) & 1, abort_flag)) return false;
                tc_fence_after();
                const uint32_t pa = tmem + PF_TM_S + b * PF_BN;
                for (int c = 0; c < CPT; ++c) {
                    int slot;
                    if (!take(slot)) return false;
                    const uint64_t vb = vd0 + (uint64_t)(slot * (CHUNK >> 4));
#pragma unroll
                    for (int kk = 0; kk < KPC / 16; ++kk) {      // keys [KPC c + 16kk, +16)
                        const uint64_t vd = vb + (kk * 16 * 128 >> 4);
                        mma_f16_ts(tmem + PF_TM_O, pa + c * (KPC / 2) + kk * 8, vd, idesc_pv,
                                   (i > 0 || c > 0 || kk > 0) ? 1u : 0u);
                        if (PRECISE) mma_f16_ts(tmem + PF_TM_O, pa + PF_TM_PLO + c * (KPC / 2) + kk * 8, vd, idesc_pv, 1u);
                    }
                    mma_commit(empty + slot);
                    ++seq;
                }
                mma_commit(p_free + b);
                return true;
            };
            bool ok = mbar_wait(q_full, 0, abort_flag);
            tc_fence_after();
            for (int j = 0; j < ntiles && ok; ++j) {
                const int b = j & 1;
                // S buffer b last held tile j-2, whose probabilities PV(j-2)
                // (issued earlier by this thread, after the softmax released
                // them) reads before this QK overwrites them: MMAs issued by
                // one thread execute in order.
                for (int c = 0; c < CPT && ok; ++c) {
                    int slot;
                    if (!take(slot)) { ok = false; break; }
                    const uint64_t kb = kd0 + (uint64_t)(slot * (CHUNK >> 4));
#pragma unroll
                    for (int e = 0; e < DPC / 64; ++e) {       // dims [DPC c + 64e, +64): query chunk
                        const uint32_t qo = ((c * (DPC / 64) + e) * PF_QCHUNK) >> 4;
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            const uint64_t kd = kb + (uint64_t)((e * 16384) >> 4) + kk * 2;
                            mma_f16_ss(tmem + PF_TM_S + b * PF_BN, qd0 + (uint64_t)(qo + kk * 2), kd, idesc_qk,
                                       (c > 0 || e > 0 || kk > 0) ? 1u : 0u);
                            if (PRECISE)
                                mma_f16_ss(tmem + PF_TM_S + b * PF_BN, qld0 + (uint64_t)(qo + kk * 2), kd, idesc_qk, 1u);
                        }
                    }
                    mma_commit(empty + slot);
                    ++seq;
                }
                if (!ok) break;
                mma_commit(s_full + b);
                if (j >= 1) ok = issue_pv(j - 1);
            }
            if (ok && ntiles > 0) issue_pv(ntiles - 1);
            // All MMAs of this thread must finish before TMEM is released.
            mma_commit(mma_done);
            const long long t0 = clock64();
            while (!mbar_try_wait(mma_done, 0) && clock64() - t0 < WAIT_LIMIT_CYCLES) {}
        }
    } else if (warp >= 4) {
        // ------------------------------------------------ softmax + epilogue
        const int wq = warp & 3, wg = (warp - 4) >> 2;
        const uint32_t t_lane = tmem + ((uint32_t)(wq * 32) << 16);
        const int r = wq * 32 + lane, t = tok0 + r;
        const bool valid = t < p.T;
        const int pos_limit = valid ? min(p.position + t, p.kv_rows - 1) : -1;   // last visible cache row
        float m_use = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < ntiles; ++j) {
            const int b = j & 1;
            if (!warp_wait_all(s_full + b, (j >> 1) & 1, abort_flag)) { ok = false; break; }
            tc_fence_after();
            float x[64];
#pragma unroll
            for (int c = 0; c < 4; ++c)
                tmem_ld16(t_lane + PF_TM_S + b * PF_BN + wg * 64 + c * 16, *reinterpret_cast<float(*)[16]>(x + c * 16));
            tmem_wait_ld();
            const int lim = pos_limit - (j * PF_BN + wg * 64);         // columns <= lim are visible
            if (__any_sync(0xffffffffu, lim < 63)) {
#pragma unroll
                for (int c = 0; c < 64; ++c) x[c] = c <= lim ? x[c] : -INFINITY;
            }
            float mp[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) mp[q] = -INFINITY;
#pragma unroll
            for (int c = 0; c < 64; ++c) mp[c & 7] = fmaxf(mp[c & 7], x[c]);
            float m_tile = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                                 fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
            // The two warpgroups agree on the row maximum; passing this
            // exchange also means both have read their score columns, so the
            // probabilities may then be written over them.
            xch[(b * 2 + wg) * 128 + r] = m_tile;
            __syncwarp();
            if (lane == 0) mbar_arrive(xbar + b);
            if (!warp_wait_all(xbar + b, (j >> 1) & 1, abort_flag)) { ok = false; break; }
            m_tile = fmaxf(m_tile, xch[(b * 2 + (wg ^ 1)) * 128 + r]) * PF_SCORE_LOG2;   // log2 units
            float factor = 1.f;
            const bool need = m_tile > m_use + PF_RESCALE_THRESHOLD;
            if (need) { factor = exp2_approx(m_use - m_tile); m_use = m_tile; l *= factor; }
            if (j > 0 && __any_sync(0xffffffffu, need)) {
                // O holds tiles < j: wait for PV(j-1), then rescale this
                // warpgroup's 128 columns of the rows in TMEM.
                if (!warp_wait_all(p_free + ((j - 1) & 1), ((j - 1) >> 1) & 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
#pragma unroll 1
                for (int c = wg * 8; c < wg * 8 + 8; ++c) {
                    float o[16];
                    tmem_ld16(t_lane + PF_TM_O + c * 16, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 16; ++e) o[e] *= factor;
                    tmem_st16(t_lane + PF_TM_O + c * 16, o);
                }
                tmem_wait_st();
            }
            const float mref = m_use == -INFINITY ? 0.f : m_use;
            // fp16 probabilities of keys [64 wg, 64 wg + 64) as 32 half2 words
            // (precise: hi = fp16(p) and lo = fp16(p - hi)).
            uint32_t hp[32], lp[PRECISE ? 32 : 1];
            float sp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < 64; c += 2) {
                const float p0 = exp2_approx(fmaf(x[c], PF_SCORE_LOG2, -mref));
                const float p1 = exp2_approx(fmaf(x[c + 1], PF_SCORE_LOG2, -mref));
                const __half2 h2 = __floats2half2_rn(p0, p1);
                hp[c / 2] = *reinterpret_cast<const uint32_t *>(&h2);
                if (PRECISE) {
                    const float2 back = __half22float2(h2);
                    const __half2 l2 = __floats2half2_rn(p0 - back.x, p1 - back.y);
                    lp[c / 2] = *reinterpret_cast<const uint32_t *>(&l2);
                }
                sp[(c >> 1) & 3] += p0 + p1;
            }
            l += (sp[0] + sp[1]) + (sp[2] + sp[3]);
            // P of keys [64 wg, 64 wg + 64) into TMEM columns [32 wg, 32 wg + 32)
            // of this S buffer, the lo halves 64 columns further.
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                tmem_st16(t_lane + PF_TM_S + b * PF_BN + wg * 32 + c * 16, *reinterpret_cast<const float(*)[16]>(hp + c * 16));
                if (PRECISE)
                    tmem_st16(t_lane + PF_TM_S + b * PF_BN + PF_TM_PLO + wg * 32 + c * 16,
                              *reinterpret_cast<const float(*)[16]>(lp + c * 16));
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full + b);
        }
        // Row sums of both warpgroups, through the exchange buffer no tile still reads.
        float *lx = xch + (ntiles & 1) * 256;
        if (ok) {
            lx[wg * 128 + r] = l;
            __syncwarp();
            if (lane == 0) mbar_arrive(lbar);
            ok = warp_wait_all(lbar, 0, abort_flag);
        }
        // Epilogue: the final PV's commit on p_free marks O complete (and every
        // MMA and K/V chunk done, so the query buffers and the ring are idle).
        // O leaves through shared memory: each lane puts its 128 columns into a
        // padded staging row, then the warp stores each row's 512 bytes at
        // once, divided by the row sum and, with a gate, times sigmoid(gate).
        if (ok && ntiles > 0 &&
            warp_wait_all(p_free + ((ntiles - 1) & 1), ((ntiles - 1) >> 1) & 1, abort_flag)) {
            tc_fence_after();
            if (valid && wg == 0 && p.lse) {
                const float lt = lx[r] + lx[128 + r];
                p.lse[(size_t)t * PF_NQ + head] = lt > 0.f ? (m_use + log2f(lt)) * PF_LN2 : -INFINITY;
            }
            constexpr int RS = 128 * 4 + 16;                            // staging row bytes (padded)
            static_assert(8 * 32 * RS <= L::SM_XCH, "O staging exceeds the query buffers and the ring");
            uint8_t *stage = smem + (warp - 4) * 32 * RS;
            uint8_t *myrow = stage + lane * RS;
#pragma unroll
            for (int c4 = 0; c4 < 2; ++c4) {
                float o[4][16];
#pragma unroll
                for (int q = 0; q < 4; ++q) tmem_ld16(t_lane + PF_TM_O + wg * 128 + c4 * 64 + q * 16, o[q]);
                tmem_wait_ld();
#pragma unroll
                for (int q = 0; q < 4; ++q)
#pragma unroll
                    for (int e = 0; e < 16; e += 4)
                        *reinterpret_cast<float4 *>(myrow + (c4 * 64 + q * 16 + e) * 4) =
                            make_float4(o[q][e], o[q][e + 1], o[q][e + 2], o[q][e + 3]);
            }
            __syncwarp();
            const int row0 = wq * 32;
            const int nvalid = max(0, min(32, p.T - tok0 - row0));      // valid rows are a prefix
            // Sixteen rows at a time, their gate values loaded before any of their
            // stores (a load the compiler cannot move above an earlier store
            // would otherwise cost one memory latency per row); sigmoid with the
            // SFU's 2^x and reciprocal (a few float ulp).
            constexpr int RB = 16;
            for (int i0 = 0; i0 < nvalid; i0 += RB) {
                float4 g[RB];
                if (p.q_gate) {
#pragma unroll
                    for (int k = 0; k < RB; ++k)
                        g[k] = i0 + k < nvalid ? *reinterpret_cast<const float4 *>(
                                                     p.q_gate + ((size_t)(tok0 + row0 + i0 + k) * PF_NQ + head) * 2 * PF_HD +
                                                     PF_HD + wg * 128 + 4 * lane)
                                               : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int k = 0; k < RB; ++k) {
                    const int i = i0 + k;
                    if (i >= nvalid) break;
                    const float lt = lx[row0 + i] + lx[128 + row0 + i];
                    const float inv = lt > 0.f ? 1.f / lt : 0.f;
                    float4 v = *reinterpret_cast<const float4 *>(stage + i * RS + lane * 16);
                    v.x *= inv; v.y *= inv; v.z *= inv; v.w *= inv;
                    if (p.q_gate) {
                        v.x *= sigmoid_fast(g[k].x); v.y *= sigmoid_fast(g[k].y);
                        v.z *= sigmoid_fast(g[k].z); v.w *= sigmoid_fast(g[k].w);
                    }
                    float *dst = p.out + ((size_t)(tok0 + row0 + i) * PF_NQ + head) * PF_HD + wg * 128;
                    *reinterpret_cast<float4 *>(dst + 4 * lane) = v;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

// 2-D fp16 map [rows][width] with 64-element x 'box_rows' boxes, 128B swizzle.
CUtensorMap pf_map(const void *base, int width, int rows, int box_rows) {
    CUtensorMap m;
    cuuint64_t dims[2] = {(cuuint64_t)width, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)width * sizeof(__half)};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims,
                                            strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return m;
}

PerDeviceOnce g_prefill_configured;

template <bool PRECISE>
void launch_prefill(float *out, float *lse, const float *q_gate, const __half *q, const __half *q_lo,
                    const __half *kc, const __half *vc, int T, int position, int kv_rows, cudaStream_t st) {
    g_prefill_configured.run([] {
        if (cudaFuncSetAttribute(prefill_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 PfLayout<false>::SMEM_BYTES) != cudaSuccess ||
            cudaFuncSetAttribute(prefill_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 PfLayout<true>::SMEM_BYTES) != cudaSuccess)
            throw std::runtime_error("cannot reserve shared memory for the prefill kernel");
    });
    if (T <= 0) return;
    const CUtensorMap mq = pf_map(q, PF_NQ * PF_HD, T, PF_QROWS);
    const CUtensorMap mql = PRECISE ? pf_map(q_lo, PF_NQ * PF_HD, T, PF_QROWS) : mq;
    const CUtensorMap mk = pf_map(kc, PF_NKV * PF_HD, kv_rows, PF_BN);
    const CUtensorMap mv = pf_map(vc, PF_NKV * PF_HD, kv_rows, PF_BN / PfLayout<PRECISE>::CPT);
    PfParams p{out, lse, q_gate, T, position, kv_rows};
    const cudaError_t e = launch_chained(prefill_kernel<PRECISE>, dim3(PF_NQ, (T + PF_QROWS - 1) / PF_QROWS),
                                         dim3(384), PfLayout<PRECISE>::SMEM_BYTES, st, mq, mql, mk, mv, p);
    if (e != cudaSuccess) throw std::runtime_error(std::string("prefill attention launch: ") + cudaGetErrorString(e));
}
}  // namespace

// Core-level causal prefill on already-prepared fp16 queries (no norm, RoPE
// or gate): out [T][24][256] = softmax(q.k/16, causal) v, optional LSE.
void prefill_core(float *out, float *lse, const __half *q, const __half *kc, const __half *vc, int T,
                  int position, cudaStream_t st) {
    launch_prefill<false>(out, lse, nullptr, q, nullptr, kc, vc, T, position, position + T, st);
}

// The attention layer's prefill after its prepare step: queries as fp16 hi /
// lo rows [T][24][256], cache rows [0, kv_rows) with token t seeing rows
// [0, position + t] (position = cache row of token 0), out = the normalised
// rows times sigmoid(gate) when q_gate is given.
void prefill_precise(float *out, const __half *q, const __half *q_lo, const float *q_gate, const __half *kc,
                     const __half *vc, int T, int position, int kv_rows, cudaStream_t st) {
    launch_prefill<true>(out, nullptr, q_gate, q, q_lo, kc, vc, T, position, kv_rows, st);
}

}  // namespace qv
