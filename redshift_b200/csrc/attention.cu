// Full-attention hot path for sm_100a: the decode/verify kernel (split-KV, all
// 6 GQA heads x T tokens of one KV head share every K/V tile, the prepare step
// of RMSNorm + partial RoPE + fp16 KV append folded in, the split combine or
// the peer exchange in its tail), the prepare kernel of the prefill regime
// (whose attention is prefill.cu's precise instantiation), and the shard
// merge kernel.
//
// Semantics follow the reference's attn_prepare / attention / attention_tiled
// (src/kernels.cu:415-503) and the CPU oracle tests/cpu_reference.py:55-89:
// scores q.k/16 over cache rows [0, position+t], softmax, P.V, times
// sigmoid(gate).
//
// Precision: 64 logical query rows per CTA.  Q is split into fp16 hi and
//    lo = fp16(q - hi) and the QK MMA's A operand (held in TMEM) interleaves them: A row 32w+i = Q_hi and
//    32w+16+i = Q_lo of query row 16w+i, so one M=128 MMA leaves both score
//    halves of a row in lanes i and i+16 of warp w, which add them while they
//    split the row's columns.  Every probability p is split the same way; the
//    PV MMA's A rows 32w+i / 32w+16+i are P_hi / P_lo of row 16w+i, so O_hi and
//    O_lo land in the same warp and are summed in the epilogue.  Scores and
//    probabilities keep ~22 mantissa bits (the reference computes them in fp32).
#include "common.cuh"
#include "hotpath.h"

#include <algorithm>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdexcept>
#include <string>

namespace qv {

constexpr int NQ = 24, NKV = 4, HD = 256, GROUP = NQ / NKV;
constexpr int BN = 64;           // cache positions per K/V tile
constexpr int TILE_BYTES = 4 * BN * 128;                      // one K or V tile, 4 boxes of 64 rows x 128 B
constexpr int DECODE_ROWS = 64;                               // logical rows of a decode CTA
constexpr float SCORE_LOG2 = 0.0625f * 1.4426950408889634f;   // (1/16) * log2(e)
constexpr float RESCALE_THRESHOLD = 8.f;                      // lazy O rescale, log2 units

constexpr int STAGES3 = 3;       // K/V tile ring depth
constexpr int MAX_DECODE_T = DECODE_ROWS / GROUP;             // largest decode / verify batch (10)
struct FaLayout {
    static constexpr int SM_KV = 0;                           // ring of (K tile, V tile)
    static constexpr int SM_KV_STAGE = 2 * TILE_BYTES;
    static constexpr int SM_P = SM_KV + STAGES3 * SM_KV_STAGE; // 2 x [128 A-rows][64 pos] fp16
    static constexpr int SM_BAR = SM_P + 2 * 128 * 128;       // mbarriers, TMEM address, abort flag
    static constexpr int SM_ROPE = SM_BAR + 256;              // decode: (cos, sin) [T][32]
    static constexpr int SMEM_BYTES = SM_ROPE + MAX_DECODE_T * 32 * 8;
};
static_assert(FaLayout::SMEM_BYTES <= 227 * 1024, "attention kernel exceeds the shared memory of a CTA");

// Rotary inverse frequencies 1e7^(-i/32), i = 0..31, as exact doubles (the
// values Python's 10000000 ** (-i / 32) yields).
__constant__ double kRopeInvFreq[32] = {
    0x1.0000000000000p+0,  0x1.3566562253c7ep-1, 0x1.75f034d79e965p-2, 0x1.c3f06b4e265cep-3,
    0x1.111aedafb9a9dp-3,  0x1.4a12ad8379eb8p-4, 0x1.8eec7def5d56cp-5, 0x1.e222ec75094e2p-6,
    0x1.235a71c5ee5ccp-6,  0x1.6020a364b1284p-7, 0x1.a99428b3d26b3p-8, 0x1.012cfaad0da13p-8,
    0x1.36d219065ac0cp-9,  0x1.77a7d87ee61b0p-10, 0x1.c603c39630446p-11, 0x1.125c04ab2d71fp-11,
    0x1.4b96be9c2da2cp-12, 0x1.90c181b38fe22p-13, 0x1.e459c57e28a47p-14, 0x1.24b0fd0e890d4p-14,
    0x1.61bea2721385fp-15, 0x1.ab88830de4ad5p-16, 0x1.025b57369650bp-16, 0x1.383f8796f72a9p-17,
    0x1.7961810874a9fp-18, 0x1.c8198c91f9fccp-19, 0x1.139e9527f964ep-19, 0x1.4d1c97f4e952fp-20,
    0x1.9298ace36f12ep-21, 0x1.e69338f8adcd3p-22, 0x1.26091b11c8665p-22, 0x1.635e883bbc816p-23,
};

// (cos, sin) of the rotary angle pos * 1e7^(-i/32).  The angle is formed in
// double precision (it reaches ~1.4e5 rad, where float would lose ~1e-2 rad)
// and reduced by 2*pi with a two-part Cody-Waite split (a 33-bit head, so
// k * head is exact for |k| < 2^20, and a tail); the reduced |x| <= pi is then
// rounded to float and evaluated with single-precision sincosf, within a few
// float ulps of cos / sin of the double angle.
__device__ __forceinline__ float2 rope_angle(int pos, int i) {
    const double theta = (double)pos * kRopeInvFreq[i];
    const double k = rint(theta * 0.15915494309189535);          // 1 / (2 pi)
    const double x = fma(-k, 0x1.0b4611a626331p-32, fma(-k, 0x1.921fb54400000p+2, theta));
    float sf, cf;
    sincosf((float)x, &sf, &cf);
    return make_float2(cf, sf);
}

// Rotary embedding of one 256-wide row spread over a warp, lane l holding
// dims [4l, 4l+4) in v (dims [0,64) live in lanes 0..15): pairs (i, i+32),
// i < 32, rotate by the angle whose (cos, sin) is cs[i].
// Branch-free, so that consecutive rows interleave: lanes that do not
// rotate use the identity (cos 1, sin 0).
__device__ __forceinline__ void rope_row(float (&v)[4], const float2 *cs, int lane, bool apply) {
    const bool rot = apply && lane < 16;
    const float sign = lane < 8 ? -1.f : 1.f;      // lane < 8: a*c - b*s;  8..15: b*c + a*s
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float partner = __shfl_xor_sync(0xffffffffu, v[e], 8);
        const float2 r = cs[4 * (lane & 7) + e];
        const float c = rot ? r.x : 1.f, sn = rot ? sign * r.y : 0.f;
        v[e] = fmaf(partner, sn, v[e] * c);
    }
}
__device__ __forceinline__ uint32_t half2_bits(__half2 h) { return *reinterpret_cast<const uint32_t *>(&h); }
// TMEM columns: S double buffer [0,128), O [128,384), Q (A operand) [384,512).
constexpr uint32_t TM_S = 0, TM_O = 128, TM_Q = 384;

// What a decode launch does with its rows once every split is done (the
// kernel tail, after a barrier over the CTAs of each KV head).
enum DecodeTail : int {
    TAIL_GATED = 0,      // out = softmax(...) V * sigmoid(gate)
    TAIL_SHARD = 1,      // out = normalised partial of this cache shard, lse = its natural-log LSE
    TAIL_EXCHANGE = 2,   // shard partial pushed to every rank's buffer, all ranks' partials merged, gated
};

struct FaParams {
    const float *q_gate;    // [T][24][512]: q = [0:256), gate = [256:512)
    float *out;             // [T][24][256]
    float *lse;             // natural-log LSE [T][24] (TAIL_SHARD)
    float *part_o;          // [4][64 rows][splits][256] unnormalised partial O of every split
    float *part_ml;         // [4][64 rows][MAXS][2] (running max in log2 units, sum)
    unsigned long long *sync;  // [4] per-KV-head barrier words (generation : arrivals)
    int T, position;        // tokens and absolute position of token 0
    int kv_begin;           // absolute position of cache row 0
    int kv_rows;            // valid cache rows
    int split_tiles, splits;
    int tail;               // DecodeTail
    const uint64_t *peers;  // TAIL_EXCHANGE: every rank's receive buffer
    int world, rank, seq;
    // The prepare step folded in: the CTA normalises and rotates its own query
    // rows from q_gate and, when its tiles hold the block's new cache rows,
    // writes their keys / values before loading them.
    const float *key, *value, *qn, *kn;
    __half *kc, *vc;        // the caches, for the append
    int append_row0;        // local cache row of token 0's key / value, or -1
    float eps;
};

// Logical query row -> (token, head): the rows of a CTA pack the 6 query heads
// of its KV head (blockIdx.y) and the T tokens.
__device__ __forceinline__ bool row_token_head(const FaParams &p, int r, int &t, int &h) {
    t = r / GROUP;
    h = blockIdx.y * GROUP + r % GROUP;
    return r < p.T * GROUP;
}

// Warp-uniform bounded wait (all lanes agree on the outcome).
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
}

// ---------------------------------------------------------------- decode tail
// After its split of the cache, a decode CTA waits at a barrier over the CTAs
// of its KV head, then combines a share of the head's rows from all splits'
// partials (rows blockIdx.x, blockIdx.x + splits, ...): the split combine
// runs inside the attention launch, on every SM, with no second kernel.
constexpr float LN2 = 0.6931471805599453f;
constexpr int MAXS = 40;                               // splits a tail combine handles (plans use <= 37)

// Peer exchange (TAIL_EXCHANGE, multi-GPU verify).  Each rank's receive
// buffer holds [2 slots][world][EX_ROWS][EX_WORDS] 64-bit words (256 O, lse,
// padding) per row t*24 + h.  Every value travels as a word {value bits,
// tag}: the reader spins on each of its words until the tag of this call
// appears, so no fence or separate flag write is needed, and it zeroes each
// word after reading it.  `seq` counts the calls on these buffers (the same
// on every rank, +1 per call): its parity picks the slot and its low 24 bits
// are in the tag.  A rank writes into a slot again two calls later, after it
// has received this rank's partials of the call in between, and that call
// started only after this one (and its zeroing) completed.  A word that
// arrives after its reader gave up (a timeout) stays behind unread, but it
// carries the tag of its own call and the next call on that slot waits for a
// different tag, so it is never taken for new data.
constexpr int EX_ROWS = MAX_DECODE_T * NQ;       // rows of the largest decode batch
constexpr int EX_WORDS = 264;                    // words per row: 256 O + lse, padded to 64 bytes
constexpr int EX_MAX_WORLD = 8;
__host__ __device__ constexpr uint32_t ex_tag(int seq) {   // high half of a filled word; never 0
    return 0x51000000u | ((uint32_t)seq & 0x00FFFFFFu);
}
__host__ __device__ constexpr size_t ex_bytes(int world) {
    return (size_t)2 * world * EX_ROWS * EX_WORDS * sizeof(uint64_t);
}

// Barrier over the `splits` CTAs of one KV head, on one 64-bit word of the
// workspace: arrivals in the low half, a generation count in the high half.
// The arrivals must be zero before the first launch on a workspace.  A CTA
// waits until the arrivals reach `splits` or the generation moves on; the
// last CTA to arrive then resets the arrivals and advances the generation in
// one atomic add (off the others' critical path: they may leave as soon as
// its arrival shows), so every launch leaves the arrivals zero, also after a
// timeout (every CTA arrives; only a waiter gives up).  A launch has at most
// (SMs / 4) CTAs per head and one CTA per SM, so all CTAs of a head are
// resident together.  Bounded: a wait past the limit raises STATUS_TIMEOUT.
__device__ bool head_barrier(unsigned long long *word, int splits, volatile int *flag) {
    fence_async_global();                              // the partials are read back by bulk copies
    __syncthreads();                                   // this CTA's partials are written
    if (threadIdx.x == 0) {
        __threadfence();                               // release them
        const unsigned long long old = atomicAdd(word, 1ull);
        bool ok = true;
        if ((uint32_t)old == (uint32_t)splits - 1) {
            atomicAdd(word, (1ull << 32) - (unsigned long long)splits);   // arrivals -> 0, generation + 1
        } else {
            const uint32_t gen = (uint32_t)(old >> 32);
            const long long start = clock64();
            while (true) {
                const unsigned long long v = ld_acquire_gpu_u64(word);
                if ((uint32_t)v >= (uint32_t)splits || (uint32_t)(v >> 32) != gen) break;
                if (clock64() - start > WAIT_LIMIT_CYCLES) { raise_status(STATUS_TIMEOUT); ok = false; break; }
            }
        }
        __threadfence();                               // acquire the other CTAs' partials
        *flag = ok ? 1 : 0;
    }
    __syncthreads();
    return *flag != 0;
}

// Bulk copy global -> shared (no tensor map), completion on the mbarrier's
// transaction count: addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)) : "memory");
}

// Split combine of decode rows ra and rb (rb < 0: ra only) of KV head g (row r
// = token r / 6, head 6g + r % 6).  A row's partials of all splits are one
// contiguous block (splits x 1 KB), and so are its splits' (max, sum) pairs
// (MAXS x 8 bytes): thread 0 brings both rows' blocks into shared memory
// (`buf`, the idle K/V ring) with bulk copies on `bar` (phase parity
// `phase`).  o[k] receives the normalised value of row k in dimension
// threadIdx.x, lse[k] its natural-log LSE.  `sh` holds 1280 floats of shared
// memory (weights and maxima in the first 2 MAXS + 8, the exchange's words
// after them, the rows' halves from float 256 on); the call ends with a CTA
// barrier.
__device__ bool combine_rows(const FaParams &p, int g, int ra, int rb, float *sh, float *buf, uint64_t *bar,
                             uint32_t phase, volatile int *abort_flag, float (&o)[2], float (&lse)[2]) {
    const int d = threadIdx.x, S = p.splits;
    const bool two = rb >= 0;
    const size_t row_a = (size_t)g * DECODE_ROWS + ra, row_b = (size_t)g * DECODE_ROWS + (two ? rb : ra);
    float *xa = buf, *xb = buf + (size_t)S * HD;                    // partials [split][256]
    float *mla = buf + 2 * (size_t)S * HD, *mlb = mla + 2 * MAXS;   // (max, sum) [MAXS][2]
    if (threadIdx.x == 0) {
        // The partials were written through the generic proxy (and acquired
        // at the barrier); the bulk copies read them through the async proxy,
        // and overwrite shared memory the CTA last used through the generic one.
        fence_async_global();
        fence_async_shared();
        const uint32_t bytes = (uint32_t)S * HD * sizeof(float), ml_bytes = 2 * MAXS * sizeof(float);
        mbar_expect_tx(bar, two ? 2 * (bytes + ml_bytes) : bytes + ml_bytes);
        bulk_load(xa, p.part_o + row_a * S * HD, bytes, bar);
        bulk_load(mla, p.part_ml + row_a * 2 * MAXS, ml_bytes, bar);
        if (two) {
            bulk_load(xb, p.part_o + row_b * S * HD, bytes, bar);
            bulk_load(mlb, p.part_ml + row_b * 2 * MAXS, ml_bytes, bar);
        }
    }
    const bool ok = mbar_wait(bar, phase, abort_flag);
    if (threadIdx.x == 0 && phase == 0) QV_STAMP(14);
    // (max, sum) of split e of row a on threads [0, S), of row b on [64, 64 + S)
    const int e = d < 64 ? d : d - 64;
    float m = -INFINITY, l = 0.f;
    if (ok && e < S && (d < 64 || (two && d < 128))) {
        const float *ml = d < 64 ? mla : mlb;
        m = ml[2 * e]; l = ml[2 * e + 1];
    }
    float *wa = sh, *wb = sh + MAXS, *red = sh + 2 * MAXS;   // red: maxima [0..3], sums [4..7]
    float M = m;
#pragma unroll
    for (int k = 16; k; k >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, k));
    if (d < 128 && (d & 31) == 0) red[d >> 5] = M;
    __syncthreads();
    const float Ma = fmaxf(red[0], red[1]), Mb = fmaxf(red[2], red[3]);
    const float w = (e < S && d < 128 && m != -INFINITY) ? exp2f(m - (d < 64 ? Ma : Mb)) : 0.f;
    if (d < MAXS) wa[d] = w;
    else if (d >= 64 && d < 64 + MAXS) wb[d - 64] = w;
    const float den_part = warp_sum(w * l);
    if (d < 128 && (d & 31) == 0) red[4 + (d >> 5)] = den_part;
    __syncthreads();
    const float den_a = red[4] + red[5], den_b = red[6] + red[7];
    // The weighted sum over the splits: thread (row, half, quad) reads four
    // dimensions of its row with 16-byte loads over half of the splits; the
    // two halves meet in shared memory.
    const int rsel = d >> 7, hsel = (d >> 6) & 1, quad = d & 63;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ok && (rsel == 0 || two)) {
        const float *x = rsel ? xb : xa, *w = rsel ? wb : wa;
        const int k0 = hsel ? S / 2 : 0, k1 = hsel ? S : S / 2;
        for (int k = k0; k < k1; ++k) {
            const float4 v = *reinterpret_cast<const float4 *>(x + (size_t)k * HD + 4 * quad);
            const float wk = w[k];
            acc.x = fmaf(wk, v.x, acc.x); acc.y = fmaf(wk, v.y, acc.y);
            acc.z = fmaf(wk, v.z, acc.z); acc.w = fmaf(wk, v.w, acc.w);
        }
    }
    float4 *part = reinterpret_cast<float4 *>(sh + 768);   // [2 rows][64 quads], the second halves
    float *res = sh + 256;                                   // [2 rows][256], the normalised rows
    if (hsel) part[rsel * 64 + quad] = acc;
    __syncthreads();
    if (!hsel) {
        const float4 b = part[rsel * 64 + quad];
        const float den = rsel ? den_b : den_a, inv = den > 0.f ? 1.f / den : 0.f;
        *reinterpret_cast<float4 *>(res + rsel * HD + 4 * quad) =
            make_float4((acc.x + b.x) * inv, (acc.y + b.y) * inv, (acc.z + b.z) * inv, (acc.w + b.w) * inv);
    }
    __syncthreads();
    o[0] = res[d];
    o[1] = res[HD + d];
    lse[0] = den_a > 0.f ? (Ma + log2f(den_a)) * LN2 : -INFINITY;
    lse[1] = den_b > 0.f ? (Mb + log2f(den_b)) * LN2 : -INFINITY;
    __syncthreads();                                   // sh and buf are free again
    return ok;
}

// Peer exchange of up to two rows (global row indices grow[k] = t*24 + h, k <
// nr): this shard's normalised values o[k] (dimension threadIdx.x) and LSEs go
// into slot [rank] of every other rank's buffer, then the other ranks' words
// of the rows are read from this rank's own buffer (all peers and both rows
// at once, so their latencies overlap; a word without this call's tag is
// re-read until it has it, bounded) and merged: sum_g exp(lse_g - LSE) o_g,
// written back into o[k].  `sh` holds 2 EX_MAX_WORLD floats; the call ends
// with a CTA barrier.
__device__ void exchange_rows(const FaParams &p, const int (&grow)[2], int nr, float (&o)[2], const float (&lse)[2],
                              float *sh) {
    const int d = threadIdx.x, world = p.world, rank = p.rank, slot = p.seq & 1;
    const uint32_t tag32 = ex_tag(p.seq);
    const uint64_t tag = (uint64_t)tag32 << 32;
    for (int k = 0; k < nr; ++k)
        for (int q = 0; q < world; ++q) {
            if (q == rank) continue;
            uint64_t *dst = reinterpret_cast<uint64_t *>(p.peers[q]) +
                            (((size_t)slot * world + rank) * EX_ROWS + grow[k]) * EX_WORDS;
            st_word_sys(dst + d, tag | __float_as_uint(o[k]));
            if (d == 0) st_word_sys(dst + HD, tag | __float_as_uint(lse[k]));
        }
    uint64_t *own = reinterpret_cast<uint64_t *>(p.peers[rank]);
    auto word_of = [&](int q, int k, int col) {
        return own + (((size_t)slot * world + q) * EX_ROWS + grow[k]) * EX_WORDS + col;
    };
    // Every word this thread needs (its dimension of the other ranks' rows, and
    // on threads 32k + q the LSE of rank q's row k) is re-read together until all
    // carry this call's tag, so the waits for the peers overlap: one round trip
    // per pass, not one per word.
    const int lk = d >> 5, lq = d & 31;
    const bool lse_reader = lk < nr && lq < world && lq != rank;
    uint64_t w[2][EX_MAX_WORLD], wl = lse_reader ? ld_word_sys(word_of(lq, lk, HD)) : 0;
#pragma unroll
    for (int k = 0; k < 2; ++k)
#pragma unroll
        for (int q = 0; q < EX_MAX_WORLD; ++q)
            w[k][q] = (k < nr && q < world && q != rank) ? ld_word_sys(word_of(q, k, d)) : ((uint64_t)tag32 << 32);
    const long long t0 = clock64();
    bool ok = true;
    while (true) {
        bool ready = !lse_reader || (uint32_t)(wl >> 32) == tag32;
#pragma unroll
        for (int k = 0; k < 2; ++k)
#pragma unroll
            for (int q = 0; q < EX_MAX_WORLD; ++q) ready = ready && (uint32_t)(w[k][q] >> 32) == tag32;
        if (ready) break;
        if (clock64() - t0 > WAIT_LIMIT_CYCLES) { raise_status(STATUS_TIMEOUT); ok = false; break; }
        if (lse_reader && (uint32_t)(wl >> 32) != tag32) wl = ld_word_sys(word_of(lq, lk, HD));
#pragma unroll
        for (int k = 0; k < 2; ++k)
#pragma unroll
            for (int q = 0; q < EX_MAX_WORLD; ++q)
                if (k < nr && q < world && q != rank && (uint32_t)(w[k][q] >> 32) != tag32) w[k][q] = ld_word_sys(word_of(q, k, d));
    }
    // read words are cleared (a late word of a timed-out call keeps its own tag)
    if (ok) {
        if (lse_reader) *word_of(lq, lk, HD) = 0;
#pragma unroll
        for (int k = 0; k < 2; ++k)
#pragma unroll
            for (int q = 0; q < EX_MAX_WORLD; ++q)
                if (k < nr && q < world && q != rank) *word_of(q, k, d) = 0;
    }
    if (lk < nr && lq < world) sh[lk * EX_MAX_WORLD + lq] = lse_reader ? (ok ? __uint_as_float((uint32_t)wl) : 0.f) : lse[lk];
    float val[2][EX_MAX_WORLD];
#pragma unroll
    for (int k = 0; k < 2; ++k)
#pragma unroll
        for (int q = 0; q < EX_MAX_WORLD; ++q) {
            val[k][q] = 0.f;
            if (k < nr && q < world) val[k][q] = q == rank ? o[k] : (ok ? __uint_as_float((uint32_t)w[k][q]) : 0.f);
        }
    const int all_ok = __syncthreads_and(ok);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        float res = 0.f;
        if (all_ok && k < nr) {
            const float *ls = sh + k * EX_MAX_WORLD;
            float Mx = -INFINITY;
            for (int q = 0; q < world; ++q) Mx = fmaxf(Mx, ls[q]);
            float num = 0.f, den = 0.f;
            if (Mx != -INFINITY) {
#pragma unroll
                for (int q = 0; q < EX_MAX_WORLD; ++q) {
                    if (q >= world || ls[q] == -INFINITY) continue;
                    const float wq = expf(ls[q] - Mx);
                    den += wq;
                    num += wq * val[k][q];
                }
            }
            res = den > 0.f ? num / den : 0.f;
        }
        o[k] = res;
    }
    __syncthreads();                                   // sh is free again
}

// The decode tail of one CTA (all 256 threads): barrier over the KV head,
// then this CTA's rows of the head (blockIdx.x, blockIdx.x + splits, ...),
// two at a time, combined and written as p.tail says.  `scratch` is a little
// shared memory, `buf` room for two rows' partials of every split, `bar` an
// mbarrier (count 1) that no earlier phase of this launch used.
__device__ void decode_tail(const FaParams &p, int g, uint8_t *scratch, float *buf, uint64_t *bar,
                            volatile int *abort_flag) {
    float *sh = reinterpret_cast<float *>(scratch);
    volatile int *flag = reinterpret_cast<volatile int *>(sh + 2 * MAXS + 8 + 2 * EX_MAX_WORLD);
    const int nrows = p.T * GROUP, d = threadIdx.x;
    auto global_row = [&](int r) { return (r / GROUP) * NQ + g * GROUP + r % GROUP; };
    // The gates of this CTA's first two rows load while the CTA waits at the barrier.
    auto load_gates = [&](int ra, int rb, float (&gate)[2]) {
        gate[0] = gate[1] = 0.f;
        if (p.tail == TAIL_SHARD) return;
        if (ra < nrows) gate[0] = p.q_gate[(size_t)global_row(ra) * 2 * HD + HD + d];
        if (rb >= 0) gate[1] = p.q_gate[(size_t)global_row(rb) * 2 * HD + HD + d];
    };
    float gate[2];
    {
        const int ra = blockIdx.x, rb = ra + p.splits < nrows ? ra + p.splits : -1;
        load_gates(ra, rb, gate);
    }
    if (!head_barrier(p.sync + g, p.splits, flag)) return;
    if (threadIdx.x == 0) QV_STAMP(7);
    uint32_t phase = 0;
    for (int ra = blockIdx.x; ra < nrows; ra += 2 * p.splits, phase ^= 1) {
        const int rb = ra + p.splits < nrows ? ra + p.splits : -1;
        const int nr = rb >= 0 ? 2 : 1;
        if (ra != (int)blockIdx.x) load_gates(ra, rb, gate);
        float o[2], lse[2];
        if (!combine_rows(p, g, ra, rb, sh, buf, bar, phase, abort_flag, o, lse)) return;
        const int grow[2] = {global_row(ra), nr == 2 ? global_row(rb) : 0};
        if (p.tail == TAIL_EXCHANGE) exchange_rows(p, grow, nr, o, lse, sh + 2 * MAXS + 8);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            if (k >= nr) break;
            if (p.tail == TAIL_SHARD) {
                p.out[(size_t)grow[k] * HD + d] = o[k];
                if (d == 0) p.lse[grow[k]] = lse[k];
            } else {
                p.out[(size_t)grow[k] * HD + d] = o[k] * sigmoidf_(gate[k]);
            }
        }
    }
    if (threadIdx.x == 0) QV_STAMP(8);
}

__global__ void __launch_bounds__(256, 1)
fa_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
          const FaParams p) {
    using L = FaLayout;
    constexpr int SOFT_WARPS = 4;                              // softmax warps
    extern __shared__ __align__(1024) uint8_t smem[];
    if (smem_addr(smem) & 1023) {           // 128B-swizzle atoms need a 1024-byte aligned base
        if (threadIdx.x == 0) raise_status(STATUS_BAD_ARGUMENT);
        return;
    }
    if (threadIdx.x == 0) QV_STAMP(0);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::SM_BAR);
    uint64_t *k_full = bars, *v_full = bars + 3, *k_empty = bars + 6, *v_empty = bars + 9,
             *s_full = bars + 12, *s_free = bars + 14, *p_full = bars + 16, *p_free = bars + 18,
             *mma_done = bars + 20, *q_ready = bars + 21, *app_done = bars + 22, *cbar = bars + 23;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::SM_BAR + 224);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::SM_BAR + 228);
    float2 *rope = reinterpret_cast<float2 *>(smem + L::SM_ROPE);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kv_head = blockIdx.y;

    // KV tile range of this CTA's split (tile = 64 cache rows, local numbering).
    const int total = (p.kv_rows + BN - 1) / BN;
    const int tile0 = blockIdx.x * p.split_tiles;
    const int ntiles = min(p.split_tiles, total - tile0);
    // The block's new cache rows that fall into this CTA's tiles.
    int app_lo = 0, app_hi = 0;
    if (p.append_row0 >= 0) {
        app_lo = max(p.append_row0, tile0 * BN);
        app_hi = min(p.append_row0 + p.T, (tile0 + ntiles) * BN);
    }
    const bool appends = app_hi > app_lo;
    const int app_tile = appends ? app_lo / BN - tile0 : ntiles;    // first tile holding a new row

    // Before anything else: L2 prefetch hints for this CTA's query rows (the
    // q half of q_gate), so that their HBM latency overlaps the previous
    // kernel's tail.  (Prefetching K/V tiles as well measured slower: the
    // extra traffic delays the query loads and thrashes L2.)
    for (int i = threadIdx.x; i < p.T * GROUP * 8; i += blockDim.x) {    // 8 lines of 128 B per row
        const int rr = i >> 3;
        prefetch_l2(p.q_gate + ((size_t)(rr / GROUP) * NQ + kv_head * GROUP + rr % GROUP) * 2 * HD + (i & 7) * 32);
    }

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES3; ++i) {
            mbar_init(k_full + i, 1); mbar_init(v_full + i, 1);
            mbar_init(k_empty + i, 1); mbar_init(v_empty + i, 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(s_full + i, 1); mbar_init(s_free + i, SOFT_WARPS);
            mbar_init(p_full + i, SOFT_WARPS); mbar_init(p_free + i, 1);
        }
        mbar_init(mma_done, 1);
        mbar_init(q_ready, 8);                     // every warp, once its query rows are in TMEM
        mbar_init(cbar, 1);
        mbar_init(app_done, 64);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) { prefetch_tmap(&tmK); prefetch_tmap(&tmV); }
    if (warp == 1) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Softmax warps 4-7: thread = TMEM lane = A row of the QK MMA; lanes i and
    // i+16 of warp w carry the hi and lo halves of query row 16w+i (one M=128
    // MMA yields both).
    const int wq = (warp - 4) & 3;
    const uint32_t t_lane = tmem + ((uint32_t)(wq * 32) << 16);
    const int half = lane >> 4;
    const int r = wq * 16 + (lane & 15);                                // logical query row
    int t = 0, h = 0;
    const bool valid = warp >= 4 && row_token_head(p, r, t, h);

    // Everything below may read what the previous kernel of the stream wrote.
    grid_dependency_wait();
    if (threadIdx.x == 0) { launch_dependents(); QV_STAMP(1); }

    // The query rows and norm weights are loaded first (from L2, ahead of the
    // bulk K/V data, which would otherwise queue in front of them on the way
    // into the SM); once every warp's rows have arrived, tiles 0..2 (all
    // three stages) go out, unless they hold new rows, which must be written
    // first, and the preparation overlaps their loads.
    const int early = min(ntiles, min(app_tile, STAGES3));
    auto issue_early = [&](int j0, int j1) {
        for (int j = j0; j < j1; ++j) {
            uint8_t *kd = smem + L::SM_KV + j * L::SM_KV_STAGE, *vd = kd + TILE_BYTES;
            const int y = (tile0 + j) * BN;
            mbar_expect_tx(k_full + j, TILE_BYTES);
            for (int c = 0; c < 4; ++c) tma_load_2d(kd + c * BN * 128, &tmK, k_full + j, kv_head * HD + c * 64, y);
            mbar_expect_tx(v_full + j, TILE_BYTES);
            for (int c = 0; c < 4; ++c) tma_load_2d(vd + c * BN * 128, &tmV, v_full + j, kv_head * HD + c * 64, y);
        }
        QV_STAMP(2);
    };
    constexpr int QR = DECODE_ROWS / 8;
    float4 xa[QR], xb[QR], n0, n1;
    {
#pragma unroll
        for (int j = 0; j < QR; ++j) {
            const int rr = warp + 8 * j;
            if (rr < p.T * GROUP) {
                const float *src = p.q_gate + ((size_t)(rr / GROUP) * NQ + kv_head * GROUP + rr % GROUP) * 2 * HD;
                xa[j] = *reinterpret_cast<const float4 *>(src + 4 * lane);
                xb[j] = *reinterpret_cast<const float4 *>(src + 128 + 4 * lane);
            } else {
                xa[j] = xb[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        n0 = *reinterpret_cast<const float4 *>(p.qn + 4 * lane);
        n1 = *reinterpret_cast<const float4 *>(p.qn + 128 + 4 * lane);
    }

    {
        // ---------------------------------------- prepare (all warps)
        // Query rows r = warp + 8j: RMSNorm with weight, rotary on dims
        // [0,64), split into fp16 hi + lo (hi: the value truncated to fp16's
        // 11 significant bits, so that lo = x - hi is exact), placed in TMEM
        // A-row order (hi of row 16g+i at A row 32g+i, lo at 32g+16+i).  The
        // rows go to TMEM through the two P buffers (idle until the first
        // softmax, which needs these queries), in two rounds of 64 columns:
        // dims [0,128) then [128,256).  A staged A row is 256 bytes, 16-byte
        // chunks XOR-swizzled by the row's low 3 bits; in each round every
        // warp copies half the columns of its TMEM lane quarter.  Warps 2-3
        // finally write the block's new keys / values, if this CTA's tiles
        // hold them.  Lane l of a row holds dims [4l,4l+4) and [128+4l,128+4l+4).
        // Rotary (cos, sin) of every (token, dim pair) while the loads are in flight.
        for (int e = threadIdx.x; e < p.T * 32; e += 256) rope[e] = rope_angle(p.position + (e >> 5), e & 31);
        float ss[QR];
#pragma unroll
        for (int j = 0; j < QR; ++j)
            ss[j] = xa[j].x * xa[j].x + xa[j].y * xa[j].y + xa[j].z * xa[j].z + xa[j].w * xa[j].w +
                    xb[j].x * xb[j].x + xb[j].y * xb[j].y + xb[j].z * xb[j].z + xb[j].w * xb[j].w;
        named_barrier(1, 256);                                    // the rotary table is complete
        // Every warp has its query rows by now (it summed their squares before
        // the barrier), so the K/V tiles no longer queue in front of them.
        if (threadIdx.x == 0) issue_early(0, early);
#pragma unroll
        for (int o = 16; o; o >>= 1) {
#pragma unroll
            for (int j = 0; j < QR; ++j) ss[j] += __shfl_xor_sync(0xffffffffu, ss[j], o);
        }
        auto split = [](float a, float b, uint32_t &hi, uint32_t &lo) {
            const float ha = __uint_as_float(__float_as_uint(a) & 0xFFFFE000u);
            const float hb = __uint_as_float(__float_as_uint(b) & 0xFFFFE000u);
            hi = half2_bits(__floats2half2_rn(ha, hb));
            lo = half2_bits(__floats2half2_rn(a - ha, b - hb));
        };
        uint32_t hw[QR][2][4];                    // [row][round] {hi0, hi1, lo0, lo1}
#pragma unroll
        for (int j = 0; j < QR; ++j) {
            const int rr = warp + 8 * j;
            const bool live = rr < p.T * GROUP;
            const float inv = rsqrtf(ss[j] / HD + p.eps);
            const float4 a = xa[j], b = xb[j];
            float x0[4] = {a.x * inv * n0.x, a.y * inv * n0.y, a.z * inv * n0.z, a.w * inv * n0.w};
            const float x1[4] = {b.x * inv * n1.x, b.y * inv * n1.y, b.z * inv * n1.z, b.w * inv * n1.w};
            rope_row(x0, rope + (live ? rr / GROUP : 0) * 32, lane, live);
            split(x0[0], x0[1], hw[j][0][0], hw[j][0][2]);
            split(x0[2], x0[3], hw[j][0][1], hw[j][0][3]);
            split(x1[0], x1[1], hw[j][1][0], hw[j][1][2]);
            split(x1[2], x1[3], hw[j][1][1], hw[j][1][3]);
        }
        uint8_t *qstage = smem + L::SM_P;                             // 128 A rows x 256 bytes
        const int sub = (lane & 1) * 8;
        const int arow = (warp & 3) * 32 + lane, col_half = warp >> 2;
        const uint32_t qdst = tmem + ((uint32_t)((warp & 3) * 32) << 16) + TM_Q + col_half * 32;
#pragma unroll
        for (int round = 0; round < 2; ++round) {
#pragma unroll
            for (int j = 0; j < QR; ++j) {
                const int rr = warp + 8 * j;
                const int ahi = 32 * (rr >> 4) + (rr & 15);
                const int p0 = (((lane >> 1) ^ (ahi & 7)) << 4) + sub;
                *reinterpret_cast<uint2 *>(qstage + ahi * 256 + p0) = make_uint2(hw[j][round][0], hw[j][round][1]);
                *reinterpret_cast<uint2 *>(qstage + (ahi + 16) * 256 + p0) = make_uint2(hw[j][round][2], hw[j][round][3]);
            }
            named_barrier(2, 256);
            // Warp w: TMEM lanes 32*(w%4).., columns 64*round + [32*(w/4), 32*(w/4)+32).
            const uint8_t *mine = qstage + arow * 256;
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                uint4 u[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    u[e] = *reinterpret_cast<const uint4 *>(mine + (((col_half * 8 + 4 * m + e) ^ (lane & 7)) << 4));
                tmem_st16(qdst + round * 64 + m * 16, *reinterpret_cast<const float(*)[16]>(u));
            }
            if (round == 0) named_barrier(3, 256);    // every warp has read round 0 before it is overwritten
        }
        {
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(q_ready);
            if (threadIdx.x == 128) QV_STAMP(3);
        }
        if ((warp == 2 || warp == 3) && appends) {
            // Append: RMSNorm + rotary of the new keys, fp16 keys / values into
            // the cache rows of this CTA's tiles, made visible to the TMA loads.
            const int k = warp - 2;
            const float4 k0 = *reinterpret_cast<const float4 *>(p.kn + 4 * lane);
            const float4 k1 = *reinterpret_cast<const float4 *>(p.kn + 128 + 4 * lane);
            for (int row = app_lo + k; row < app_hi; row += 2) {
                const int tt = row - p.append_row0;
                const float *ks = p.key + ((size_t)tt * NKV + kv_head) * HD;
                const float *vs = p.value + ((size_t)tt * NKV + kv_head) * HD;
                const float4 a = *reinterpret_cast<const float4 *>(ks + 4 * lane);
                const float4 b = *reinterpret_cast<const float4 *>(ks + 128 + 4 * lane);
                const float4 va = *reinterpret_cast<const float4 *>(vs + 4 * lane);
                const float4 vb = *reinterpret_cast<const float4 *>(vs + 128 + 4 * lane);
                float sk = a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w + b.x * b.x + b.y * b.y + b.z * b.z +
                           b.w * b.w;
                sk = warp_sum(sk);
                const float inv = rsqrtf(sk / HD + p.eps);
                float x0[4] = {a.x * inv * k0.x, a.y * inv * k0.y, a.z * inv * k0.z, a.w * inv * k0.w};
                rope_row(x0, rope + tt * 32, lane, true);
                __half *kd = p.kc + ((size_t)row * NKV + kv_head) * HD;
                __half *vd = p.vc + ((size_t)row * NKV + kv_head) * HD;
                *reinterpret_cast<uint2 *>(kd + 4 * lane) =
                    make_uint2(half2_bits(__floats2half2_rn(x0[0], x0[1])), half2_bits(__floats2half2_rn(x0[2], x0[3])));
                *reinterpret_cast<uint2 *>(kd + 128 + 4 * lane) =
                    make_uint2(half2_bits(__floats2half2_rn(b.x * inv * k1.x, b.y * inv * k1.y)),
                               half2_bits(__floats2half2_rn(b.z * inv * k1.z, b.w * inv * k1.w)));
                *reinterpret_cast<uint2 *>(vd + 4 * lane) =
                    make_uint2(half2_bits(__floats2half2_rn(va.x, va.y)), half2_bits(__floats2half2_rn(va.z, va.w)));
                *reinterpret_cast<uint2 *>(vd + 128 + 4 * lane) =
                    make_uint2(half2_bits(__floats2half2_rn(vb.x, vb.y)), half2_bits(__floats2half2_rn(vb.z, vb.w)));
            }
            fence_async_global();
            mbar_arrive(app_done);
        }
    }

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        // K tiles are released after QK, V tiles after PV, so the next K load
        // overlaps the softmax and PV of the current tile.
        if (lane == 0) {
            int k_issued = early, v_issued = early;        // tiles issued before the query preparation
            for (int j = early; j < ntiles; ++j) {
                const int s = j % STAGES3;
                const uint32_t use = (uint32_t)(j / STAGES3);
                const int y = (tile0 + j) * BN;
                uint8_t *kd = smem + L::SM_KV + s * L::SM_KV_STAGE, *vd = kd + TILE_BYTES;
                if (j == app_tile && !mbar_wait(app_done, 0, abort_flag)) break;   // new rows written
                if (j >= STAGES3 && !mbar_wait(k_empty + s, (use - 1) & 1, abort_flag)) break;
                mbar_expect_tx(k_full + s, TILE_BYTES);
                for (int c = 0; c < 4; ++c) tma_load_2d(kd + c * BN * 128, &tmK, k_full + s, kv_head * HD + c * 64, y);
                k_issued = j + 1;
                if (j >= STAGES3 && !mbar_wait(v_empty + s, (use - 1) & 1, abort_flag)) break;
                mbar_expect_tx(v_full + s, TILE_BYTES);
                for (int c = 0; c < 4; ++c) tma_load_2d(vd + c * BN * 128, &tmV, v_full + s, kv_head * HD + c * 64, y);
                v_issued = j + 1;
            }
            QV_STAMP(9);
            // Drain: every issued load must land before the CTA may exit.
            const long long t0 = clock64();
            for (int j = max(0, k_issued - STAGES3); j < k_issued; ++j)
                while (!mbar_try_wait(k_full + j % STAGES3, (j / STAGES3) & 1) && clock64() - t0 < WAIT_LIMIT_CYCLES) {}
            for (int j = max(0, v_issued - STAGES3); j < v_issued; ++j)
                while (!mbar_try_wait(v_full + j % STAGES3, (j / STAGES3) & 1) && clock64() - t0 < WAIT_LIMIT_CYCLES) {}
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc_qk = idesc_f16(128, BN, false, false);
            const uint32_t idesc_pv = idesc_f16(128, HD, false, true);
            auto issue_pv = [&](int i) -> bool {
                const int b = i & 1, s = i % STAGES3;
                if (!mbar_wait(p_full + b, (i >> 1) & 1, abort_flag)) return false;
                if (!mbar_wait(v_full + s, (i / STAGES3) & 1, abort_flag)) return false;
                tc_fence_after();
                const uint32_t pa = smem_addr(smem + L::SM_P + b * 128 * 128);
                const uint32_t vb = smem_addr(smem + L::SM_KV + s * L::SM_KV_STAGE + TILE_BYTES);
#pragma unroll
                for (int k = 0; k < BN / 16; ++k)     // P (hi / lo rows) from shared memory
                    mma_f16_ss(tmem + TM_O, sw128_desc(pa + k * 32, 16, 1024),
                               sw128_desc(vb + k * 16 * 128, BN * 128, 1024), idesc_pv,
                               (i > 0 || k > 0) ? 1u : 0u);
                mma_commit(p_free + b);
                mma_commit(v_empty + s);
                return true;
            };
            bool ok = mbar_wait(q_ready, 0, abort_flag);
            tc_fence_after();
            for (int j = 0; j < ntiles && ok; ++j) {
                const int b = j & 1, s = j % STAGES3;
                if (!mbar_wait(k_full + s, (j / STAGES3) & 1, abort_flag)) { ok = false; break; }
                // S buffer b is reusable once the softmax has read tile j-2.
                if (j >= 2 && !mbar_wait(s_free + b, ((j >> 1) - 1) & 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t kb = smem_addr(smem + L::SM_KV + s * L::SM_KV_STAGE);
#pragma unroll
                for (int k = 0; k < HD / 16; ++k)
                    mma_f16_ts(tmem + TM_S + b * BN, tmem + TM_Q + k * 8,
                               sw128_desc(kb + (k >> 2) * (BN * 128) + (k & 3) * 32, 16, 1024),
                               idesc_qk, k > 0 ? 1u : 0u);
                mma_commit(s_full + b);
                mma_commit(k_empty + s);
                if (j >= 1) ok = issue_pv(j - 1);
            }
            if (ok && ntiles > 0) issue_pv(ntiles - 1);
            QV_STAMP(10);
            // All MMAs of this thread must finish before TMEM is released.
            mma_commit(mma_done);
            const long long t0 = clock64();
            while (!mbar_try_wait(mma_done, 0) && clock64() - t0 < WAIT_LIMIT_CYCLES) {}
        }
    } else if (warp >= 4) {
        // ------------------------------------------------ softmax + epilogue
        // Each thread handles 32 columns of its row per tile: lane i keeps
        // columns [0,32) and lane i+16 columns [32,64) of row 16w+i, each summing
        // the hi and lo score halves, and each writes the hi and lo
        // probabilities of its columns.
        constexpr int NC = 32;                                     // columns per thread
        const int cpart = half;                                    // which 32 columns
        const int pos_limit = valid ? p.position + t - p.kv_begin : -1;   // last visible local row
        const int arow_hi = wq * 32 + (lane & 15);                 // A rows of P (hi, lo)
        const int arow_lo = arow_hi + 16;
        float m_use = -INFINITY, l = 0.f;
        for (int j = 0; j < ntiles; ++j) {
            const int b = j & 1;
            if (!warp_wait(s_full + b, (j >> 1) & 1, abort_flag)) break;
            if (j == 0 && threadIdx.x == 128) QV_STAMP(4);
            tc_fence_after();
            float x[64];
#pragma unroll
            for (int c = 0; c < 4; ++c)
                tmem_ld16(t_lane + TM_S + b * BN + c * 16, *reinterpret_cast<float(*)[16]>(x + c * 16));
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free + b);
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                const float recv = __shfl_xor_sync(0xffffffffu, half ? x[c] : x[32 + c], 16);
                x[c] = (half ? x[32 + c] : x[c]) + recv;
            }
            const int key0 = (tile0 + j) * BN + cpart * 32;
            const int lim = min(pos_limit, p.kv_rows - 1) - key0;     // columns <= lim are visible
            // Row max and (below) row sum over 8 / 4 independent partials, so
            // neither is one long dependent chain.
            float mp[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) mp[q] = -INFINITY;
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                x[c] = c <= lim ? x[c] : -INFINITY;
                mp[c & 7] = fmaxf(mp[c & 7], x[c]);
            }
            float m_tile = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                                 fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
            m_tile = fmaxf(m_tile, __shfl_xor_sync(0xffffffffu, m_tile, 16));
            m_tile *= SCORE_LOG2;                                  // log2 units (-inf stays -inf)
            float factor = 1.f;
            const bool need = m_tile > m_use + RESCALE_THRESHOLD;
            if (need) { factor = exp2_approx(m_use - m_tile); m_use = m_tile; l *= factor; }
            if (j > 0 && __any_sync(0xffffffffu, need)) {
                // O already holds tiles < j: wait for PV(j-1), then rescale rows in
                // TMEM.
                if (!warp_wait(p_free + ((j - 1) & 1), ((j - 1) >> 1) & 1, abort_flag)) break;
                tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < HD / 16; ++c) {
                    float o[16];
                    tmem_ld16(t_lane + TM_O + c * 16, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 16; ++e) o[e] *= factor;
                    tmem_st16(t_lane + TM_O + c * 16, o);
                }
                tmem_wait_st();
            }
            const float mref = m_use == -INFINITY ? 0.f : m_use;
            uint32_t hi[NC / 2], lo[NC / 2];
            float sp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < NC; c += 2) {
                const float p0 = exp2_approx(fmaf(x[c], SCORE_LOG2, -mref));
                const float p1 = exp2_approx(fmaf(x[c + 1], SCORE_LOG2, -mref));
                const __half2 hp = __floats2half2_rn(p0, p1);
                hi[c / 2] = *reinterpret_cast<const uint32_t *>(&hp);
                const float2 back = __half22float2(hp);
                const __half2 lp = __floats2half2_rn(p0 - back.x, p1 - back.y);
                lo[c / 2] = *reinterpret_cast<const uint32_t *>(&lp);
                sp[(c >> 1) & 3] += p0 + p1;
            }
            l += (sp[0] + sp[1]) + (sp[2] + sp[3]);
            if (j >= 2 && !warp_wait(p_free + b, ((j - 2) >> 1) & 1, abort_flag)) break;
            uint8_t *pbuf = smem + L::SM_P + b * 128 * 128;
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const int unit = cpart * 4 + w;
                *reinterpret_cast<uint4 *>(pbuf + arow_hi * 128 + ((unit ^ (arow_hi & 7)) << 4)) =
                    make_uint4(hi[4 * w], hi[4 * w + 1], hi[4 * w + 2], hi[4 * w + 3]);
                *reinterpret_cast<uint4 *>(pbuf + arow_lo * 128 + ((unit ^ (arow_lo & 7)) << 4)) =
                    make_uint4(lo[4 * w], lo[4 * w + 1], lo[4 * w + 2], lo[4 * w + 3]);
            }
            fence_async_shared();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full + b);
        }
        if (threadIdx.x == 128) QV_STAMP(5);
        // The row's running max and sum, for the split combine.
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        if (valid && half == 0) {
            const size_t slot = ((size_t)kv_head * DECODE_ROWS + r) * MAXS + blockIdx.x;
            p.part_ml[slot * 2] = m_use;
            p.part_ml[slot * 2 + 1] = l;
        }
    }
    // ------------------------------------------------ epilogue (all 8 warps)
    // The final PV's commit on p_free marks O complete (and every K/V tile
    // consumed, so the ring is idle).  Warps w and w+4 share TMEM lane
    // quarter w%4 (O_hi of row 16(w%4)+i in lane i, O_lo in lane 16+i) and
    // take O columns [0,128) (warps 4-7) and [128,256) (warps 0-3): each lane
    // puts its lane's columns into a padded staging row, then the warp
    // stores each of its rows, the sum of its hi and lo staging rows, as
    // 512-byte pieces of this split's unnormalised partial.
    __syncwarp();                                      // warps 0 and 1: lane 0 is back from its role
    named_barrier(5, 256);
    const bool o_ready = ntiles > 0 &&
                         warp_wait(p_free + ((ntiles - 1) & 1), ((ntiles - 1) >> 1) & 1, abort_flag);
    if (o_ready) {
        tc_fence_after();
        if (threadIdx.x == 128) QV_STAMP(12);
        const int chalf = warp < 4 ? 1 : 0;
        constexpr int RS = 128 * 4 + 16;                       // staging row bytes (padded)
        static_assert(8 * 32 * RS <= STAGES3 * L::SM_KV_STAGE, "O staging exceeds the K/V ring");
        uint8_t *stage = smem + L::SM_KV + warp * 32 * RS;
        uint8_t *myrow = stage + lane * RS;
        const uint32_t ocol = t_lane + TM_O + chalf * 128;
#pragma unroll
        for (int c4 = 0; c4 < 2; ++c4) {                       // 64 columns per TMEM round trip
            float o[4][16];
#pragma unroll
            for (int q = 0; q < 4; ++q) tmem_ld16(ocol + c4 * 64 + q * 16, o[q]);
            tmem_wait_ld();
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int e = 0; e < 16; e += 4)
                    *reinterpret_cast<float4 *>(myrow + (c4 * 64 + q * 16 + e) * 4) =
                        make_float4(o[q][e], o[q][e + 1], o[q][e + 2], o[q][e + 3]);
        }
        __syncwarp();
        if (threadIdx.x == 128) QV_STAMP(13);
        // The valid logical rows of a CTA are a prefix, so are this warp's.
        const int row0 = wq * 16;
        const int nvalid = max(0, min(16, p.T * GROUP - row0));
        const int col = 4 * lane;
#pragma unroll 4
        for (int i = 0; i < nvalid; ++i) {
            const int rr = row0 + i;
            float4 v = *reinterpret_cast<const float4 *>(stage + i * RS + col * 4);
            const float4 w = *reinterpret_cast<const float4 *>(stage + (i + 16) * RS + col * 4);
            v.x += w.x; v.y += w.y; v.z += w.z; v.w += w.w;
            float *dst = p.part_o + (((size_t)kv_head * DECODE_ROWS + rr) * p.splits + blockIdx.x) * HD;
            *reinterpret_cast<float4 *>(dst + chalf * 128 + col) = v;
        }
        if (threadIdx.x == 128) QV_STAMP(6);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
    if (threadIdx.x == 0) QV_STAMP(11);
    // The split combine of this CTA's share of the KV head's rows (the K/V
    // ring and the P buffers are idle now; the P region is scratch).
    decode_tail(p, kv_head, smem + L::SM_P, reinterpret_cast<float *>(smem + L::SM_KV), cbar, abort_flag);
}

// ---------------------------------------------------------------- prepare
// One block per token, 8 warps; warp w prepares rows w, w+8, w+16 (and w+24)
// of the token's 28: the 24 query heads, then the 4 key heads.  RMSNorm with
// weight, rotary embedding on dims [0,64) as pairs (i, i+32) with angle
// (position+t) * 1e7^(-i/32) evaluated in double precision (the token's 32
// angles once per block), queries written as fp16 hi / lo operand rows,
// keys / values rounded to fp16 into the cache.  Lane l of a row holds dims
// [4l,4l+4) and [128+4l,128+4l+4), as in the decode kernel's prepare step.
// Used by the prefill regime; decode batches fold this step into fa_kernel.
__global__ void __launch_bounds__(256)
attn_prepare_kernel(const float *q_gate, const float *key, const float *value, const float *qn,
                    const float *kn, __half *qw, __half *qw_lo, __half *kc, __half *vc, int position,
                    int append_row0, float eps) {
    constexpr int ROWS = NQ + NKV, RPW = (ROWS + 7) / 8;          // rows per token, per warp
    const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __shared__ float2 cs[32];
    grid_dependency_wait();
    launch_dependents();
    float4 a[RPW], b[RPW];
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
        const int h = warp + 8 * j;
        if (h < ROWS) {
            const float *src = h < NQ ? q_gate + ((size_t)t * NQ + h) * 2 * HD : key + ((size_t)t * NKV + h - NQ) * HD;
            a[j] = *reinterpret_cast<const float4 *>(src + 4 * lane);
            b[j] = *reinterpret_cast<const float4 *>(src + 128 + 4 * lane);
        }
    }
    if (threadIdx.x < 32) cs[threadIdx.x] = rope_angle(position + t, threadIdx.x);
    __syncthreads();
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
        const int h = warp + 8 * j;
        if (h >= ROWS) continue;
        const bool isq = h < NQ;
        const float *nw = isq ? qn : kn;
        const float4 n0 = *reinterpret_cast<const float4 *>(nw + 4 * lane);
        const float4 n1 = *reinterpret_cast<const float4 *>(nw + 128 + 4 * lane);
        const float4 u = a[j], v = b[j];
        const float ss = warp_sum(u.x * u.x + u.y * u.y + u.z * u.z + u.w * u.w + v.x * v.x + v.y * v.y +
                                  v.z * v.z + v.w * v.w);
        const float inv = rsqrtf(ss / HD + eps);
        float x0[4] = {u.x * inv * n0.x, u.y * inv * n0.y, u.z * inv * n0.z, u.w * inv * n0.w};
        const float x1[4] = {v.x * inv * n1.x, v.y * inv * n1.y, v.z * inv * n1.z, v.w * inv * n1.w};
        rope_row(x0, cs, lane, true);
        if (isq) {
            __half *hi = qw + ((size_t)t * NQ + h) * HD, *lo = qw_lo + ((size_t)t * NQ + h) * HD;
#pragma unroll
            for (int part = 0; part < 2; ++part) {
                const float *x = part ? x1 : x0;
                const __half2 h0 = __floats2half2_rn(x[0], x[1]), h1 = __floats2half2_rn(x[2], x[3]);
                const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
                *reinterpret_cast<uint2 *>(hi + part * 128 + 4 * lane) = make_uint2(half2_bits(h0), half2_bits(h1));
                *reinterpret_cast<uint2 *>(lo + part * 128 + 4 * lane) =
                    make_uint2(half2_bits(__floats2half2_rn(x[0] - f0.x, x[1] - f0.y)),
                               half2_bits(__floats2half2_rn(x[2] - f1.x, x[3] - f1.y)));
            }
        } else if (append_row0 >= 0) {
            const int kh = h - NQ;
            const size_t o = ((size_t)(append_row0 + t) * NKV + kh) * HD;
            const float *vs = value + ((size_t)t * NKV + kh) * HD;
            const float4 va = *reinterpret_cast<const float4 *>(vs + 4 * lane);
            const float4 vb = *reinterpret_cast<const float4 *>(vs + 128 + 4 * lane);
            *reinterpret_cast<uint2 *>(kc + o + 4 * lane) =
                make_uint2(half2_bits(__floats2half2_rn(x0[0], x0[1])), half2_bits(__floats2half2_rn(x0[2], x0[3])));
            *reinterpret_cast<uint2 *>(kc + o + 128 + 4 * lane) =
                make_uint2(half2_bits(__floats2half2_rn(x1[0], x1[1])), half2_bits(__floats2half2_rn(x1[2], x1[3])));
            *reinterpret_cast<uint2 *>(vc + o + 4 * lane) =
                make_uint2(half2_bits(__floats2half2_rn(va.x, va.y)), half2_bits(__floats2half2_rn(va.z, va.w)));
            *reinterpret_cast<uint2 *>(vc + o + 128 + 4 * lane) =
                make_uint2(half2_bits(__floats2half2_rn(vb.x, vb.y)), half2_bits(__floats2half2_rn(vb.z, vb.w)));
        }
    }
}

// Merge per-GPU shard partials (normalised O, natural-log LSE) into the gated
// output: O = sum_g exp(lse_g - LSE) O_g, times sigmoid(gate).
__global__ void __launch_bounds__(256)
attn_merge_kernel(float *out, const float *parts, const float *lses, int shards, int T,
                  const float *q_gate) {
    const int t = blockIdx.x / NQ, h = blockIdx.x % NQ, d = threadIdx.x;
    const size_t row = (size_t)t * NQ + h, stride_o = (size_t)T * NQ * HD, stride_l = (size_t)T * NQ;
    grid_dependency_wait();
    launch_dependents();
    float M = -INFINITY;
    for (int g = 0; g < shards; ++g) M = fmaxf(M, lses[g * stride_l + row]);
    float num = 0.f, den = 0.f;
    if (M != -INFINITY)
        for (int g = 0; g < shards; ++g) {
            const float L = lses[g * stride_l + row];
            if (L == -INFINITY) continue;
            const float w = expf(L - M);
            den += w;
            num += w * parts[g * stride_o + row * HD + d];
        }
    out[row * HD + d] = (den > 0.f ? num / den : 0.f) * sigmoidf_(q_gate[row * 2 * HD + HD + d]);
}

// ======================================================================= host
namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void *ptr = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !ptr)
            throw std::runtime_error("cuTensorMapEncodeTiled is unavailable");
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// 2-D map over a [rows][4*256] fp16 cache: box = 64 dims x 64 rows, 128B swizzle.
CUtensorMap cache_map(const void *base, int rows) {
    CUtensorMap m;
    cuuint64_t dims[2] = {(cuuint64_t)NKV * HD, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)NKV * HD * sizeof(__half)};
    cuuint32_t box[2] = {64, (cuuint32_t)BN};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims,
                                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return m;
}

// The shared-memory limit of a kernel is a per-device attribute: set it on
// every device the process launches on.
PerDeviceOnce g_configured;
void configure() {
    g_configured.run([] {
        if (cudaFuncSetAttribute(fa_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FaLayout::SMEM_BYTES) !=
            cudaSuccess)
            throw std::runtime_error("cannot reserve shared memory for the attention kernel");
    });
}

struct Split { int tiles, splits; };
// CTAs per KV head of a decode launch: a quarter of the SMs (37 on B200), so
// that the four heads fill one wave with one CTA per SM and the CTAs of a
// head, which meet at the tail barrier, are all resident at once.  Without a
// device (host-side size queries) the B200 figure is used.
int decode_ctas_per_head() {
    int dev = -1, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        sms = 148;
    }
    return std::max(1, std::min(37, sms / NKV));
}
// Split-KV plan: whole tiles per split, at most decode_ctas_per_head() splits.
Split decode_split(int kv_rows) {
    const int total = std::max(1, (kv_rows + BN - 1) / BN);
    const int ctas = decode_ctas_per_head();
    const int per = (total + ctas - 1) / ctas;
    static_assert(37 <= MAXS, "the tail combine handles up to MAXS splits");
    return {per, (total + per - 1) / per};
}
size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
bool decode_regime(int T) { return T * GROUP <= DECODE_ROWS; }

void launch_fa(const CUtensorMap &mk, const CUtensorMap &mv, const FaParams &p, dim3 grid, cudaStream_t st) {
    const cudaError_t e = launch_chained(fa_kernel, grid, dim3(256), FaLayout::SMEM_BYTES, st,
                                         mk, mv, p);
    if (e != cudaSuccess) throw std::runtime_error(std::string("attention kernel launch: ") + cudaGetErrorString(e));
}

// Decode workspace: the tail barrier's words (256 bytes: one 64-bit word per
// KV head, generation : arrivals; the arrivals must be zero before the first
// launch on the workspace and every launch leaves them zero), then the split
// partials.
constexpr size_t SYNC_BYTES = 256;
struct DecodeParts { unsigned long long *sync; float *o, *ml; };
size_t decode_parts_bytes(const Split &sp) {
    return SYNC_BYTES + align256((size_t)NKV * sp.splits * DECODE_ROWS * HD * sizeof(float)) +
           align256((size_t)NKV * DECODE_ROWS * MAXS * 2 * sizeof(float));
}
DecodeParts decode_parts(void *ws, const Split &sp) {
    uint8_t *w = static_cast<uint8_t *>(ws);
    float *o = reinterpret_cast<float *>(w + SYNC_BYTES);
    float *ml = reinterpret_cast<float *>(w + SYNC_BYTES + align256((size_t)NKV * sp.splits * DECODE_ROWS * HD * sizeof(float)));
    return {reinterpret_cast<unsigned long long *>(w), o, ml};
}

// Split-KV decode / verify, one launch: the CTAs normalise and rotate the
// queries, append the new keys / values (when `append`), attend over their
// split, and at the tail combine the splits and write the rows as `tail`
// says (out = gated output, or shard partial with lse, or the peer exchange).
void launch_decode(float *out, float *lse, __half *kc, __half *vc, const float *q_gate, const float *key,
                   const float *value, const float *qn, const float *kn, int T, int position, int kv_begin,
                   int kv_rows, bool append, float eps, void *ws, size_t ws_bytes, DecodeTail tail,
                   const uint64_t *peers, int world, int rank, int seq, cudaStream_t st) {
    configure();
    const Split sp = decode_split(kv_rows);
    if (ws_bytes < decode_parts_bytes(sp)) throw std::invalid_argument("attention workspace too small");
    const DecodeParts parts = decode_parts(ws, sp);
    const CUtensorMap mk = cache_map(kc, kv_rows), mv = cache_map(vc, kv_rows);
    FaParams p{};
    p.q_gate = q_gate; p.out = out; p.lse = lse; p.T = T; p.position = position; p.kv_begin = kv_begin;
    p.kv_rows = kv_rows; p.split_tiles = sp.tiles; p.splits = sp.splits;
    p.part_o = parts.o; p.part_ml = parts.ml; p.sync = parts.sync;
    p.tail = tail; p.peers = peers; p.world = world; p.rank = rank; p.seq = seq;
    p.key = key; p.value = value; p.qn = qn; p.kn = kn; p.kc = kc; p.vc = vc;
    p.append_row0 = append ? position - kv_begin : -1; p.eps = eps;
    launch_fa(mk, mv, p, dim3(sp.splits, NKV), st);
}
}  // namespace

size_t attention_workspace_bytes(int T, int kv_rows) {
    if (decode_regime(T)) return decode_parts_bytes(decode_split(kv_rows));
    return 2 * align256((size_t)T * NQ * HD * sizeof(__half));     // prefill: Q hi and lo, direct output
}

int attention_max_shard_batch() { return MAX_DECODE_T; }

// One attention layer over a device cache holding absolute positions
// [kv_begin, kv_begin + kv_rows).  New rows are appended at local row
// position - kv_begin when append is true.  Writes either the final gated
// output (shard_lse == nullptr) or a normalised partial + LSE (shard mode).
// Decode / verify batches (T <= 10) use the split-KV regime (one launch, the
// split combine in its tail); longer blocks use the prefill regime: a prepare
// launch, then prefill.cu's precise kernel (128 queries per CTA, 128-key tiles).
void attention_run(float *out, float *shard_lse, __half *kc, __half *vc, const float *q_gate,
                   const float *key, const float *value, const float *qn, const float *kn, int T,
                   int position, int kv_begin, int kv_rows, bool append, float eps, void *ws,
                   size_t ws_bytes, cudaStream_t st) {
    if (ws_bytes < attention_workspace_bytes(T, kv_rows)) throw std::invalid_argument("attention workspace too small");
    if (decode_regime(T)) {
        launch_decode(out, shard_lse, kc, vc, q_gate, key, value, qn, kn, T, position, kv_begin, kv_rows, append, eps,
                      ws, ws_bytes, shard_lse ? TAIL_SHARD : TAIL_GATED, nullptr, 1, 0, 0, st);
        return;
    }
    if (shard_lse) throw std::invalid_argument("shard partials are limited to decode batches");
    configure();
    uint8_t *w = static_cast<uint8_t *>(ws);
    const size_t q_bytes = align256((size_t)T * NQ * HD * sizeof(__half));
    __half *qw = reinterpret_cast<__half *>(w), *qw_lo = reinterpret_cast<__half *>(w + q_bytes);
    const cudaError_t e = launch_chained(attn_prepare_kernel, dim3(T), dim3(256), 0, st, q_gate, key, value,
                                         qn, kn, qw, qw_lo, kc, vc, position, append ? position - kv_begin : -1, eps);
    if (e != cudaSuccess) throw std::runtime_error(std::string("attention prepare: ") + cudaGetErrorString(e));
    prefill_precise(out, qw, qw_lo, q_gate, kc, vc, T, position - kv_begin, kv_rows, st);
}

size_t attention_exchange_bytes(int world) { return ex_bytes(world); }
int attention_exchange_max_world() { return EX_MAX_WORLD; }

// Shard attention + all-to-all exchange + merge, one launch (the exchange is
// the decode kernel's tail, see exchange_rows).
void attention_shard_exchange(float *out, __half *kc, __half *vc, const float *q_gate, const float *key,
                              const float *value, const float *qn, const float *kn, int T, int position,
                              int kv_begin, int kv_rows, bool append, float eps, const uint64_t *peers,
                              int world, int rank, int seq, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (!decode_regime(T)) throw std::invalid_argument("the exchange supports decode batches only");
    if (world < 1 || world > EX_MAX_WORLD || rank < 0 || rank >= world || seq < 0)
        throw std::invalid_argument("invalid exchange group");
    if (ws_bytes < attention_workspace_bytes(T, kv_rows)) throw std::invalid_argument("attention workspace too small");
    launch_decode(out, nullptr, kc, vc, q_gate, key, value, qn, kn, T, position, kv_begin, kv_rows, append, eps, ws,
                  ws_bytes, TAIL_EXCHANGE, peers, world, rank, seq, st);
}

void attention_merge(float *out, const float *parts, const float *lses, int shards, int T,
                     const float *q_gate, cudaStream_t st) {
    const cudaError_t e = launch_chained(attn_merge_kernel, dim3(T * NQ), dim3(256), 0, st, out, parts, lses, shards,
                                         T, q_gate);
    if (e != cudaSuccess) throw std::runtime_error(std::string("attention merge: ") + cudaGetErrorString(e));
}

}  // namespace qv
