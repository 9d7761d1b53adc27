// Full-attention hot path for sm_100a: prepare (RMSNorm + partial RoPE + fp16
// KV append), a tcgen05/TMEM FlashAttention kernel that serves both the
// decode/verify regime (split-KV, all 6 GQA heads x T tokens of one KV head
// share every K/V tile) and causal prefill (a tile of query positions of one
// head per CTA), and the split/shard combine kernels.
//
// Semantics follow the reference's attn_prepare / attention / attention_tiled
// (src/kernels.cu:415-503) and the CPU oracle tests/cpu_reference.py:55-89:
// scores q.k/16 over cache rows [0, position+t], softmax, P.V, times
// sigmoid(gate).
//
// Two precision modes of the FlashAttention kernel:
//  * PRECISE (decode / verify and reference-semantics prefill): 64 query rows
//    per CTA.  Q is split into fp16 hi = fp16(q) and lo = fp16(q - hi) and the
//    QK MMA's A operand (held in TMEM) interleaves them: A row 32w+i = Q_hi and
//    32w+16+i = Q_lo of query row 16w+i, so one M=128 MMA leaves both score
//    halves of a row in lanes i and i+16 of warp w, which add them while they
//    split the row's columns.  Every probability p is split the same way; the
//    PV MMA's A rows 32w+i / 32w+16+i are P_hi / P_lo of row 16w+i, so O_hi and
//    O_lo land in the same warp and are summed in the epilogue.  Scores and
//    probabilities keep ~22 mantissa bits (the reference computes them in fp32).
//  * FAST (core prefill, benchmark configuration 3): M=128 query rows and fp16 P.
#include "common.cuh"
#include "hotpath.h"

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
template <bool PRECISE> struct FaLayout {
    static constexpr int QROWS = PRECISE ? 64 : 128;          // logical query rows per CTA
    static constexpr int SM_KV = 0;                           // ring of (K tile, V tile)
    static constexpr int SM_KV_STAGE = 2 * TILE_BYTES;
    static constexpr int SM_P = SM_KV + STAGES3 * SM_KV_STAGE; // 2 x [128 A-rows][64 pos] fp16
    static constexpr int SM_BAR = SM_P + 2 * 128 * 128;       // mbarriers, TMEM address, abort flag
    static constexpr int SM_ROPE = SM_BAR + 256;              // decode: (cos, sin) [T][32]
    static constexpr int SMEM_BYTES = SM_ROPE + MAX_DECODE_T * 32 * 8;
};
static_assert(FaLayout<true>::SMEM_BYTES <= 227 * 1024, "attention kernel exceeds the shared memory of a CTA");

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

struct FaParams {
    const __half *q;        // prepared queries [T][24][256] (fp16 of q)
    const __half *q_lo;     // fp16 of (q - fp16(q)) (PRECISE)
    const float *q_gate;    // [T][24][512], gate = [256:512) (direct mode), may be null
    float *out;             // [T][24][256] (direct mode)
    float *lse;             // optional natural-log LSE [T][24] (direct mode)
    float *part_o;          // [4][splits][64][256] unnormalised partial O (split mode)
    float *part_ml;         // [4][splits][64][2]  (running max in log2 units, sum)
    int T, position;        // tokens and absolute position of token 0
    int kv_begin;           // absolute position of cache row 0
    int kv_rows;            // valid cache rows
    int mode;               // 0 = decode (GQA-packed rows), 1 = prefill (head-major rows)
    int split_tiles, splits;
    int direct;             // 1: write final output; 0: write split partials
    // Decode with the prepare step folded in (fused = 1): the CTA normalises
    // and rotates its own query rows from q_gate and, when its tiles hold the
    // block's new cache rows, writes their keys / values before loading them.
    int fused;
    const float *key, *value, *qn, *kn;
    __half *kc, *vc;        // the caches, for the append
    int append_row0;        // local cache row of token 0's key / value, or -1
    float eps;
};

// Logical query row -> (token, head).  Decode packs the 6 heads of one KV head
// and the T tokens; prefill takes QROWS consecutive tokens of one head.
template <int QROWS>
__device__ __forceinline__ bool row_token_head(const FaParams &p, int r, int &t, int &h) {
    if (p.mode == 0) {
        t = r / GROUP;
        h = blockIdx.y * GROUP + r % GROUP;
        return r < p.T * GROUP;
    }
    t = (gridDim.y - 1 - blockIdx.y) * QROWS + r;
    h = blockIdx.x;
    return t < p.T;
}

// Warp-uniform bounded wait (all lanes agree on the outcome).
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
}

template <bool PRECISE>
__global__ void __launch_bounds__(PRECISE ? 256 : 384, 1)
fa_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
          const FaParams p) {
    using L = FaLayout<PRECISE>;
    constexpr int QROWS = L::QROWS;
    constexpr int SOFT_WARPS = PRECISE ? 4 : 8;                // softmax warps
    extern __shared__ __align__(1024) uint8_t smem[];
    if (smem_addr(smem) & 1023) {           // 128B-swizzle atoms need a 1024-byte aligned base
        if (threadIdx.x == 0) raise_status(STATUS_BAD_ARGUMENT);
        return;
    }
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::SM_BAR);
    uint64_t *k_full = bars, *v_full = bars + 3, *k_empty = bars + 6, *v_empty = bars + 9,
             *s_full = bars + 12, *s_free = bars + 14, *p_full = bars + 16, *p_free = bars + 18,
             *mma_done = bars + 20, *q_ready = bars + 21, *app_done = bars + 22, *xbar = bars + 23,
             *lbar = bars + 25;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::SM_BAR + 224);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::SM_BAR + 228);
    float2 *rope = reinterpret_cast<float2 *>(smem + L::SM_ROPE);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kv_head = p.mode == 0 ? blockIdx.y : blockIdx.x / GROUP;

    // KV tile range of this CTA (tile = 64 cache rows, local numbering).
    int tile0, ntiles;
    if (p.mode == 0) {
        const int total = (p.kv_rows + BN - 1) / BN;
        tile0 = blockIdx.x * p.split_tiles;
        ntiles = min(p.split_tiles, total - tile0);
    } else {
        const int qtile = gridDim.y - 1 - blockIdx.y;
        const int last_tok = min(p.T, (qtile + 1) * QROWS) - 1;
        const int limit = min(p.kv_rows, p.position + last_tok - p.kv_begin + 1);
        tile0 = 0;
        ntiles = (limit + BN - 1) / BN;
    }
    // Fused decode: the block's new cache rows that fall into this CTA's tiles.
    int app_lo = 0, app_hi = 0;
    if (p.fused && p.append_row0 >= 0) {
        app_lo = max(p.append_row0, tile0 * BN);
        app_hi = min(p.append_row0 + p.T, (tile0 + ntiles) * BN);
    }
    const bool appends = app_hi > app_lo;
    const int app_tile = appends ? app_lo / BN - tile0 : ntiles;    // first tile holding a new row

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES3; ++i) {
            mbar_init(k_full + i, 1); mbar_init(v_full + i, 1);
            mbar_init(k_empty + i, 1); mbar_init(v_empty + i, 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(s_full + i, 1); mbar_init(s_free + i, SOFT_WARPS);
            mbar_init(p_full + i, SOFT_WARPS); mbar_init(p_free + i, 1);
            mbar_init(xbar + i, SOFT_WARPS);
        }
        mbar_init(mma_done, 1);
        mbar_init(q_ready, p.fused ? 8 : 4);      // every warp (fused) or softmax warps 4-7
        mbar_init(lbar, 4);
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

    // Softmax warps 4-7 (and 8-11 in FAST): thread = TMEM lane = A row of the
    // QK MMA.  FAST: A row = query row; warpgroup wg (warps 4-7 / 8-11) takes
    // columns [32 wg, 32 wg + 32) of every S tile.  PRECISE: lanes i and i+16
    // of warp w carry the hi and lo halves of query row 16w+i (one M=128 MMA
    // yields both).
    const int wq = (warp - 4) & 3, wg = PRECISE ? 0 : ((warp - 4) >> 2);
    const uint32_t t_lane = tmem + ((uint32_t)(wq * 32) << 16);
    const int half = PRECISE ? (lane >> 4) : 0;
    const int r = PRECISE ? wq * 16 + (lane & 15) : wq * 32 + lane;     // logical query row
    int t = 0, h = 0;
    const bool valid = warp >= 4 && row_token_head<QROWS>(p, r, t, h);

    // Everything below may read what the previous kernel of the stream wrote.
    grid_dependency_wait();
    if (threadIdx.x == 0) launch_dependents();

    // Fused decode: tiles 0 and 1 (stages 0 and 1) go out before the queries
    // are prepared, unless they hold new rows, which must be written first;
    // stage 2 stages the queries, so tile 2 waits for them.
    const int early = (PRECISE && p.fused) ? min(ntiles, min(app_tile, 2)) : 0;
    if (threadIdx.x == 0) {
        for (int j = 0; j < early; ++j) {
            uint8_t *kd = smem + L::SM_KV + j * L::SM_KV_STAGE, *vd = kd + TILE_BYTES;
            const int y = (tile0 + j) * BN;
            mbar_expect_tx(k_full + j, TILE_BYTES);
            for (int c = 0; c < 4; ++c) tma_load_2d(kd + c * BN * 128, &tmK, k_full + j, kv_head * HD + c * 64, y);
            mbar_expect_tx(v_full + j, TILE_BYTES);
            for (int c = 0; c < 4; ++c) tma_load_2d(vd + c * BN * 128, &tmV, v_full + j, kv_head * HD + c * 64, y);
        }
    }

    if (PRECISE && p.fused) {
        // ---------------------------------------- fused prepare (all warps)
        // Query rows r = warp + 8j: RMSNorm with weight, rotary on dims
        // [0,64), split into fp16 hi + lo (hi: the value truncated to fp16's
        // 11 significant bits, so that lo = x - hi is exact), written in TMEM
        // A-row order (hi of row 16g+i at A row 32g+i, lo at 32g+16+i; 512 bytes
        // per A row, 16-byte chunks XOR-swizzled by the row's low 3 bits) into
        // the third K/V stage, which the producer leaves idle until the
        // queries are staged (tiles 0 and 1 are already on their way).  Each warp then copies half the columns of its
        // TMEM lane quarter; warps 2-3 finally write the block's new keys /
        // values, if this CTA's tiles hold them.  Lane l of a row holds dims
        // [4l,4l+4) and [128+4l,128+4l+4).
        constexpr int QR = DECODE_ROWS / 8;
        float4 xa[QR], xb[QR];
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
        // Rotary (cos, sin) of every (token, dim pair) while the loads are in flight.
        for (int e = threadIdx.x; e < p.T * 32; e += 256) rope[e] = rope_angle(p.position + (e >> 5), e & 31);
        named_barrier(1, 256);
        const float4 n0 = *reinterpret_cast<const float4 *>(p.qn + 4 * lane);
        const float4 n1 = *reinterpret_cast<const float4 *>(p.qn + 128 + 4 * lane);
        float ss[QR];
#pragma unroll
        for (int j = 0; j < QR; ++j)
            ss[j] = xa[j].x * xa[j].x + xa[j].y * xa[j].y + xa[j].z * xa[j].z + xa[j].w * xa[j].w +
                    xb[j].x * xb[j].x + xb[j].y * xb[j].y + xb[j].z * xb[j].z + xb[j].w * xb[j].w;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
#pragma unroll
            for (int j = 0; j < QR; ++j) ss[j] += __shfl_xor_sync(0xffffffffu, ss[j], o);
        }
        uint8_t *qstage = smem + L::SM_KV + 2 * L::SM_KV_STAGE;     // third K/V stage
        const int sub = (lane & 1) * 8;
        auto split = [](float a, float b, uint32_t &hi, uint32_t &lo) {
            const float ha = __uint_as_float(__float_as_uint(a) & 0xFFFFE000u);
            const float hb = __uint_as_float(__float_as_uint(b) & 0xFFFFE000u);
            hi = half2_bits(__floats2half2_rn(ha, hb));
            lo = half2_bits(__floats2half2_rn(a - ha, b - hb));
        };
#pragma unroll
        for (int j = 0; j < QR; ++j) {
            const int rr = warp + 8 * j;
            const bool live = rr < p.T * GROUP;
            const float inv = rsqrtf(ss[j] / HD + p.eps);
            const float4 a = xa[j], b = xb[j];
            float x0[4] = {a.x * inv * n0.x, a.y * inv * n0.y, a.z * inv * n0.z, a.w * inv * n0.w};
            const float x1[4] = {b.x * inv * n1.x, b.y * inv * n1.y, b.z * inv * n1.z, b.w * inv * n1.w};
            rope_row(x0, rope + (live ? rr / GROUP : 0) * 32, lane, live);
            uint32_t h0, h1, g0, g1, l0, l1, m0, m1;
            split(x0[0], x0[1], h0, l0);
            split(x0[2], x0[3], h1, l1);
            split(x1[0], x1[1], g0, m0);
            split(x1[2], x1[3], g1, m1);
            const int ahi = 32 * (rr >> 4) + (rr & 15), sw = ahi & 7;
            uint8_t *hrow = qstage + ahi * 512, *lrow = hrow + 16 * 512;
            const int p0 = (((lane >> 1) ^ sw) << 4) + sub, p1 = (((16 + (lane >> 1)) ^ sw) << 4) + sub;
            *reinterpret_cast<uint2 *>(hrow + p0) = make_uint2(h0, h1);
            *reinterpret_cast<uint2 *>(hrow + p1) = make_uint2(g0, g1);
            *reinterpret_cast<uint2 *>(lrow + p0) = make_uint2(l0, l1);
            *reinterpret_cast<uint2 *>(lrow + p1) = make_uint2(m0, m1);
        }
        named_barrier(2, 256);
        {
            // Warp w: TMEM lanes 32*(w%4).., Q columns [64*(w/4), 64*(w/4)+64).
            const int arow = (warp & 3) * 32 + lane, half_cols = warp >> 2;
            const uint8_t *mine = qstage + arow * 512;
            const uint32_t qdst = tmem + ((uint32_t)((warp & 3) * 32) << 16) + TM_Q + half_cols * 64;
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                uint4 u[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    u[e] = *reinterpret_cast<const uint4 *>(mine + (((half_cols * 16 + 4 * m + e) ^ (lane & 7)) << 4));
                tmem_st16(qdst + m * 16, *reinterpret_cast<const float(*)[16]>(u));
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(q_ready);
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
    } else if (warp >= 4 && warp < 8) {
        // Stage this lane's prepared query row (256 fp16 = 128 columns) into TMEM.
        const __half *src = (PRECISE && half) ? p.q_lo : p.q;
        const uint4 *row = reinterpret_cast<const uint4 *>(src + ((size_t)t * NQ + h) * HD);
#pragma unroll 2
        for (int c = 0; c < 8; ++c) {
            uint4 u[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) u[e] = valid ? row[c * 4 + e] : make_uint4(0, 0, 0, 0);
            tmem_st16(t_lane + TM_Q + c * 16, *reinterpret_cast<const float(*)[16]>(u));
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(q_ready);
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
                // Fused decode: stage 2 holds the staged queries until they are in TMEM.
                if (PRECISE && p.fused && j == 2 && !mbar_wait(q_ready, 0, abort_flag)) break;
                mbar_expect_tx(k_full + s, TILE_BYTES);
                for (int c = 0; c < 4; ++c) tma_load_2d(kd + c * BN * 128, &tmK, k_full + s, kv_head * HD + c * 64, y);
                k_issued = j + 1;
                if (j >= STAGES3 && !mbar_wait(v_empty + s, (use - 1) & 1, abort_flag)) break;
                mbar_expect_tx(v_full + s, TILE_BYTES);
                for (int c = 0; c < 4; ++c) tma_load_2d(vd + c * BN * 128, &tmV, v_full + s, kv_head * HD + c * 64, y);
                v_issued = j + 1;
            }
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
                for (int k = 0; k < BN / 16; ++k) {
                    if (PRECISE)      // P (hi / lo rows) from shared memory
                        mma_f16_ss(tmem + TM_O, sw128_desc(pa + k * 32, 16, 1024),
                                   sw128_desc(vb + k * 16 * 128, BN * 128, 1024), idesc_pv,
                                   (i > 0 || k > 0) ? 1u : 0u);
                    else              // P written over its S tile in TMEM (fp16, 2 per column)
                        mma_f16_ts(tmem + TM_O, tmem + TM_S + b * BN + k * 8,
                                   sw128_desc(vb + k * 16 * 128, BN * 128, 1024), idesc_pv,
                                   (i > 0 || k > 0) ? 1u : 0u);
                }
                mma_commit(p_free + b);
                mma_commit(v_empty + s);
                return true;
            };
            bool ok = mbar_wait(q_ready, 0, abort_flag);
            tc_fence_after();
            for (int j = 0; j < ntiles && ok; ++j) {
                const int b = j & 1, s = j % STAGES3;
                if (!mbar_wait(k_full + s, (j / STAGES3) & 1, abort_flag)) { ok = false; break; }
                // S buffer b is reusable once the softmax has read tile j-2.  FAST:
                // implied by the p_full wait before PV(j-2) (issued above by this
                // thread), and tile j-2's P, kept in this buffer, is read by PV(j-2)
                // before this QK writes it: tcgen05.mma issued by one thread execute
                // in issue order.
                if (PRECISE && j >= 2 && !mbar_wait(s_free + b, ((j >> 1) - 1) & 1, abort_flag)) { ok = false; break; }
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
            // All MMAs of this thread must finish before TMEM is released.
            mma_commit(mma_done);
            const long long t0 = clock64();
            while (!mbar_try_wait(mma_done, 0) && clock64() - t0 < WAIT_LIMIT_CYCLES) {}
        }
    } else if (warp >= 4) {
        // ------------------------------------------------ softmax + epilogue
        // Each thread handles 32 columns of its row per tile.  FAST: warpgroup
        // wg takes columns [32 wg, 32 wg + 32); the two warpgroups agree on the
        // row maximum through a shared-memory exchange (an mbarrier per S
        // buffer) and keep separate row sums, added after the last tile.
        // PRECISE: lane i keeps columns [0,32) and lane i+16 columns [32,64) of
        // row 16w+i, each summing the hi and lo score halves, and each writes
        // the hi and lo probabilities of its columns.
        constexpr int NC = 32;                                     // columns per thread
        const int cpart = PRECISE ? half : wg;                     // which 32 columns
        float *xch = reinterpret_cast<float *>(smem + L::SM_ROPE);  // FAST: [2 buffers][2 wg][128 rows]
        const int pos_limit = valid ? p.position + t - p.kv_begin : -1;   // last visible local row
        const int arow_hi = PRECISE ? wq * 32 + (lane & 15) : r;         // A rows of P (hi, lo)
        const int arow_lo = arow_hi + 16;
        float m_use = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < ntiles; ++j) {
            const int b = j & 1;
            if (!warp_wait(s_full + b, (j >> 1) & 1, abort_flag)) { ok = false; break; }
            tc_fence_after();
            float x[64];
            if (PRECISE) {
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    tmem_ld16(t_lane + TM_S + b * BN + c * 16, *reinterpret_cast<float(*)[16]>(x + c * 16));
            } else {
#pragma unroll
                for (int c = 0; c < 2; ++c)
                    tmem_ld16(t_lane + TM_S + b * BN + wg * 32 + c * 16, *reinterpret_cast<float(*)[16]>(x + c * 16));
            }
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free + b);
            if (PRECISE) {
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const float recv = __shfl_xor_sync(0xffffffffu, half ? x[c] : x[32 + c], 16);
                    x[c] = (half ? x[32 + c] : x[c]) + recv;
                }
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
            if (PRECISE) {
                m_tile = fmaxf(m_tile, __shfl_xor_sync(0xffffffffu, m_tile, 16));
            } else {
                xch[(b * 2 + wg) * 128 + r] = m_tile;
                __syncwarp();
                if (lane == 0) mbar_arrive(xbar + b);
                if (!warp_wait(xbar + b, (j >> 1) & 1, abort_flag)) { ok = false; break; }
                m_tile = fmaxf(m_tile, xch[(b * 2 + (wg ^ 1)) * 128 + r]);
            }
            m_tile *= SCORE_LOG2;                                  // log2 units (-inf stays -inf)
            float factor = 1.f;
            const bool need = m_tile > m_use + RESCALE_THRESHOLD;
            if (need) { factor = exp2_approx(m_use - m_tile); m_use = m_tile; l *= factor; }
            if (j > 0 && __any_sync(0xffffffffu, need)) {
                // O already holds tiles < j: wait for PV(j-1), then rescale rows in
                // TMEM (FAST: each warpgroup its half of the columns).
                if (!warp_wait(p_free + ((j - 1) & 1), ((j - 1) >> 1) & 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                constexpr int CH = PRECISE ? HD / 16 : HD / 32;
#pragma unroll 1
                for (int c = wg * CH; c < wg * CH + CH; ++c) {
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
            uint32_t hi[NC / 2], lo[PRECISE ? NC / 2 : 1];
            float sp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < NC; c += 2) {
                const float p0 = exp2_approx(fmaf(x[c], SCORE_LOG2, -mref));
                const float p1 = exp2_approx(fmaf(x[c + 1], SCORE_LOG2, -mref));
                const __half2 hp = __floats2half2_rn(p0, p1);
                hi[c / 2] = *reinterpret_cast<const uint32_t *>(&hp);
                if (PRECISE) {
                    const float2 back = __half22float2(hp);
                    const __half2 lp = __floats2half2_rn(p0 - back.x, p1 - back.y);
                    lo[c / 2] = *reinterpret_cast<const uint32_t *>(&lp);
                }
                sp[(c >> 1) & 3] += p0 + p1;
            }
            l += (sp[0] + sp[1]) + (sp[2] + sp[3]);
            if (PRECISE) {
                if (j >= 2 && !warp_wait(p_free + b, ((j - 2) >> 1) & 1, abort_flag)) { ok = false; break; }
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
            } else {
                // fp16 P of columns [32 wg, 32 wg + 32) into TMEM columns [16 wg, 16 wg + 16)
                // of this S buffer: S columns both warpgroups have read (they passed
                // the exchange), and which the QK MMA rewrites only after this
                // tile's PV (issued earlier by the same thread) has consumed them.
                tmem_st16(t_lane + TM_S + b * BN + wg * 16, *reinterpret_cast<const float(*)[16]>(hi));
                tmem_wait_st();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full + b);
        }
        if (PRECISE) l += __shfl_xor_sync(0xffffffffu, l, 16);
        if (!PRECISE) {
            // Warpgroup 1 hands its row sums to warpgroup 0, which writes the output.
            float *lx = xch + (ntiles & 1) * 256;     // the exchange buffer no tile still reads
            if (wg == 1) {
                lx[r] = l;
                __syncwarp();
                if (lane == 0) mbar_arrive(lbar);
                ok = false;                            // the epilogue is warpgroup 0's
            } else if (ok && warp_wait(lbar, 0, abort_flag)) {
                l += lx[r];
            } else {
                ok = false;
            }
        }
        // Epilogue: the final PV's commit on p_free marks O complete (and every
        // K/V tile consumed, so the ring is idle).  O leaves through shared
        // memory: every lane puts its TMEM lane (PRECISE: O_hi in lanes i,
        // O_lo in lanes 16+i) into a padded staging row, then the warp stores
        // each output row (the sum of its hi and lo rows) as 512-byte pieces.
        if (ok && ntiles > 0 && warp_wait(p_free + ((ntiles - 1) & 1), ((ntiles - 1) >> 1) & 1, abort_flag)) {
            tc_fence_after();
            constexpr int WROWS = PRECISE ? 16 : 32;               // logical rows of this warp
            constexpr int RSTRIDE = HD * 4 + 16;                   // staging row bytes (padded)
            static_assert(4 * 32 * RSTRIDE <= STAGES3 * L::SM_KV_STAGE, "O staging exceeds the K/V ring");
            uint8_t *stage = smem + L::SM_KV + wq * 32 * RSTRIDE;
            const float inv = p.direct ? (l > 0.f ? 1.f / l : 0.f) : 1.f;
            if (valid && (!PRECISE || half == 0)) {
                if (p.direct) {
                    if (p.lse) p.lse[(size_t)t * NQ + h] = l > 0.f ? (m_use + log2f(l)) * 0.6931471805599453f : -INFINITY;
                } else {
                    const size_t slot = ((size_t)kv_head * p.splits + blockIdx.x) * DECODE_ROWS + r;
                    p.part_ml[slot * 2] = m_use;
                    p.part_ml[slot * 2 + 1] = l;
                }
            }
            uint8_t *myrow = stage + lane * RSTRIDE;
#pragma unroll 1
            for (int c4 = 0; c4 < HD / 64; ++c4) {                 // 64 columns per TMEM round trip
                float o[4][16];
#pragma unroll
                for (int q = 0; q < 4; ++q) tmem_ld16(t_lane + TM_O + c4 * 64 + q * 16, o[q]);
                tmem_wait_ld();
#pragma unroll
                for (int q = 0; q < 4; ++q)
#pragma unroll
                    for (int e = 0; e < 16; e += 4)
                        *reinterpret_cast<float4 *>(myrow + (c4 * 64 + q * 16 + e) * 4) =
                            make_float4(o[q][e] * inv, o[q][e + 1] * inv, o[q][e + 2] * inv, o[q][e + 3] * inv);
            }
            __syncwarp();
            // The valid logical rows of a CTA are a prefix, so are this warp's.
            const int row0 = PRECISE ? wq * 16 : wq * 32;
            const int nvalid = max(0, min(WROWS, (p.mode == 0 ? p.T * GROUP
                                                              : p.T - (int)(gridDim.y - 1 - blockIdx.y) * QROWS) - row0));
#pragma unroll 4
            for (int i = 0; i < nvalid; ++i) {
                const int rr = row0 + i;
                int tt, hh;
                row_token_head<QROWS>(p, rr, tt, hh);
                float *dst = p.direct ? p.out + ((size_t)tt * NQ + hh) * HD
                                      : p.part_o + (((size_t)kv_head * p.splits + blockIdx.x) * DECODE_ROWS + rr) * HD;
                const float *gate = p.direct && p.q_gate ? p.q_gate + ((size_t)tt * NQ + hh) * 2 * HD + HD : nullptr;
#pragma unroll
                for (int part = 0; part < 2; ++part) {
                    const int col = part * 128 + 4 * lane;
                    float4 v = *reinterpret_cast<const float4 *>(stage + i * RSTRIDE + col * 4);
                    if (PRECISE) {
                        const float4 w = *reinterpret_cast<const float4 *>(stage + (i + 16) * RSTRIDE + col * 4);
                        v.x += w.x; v.y += w.y; v.z += w.z; v.w += w.w;
                    }
                    if (gate) {
                        const float4 g = *reinterpret_cast<const float4 *>(gate + col);
                        v.x *= sigmoidf_(g.x); v.y *= sigmoidf_(g.y);
                        v.z *= sigmoidf_(g.z); v.w *= sigmoidf_(g.w);
                    }
                    *reinterpret_cast<float4 *>(dst + col) = v;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------- prepare
// One block per (head, token): 24 query heads then 4 key heads.  RMSNorm with
// weight, rotary embedding on dims [0,64) as pairs (i, i+32) with angle
// (position+t) * 1e7^(-i/32) evaluated in double precision, queries written
// as fp16 operand rows, keys/values rounded to fp16 into the cache.  Used by
// the prefill regime; decode batches fold this step into fa_kernel.
__global__ void __launch_bounds__(256)
attn_prepare_kernel(const float *q_gate, const float *key, const float *value, const float *qn,
                    const float *kn, __half *qw, __half *qw_lo, __half *kc, __half *vc, int position,
                    int append_row0, float eps) {
    const int t = blockIdx.x, h = blockIdx.y, i = threadIdx.x;
    const bool isq = h < NQ;
    const int kh = h - NQ;
    grid_dependency_wait();
    launch_dependents();
    const float *src = isq ? q_gate + ((size_t)t * NQ + h) * 2 * HD : key + ((size_t)t * NKV + kh) * HD;
    __shared__ float row[HD], red[8];
    const float x = src[i];
    float ss = warp_sum(x * x);
    if ((i & 31) == 0) red[i >> 5] = ss;
    __syncthreads();
    ss = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) ss += red[w];
    const float inv = rsqrtf(ss / HD + eps);
    row[i] = x * inv * (isq ? qn : kn)[i];
    __syncthreads();
    if (i < 32) {
        const float2 cs = rope_angle(position + t, i);
        const float c = cs.x, s = cs.y, a = row[i], b = row[i + 32];
        row[i] = a * c - b * s;
        row[i + 32] = a * s + b * c;
    }
    __syncthreads();
    if (isq) {
        const __half hi = __float2half_rn(row[i]);
        qw[((size_t)t * NQ + h) * HD + i] = hi;
        if (qw_lo) qw_lo[((size_t)t * NQ + h) * HD + i] = __float2half_rn(row[i] - __half2float(hi));
    } else if (append_row0 >= 0) {
        const size_t o = ((size_t)(append_row0 + t) * NKV + kh) * HD + i;
        kc[o] = __float2half_rn(row[i]);
        vc[o] = __float2half_rn(value[((size_t)t * NKV + kh) * HD + i]);
    }
}

// ---------------------------------------------------------------- combine
// Merge the split partials of one (token, head) row: weights from the
// per-split (max, sum) are formed once in shared memory, then each thread
// (one output dimension) streams the splits with 8 independent loads in
// flight.  final_gate 1: gated output; 0: normalised partial + natural-log LSE.
constexpr int MAX_SPLITS = 64;
__global__ void __launch_bounds__(256)
attn_combine_kernel(float *out, float *out_lse, const float *part_o, const float *part_ml,
                    const float *q_gate, int splits, int final_gate) {
    const int t = blockIdx.x / NQ, h = blockIdx.x % NQ, d = threadIdx.x;
    const int g = h / GROUP, r = t * GROUP + h % GROUP;
    __shared__ float wgt[MAX_SPLITS], red[2], den_s;
    const size_t slot0 = (size_t)g * splits * DECODE_ROWS + r;     // slot(s) = slot0 + s*DECODE_ROWS
    grid_dependency_wait();
    launch_dependents();
    // Every split's value and (max, sum) are loaded before any is used: one
    // memory round trip.
    const float *src = part_o + slot0 * HD + d;
    float v[MAX_SPLITS];
#pragma unroll
    for (int e = 0; e < MAX_SPLITS; ++e) v[e] = e < splits ? src[(size_t)e * DECODE_ROWS * HD] : 0.f;
    float m = -INFINITY, l = 0.f;
    if (d < splits) {
        const float2 ml = *reinterpret_cast<const float2 *>(part_ml + (slot0 + (size_t)d * DECODE_ROWS) * 2);
        m = ml.x; l = ml.y;
    }
    float M = m;
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    if (d < 64 && (d & 31) == 0) red[d >> 5] = M;
    __syncthreads();
    M = fmaxf(red[0], red[1]);
    const float w = (d < splits && m != -INFINITY) ? exp2f(m - M) : 0.f;
    if (d < MAX_SPLITS) wgt[d] = w;     // zero for d >= splits
    float den = w * l;
#pragma unroll
    for (int o = 16; o; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    __syncthreads();
    if (d < 64 && (d & 31) == 0) red[d >> 5] = den;
    __syncthreads();
    if (d == 0) den_s = red[0] + red[1];
    __syncthreads();
    den = den_s;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int e = 0; e < MAX_SPLITS; ++e) acc[e & 3] += wgt[e] * v[e];
    const float num = (acc[0] + acc[1]) + (acc[2] + acc[3]);
    const size_t o = ((size_t)t * NQ + h) * HD + d;
    if (final_gate) {
        out[o] = (den > 0.f ? num / den : 0.f) * sigmoidf_(q_gate[((size_t)t * NQ + h) * 2 * HD + HD + d]);
    } else {
        out[o] = den > 0.f ? num / den : 0.f;
        if (d == 0) out_lse[(size_t)t * NQ + h] = den > 0.f ? (M + log2f(den)) * 0.6931471805599453f : -INFINITY;
    }
}

// ---------------------------------------------------------------- fused shard exchange
// Multi-GPU verify: one CTA per (token, head) row combines this shard's split
// partials of the row, stores the normalised partial and its LSE into slot
// [rank] of every other rank's receive buffer (peer memory over NVLink), then
// reads the other ranks' partials of the row from its own buffer and merges
// them (O = sum_g exp(lse_g - LSE) O_g, times sigmoid(gate)).
//
// Every value travels as a 64-bit word {value bits, tag}: the reader spins on
// each of its words until the tag of this call appears, so no fence or
// separate flag write is needed, and it zeroes each word after reading it.
// Receive buffer of each rank: [2 slots][world][EX_ROWS][EX_WORDS] words (256
// O, lse, padding).  `seq` counts the calls on these buffers (the same on
// every rank, +1 per call): its parity picks the slot and its low 24 bits are
// in the tag.  A rank writes into a slot again two calls later, after it has
// received this rank's partials of the call in between, and that call started
// only after this one (and its zeroing) completed.  A word that arrives after
// its reader gave up (a timeout) stays behind unread, but it carries the tag
// of its own call and the next call on that slot waits for a different tag,
// so it is never taken for new data.  The CTAs of one launch hold no shared
// memory to speak of, so all of them are resident at once and every awaited
// word has a running writer on its rank.
constexpr int EX_ROWS = MAX_DECODE_T * NQ;       // rows of the largest decode batch
constexpr int EX_WORDS = 264;                    // words per row: 256 O + lse, padded to 64 bytes
constexpr int EX_MAX_WORLD = 8;
__host__ __device__ constexpr uint32_t ex_tag(int seq) {   // high half of a filled word; never 0
    return 0x51000000u | ((uint32_t)seq & 0x00FFFFFFu);
}
__host__ __device__ constexpr size_t ex_bytes(int world) {
    return (size_t)2 * world * EX_ROWS * EX_WORDS * sizeof(uint64_t);
}

__global__ void __launch_bounds__(256)
attn_exchange_kernel(float *out, const float *part_o, const float *part_ml, int splits, const float *q_gate,
                     const uint64_t *peers, int world, int rank, int seq) {
    const int d = threadIdx.x, row = blockIdx.x, slot = seq & 1;
    const uint32_t tag32 = ex_tag(seq);
    const int t = row / NQ, h = row % NQ, g = h / GROUP, r = t * GROUP + h % GROUP;
    __shared__ float wgt[MAX_SPLITS], red[2], den_s, lse_s[EX_MAX_WORLD];
    grid_dependency_wait();
    launch_dependents();
    // ---- this shard's partial of the row (split combine, one round trip)
    const size_t slot0 = (size_t)g * splits * DECODE_ROWS + r;
    const float *src = part_o + slot0 * HD + d;
    float v[MAX_SPLITS];
#pragma unroll
    for (int e = 0; e < MAX_SPLITS; ++e) v[e] = e < splits ? src[(size_t)e * DECODE_ROWS * HD] : 0.f;
    float m = -INFINITY, l = 0.f;
    if (d < splits) {
        const float2 ml = *reinterpret_cast<const float2 *>(part_ml + (slot0 + (size_t)d * DECODE_ROWS) * 2);
        m = ml.x; l = ml.y;
    }
    float M = m;
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    if (d < 64 && (d & 31) == 0) red[d >> 5] = M;
    __syncthreads();
    M = fmaxf(red[0], red[1]);
    const float w = (d < splits && m != -INFINITY) ? exp2f(m - M) : 0.f;
    if (d < MAX_SPLITS) wgt[d] = w;
    float den = w * l;
#pragma unroll
    for (int o = 16; o; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    __syncthreads();
    if (d < 64 && (d & 31) == 0) red[d >> 5] = den;
    __syncthreads();
    if (d == 0) den_s = red[0] + red[1];
    __syncthreads();
    den = den_s;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int e = 0; e < MAX_SPLITS; ++e) acc[e & 3] += wgt[e] * v[e];
    const float o = den > 0.f ? ((acc[0] + acc[1]) + (acc[2] + acc[3])) / den : 0.f;
    const float lse = den > 0.f ? (M + log2f(den)) * 0.6931471805599453f : -INFINITY;

    // ---- push it to every other rank
    const uint64_t tag = (uint64_t)tag32 << 32;
    for (int q = 0; q < world; ++q) {
        if (q == rank) continue;
        uint64_t *dst = reinterpret_cast<uint64_t *>(peers[q]) +
                        (((size_t)slot * world + rank) * EX_ROWS + row) * EX_WORDS;
        st_word_sys(dst + d, tag | __float_as_uint(o));
        if (d == 0) st_word_sys(dst + HD, tag | __float_as_uint(lse));
    }

    // ---- receive the other ranks' partials of the row and merge.  The words of
    //      all peers are read at once, so their latencies overlap; a word whose
    //      flag is not there yet is re-read until it is (bounded).
    uint64_t *own = reinterpret_cast<uint64_t *>(peers[rank]);
    const long long t0 = clock64();
    bool ok = true;
    auto finish = [&](uint64_t *word, uint64_t x, float fallback) {
        while ((uint32_t)(x >> 32) != tag32) {
            if (clock64() - t0 > WAIT_LIMIT_CYCLES) { raise_status(STATUS_TIMEOUT); ok = false; return fallback; }
            x = ld_word_sys(word);
        }
        *word = 0;
        return __uint_as_float((uint32_t)x);
    };
    auto word_of = [&](int q, int col) {
        return own + (((size_t)slot * world + q) * EX_ROWS + row) * EX_WORDS + col;
    };
    uint64_t first[EX_MAX_WORLD], lse_first = 0;
    const bool lse_reader = d < world && d != rank;
    if (lse_reader) lse_first = ld_word_sys(word_of(d, HD));
#pragma unroll
    for (int q = 0; q < EX_MAX_WORLD; ++q)
        first[q] = (q < world && q != rank) ? ld_word_sys(word_of(q, d)) : 0;
    if (d < world) {
        float x = lse;
        if (lse_reader) x = finish(word_of(d, HD), lse_first, x);
        lse_s[d] = x;
    }
    float val[EX_MAX_WORLD];
#pragma unroll
    for (int q = 0; q < EX_MAX_WORLD; ++q) {
        val[q] = 0.f;
        if (q < world) {
            if (q == rank) val[q] = o;
            else val[q] = finish(word_of(q, d), first[q], 0.f);
        }
    }
    const int all_ok = __syncthreads_and(ok);
    float res = 0.f;
    if (all_ok) {
        float Mx = -INFINITY;
        for (int q = 0; q < world; ++q) Mx = fmaxf(Mx, lse_s[q]);
        float num = 0.f, dsum = 0.f;
        if (Mx != -INFINITY) {
#pragma unroll
            for (int q = 0; q < EX_MAX_WORLD; ++q) {
                if (q >= world || lse_s[q] == -INFINITY) continue;
                const float wq = expf(lse_s[q] - Mx);
                dsum += wq;
                num += wq * val[q];
            }
        }
        res = dsum > 0.f ? num / dsum : 0.f;
    }
    out[((size_t)t * NQ + h) * HD + d] = res * sigmoidf_(q_gate[((size_t)t * NQ + h) * 2 * HD + HD + d]);
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

void check_launch(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// The shared-memory limit of a kernel is a per-device attribute: set it on
// every device the process launches on.
PerDeviceOnce g_configured;
void configure() {
    g_configured.run([] {
        if (cudaFuncSetAttribute(fa_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 FaLayout<true>::SMEM_BYTES) != cudaSuccess ||
            cudaFuncSetAttribute(fa_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 FaLayout<false>::SMEM_BYTES) != cudaSuccess)
            throw std::runtime_error("cannot reserve shared memory for the attention kernel");
    });
}

struct Split { int tiles, splits; };
// Split-KV plan: about 37 CTAs per KV head (148 SMs / 4 heads), whole tiles
// per split.  The plan depends only on the cache length.
Split decode_split(int kv_rows) {
    const int total = (kv_rows + BN - 1) / BN;
    const int per = (total + 36) / 37;
    static_assert(37 <= MAX_SPLITS, "combine kernel handles up to MAX_SPLITS splits");
    return {per, (total + per - 1) / per};
}
size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
bool decode_regime(int T) { return T * GROUP <= DECODE_ROWS; }

template <bool PRECISE>
void launch_fa(const CUtensorMap &mk, const CUtensorMap &mv, const FaParams &p, dim3 grid, cudaStream_t st) {
    const cudaError_t e = launch_chained(fa_kernel<PRECISE>, grid, dim3(PRECISE ? 256 : 384), FaLayout<PRECISE>::SMEM_BYTES, st,
                                         mk, mv, p);
    if (e != cudaSuccess) throw std::runtime_error(std::string("attention kernel launch: ") + cudaGetErrorString(e));
}

// Split partials of a decode / verify launch inside the workspace.
struct DecodeParts { float *o, *ml; };
size_t decode_parts_bytes(const Split &sp) {
    return align256((size_t)NKV * sp.splits * DECODE_ROWS * HD * sizeof(float)) +
           align256((size_t)NKV * sp.splits * DECODE_ROWS * 2 * sizeof(float));
}
DecodeParts decode_parts(void *ws, const Split &sp) {
    float *o = static_cast<float *>(ws);
    float *ml = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(ws) +
                                          align256((size_t)NKV * sp.splits * DECODE_ROWS * HD * sizeof(float)));
    return {o, ml};
}

// Split-KV decode / verify with the prepare step folded in: one launch
// normalises and rotates the queries, appends the new keys / values (when
// `append`) and writes the split partials of every (token, head) row.
Split launch_decode(__half *kc, __half *vc, const float *q_gate, const float *key, const float *value,
                    const float *qn, const float *kn, int T, int position, int kv_begin, int kv_rows, bool append,
                    float eps, const DecodeParts &parts, cudaStream_t st) {
    configure();
    const CUtensorMap mk = cache_map(kc, kv_rows), mv = cache_map(vc, kv_rows);
    const Split sp = decode_split(kv_rows);
    FaParams p{};
    p.q_gate = q_gate; p.T = T; p.position = position; p.kv_begin = kv_begin; p.kv_rows = kv_rows;
    p.mode = 0; p.split_tiles = sp.tiles; p.splits = sp.splits; p.direct = 0;
    p.part_o = parts.o; p.part_ml = parts.ml;
    p.fused = 1; p.key = key; p.value = value; p.qn = qn; p.kn = kn; p.kc = kc; p.vc = vc;
    p.append_row0 = append ? position - kv_begin : -1; p.eps = eps;
    launch_fa<true>(mk, mv, p, dim3(sp.splits, NKV), st);
    return sp;
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
// Decode / verify batches (T <= 10) use the split-KV regime (one fused
// launch + the split combine); longer blocks use the prefill regime with 64
// query rows per CTA after a prepare launch; both are PRECISE.
void attention_run(float *out, float *shard_lse, __half *kc, __half *vc, const float *q_gate,
                   const float *key, const float *value, const float *qn, const float *kn, int T,
                   int position, int kv_begin, int kv_rows, bool append, float eps, void *ws,
                   size_t ws_bytes, cudaStream_t st) {
    if (ws_bytes < attention_workspace_bytes(T, kv_rows)) throw std::invalid_argument("attention workspace too small");
    if (decode_regime(T)) {
        const DecodeParts parts = decode_parts(ws, decode_split(kv_rows));
        const Split sp = launch_decode(kc, vc, q_gate, key, value, qn, kn, T, position, kv_begin, kv_rows, append,
                                       eps, parts, st);
        const cudaError_t e = launch_chained(attn_combine_kernel, dim3(T * NQ), dim3(256), 0, st, out, shard_lse,
                                             parts.o, parts.ml, q_gate, sp.splits, shard_lse ? 0 : 1);
        if (e != cudaSuccess) throw std::runtime_error(std::string("attention combine: ") + cudaGetErrorString(e));
        return;
    }
    if (shard_lse) throw std::invalid_argument("shard partials are limited to decode batches");
    configure();
    uint8_t *w = static_cast<uint8_t *>(ws);
    const size_t q_bytes = align256((size_t)T * NQ * HD * sizeof(__half));
    __half *qw = reinterpret_cast<__half *>(w), *qw_lo = reinterpret_cast<__half *>(w + q_bytes);
    const cudaError_t e = launch_chained(attn_prepare_kernel, dim3(T, NQ + NKV), dim3(256), 0, st, q_gate, key, value,
                                         qn, kn, qw, qw_lo, kc, vc, position, append ? position - kv_begin : -1, eps);
    if (e != cudaSuccess) throw std::runtime_error(std::string("attention prepare: ") + cudaGetErrorString(e));
    const CUtensorMap mk = cache_map(kc, kv_rows), mv = cache_map(vc, kv_rows);
    FaParams p{};
    p.q = qw; p.q_lo = qw_lo; p.q_gate = q_gate; p.T = T; p.position = position;
    p.kv_begin = kv_begin; p.kv_rows = kv_rows;
    p.mode = 1; p.direct = 1; p.out = out; p.splits = 1;
    constexpr int R = FaLayout<true>::QROWS;
    launch_fa<true>(mk, mv, p, dim3(NQ, (T + R - 1) / R), st);
}

size_t attention_exchange_bytes(int world) { return ex_bytes(world); }
int attention_exchange_max_world() { return EX_MAX_WORLD; }

// Shard attention + fused all-to-all exchange + merge (see attn_exchange_kernel).
void attention_shard_exchange(float *out, __half *kc, __half *vc, const float *q_gate, const float *key,
                              const float *value, const float *qn, const float *kn, int T, int position,
                              int kv_begin, int kv_rows, bool append, float eps, const uint64_t *peers,
                              int world, int rank, int seq, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (!decode_regime(T)) throw std::invalid_argument("the exchange supports decode batches only");
    if (world < 1 || world > EX_MAX_WORLD || rank < 0 || rank >= world || seq < 0)
        throw std::invalid_argument("invalid exchange group");
    if (ws_bytes < attention_workspace_bytes(T, kv_rows)) throw std::invalid_argument("attention workspace too small");
    const DecodeParts parts = decode_parts(ws, decode_split(kv_rows));
    const Split sp = launch_decode(kc, vc, q_gate, key, value, qn, kn, T, position, kv_begin, kv_rows, append, eps,
                                   parts, st);
    const cudaError_t e = launch_chained(attn_exchange_kernel, dim3(T * NQ), dim3(256), 0, st, out, parts.o, parts.ml,
                                         sp.splits, q_gate, peers, world, rank, seq);
    if (e != cudaSuccess) throw std::runtime_error(std::string("attention exchange: ") + cudaGetErrorString(e));
}

void attention_merge(float *out, const float *parts, const float *lses, int shards, int T,
                     const float *q_gate, cudaStream_t st) {
    const cudaError_t e = launch_chained(attn_merge_kernel, dim3(T * NQ), dim3(256), 0, st, out, parts, lses, shards,
                                         T, q_gate);
    if (e != cudaSuccess) throw std::runtime_error(std::string("attention merge: ") + cudaGetErrorString(e));
}

// Core-level causal prefill on already-prepared fp16 queries (no norm, RoPE
// or gate): out [T][24][256] = softmax(q.k/16, causal) v, optional LSE.
// FAST mode: 128 query rows per CTA, fp16 probabilities.
void prefill_core(float *out, float *lse, const __half *q, const __half *kc, const __half *vc, int T,
                  int position, cudaStream_t st) {
    configure();
    const int kv_rows = position + T;
    const CUtensorMap mk = cache_map(kc, kv_rows), mv = cache_map(vc, kv_rows);
    FaParams p{};
    p.q = q; p.T = T; p.position = position; p.kv_begin = 0; p.kv_rows = kv_rows;
    p.mode = 1; p.direct = 1; p.out = out; p.lse = lse; p.splits = 1;
    constexpr int R = FaLayout<false>::QROWS;
    launch_fa<false>(mk, mv, p, dim3(NQ, (T + R - 1) / R), st);
    check_launch("prefill attention");
}

}  // namespace qv
