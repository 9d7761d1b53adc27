// Chunked gated-DeltaNet prefill on tcgen05 (chunk C = 64 tokens, D = 128).
//
// Same semantics as the token recurrence (cpu_reference.py:35-47 and the
// reference's k_gdn_scan, src/kernels.cu:331-349): per value head h (key head
// h % Hk), with k^ = k/|k|, q^ = q/(|q| sqrt(D)), a_t = exp(decay*softplus(
// alpha_t + bias)) and beta_t = sigmoid(beta_t),
//     S_t = a_t S_{t-1} + d_t k^_t^T,  d_t = beta_t (v_t - a_t S_{t-1} k^_t),
//     o_t = S_t q^_t.
// Over a chunk with state S_0 at its start, g_t = a_1 ... a_t (inside the
// chunk) and G(t,s) = g_t / g_s, the recurrence is linear in the d's:
//     (I + B) d = beta (v - g S_0 k^),  B_ts = beta_t G(t,s) (k^_t.k^_s), s < t,
// so with T = (I + B)^-1 diag(beta) (the WY / UT transform):
//     U = T V,  W = T diag(g) K^,  Delta = U - W S_0^T,
//     O = diag(g) Q^ S_0^T + Mq Delta,  Mq_ts = G(t,s) (q^_t.k^_s), s <= t,
//     S_C = g_C S_0 + Delta^T diag(g_C / g) K^.
//
// Two kernels:
//  * gdn_prep_kernel, one CTA per (chunk, value head), all chunks in
//    parallel: normalised K^, Q^ in shared memory, K^K^^T and Q^K^^T in one
//    M=128 tcgen05 MMA, the masked / decayed matrices on CUDA cores, T by
//    forward substitution (each thread pair owns one column), and the per-
//    token scale factors.  Writes T (fp16 hi + lo), T diag(g/|k|) (fp16), Mq
//    (fp16) and the scales to the workspace.
//  * gdn_scan_kernel, one CTA per (value head, half of the state's rows),
//    sequential over chunks: every chunk's operands arrive by TMA one chunk
//    ahead; U, W and Q S^T, then Delta, then Mq Delta and the rank-64 state
//    update are M=64 tcgen05 MMAs with fp32 accumulators in TMEM; the state
//    stays in TMEM (fp32) for the whole prefill and is rounded to fp16 only
//    as an MMA operand.  The raw fp16 K and Q tiles are the MMA operands
//    directly: the per-token normalisations and decays are folded into T
//    diag(g/|k|), into the output row scale and into the Delta operand of
//    the state update.
// Operand precision (fp32 accumulation throughout): T and the state-update
// Delta are split into fp16 hi + lo; the rest is fp16.  Against the fp64
// recurrence this keeps the state within ~3e-4 (max-relative) over 4096
// tokens.
#include "common.cuh"
#include "hotpath.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdexcept>
#include <string>

namespace qv {

namespace {
constexpr int GC = 64;                 // tokens per chunk
constexpr int GD = 128;                // key / value head dimension
constexpr int TILE = GC * GC * 2;      // one 64x64 fp16 tile (8 KB)

struct GdnPrep {
    const __half *q, *k;               // [L][Hk][128]
    const float *alpha, *beta;         // [L][Hv] raw
    const float *decay, *bias;         // [Hv]
    __half *tt_hi, *tt_lo, *ttp, *mq;  // [Hv][nch][64][64]
    float *sc;                         // [Hv][nch][64][4]
    int L, Hk, Hv, nch;
};

// Byte offset of element `col` (a multiple of 4) of row `row` in a K-major,
// 128-byte-swizzled operand of `rows` rows: 64-element blocks of rows x 128 B,
// 16-byte chunks XOR-swizzled by the row's low 3 bits.
__device__ __forceinline__ uint32_t sw_off(int rows, int row, int col) {
    const int blk = col >> 6, within = col & 63;
    return (uint32_t)(blk * rows * 128 + row * 128 + ((((within >> 3) ^ (row & 7))) << 4) + (within & 7) * 2);
}

__device__ __forceinline__ uint2 pack4(float a, float b, float c, float d) {
    __half2 x = __floats2half2_rn(a, b), y = __floats2half2_rn(c, d);
    return make_uint2(*reinterpret_cast<uint32_t *>(&x), *reinterpret_cast<uint32_t *>(&y));
}

// ------------------------------------------------------------------ prep
constexpr int PREP_SA = 0;                       // A: [2 blocks][128 rows][128 B] (K^ rows 0-63, Q^ rows 64-127)
constexpr int PREP_SB = 32768;                   // B: [2 blocks][64 rows][128 B] (K^)
constexpr int PREP_BM = 49152;                   // fp32 [64][65]
constexpr int PREP_SMALL = PREP_BM + 64 * 65 * 4;
constexpr int PREP_SMEM = PREP_SMALL + 4 * 64 * 4 + 64;

__global__ void __launch_bounds__(128) gdn_prep_kernel(const GdnPrep p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    if (smem_addr(smem) & 1023) {
        if (threadIdx.x == 0) raise_status(STATUS_BAD_ARGUMENT);
        return;
    }
    uint8_t *sa = smem + PREP_SA, *sb = smem + PREP_SB;
    float *bm = reinterpret_cast<float *>(smem + PREP_BM);
    float *gam = reinterpret_cast<float *>(smem + PREP_SMALL), *bet = gam + 64, *ik = bet + 64, *iq = ik + 64;
    uint64_t *bar = reinterpret_cast<uint64_t *>(iq + 64);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bar + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(bar + 2);
    const int c = blockIdx.x, h = blockIdx.y, kh = h % p.Hk;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = c * GC, n = min(GC, p.L - t0);
    if (tid == 0) { mbar_init(bar, 1); *abort_flag = 0; fence_barrier_init(); }
    if (warp == 0) { tmem_alloc(tslot, 64); tmem_relinquish(); }
    grid_dependency_wait();
    if (tid == 0) launch_dependents();

    // (1) normalised keys / queries as fp16 MMA operands
    for (int i = 0; i < 16; ++i) {
        const int t = warp * 16 + i;
        uint2 kr = make_uint2(0, 0), qr = make_uint2(0, 0);
        if (t < n) {
            kr = *reinterpret_cast<const uint2 *>(p.k + ((size_t)(t0 + t) * p.Hk + kh) * GD + 4 * lane);
            qr = *reinterpret_cast<const uint2 *>(p.q + ((size_t)(t0 + t) * p.Hk + kh) * GD + 4 * lane);
        }
        const float2 k01 = __half22float2(*reinterpret_cast<__half2 *>(&kr.x));
        const float2 k23 = __half22float2(*reinterpret_cast<__half2 *>(&kr.y));
        const float2 q01 = __half22float2(*reinterpret_cast<__half2 *>(&qr.x));
        const float2 q23 = __half22float2(*reinterpret_cast<__half2 *>(&qr.y));
        const float sk = warp_sum(k01.x * k01.x + k01.y * k01.y + k23.x * k23.x + k23.y * k23.y);
        const float sq = warp_sum(q01.x * q01.x + q01.y * q01.y + q23.x * q23.x + q23.y * q23.y);
        const float rk = rsqrtf(sk + 1e-6f), rq = rsqrtf(sq + 1e-6f) * rsqrtf((float)GD);
        if (lane == 0) { ik[t] = rk; iq[t] = rq; }
        const uint2 kn = pack4(k01.x * rk, k01.y * rk, k23.x * rk, k23.y * rk);
        const uint2 qn = pack4(q01.x * rq, q01.y * rq, q23.x * rq, q23.y * rq);
        *reinterpret_cast<uint2 *>(sa + sw_off(128, t, 4 * lane)) = kn;
        *reinterpret_cast<uint2 *>(sa + sw_off(128, 64 + t, 4 * lane)) = qn;
        *reinterpret_cast<uint2 *>(sb + sw_off(64, t, 4 * lane)) = kn;
    }
    // (2) log decays, their inclusive prefix sum over the chunk, and beta
    if (warp == 0) {
        float g[2], b[2];
        const float dh = p.decay[h], bh = p.bias[h];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int t = 2 * lane + e;
            g[e] = 0.f; b[e] = 0.f;
            if (t < n) {
                const size_t idx = (size_t)(t0 + t) * p.Hv + h;
                g[e] = dh * softplusf_(p.alpha[idx] + bh);
                b[e] = sigmoidf_(p.beta[idx]);
            }
        }
        float s = g[0] + g[1];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float u = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += u;
        }
        gam[2 * lane] = s - g[1];
        gam[2 * lane + 1] = s;
        bet[2 * lane] = b[0];
        bet[2 * lane + 1] = b[1];
    }
    fence_async_shared();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    // (3) [K^; Q^] K^^T: M=128, N=64, K=128
    if (tid == 0) {
        const uint32_t a0 = smem_addr(sa), b0 = smem_addr(sb), idesc = idesc_f16(128, 64, false, false);
#pragma unroll
        for (int k = 0; k < GD / 16; ++k)
            mma_f16_ss(tmem, sw128_desc(a0 + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024),
                       sw128_desc(b0 + (k >> 2) * 8192 + (k & 3) * 32, 16, 1024), idesc, k > 0 ? 1u : 0u);
        mma_commit(bar);
    }
    const bool ok = mbar_wait(bar, 0, abort_flag);
    tc_fence_after();
    // (4) row tid of the product: B (tid < 64) or Mq (tid >= 64)
    float x[64];
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + q4 * 16, *reinterpret_cast<float(*)[16]>(x + q4 * 16));
    tmem_wait_ld();
    const size_t unit = (size_t)h * p.nch + c;
    if (tid < 64) {
        const int t = tid;
        const float gt = gam[t], bt = bet[t];
#pragma unroll
        for (int s = 0; s < 64; ++s) bm[t * 65 + s] = s < t ? bt * expf(gt - gam[s]) * x[s] : 0.f;
    } else {
        const int t = tid - 64;
        const float gt = gam[t];
        uint4 *dst = reinterpret_cast<uint4 *>(p.mq + (unit * GC + t) * GC);
#pragma unroll
        for (int s8 = 0; s8 < 8; ++s8) {
            float m[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int s = s8 * 8 + e;
                m[e] = s <= t ? expf(gt - gam[s]) * x[s] : 0.f;
            }
            const uint2 lo = pack4(m[0], m[1], m[2], m[3]), hi = pack4(m[4], m[5], m[6], m[7]);
            dst[s8] = make_uint4(lo.x, lo.y, hi.x, hi.y);
        }
    }
    __syncthreads();

    // (5) X = (I + B)^-1 by forward substitution: thread pair (j, par) owns
    //     column j, par splits the dot products (even / odd s).
    const int j = tid >> 1, par = tid & 1;
    float xc[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) {
        float acc = 0.f;
#pragma unroll
        for (int s = 0; s < i; ++s)
            if ((s & 1) == par) acc += bm[i * 65 + s] * xc[s];
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        xc[i] = (i == j ? 1.f : 0.f) - acc;
    }
    // (6) T = X diag(beta) and T diag(g / |k|), stored transposed (row j of
    //     T^T = column j of T), half a row per thread.
    {
        const float bj = bet[j], wj = bj * expf(gam[j]) * ik[j];
        const size_t row = (unit * GC + j) * GC + 32 * par;
        uint4 *ph = reinterpret_cast<uint4 *>(p.tt_hi + row), *pl = reinterpret_cast<uint4 *>(p.tt_lo + row);
        uint4 *pp = reinterpret_cast<uint4 *>(p.ttp + row);
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
            float hv[8], lv[8], pv[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float xv = par ? xc[32 + q8 * 8 + e] : xc[q8 * 8 + e];     // compile-time indices
                const float v = xv * bj;
                const float hh = __half2float(__float2half_rn(v));
                hv[e] = hh; lv[e] = v - hh;
                pv[e] = xv * wj;
            }
            uint2 a = pack4(hv[0], hv[1], hv[2], hv[3]), b = pack4(hv[4], hv[5], hv[6], hv[7]);
            ph[q8] = make_uint4(a.x, a.y, b.x, b.y);
            a = pack4(lv[0], lv[1], lv[2], lv[3]); b = pack4(lv[4], lv[5], lv[6], lv[7]);
            pl[q8] = make_uint4(a.x, a.y, b.x, b.y);
            a = pack4(pv[0], pv[1], pv[2], pv[3]); b = pack4(pv[4], pv[5], pv[6], pv[7]);
            pp[q8] = make_uint4(a.x, a.y, b.x, b.y);
        }
    }
    // (7) per-token scales: {g_t / (|q_t| sqrt D), (g_C / g_t) / |k_t|, g_C, 0}
    if (tid < 64) {
        const int t = tid;
        const float gl = gam[n - 1];
        const float4 v = t < n ? make_float4(expf(gam[t]) * iq[t], expf(gl - gam[t]) * ik[t], expf(gl), 0.f)
                               : make_float4(0.f, 0.f, expf(gl), 0.f);
        reinterpret_cast<float4 *>(p.sc)[unit * GC + t] = v;
    }
    (void)ok;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, 64);
}

// ------------------------------------------------------------------ scan
struct GdnScan {
    float *out;                        // [L][Hv][128]
    float *state;                      // [Hv][128][128] in / out
    int L, Hv, Hk, nch;
};

// Shared memory of the scan CTA.  Per buffer: T^T hi, T^T lo, (T diag(g/|k|))^T,
// Mq (8 KB each), K and Q (two 64-dim boxes each, 16 KB), V half (8 KB) and
// the scales (1 KB).
constexpr int SB_TH = 0, SB_TL = TILE, SB_TP = 2 * TILE, SB_MQ = 3 * TILE, SB_K = 4 * TILE, SB_Q = 6 * TILE,
              SB_V = 8 * TILE, SB_SC = 9 * TILE, SB_BYTES = 9 * TILE + 1024;
constexpr int SCAN_BUF = 0;                                        // 2 buffers
constexpr int SCAN_NW = 2 * 75776;                                 // -W, K-major [64][128] (16 KB)
constexpr int SCAN_DL = SCAN_NW + 2 * TILE;                        // Delta, [tokens][Dv] (8 KB)
constexpr int SCAN_DH = SCAN_DL + TILE;                            // Delta' hi, lo (8 KB each)
constexpr int SCAN_DLO = SCAN_DH + TILE;
constexpr int SCAN_SH = SCAN_DLO + TILE;                           // S half, K-major [64][128] (16 KB)
constexpr int SCAN_BAR = SCAN_SH + 2 * TILE;
constexpr int SCAN_SMEM = SCAN_BAR + 128;
static_assert(SB_BYTES == 74752, "buffer layout");
static_assert(75776 % 1024 == 0 && 75776 >= SB_BYTES, "buffer stride");
static_assert(SCAN_SMEM <= 227 * 1024, "scan kernel shared memory");
// TMEM columns
constexpr uint32_t TU = 0, TW = 64, TO1 = 192, TO2 = 256, TS = 320;

__device__ __forceinline__ void tma2(void *dst, const CUtensorMap *m, uint64_t *bar, int x, int y) {
    tma_load_2d(dst, m, bar, x, y);
}

__global__ void __launch_bounds__(256, 1)
gdn_scan_kernel(const __grid_constant__ CUtensorMap mTh, const __grid_constant__ CUtensorMap mTl,
                const __grid_constant__ CUtensorMap mTp, const __grid_constant__ CUtensorMap mMq,
                const __grid_constant__ CUtensorMap mK, const __grid_constant__ CUtensorMap mQ,
                const __grid_constant__ CUtensorMap mV, const __grid_constant__ CUtensorMap mSc, const GdnScan p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    if (smem_addr(smem) & 1023) {
        if (threadIdx.x == 0) raise_status(STATUS_BAD_ARGUMENT);
        return;
    }
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + SCAN_BAR);
    uint64_t *full = bars, *bm1 = bars + 2, *bm3 = bars + 3, *bm5 = bars + 4;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 6);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 7);
    const int half = blockIdx.x, h = blockIdx.y, kh = h % p.Hk;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, quad = warp & 3, side = warp >> 2;
    const int row = 16 * quad + (lane & 15);          // M=64 accumulator row held by this thread
    const bool holds = lane < 16;
    const uint32_t tq = (uint32_t)(quad * 32) << 16;  // this warp's TMEM lane quarter

    if (tid == 0) {
        mbar_init(full, 1); mbar_init(full + 1, 1);
        mbar_init(bm1, 1); mbar_init(bm3, 1); mbar_init(bm5, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&mTh); prefetch_tmap(&mTl); prefetch_tmap(&mTp); prefetch_tmap(&mMq);
        prefetch_tmap(&mK); prefetch_tmap(&mQ); prefetch_tmap(&mV); prefetch_tmap(&mSc);
    }
    if (warp == 0) { tmem_alloc(tslot, 512); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    grid_dependency_wait();
    if (tid == 0) launch_dependents();

    auto issue_loads = [&](int c) {
        uint8_t *b = smem + SCAN_BUF + (c & 1) * 75776;
        uint64_t *f = full + (c & 1);
        const int unit_row = (h * p.nch + c) * GC;
        mbar_expect_tx(f, SB_BYTES);
        tma2(b + SB_TH, &mTh, f, 0, unit_row);
        tma2(b + SB_TL, &mTl, f, 0, unit_row);
        tma2(b + SB_TP, &mTp, f, 0, unit_row);
        tma2(b + SB_MQ, &mMq, f, 0, unit_row);
        tma2(b + SB_K, &mK, f, kh * GD, c * GC);
        tma2(b + SB_K + TILE, &mK, f, kh * GD + 64, c * GC);
        tma2(b + SB_Q, &mQ, f, kh * GD, c * GC);
        tma2(b + SB_Q + TILE, &mQ, f, kh * GD + 64, c * GC);
        tma2(b + SB_V, &mV, f, h * GD + half * 64, c * GC);
        tma2(b + SB_SC, &mSc, f, 0, unit_row);
    };
    if (tid == 0) issue_loads(0);

    // Initial state rows (value dims half*64 + row) into TMEM (fp32) and the
    // fp16 operand image (K-major [64][128]); this thread covers 64 columns.
    uint8_t *sh = smem + SCAN_SH;
    float *srow = p.state + ((size_t)h * GD + half * 64 + row) * GD + side * 64;
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {
        float v[16];
#pragma unroll
        for (int e = 0; e < 16; e += 4) {
            const float4 f = holds ? *reinterpret_cast<const float4 *>(srow + q4 * 16 + e) : make_float4(0.f, 0.f, 0.f, 0.f);
            v[e] = f.x; v[e + 1] = f.y; v[e + 2] = f.z; v[e + 3] = f.w;
        }
        tmem_st16(tmem + tq + TS + side * 64 + q4 * 16, v);
        if (holds) {
#pragma unroll
            for (int e = 0; e < 16; e += 4)
                *reinterpret_cast<uint2 *>(sh + sw_off(64, row, side * 64 + q4 * 16 + e)) =
                    pack4(v[e], v[e + 1], v[e + 2], v[e + 3]);
        }
    }
    tmem_wait_st();
    fence_async_shared();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    const uint32_t sh_a = smem_addr(sh), nw_a = smem_addr(smem + SCAN_NW), dl_a = smem_addr(smem + SCAN_DL);
    const uint32_t dh_a = smem_addr(smem + SCAN_DH), dlo_a = smem_addr(smem + SCAN_DLO);
    uint8_t *nw = smem + SCAN_NW, *dl = smem + SCAN_DL, *dhi = smem + SCAN_DH, *dlo = smem + SCAN_DLO;
    for (int c = 0; c < p.nch; ++c) {
        const int b = c & 1;
        uint8_t *buf = smem + SCAN_BUF + b * 75776;
        const uint32_t ba = smem_addr(buf);
        if (tid == 0 && c + 1 < p.nch) issue_loads(c + 1);
        mbar_wait(full + b, (uint32_t)(c >> 1) & 1, abort_flag);
        // ---- U = T V, W = T diag(g/|k|) K, O1 = Q S^T
        if (tid == 0) {
            tc_fence_after();
            const uint32_t i_u = idesc_f16(64, 64, true, true), i_w = idesc_f16(64, 128, true, true);
            const uint32_t i_o = idesc_f16(64, 64, false, false);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                mma_f16_ss(tmem + TU, sw128_desc(ba + SB_TH + k * 2048, TILE, 1024),
                           sw128_desc(ba + SB_V + k * 2048, TILE, 1024), i_u, k > 0 ? 1u : 0u);
                mma_f16_ss(tmem + TU, sw128_desc(ba + SB_TL + k * 2048, TILE, 1024),
                           sw128_desc(ba + SB_V + k * 2048, TILE, 1024), i_u, 1u);
                mma_f16_ss(tmem + TW, sw128_desc(ba + SB_TP + k * 2048, TILE, 1024),
                           sw128_desc(ba + SB_K + k * 2048, TILE, 1024), i_w, k > 0 ? 1u : 0u);
            }
#pragma unroll
            for (int k = 0; k < GD / 16; ++k)
                mma_f16_ss(tmem + TO1, sw128_desc(ba + SB_Q + (k >> 2) * TILE + (k & 3) * 32, 16, 1024),
                           sw128_desc(sh_a + (k >> 2) * TILE + (k & 3) * 32, 16, 1024), i_o, k > 0 ? 1u : 0u);
            mma_commit(bm1);
        }
        mbar_wait(bm1, (uint32_t)c & 1, abort_flag);
        tc_fence_after();
        // ---- -W into a K-major fp16 operand (this thread: token `row`, 64 of the 128 columns)
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
            float v[16];
            tmem_ld16(tmem + tq + TW + side * 64 + q4 * 16, v);
            tmem_wait_ld();
            if (holds) {
#pragma unroll
                for (int e = 0; e < 16; e += 4)
                    *reinterpret_cast<uint2 *>(nw + sw_off(64, row, side * 64 + q4 * 16 + e)) =
                        pack4(-v[e], -v[e + 1], -v[e + 2], -v[e + 3]);
            }
        }
        fence_async_shared();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (*abort_flag) break;
        // ---- Delta = U - W S^T
        if (tid == 0) {
            const uint32_t i_d = idesc_f16(64, 64, false, false);
#pragma unroll
            for (int k = 0; k < GD / 16; ++k)
                mma_f16_ss(tmem + TU, sw128_desc(nw_a + (k >> 2) * TILE + (k & 3) * 32, 16, 1024),
                           sw128_desc(sh_a + (k >> 2) * TILE + (k & 3) * 32, 16, 1024), i_d, 1u);
            mma_commit(bm3);
        }
        mbar_wait(bm3, (uint32_t)c & 1, abort_flag);
        tc_fence_after();
        // ---- Delta (fp16, for Mq Delta) and Delta' = Delta * (g_C/g_t)/|k_t| (hi + lo, for the
        //      state update), both [tokens][Dv] images; state scaled by g_C in TMEM.
        {
            const float4 sc = reinterpret_cast<const float4 *>(buf + SB_SC)[row];
            const float gC = reinterpret_cast<const float4 *>(buf + SB_SC)[0].z;
#pragma unroll
            for (int q2 = 0; q2 < 2; ++q2) {
                float v[16];
                tmem_ld16(tmem + tq + TU + side * 32 + q2 * 16, v);
                tmem_wait_ld();
                if (holds) {
#pragma unroll
                    for (int e = 0; e < 16; e += 4) {
                        const int col = side * 32 + q2 * 16 + e;          // Dv column within the half
                        const uint32_t off = sw_off(64, row, col);        // [tokens rows][64 Dv], one block
                        *reinterpret_cast<uint2 *>(dl + off) = pack4(v[e], v[e + 1], v[e + 2], v[e + 3]);
                        float d[4] = {v[e] * sc.y, v[e + 1] * sc.y, v[e + 2] * sc.y, v[e + 3] * sc.y};
                        float hh[4], ll[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) { hh[u] = __half2float(__float2half_rn(d[u])); ll[u] = d[u] - hh[u]; }
                        *reinterpret_cast<uint2 *>(dhi + off) = pack4(hh[0], hh[1], hh[2], hh[3]);
                        *reinterpret_cast<uint2 *>(dlo + off) = pack4(ll[0], ll[1], ll[2], ll[3]);
                    }
                }
            }
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
                float v[16];
                tmem_ld16(tmem + tq + TS + side * 64 + q4 * 16, v);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 16; ++e) v[e] *= gC;
                tmem_st16(tmem + tq + TS + side * 64 + q4 * 16, v);
            }
            tmem_wait_st();
        }
        fence_async_shared();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (*abort_flag) break;
        // ---- O2 = Mq Delta;  S += Delta'^T K
        if (tid == 0) {
            const uint32_t i_m = idesc_f16(64, 64, false, true), i_s = idesc_f16(64, 128, true, true);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                mma_f16_ss(tmem + TO2, sw128_desc(ba + SB_MQ + k * 32, 16, 1024),
                           sw128_desc(dl_a + k * 2048, TILE, 1024), i_m, k > 0 ? 1u : 0u);
                mma_f16_ss(tmem + TS, sw128_desc(dh_a + k * 2048, TILE, 1024),
                           sw128_desc(ba + SB_K + k * 2048, TILE, 1024), i_s, 1u);
                mma_f16_ss(tmem + TS, sw128_desc(dlo_a + k * 2048, TILE, 1024),
                           sw128_desc(ba + SB_K + k * 2048, TILE, 1024), i_s, 1u);
            }
            mma_commit(bm5);
        }
        mbar_wait(bm5, (uint32_t)c & 1, abort_flag);
        tc_fence_after();
        // ---- outputs O = (g_t/(|q_t| sqrt D)) Q S^T + Mq Delta, then the new state's fp16 image
        {
            const int t = c * GC + row;
            const float so = reinterpret_cast<const float4 *>(buf + SB_SC)[row].x;
            float *orow = p.out + ((size_t)t * p.Hv + h) * GD + half * 64 + side * 32;
#pragma unroll
            for (int q2 = 0; q2 < 2; ++q2) {
                float a[16], bb[16];
                tmem_ld16(tmem + tq + TO1 + side * 32 + q2 * 16, a);
                tmem_ld16(tmem + tq + TO2 + side * 32 + q2 * 16, bb);
                tmem_wait_ld();
                if (holds && t < p.L) {
#pragma unroll
                    for (int e = 0; e < 16; e += 4)
                        *reinterpret_cast<float4 *>(orow + q2 * 16 + e) =
                            make_float4(a[e] * so + bb[e], a[e + 1] * so + bb[e + 1], a[e + 2] * so + bb[e + 2],
                                        a[e + 3] * so + bb[e + 3]);
                }
            }
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
                float v[16];
                tmem_ld16(tmem + tq + TS + side * 64 + q4 * 16, v);
                tmem_wait_ld();
                if (holds) {
#pragma unroll
                    for (int e = 0; e < 16; e += 4)
                        *reinterpret_cast<uint2 *>(sh + sw_off(64, row, side * 64 + q4 * 16 + e)) =
                            pack4(v[e], v[e + 1], v[e + 2], v[e + 3]);
                }
            }
        }
        fence_async_shared();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (*abort_flag) break;
    }
    // Final state rows back to global memory (fp32).
    if (!*abort_flag) {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
            float v[16];
            tmem_ld16(tmem + tq + TS + side * 64 + q4 * 16, v);
            tmem_wait_ld();
            if (holds) {
#pragma unroll
                for (int e = 0; e < 16; e += 4)
                    *reinterpret_cast<float4 *>(srow + q4 * 16 + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
            }
        }
    }
    // Every issued load must land before the CTA may exit.
    if (tid == 0) {
        const long long t0 = clock64();
        for (int c = max(0, p.nch - 2); c < p.nch; ++c)
            while (!mbar_try_wait(full + (c & 1), (uint32_t)(c >> 1) & 1) && clock64() - t0 < WAIT_LIMIT_CYCLES) {}
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------------ host
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

// 2-D map over a row-major [rows][cols] array with a {box_x, box_y} box.
CUtensorMap map2d(const void *base, CUtensorMapDataType type, size_t esize, uint64_t cols, uint64_t rows,
                  uint32_t box_x, uint32_t box_y, bool swizzle) {
    CUtensorMap m;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * esize};
    cuuint32_t box[2] = {box_x, box_y};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_fn()(&m, type, 2, const_cast<void *>(base), dims, strides, box, estr,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                                   swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return m;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct GdnWorkspace { __half *th, *tl, *tp, *mq; float *sc; };
GdnWorkspace carve(void *ws, int Hv, int nch) {
    const size_t tile_bytes = align256((size_t)Hv * nch * GC * GC * sizeof(__half));
    uint8_t *w = static_cast<uint8_t *>(ws);
    GdnWorkspace g;
    g.th = reinterpret_cast<__half *>(w);
    g.tl = reinterpret_cast<__half *>(w + tile_bytes);
    g.tp = reinterpret_cast<__half *>(w + 2 * tile_bytes);
    g.mq = reinterpret_cast<__half *>(w + 3 * tile_bytes);
    g.sc = reinterpret_cast<float *>(w + 4 * tile_bytes);
    return g;
}

bool gdn_configured = false;
}  // namespace

size_t delta_chunked_workspace_bytes(int T, int Hv) {
    const int nch = (T + GC - 1) / GC;
    return 4 * align256((size_t)Hv * nch * GC * GC * sizeof(__half)) + align256((size_t)Hv * nch * GC * 4 * sizeof(float));
}

void delta_chunked(float *out, float *state, const __half *q, const __half *k, const __half *v, const float *alpha,
                   const float *beta, const float *decay, const float *bias, int T, int Hk, int Hv, int D, void *ws,
                   size_t ws_bytes, cudaStream_t st) {
    if (D != GD) throw std::invalid_argument("the chunked DeltaNet path needs head dimension 128");
    if (T < 1 || Hk < 1 || Hv < 1) throw std::invalid_argument("invalid DeltaNet dimensions");
    if (ws_bytes < delta_chunked_workspace_bytes(T, Hv)) throw std::invalid_argument("DeltaNet workspace too small");
    if (!gdn_configured) {
        if (cudaFuncSetAttribute(gdn_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PREP_SMEM) != cudaSuccess ||
            cudaFuncSetAttribute(gdn_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SCAN_SMEM) != cudaSuccess)
            throw std::runtime_error("cannot reserve shared memory for the chunked DeltaNet kernels");
        gdn_configured = true;
    }
    const int nch = (T + GC - 1) / GC;
    const GdnWorkspace w = carve(ws, Hv, nch);
    GdnPrep pp{q, k, alpha, beta, decay, bias, w.th, w.tl, w.tp, w.mq, w.sc, T, Hk, Hv, nch};
    cudaError_t e = launch_chained(gdn_prep_kernel, dim3(nch, Hv), dim3(128), PREP_SMEM, st, pp);
    if (e != cudaSuccess) throw std::runtime_error(std::string("DeltaNet chunk prep: ") + cudaGetErrorString(e));
    const uint64_t units = (uint64_t)Hv * nch * GC;
    const CUtensorMap mTh = map2d(w.th, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, GC, units, 64, 64, true);
    const CUtensorMap mTl = map2d(w.tl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, GC, units, 64, 64, true);
    const CUtensorMap mTp = map2d(w.tp, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, GC, units, 64, 64, true);
    const CUtensorMap mMq = map2d(w.mq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, GC, units, 64, 64, true);
    const CUtensorMap mK = map2d(k, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)Hk * GD, T, 64, 64, true);
    const CUtensorMap mQ = map2d(q, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)Hk * GD, T, 64, 64, true);
    const CUtensorMap mV = map2d(v, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)Hv * GD, T, 64, 64, true);
    const CUtensorMap mSc = map2d(w.sc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, 4, units, 4, 64, false);
    GdnScan sp{out, state, T, Hv, Hk, nch};
    e = launch_chained(gdn_scan_kernel, dim3(2, Hv), dim3(256), SCAN_SMEM, st, mTh, mTl, mTp, mMq, mK, mQ, mV, mSc, sp);
    if (e != cudaSuccess) throw std::runtime_error(std::string("DeltaNet chunk scan: ") + cudaGetErrorString(e));
}

}  // namespace qv
