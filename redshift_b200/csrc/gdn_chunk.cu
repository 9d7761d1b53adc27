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
#include <type_traits>

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
constexpr int PREP_BM = 49152;                   // fp32 [64][BMS]
constexpr int BMS = 68;                          // row stride: 16-byte rows, conflict-free row stores
constexpr int PREP_SMALL = PREP_BM + 64 * BMS * 4;
constexpr int PREP_SMEM = PREP_SMALL + 4 * 64 * 4 + 64;

__global__ void __launch_bounds__(128, 3) gdn_prep_kernel(const GdnPrep p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    if (smem_addr(smem) & 1023) {
        if (threadIdx.x == 0) raise_status(STATUS_BAD_ARGUMENT);
        return;
    }
    uint8_t *sa = smem + PREP_SA, *sb = smem + PREP_SB;
    float *bm = reinterpret_cast<float *>(smem + PREP_BM);
    // log2-scaled cumulative log decay, beta, 1/|k|, 1/(|q| sqrt D)
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

    // Raw decay inputs of this lane's two tokens (warp 0), loaded with the
    // keys / queries so that both arrive in one round trip.
    float al_raw[2] = {0.f, 0.f}, be_raw[2] = {0.f, 0.f};
    if (warp == 0) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int t = 2 * lane + e;
            if (t < n) {
                const size_t idx = (size_t)(t0 + t) * p.Hv + h;
                al_raw[e] = p.alpha[idx];
                be_raw[e] = p.beta[idx];
            }
        }
    }
    // (1) normalised keys / queries as fp16 MMA operands: warp w takes tokens
    //     16w..16w+15, lane l dims [4l, 4l+4); the 32 sums reduce together.
    {
        uint2 kr[16], qr[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int t = warp * 16 + i;
            kr[i] = qr[i] = make_uint2(0, 0);
            if (t < n) {
                kr[i] = *reinterpret_cast<const uint2 *>(p.k + ((size_t)(t0 + t) * p.Hk + kh) * GD + 4 * lane);
                qr[i] = *reinterpret_cast<const uint2 *>(p.q + ((size_t)(t0 + t) * p.Hk + kh) * GD + 4 * lane);
            }
        }
        float sk[16], sq[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float2 a = __half22float2(*reinterpret_cast<__half2 *>(&kr[i].x));
            const float2 b = __half22float2(*reinterpret_cast<__half2 *>(&kr[i].y));
            const float2 e = __half22float2(*reinterpret_cast<__half2 *>(&qr[i].x));
            const float2 f = __half22float2(*reinterpret_cast<__half2 *>(&qr[i].y));
            sk[i] = a.x * a.x + a.y * a.y + b.x * b.x + b.y * b.y;
            sq[i] = e.x * e.x + e.y * e.y + f.x * f.x + f.y * f.y;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                sk[i] += __shfl_xor_sync(0xffffffffu, sk[i], o);
                sq[i] += __shfl_xor_sync(0xffffffffu, sq[i], o);
            }
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int t = warp * 16 + i;
            const float rk = rsqrtf(sk[i] + 1e-6f), rq = rsqrtf(sq[i] + 1e-6f) * rsqrtf((float)GD);
            if (lane == 0) { ik[t] = rk; iq[t] = rq; }
            const float2 a = __half22float2(*reinterpret_cast<__half2 *>(&kr[i].x));
            const float2 b = __half22float2(*reinterpret_cast<__half2 *>(&kr[i].y));
            const float2 e = __half22float2(*reinterpret_cast<__half2 *>(&qr[i].x));
            const float2 f = __half22float2(*reinterpret_cast<__half2 *>(&qr[i].y));
            const uint2 kn = pack4(a.x * rk, a.y * rk, b.x * rk, b.y * rk);
            const uint2 qn = pack4(e.x * rq, e.y * rq, f.x * rq, f.y * rq);
            *reinterpret_cast<uint2 *>(sa + sw_off(128, t, 4 * lane)) = kn;
            *reinterpret_cast<uint2 *>(sa + sw_off(128, 64 + t, 4 * lane)) = qn;
            *reinterpret_cast<uint2 *>(sb + sw_off(64, t, 4 * lane)) = kn;
        }
    }
    // (2) log decays, their inclusive prefix sum over the chunk (log2 units),
    //     and beta
    if (warp == 0) {
        float g[2], b[2];
        const float dh = p.decay[h], bh = p.bias[h];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int t = 2 * lane + e;
            g[e] = 0.f; b[e] = 0.f;
            if (t < n) {
                g[e] = dh * softplusf_(al_raw[e] + bh) * 1.4426950408889634f;
                b[e] = sigmoidf_(be_raw[e]);
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
    mbar_wait(bar, 0, abort_flag);
    tc_fence_after();
    // (4) row tid of the product: B = beta_t G(t,s) k^_t.k^_s, s < t (tid < 64)
    //     or Mq = G(t,s) q^_t.k^_s, s <= t (tid >= 64); G(t,s) = 2^(gam_t - gam_s).
    {
        float x[64];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4)
            tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + q4 * 16, *reinterpret_cast<float(*)[16]>(x + q4 * 16));
        tmem_wait_ld();
        const size_t unit = (size_t)h * p.nch + c;
        if (tid < 64) {
            const int t = tid;
            const float gt = gam[t], bt = bet[t];
#pragma unroll
            for (int s4 = 0; s4 < 64; s4 += 4) {
                float4 v;
                v.x = s4 < t ? bt * exp2_approx(gt - gam[s4]) * x[s4] : 0.f;
                v.y = s4 + 1 < t ? bt * exp2_approx(gt - gam[s4 + 1]) * x[s4 + 1] : 0.f;
                v.z = s4 + 2 < t ? bt * exp2_approx(gt - gam[s4 + 2]) * x[s4 + 2] : 0.f;
                v.w = s4 + 3 < t ? bt * exp2_approx(gt - gam[s4 + 3]) * x[s4 + 3] : 0.f;
                *reinterpret_cast<float4 *>(bm + t * BMS + s4) = v;
            }
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
                    m[e] = s <= t ? exp2_approx(gt - gam[s]) * x[s] : 0.f;
                }
                const uint2 lo = pack4(m[0], m[1], m[2], m[3]), hi = pack4(m[4], m[5], m[6], m[7]);
                dst[s8] = make_uint4(lo.x, lo.y, hi.x, hi.y);
            }
        }
    }
    __syncthreads();

    // (5) X = (I + B)^-1 (unit lower triangular) by forward substitution, one
    //     thread per column j (warps 0 and 1); column j is zero above row j,
    //     so warp 1 (j >= 32) starts at row 32.  (6) The owner of column j then
    //     writes row j of T^T, T = X diag(beta), as fp16 hi + lo, and of
    //     (T diag(g / |k|))^T as fp16.  (7) Warps 2-3 write the per-token scales
    //     {g_t / (|q_t| sqrt D), (g_C / g_t) / |k_t|, g_C, 0}.
    const size_t unit = (size_t)h * p.nch + c;
    auto solve_and_store = [&](auto first_row) {
        constexpr int R0 = decltype(first_row)::value;
        const int j = tid;
        float xv[64];
#pragma unroll
        for (int i = 0; i < R0; ++i) xv[i] = 0.f;
#pragma unroll
        for (int i = R0; i < 64; ++i) {
            float a0 = 0.f, a1 = 0.f;
            const float *brow = bm + i * BMS;
#pragma unroll
            for (int s4 = R0; s4 < (i & ~3); s4 += 4) {
                const float4 b4 = *reinterpret_cast<const float4 *>(brow + s4);
                a0 += b4.x * xv[s4]; a1 += b4.y * xv[s4 + 1];
                a0 += b4.z * xv[s4 + 2]; a1 += b4.w * xv[s4 + 3];
            }
#pragma unroll
            for (int s = (i & ~3) > R0 ? (i & ~3) : R0; s < i; ++s) a0 += brow[s] * xv[s];
            xv[i] = (i == j ? 1.f : 0.f) - (a0 + a1);
        }
        const float bj = bet[j], wj = bj * exp2f(gam[j]) * ik[j];
        const size_t row = (unit * GC + j) * GC;
        uint4 *ph = reinterpret_cast<uint4 *>(p.tt_hi + row), *pl = reinterpret_cast<uint4 *>(p.tt_lo + row);
        uint4 *pp = reinterpret_cast<uint4 *>(p.ttp + row);
#pragma unroll
        for (int q8 = 0; q8 < 8; ++q8) {
            float hv[8], lv[8], pv[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float xe = xv[q8 * 8 + e];
                const float v = xe * bj;
                const float hh = __half2float(__float2half_rn(v));
                hv[e] = hh; lv[e] = v - hh;
                pv[e] = xe * wj;
            }
            uint2 a = pack4(hv[0], hv[1], hv[2], hv[3]), b = pack4(hv[4], hv[5], hv[6], hv[7]);
            ph[q8] = make_uint4(a.x, a.y, b.x, b.y);
            a = pack4(lv[0], lv[1], lv[2], lv[3]); b = pack4(lv[4], lv[5], lv[6], lv[7]);
            pl[q8] = make_uint4(a.x, a.y, b.x, b.y);
            a = pack4(pv[0], pv[1], pv[2], pv[3]); b = pack4(pv[4], pv[5], pv[6], pv[7]);
            pp[q8] = make_uint4(a.x, a.y, b.x, b.y);
        }
    };
    if (warp == 0) solve_and_store(std::integral_constant<int, 0>{});
    else if (warp == 1) solve_and_store(std::integral_constant<int, 32>{});
    else if (tid >= 64) {
        const int t = tid - 64;
        const float gl = gam[n - 1];
        const float4 v = t < n ? make_float4(exp2f(gam[t]) * iq[t], exp2f(gl - gam[t]) * ik[t], exp2f(gl), 0.f)
                               : make_float4(0.f, 0.f, exp2f(gl), 0.f);
        reinterpret_cast<float4 *>(p.sc)[unit * GC + t] = v;
    }
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
    uint64_t *full = bars, *bm1 = bars + 2, *bm3 = bars + 3, *bm5 = bars + 4, *bm4 = bars + 5;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 6);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 7);
    const int half = blockIdx.x, h = blockIdx.y, kh = h % p.Hk;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, quad = warp & 3, side = warp >> 2;
    const int row = 16 * quad + (lane & 15);          // M=64 accumulator row held by this thread
    const bool holds = lane < 16;
    const uint32_t tq = (uint32_t)(quad * 32) << 16;  // this warp's TMEM lane quarter

    if (tid == 0) {
        mbar_init(full, 1); mbar_init(full + 1, 1);
        mbar_init(bm1, 1); mbar_init(bm3, 1); mbar_init(bm4, 1); mbar_init(bm5, 1);
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
    int last_issued = min(p.nch, 2) - 1;          // (thread 0) latest chunk whose loads are in flight
    if (tid == 0) {
        issue_loads(0);
        if (p.nch > 1) issue_loads(1);
    }
    uint8_t *sh = smem + SCAN_SH, *nw = smem + SCAN_NW, *dl = smem + SCAN_DL;
    uint8_t *dhi = smem + SCAN_DH, *dlo = smem + SCAN_DLO;
    const uint32_t sh_a = smem_addr(sh), nw_a = smem_addr(nw), dl_a = smem_addr(dl);
    const uint32_t dh_a = smem_addr(dhi), dlo_a = smem_addr(dlo);
    auto buf_of = [&](int c) { return smem + SCAN_BUF + (c & 1) * 75776; };

    // Initial state rows (value dims half*64 + row) into TMEM, fp32; this
    // thread covers 64 columns.
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
    }
    tmem_wait_st();

    // U = T V and W = T diag(g/|k|) K of chunk c (independent of the state).
    // Shared-memory descriptors are formed once per operand base; a K step
    // adds its byte offset / 16 to the start-address field (every address
    // here is below 256 KB, so the 14-bit field never carries).
    auto kmaj = [](uint32_t a) { return sw128_desc(a, 16, 1024); };
    auto mnmaj = [](uint32_t a) { return sw128_desc(a, TILE, 1024); };
    auto koff = [](int k) { return (uint64_t)((k >> 2) * (TILE >> 4) + (k & 3) * 2); };   // K-major, K = 16 k
    auto moff = [](int k) { return (uint64_t)(k * 128); };                                // MN-major, K = 16 k
    const uint64_t d_sh = kmaj(sh_a), d_nw = kmaj(nw_a), d_dl = mnmaj(dl_a), d_dh = mnmaj(dh_a), d_dlo = mnmaj(dlo_a);
    const uint32_t i_u = idesc_f16(64, 64, true, true), i_w = idesc_f16(64, 128, true, true);
    const uint32_t i_d = idesc_f16(64, 64, false, false), i_m = idesc_f16(64, 64, false, true);
    const uint32_t i_s = idesc_f16(64, 128, true, true);
    auto issue_uw = [&](int c) {
        const uint32_t ba = smem_addr(buf_of(c));
        const uint64_t th = mnmaj(ba + SB_TH), tl = mnmaj(ba + SB_TL), tp = mnmaj(ba + SB_TP);
        const uint64_t dv = mnmaj(ba + SB_V), dk = mnmaj(ba + SB_K);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            mma_f16_ss(tmem + TU, th + moff(k), dv + moff(k), i_u, k > 0 ? 1u : 0u);
            mma_f16_ss(tmem + TU, tl + moff(k), dv + moff(k), i_u, 1u);
            mma_f16_ss(tmem + TW, tp + moff(k), dk + moff(k), i_w, k > 0 ? 1u : 0u);
        }
    };
    // Warps 0-3: the state (fp32, TMEM) becomes the fp16 operand image of the
    // next chunk and is pre-scaled there by that chunk's g_C (the state update
    // accumulates onto g_C S).  Each active thread: one state row, 128 columns.
    auto convert_state = [&](int c_next) {
        const float gC = reinterpret_cast<const float4 *>(buf_of(c_next) + SB_SC)[0].z;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            float v[4][16];
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) tmem_ld16(tmem + tq + TS + hh * 64 + q4 * 16, v[q4]);
            tmem_wait_ld();
            if (holds) {
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4)
#pragma unroll
                    for (int e = 0; e < 16; e += 4)
                        *reinterpret_cast<uint2 *>(sh + sw_off(64, row, hh * 64 + q4 * 16 + e)) =
                            pack4(v[q4][e], v[q4][e + 1], v[q4][e + 2], v[q4][e + 3]);
            }
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
#pragma unroll
                for (int e = 0; e < 16; ++e) v[q4][e] *= gC;
                tmem_st16(tmem + tq + TS + hh * 64 + q4 * 16, v[q4]);
            }
        }
        tmem_wait_st();
    };
    // Warps 4-7: -W of chunk c into its K-major fp16 operand (one token row,
    // 128 columns per active thread).
    auto convert_w = [&]() {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            float v[4][16];
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) tmem_ld16(tmem + tq + TW + hh * 64 + q4 * 16, v[q4]);
            tmem_wait_ld();
            if (holds) {
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4)
#pragma unroll
                    for (int e = 0; e < 16; e += 4)
                        *reinterpret_cast<uint2 *>(nw + sw_off(64, row, hh * 64 + q4 * 16 + e)) =
                            pack4(-v[q4][e], -v[q4][e + 1], -v[q4][e + 2], -v[q4][e + 3]);
            }
        }
    };
    // Warps 4-7: outputs of chunk c, O = (g_t/(|q_t| sqrt D)) Q S^T + Mq Delta.
    auto readout = [&](int c) {
        const int t = c * GC + row;
        const float so = reinterpret_cast<const float4 *>(buf_of(c) + SB_SC)[row].x;
        float *orow = p.out + ((size_t)t * p.Hv + h) * GD + half * 64;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            float a[2][16], bb[2][16];
#pragma unroll
            for (int q2 = 0; q2 < 2; ++q2) {
                tmem_ld16(tmem + tq + TO1 + hh * 32 + q2 * 16, a[q2]);
                tmem_ld16(tmem + tq + TO2 + hh * 32 + q2 * 16, bb[q2]);
            }
            tmem_wait_ld();
            if (holds && t < p.L) {
#pragma unroll
                for (int q2 = 0; q2 < 2; ++q2)
#pragma unroll
                    for (int e = 0; e < 16; e += 4)
                        *reinterpret_cast<float4 *>(orow + hh * 32 + q2 * 16 + e) =
                            make_float4(a[q2][e] * so + bb[q2][e], a[q2][e + 1] * so + bb[q2][e + 1],
                                        a[q2][e + 2] * so + bb[q2][e + 2], a[q2][e + 3] * so + bb[q2][e + 3]);
            }
        }
    };
    auto cta_sync = [&]() {
        fence_async_shared();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    };

    // Two issuing threads: thread 0 (warp 0) issues the chain that carries
    // the state (Delta, then the state update), thread 128 (warp 4) the
    // products off that chain (Q S^T, and the next chunk's U and W).
    // Prologue: chunk 0's U, W; the state image of chunk 0; -W of chunk 0.
    // (Warps 0-3 convert state columns that warps 4-7 stored above.)
    cta_sync();
    mbar_wait(full, 0, abort_flag);
    if (tid == 128) {
        tc_fence_after();
        issue_uw(0);
        mma_commit(bm1);
    }
    if (side == 0) {
        convert_state(0);
    } else {
        mbar_wait(bm1, 0, abort_flag);
        tc_fence_after();
        convert_w();
    }
    cta_sync();

    for (int c = 0; c < p.nch && !*abort_flag; ++c) {
        const uint32_t ba = smem_addr(buf_of(c));
        // ---- Delta = U - W S^T (thread 0) and O1 = Q S^T (thread 128)
        if (tid == 0) {
#pragma unroll
            for (int k = 0; k < GD / 16; ++k) mma_f16_ss(tmem + TU, d_nw + koff(k), d_sh + koff(k), i_d, 1u);
            mma_commit(bm3);
        } else if (tid == 128) {
            const uint64_t dq = kmaj(ba + SB_Q);
#pragma unroll
            for (int k = 0; k < GD / 16; ++k)
                mma_f16_ss(tmem + TO1, dq + koff(k), d_sh + koff(k), i_d, k > 0 ? 1u : 0u);
            mma_commit(bm4);
        }
        mbar_wait(bm3, (uint32_t)c & 1, abort_flag);
        tc_fence_after();
        // ---- Delta (fp16, for Mq Delta) and Delta' = Delta (g_C/g_t)/|k_t| (hi + lo, for the
        //      state update), both [tokens][Dv] images; this thread: 32 of the 64 columns.
        {
            const float sy = reinterpret_cast<const float4 *>(buf_of(c) + SB_SC)[row].y;
            float dv[2][16];
#pragma unroll
            for (int q2 = 0; q2 < 2; ++q2) tmem_ld16(tmem + tq + TU + side * 32 + q2 * 16, dv[q2]);
            tmem_wait_ld();
            if (holds) {
#pragma unroll
                for (int q2 = 0; q2 < 2; ++q2)
#pragma unroll
                    for (int e = 0; e < 16; e += 4) {
                        const float *v = dv[q2] + e;
                        const uint32_t off = sw_off(64, row, side * 32 + q2 * 16 + e);
                        *reinterpret_cast<uint2 *>(dl + off) = pack4(v[0], v[1], v[2], v[3]);
                        float hh[4], ll[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const float d = v[u] * sy;
                            hh[u] = __half2float(__float2half_rn(d));
                            ll[u] = d - hh[u];
                        }
                        *reinterpret_cast<uint2 *>(dhi + off) = pack4(hh[0], hh[1], hh[2], hh[3]);
                        *reinterpret_cast<uint2 *>(dlo + off) = pack4(ll[0], ll[1], ll[2], ll[3]);
                    }
            }
        }
        cta_sync();
        // ---- O2 = Mq Delta and S = g_C S + Delta'^T K (thread 0); U, W of the next chunk (thread 128)
        if (tid == 0) {
            const uint64_t dmq = kmaj(ba + SB_MQ), dk = mnmaj(ba + SB_K);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                mma_f16_ss(tmem + TO2, dmq + (uint64_t)(k * 2), d_dl + moff(k), i_m, k > 0 ? 1u : 0u);
                mma_f16_ss(tmem + TS, d_dh + moff(k), dk + moff(k), i_s, 1u);
                mma_f16_ss(tmem + TS, d_dlo + moff(k), dk + moff(k), i_s, 1u);
            }
            mma_commit(bm5);
        } else if (tid == 128 && c + 1 < p.nch) {
            if (mbar_wait(full + ((c + 1) & 1), (uint32_t)((c + 1) >> 1) & 1, abort_flag)) {
                tc_fence_after();
                issue_uw(c + 1);
            }
            mma_commit(bm1);
        }
        // ---- warps 0-3: next state image (+ g_C scaling); warps 4-7: outputs, next -W
        mbar_wait(bm5, (uint32_t)c & 1, abort_flag);
        mbar_wait(bm4, (uint32_t)c & 1, abort_flag);      // Q S^T has read the state image
        tc_fence_after();
        if (side == 0) {
            if (c + 1 < p.nch) {
                mbar_wait(full + ((c + 1) & 1), (uint32_t)((c + 1) >> 1) & 1, abort_flag);
                convert_state(c + 1);
            }
        } else {
            readout(c);
            if (c + 1 < p.nch) {
                mbar_wait(bm1, (uint32_t)(c + 1) & 1, abort_flag);
                tc_fence_after();
                convert_w();
            }
        }
        cta_sync();
        // This chunk's buffer is free again: the loads of chunk c+2 go into it.
        if (tid == 0 && c + 2 < p.nch) { issue_loads(c + 2); last_issued = c + 2; }
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
        for (int c = max(0, last_issued - 1); c <= last_issued; ++c)
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

// The shared-memory limit of a kernel is a per-device attribute.
PerDeviceOnce g_gdn_configured;
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
    g_gdn_configured.run([] {
        if (cudaFuncSetAttribute(gdn_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PREP_SMEM) != cudaSuccess ||
            cudaFuncSetAttribute(gdn_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SCAN_SMEM) != cudaSuccess)
            throw std::runtime_error("cannot reserve shared memory for the chunked DeltaNet kernels");
    });
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
