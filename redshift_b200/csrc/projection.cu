// Quantized projections for verify batches (T <= 8): out[t][row] = sum_k W[row][k] x[t][k]
// with W in the GGUF block formats the reference model uses (src/kernels.cu:31-273,
// 506-552; kinds 8 = Q8_0, 12 = Q4_K, 14 = Q6_K).
//
// On the tensor cores (tcgen05, kind::f16, fp32 accumulators in TMEM), HBM-bound:
//  * A = the integer quants of 128 weight rows (Q8_0: q, Q4_K: the 4-bit q, Q6_K:
//    q - 32), exact as fp16; the per-row block scales stay out of the MMA;
//  * B = the activations of 8 tokens as N = 16 columns: per 32-column block x is
//    scaled by a power of two into [2^14, 2^15) at its maximum and split into
//    fp16 hi + lo (22 significant bits); the fast variant (the reference's
//    dp4a-path semantics, runtime.h:17-20) instead quantises x per 32-column
//    block to 16-bit integers q16 = round(x / s), s = max|x| / 32639, round half
//    away from zero, split into bytes q16 = 256 hi + lo, so its products are
//    exact integers;
//  * one M=128 N=16 K=16 MMA per 16 columns; after every scale group (32
//    columns, 16 for Q6_K) the accumulator is read back and
//    acc[t] += (c D_hi + D_lo) * f_tb * s_row - m_row * xsum_tb
//    (c = 1 or 256, f_tb the block's activation factor, s_row the row's block
//    scale: Q8_0 d, Q4_K d*sc, Q6_K d*sc; the Q4_K minimum dmin*m times the
//    block's sum of the exact activations), in fp32.
// Per CTA of 128 rows, 640 threads:
//  * warps 16-17: raw GGUF bytes of each 256-column chunk of the 128 rows into a
//    ring, by asynchronous 8-byte copies (lane = row; a row's later words hit
//    the L1 lines its first ones brought in), each row's chunk as its
//    8-byte-aligned superset (the formats only guarantee 2-byte alignment);
//    their completion is tracked on the ring slot's mbarrier;
//  * warps 8-15: two threads per row, one per 128-column half of a chunk: quants
//    to the swizzled fp16 A tile, the row's block scales, and (per half) the B
//    tile of the 8 tokens with its per-block factors and sums;
//  * warps 18-19: MMA issuers (alternate stages), 32 TMEM accumulator slots of
//    16 columns (8 stages of slack between the MMAs and the readback);
//  * warps 0-7: readback, thread = (row = TMEM lane, 4 of the 8 tokens).
#include "common.cuh"
#include "hotpath.h"

#include <stdexcept>
#include <string>

namespace qv {
namespace {

constexpr int PM_ROWS = 128;                 // weight rows per CTA (MMA M)
constexpr int PM_T = 8;                      // tokens
constexpr int PM_CC = 256;                   // columns per chunk (a K-quant super-block)
constexpr int PM_HC = 128;                   // columns per stage (half a chunk)
constexpr int PM_NS = 32;                    // TMEM accumulator slots (all 512 columns)
constexpr int PM_THREADS = 640;
constexpr int PM_A_BYTES = PM_ROWS * PM_HC * 2;      // 32 KB: 2 swizzle atoms of [128 rows][128 B]
constexpr int PM_B_BYTES = 16 * PM_HC * 2;           // 4 KB: 2 atoms of [16 rows][128 B]

// Shared-memory layout per format: NA stages of A / B / scales and a raw ring.
// Q4_K (raw chunks by tensor loads, 18 KB each) trades raw-ring depth for a
// fourth operand stage, which lets the converters run further ahead.
template <int KIND> struct PmLayout {
    static constexpr int NA = KIND == 12 ? 4 : 3;
    static constexpr int NG = KIND == 14 ? 8 : 4;                 // scale groups per stage
    static constexpr int SM_A = 0;
    static constexpr int SM_B = SM_A + NA * PM_A_BYTES;
    static constexpr int SM_SW = SM_B + NA * PM_B_BYTES;          // [NA][128 rows][NG] row scales
    static constexpr int SM_MN = SM_SW + NA * PM_ROWS * NG * 4;   // [NA][128 rows][4 blocks] Q4_K minima
    static constexpr int SM_F = SM_MN + NA * PM_ROWS * 4 * 4;     // [NA][8 tokens][4 blocks] activation factors (x 2^24)
    static constexpr int SM_XS = SM_F + NA * PM_T * 4 * 4;        // [NA][8 tokens][4 blocks] activation sums
    static constexpr int SM_BS = SM_XS + NA * PM_T * 4 * 4;       // [NA][8 tokens][8 groups of 16] quant-bias terms
    static constexpr int SM_BAR = SM_BS + NA * PM_T * 8 * 4;
    static constexpr int SM_RAW = (SM_BAR + 1024 + 127) / 128 * 128;
    static constexpr int RAW_BYTES = 227 * 1024 - SM_RAW;
    static constexpr int SMEM = SM_RAW + RAW_BYTES;
    static_assert(SM_B % 1024 == 0 && PM_B_BYTES % 1024 == 0, "operand tiles need 1024-byte alignment");
};

template <int KIND> struct PmFormat {
    static constexpr int SB = KIND == 8 ? 32 : 256;                      // columns per GGUF block
    static constexpr int BB = KIND == 8 ? 34 : (KIND == 12 ? 144 : 210); // bytes per GGUF block
    static constexpr int CB = PM_CC / SB * BB;                           // bytes of a full chunk of a row
    // raw row slot of the copy path: the row's chunk as its 16-byte-aligned
    // superset (up to 14 bytes before and after an even start); the tensor
    // path lands rows packed at the chunk's own pitch CB (a multiple of 16)
    static constexpr int RS_COPY = (CB + 28 + 15) / 16 * 16;
    static constexpr int G = KIND == 14 ? 16 : 32;                       // columns per scale group
    static_assert(PmLayout<KIND>::RAW_BYTES / (PM_ROWS * RS_COPY) >= 2, "raw ring too shallow");
};

// Byte offset of element `col` (a multiple of 8) of row `row` in a K-major,
// 128-byte-swizzled operand of `rows` rows: 64-element atoms of rows x 128 B,
// 16-byte chunks XOR-swizzled by the row's low 3 bits.
__device__ __forceinline__ uint32_t pm_sw(int rows, int row, int col) {
    return (uint32_t)((col >> 6) * rows * 128 + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4));
}
// 32-bit little-endian word at a shared-memory byte address of any alignment.
__device__ __forceinline__ uint32_t pm_word(const uint8_t *p) {
    const uint32_t a = smem_addr(p), a0 = a & ~3u;
    uint32_t w0, w1;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(w0) : "r"(a0));
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(w1) : "r"(a0 + 4));
    return __funnelshift_r(w0, w1, (a & 3) * 8);
}
__device__ __forceinline__ float pm_half(const uint8_t *p) {       // 2-byte aligned fp16
    return __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(p)));
}
// 32 lanes x 32 bit, 4 consecutive TMEM columns.
__device__ __forceinline__ void pm_tmem_ld4(uint32_t taddr, float (&v)[4]) {
    uint32_t r0, r1, r2, r3;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(taddr));
    v[0] = __uint_as_float(r0); v[1] = __uint_as_float(r1); v[2] = __uint_as_float(r2); v[3] = __uint_as_float(r3);
}
__device__ __forceinline__ bool pm_wait_warp(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
}

struct PmArgs {
    float *out;             // [T][rows]
    const uint8_t *w;       // rows x row_bytes, 16-byte aligned
    const float *x;         // [T][width]
    size_t w_bytes;         // total weight bytes (the end of w)
    int T, width, rows;
    int tma;                // 1: rows are 16-byte multiples, chunks arrive by the tensor map
};

// 3-D tile load global -> shared (16-byte pieces x pieces x rows), completion on
// the mbarrier's transaction count.
__device__ __forceinline__ void pm_tma_load_3d(void *dst, const void *tmap, uint64_t *bar, int x, int y, int z) {
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4, %5}], [%2];"
                 :: "r"(smem_addr(dst)), "l"(tmap), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z) : "memory");
}

template <int KIND, bool FAST>
__global__ void __launch_bounds__(PM_THREADS, 1) qmm_tc_kernel(const __grid_constant__ CUtensorMap tmW, const PmArgs a) {
    using F = PmFormat<KIND>;
    using L = PmLayout<KIND>;
    constexpr int G = F::G, NGH = PM_HC / G, NA = L::NA;               // groups per stage, operand stages
    const int RS = a.tma ? F::CB : F::RS_COPY;                          // raw row pitch
    const int R = min(4, L::RAW_BYTES / (PM_ROWS * RS));                // raw ring depth
    extern __shared__ __align__(1024) uint8_t smem[];
    if (smem_addr(smem) & 1023) {
        if (threadIdx.x == 0) raise_status(STATUS_BAD_ARGUMENT);
        return;
    }
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::SM_BAR);
    uint64_t *raw_full = bars, *raw_empty = bars + 4, *a_full = bars + 8, *a_empty = bars + 12, *s_empty = bars + 16,
             *d_full = bars + 20, *d_empty = d_full + PM_NS, *mma_done = d_empty + PM_NS;     // mma_done: one per issuer
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    static_assert((20 + 2 * PM_NS + 2) * 8 + 8 <= 1024 && NA <= 4, "mbarriers exceed their region");
    float *sw = reinterpret_cast<float *>(smem + L::SM_SW), *mn = reinterpret_cast<float *>(smem + L::SM_MN);
    float *fs = reinterpret_cast<float *>(smem + L::SM_F), *xs = reinterpret_cast<float *>(smem + L::SM_XS);
    float *bs = reinterpret_cast<float *>(smem + L::SM_BS);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * PM_ROWS;
    const int nrows = min(PM_ROWS, a.rows - row0);
    const size_t row_bytes = (size_t)(a.width / F::SB) * F::BB;
    const int nchunks = (a.width + PM_CC - 1) / PM_CC;

    if (threadIdx.x == 0) {
        for (int i = 0; i < R; ++i) { mbar_init(raw_full + i, a.tma ? 1 : 64); mbar_init(raw_empty + i, 8); }
        for (int i = 0; i < NA; ++i) { mbar_init(a_full + i, 4); mbar_init(a_empty + i, 1); mbar_init(s_empty + i, 8); }
        for (int i = 0; i < PM_NS; ++i) { mbar_init(d_full + i, 1); mbar_init(d_empty + i, 8); }
        mbar_init(mma_done, 1);
        mbar_init(mma_done + 1, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 18) { tmem_alloc(tmem_slot, PM_NS * 16); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    grid_dependency_wait();
    if (threadIdx.x == 0) launch_dependents();

    // groups of stage u (chunk u / 2, half u % 2); only a partial last Q8_0 chunk has fewer
    auto stage_groups = [&](int u) {
        const int len = min(PM_CC, a.width - (u >> 1) * PM_CC) - (u & 1) * PM_HC;
        return len <= 0 ? 0 : min(NGH, len / G);
    };
    const int nstages = 2 * nchunks;

    if (warp == 16 || warp == 17) {
        // ------------------------------------------------ raw bytes producers
        const uintptr_t wbase = reinterpret_cast<uintptr_t>(a.w), wend = wbase + a.w_bytes;
        if (a.tma) {
            // one tensor load per chunk: pieces [c CB/16, (c+1) CB/16) of the 128
            // rows (rows past the matrix read as zeros)
            if (warp == 16 && lane == 0) {
                prefetch_tmap(&tmW);
                int issued = 0;
                for (int c = 0; c < nchunks; ++c) {
                    const int slot = c % R;
                    if (c >= R && !mbar_wait(raw_empty + slot, ((c / R) - 1) & 1, abort_flag)) break;
                    mbar_expect_tx(raw_full + slot, PM_ROWS * F::CB);
                    pm_tma_load_3d(smem + L::SM_RAW + slot * PM_ROWS * RS, &tmW, raw_full + slot, 0, c * (F::CB / 16), row0);
                    issued = c + 1;
                }
                const long long t0 = clock64();
                for (int c = max(0, issued - R); c < issued; ++c)
                    while (!mbar_try_wait(raw_full + c % R, (c / R) & 1) && clock64() - t0 < WAIT_LIMIT_CYCLES) {}
            }
        } else {
            // 16-byte asynchronous copies, half a warp per row (coalesced): lane l
            // of warp 16 + p copies pieces l % 16 (+ 16) of rows 64 p + 2 i + l / 16
            for (int c = 0; c < nchunks; ++c) {
                const int slot = c % R;
                if (c >= R && !pm_wait_warp(raw_empty + slot, ((c / R) - 1) & 1, abort_flag)) break;
                const int cb = min(PM_CC, a.width - c * PM_CC) / F::SB * F::BB;
                uint8_t *dst0 = smem + L::SM_RAW + slot * PM_ROWS * RS;
                for (int i = 0; i < 32; ++i) {
                    const int r = (warp - 16) * 64 + 2 * i + (lane >> 4);
                    if (r >= nrows) break;
                    const uintptr_t st = wbase + (size_t)(row0 + r) * row_bytes + (size_t)c * F::CB;
                    const uintptr_t a0 = st & ~uintptr_t(15), a1 = (st + cb + 15) & ~uintptr_t(15);
#pragma unroll
                    for (int pc = 0; pc < 2; ++pc) {
                        const uintptr_t src = a0 + 16 * ((lane & 15) + 16 * pc);
                        if (src >= a1) continue;
                        uint8_t *dst = dst0 + r * RS + (src - a0);
                        if (src + 16 <= wend) {
                            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_addr(dst)), "l"(src) : "memory");
                        } else {
                            // the matrix's last piece, past the end of the buffer: its
                            // bytes up to the end (the buffer size is even) by plain loads
                            for (uintptr_t b = src; b < wend; b += 2)
                                *reinterpret_cast<uint16_t *>(dst + (b - src)) = *reinterpret_cast<const uint16_t *>(b);
                        }
                    }
                }
                // the slot's mbarrier counts this lane once its copies have landed
                asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" :: "r"(smem_addr(raw_full + slot)) : "memory");
            }
            // every issued copy must land before the CTA may exit
            asm volatile("cp.async.wait_all;" ::: "memory");
        }
    } else if (warp == 18 || warp == 19) {
        // ------------------------------------------------ MMA issuers: warp 18 + i
        // takes the stages u with u % 2 == i (one thread's issue rate is below
        // the tensor core's at N = 16). The operand descriptors of stage 0 are
        // formed once; a stage and a K step only move their start-address
        // field (address >> 4, in the low 14 bits: shared-memory addresses stay
        // below 2^18, so no carry).
        const int issuer = warp - 18;
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(128, 16, false, false);
            const uint64_t ad0 = sw128_desc(smem_addr(smem + L::SM_A), 16, 1024);
            const uint64_t bd0 = sw128_desc(smem_addr(smem + L::SM_B), 16, 1024);
            int gseq = 0;
            bool ok = true;
            for (int u = 0; u < nstages && ok; ++u) {
                const int st = u % NA;
                const int ng = stage_groups(u);
                if ((u & 1) != issuer) { gseq += ng; continue; }
                if (!mbar_wait(a_full + st, (u / NA) & 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint64_t ad = ad0 + (uint64_t)(st * PM_A_BYTES >> 4), bd = bd0 + (uint64_t)(st * PM_B_BYTES >> 4);
#pragma unroll
                for (int g = 0; g < NGH; ++g) {
                    if (g >= ng) break;
                    const int q = gseq + g, slot = q % PM_NS;
                    if (q >= PM_NS) {
                        if (!mbar_wait(d_empty + slot, ((q / PM_NS) - 1) & 1, abort_flag)) { ok = false; break; }
                        tc_fence_after();
                    }
#pragma unroll
                    for (int kk = 0; kk < G / 16; ++kk) {
                        const int k = g * G + kk * 16;                  // column within the stage (compile-time)
                        mma_f16_ss(tmem + slot * 16, ad + (uint64_t)(((k >> 6) * (PM_ROWS * 128) + (k & 63) * 2) >> 4),
                                   bd + (uint64_t)(((k >> 6) * (16 * 128) + (k & 63) * 2) >> 4), idesc, kk > 0 ? 1u : 0u);
                    }
                    mma_commit(d_full + slot);
                }
                gseq += ng;
                mma_commit(a_empty + st);
            }
            mma_commit(mma_done + issuer);
            const long long t0 = clock64();
            while (!mbar_try_wait(mma_done + issuer, 0) && clock64() - t0 < WAIT_LIMIT_CYCLES) {}
        }
    } else if (warp >= 8 && warp < 16) {
        // ------------------------------------------------ converters
        const int h = (warp - 8) >> 2, r = ((warp - 8) & 3) * 32 + lane, ib = r;   // thread index within its half
        // thread ib's activations: token ib / 16, columns 8 (ib % 16) .. + 8 of
        // each of its stages, loaded one stage ahead
        const int t = ib >> 4, kx = 8 * (ib & 15);
        const float *xrow = a.x + (size_t)t * a.width + h * PM_HC + kx;
        float4 xn0 = make_float4(0.f, 0.f, 0.f, 0.f), xn1 = xn0;
        if (t < a.T && kx < stage_groups(h) * G) {
            xn0 = reinterpret_cast<const float4 *>(xrow)[0];
            xn1 = reinterpret_cast<const float4 *>(xrow)[1];
        }
        bool ok = true;
        for (int c = 0; c < nchunks && ok; ++c) {
            const int u = 2 * c + h, st = u % NA;
            const int ng = stage_groups(u);
            float xv[8];
            xv[0] = xn0.x; xv[1] = xn0.y; xv[2] = xn0.z; xv[3] = xn0.w;
            xv[4] = xn1.x; xv[5] = xn1.y; xv[6] = xn1.z; xv[7] = xn1.w;
            xn0 = xn1 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (c + 1 < nchunks && t < a.T && kx < stage_groups(u + 2) * G) {
                xn0 = reinterpret_cast<const float4 *>(xrow + (c + 1) * PM_CC)[0];
                xn1 = reinterpret_cast<const float4 *>(xrow + (c + 1) * PM_CC)[1];
            }
            if (u >= NA) {
                if (!pm_wait_warp(a_empty + st, ((u / NA) - 1) & 1, abort_flag)) { ok = false; break; }
                if (!pm_wait_warp(s_empty + st, ((u / NA) - 1) & 1, abort_flag)) { ok = false; break; }
            }
            float m = 0.f, xsum = 0.f, bsum = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) { m = fmaxf(m, fabsf(xv[e])); xsum += xv[e]; }
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
            uint32_t bh[4], bl[4];
            float fac;
            if (FAST) {
                const float scale = m / 32639.f;
                int qv[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    float q = 0.f;
                    if (scale != 0.f) {
                        const float ratio = xv[e] / scale;
                        q = copysignf(floorf(fabsf(ratio) + 0.5f), ratio);
                    }
                    qv[e] = (int)q;
                    bsum += q;
                }
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                    const __half2 hh = __floats2half2_rn((float)(qv[e] >> 8), (float)(qv[e + 1] >> 8));
                    const __half2 ll = __floats2half2_rn((float)(qv[e] & 255), (float)(qv[e + 1] & 255));
                    bh[e / 2] = *reinterpret_cast<const uint32_t *>(&hh);
                    bl[e / 2] = *reinterpret_cast<const uint32_t *>(&ll);
                }
                fac = scale;
            } else {
                // power-of-two scale taking the block maximum into [2^14, 2^15)
                int ex = m > 0.f ? ((__float_as_int(m) >> 23) & 255) - 127 : 0;
                ex = min(max(ex, -100), 100);
                const float sc = __int_as_float((127 + 14 - ex) << 23);
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                    const float y0 = xv[e] * sc, y1 = xv[e + 1] * sc;
                    const __half2 hh = __floats2half2_rn(y0, y1);
                    const float2 back = __half22float2(hh);
                    const __half2 ll = __floats2half2_rn(y0 - back.x, y1 - back.y);
                    const float2 lb = __half22float2(ll);
                    bsum += (back.x + lb.x) + (back.y + lb.y);
                    bh[e / 2] = *reinterpret_cast<const uint32_t *>(&hh);
                    bl[e / 2] = *reinterpret_cast<const uint32_t *>(&ll);
                }
                fac = __int_as_float((127 - 14 + ex) << 23);
            }
            xsum += __shfl_xor_sync(0xffffffffu, xsum, 1);
            xsum += __shfl_xor_sync(0xffffffffu, xsum, 2);
            bsum += __shfl_xor_sync(0xffffffffu, bsum, 1);          // per 16 columns
            uint8_t *bt = smem + L::SM_B + st * PM_B_BYTES;
            *reinterpret_cast<uint4 *>(bt + pm_sw(16, t, kx)) = make_uint4(bh[0], bh[1], bh[2], bh[3]);
            *reinterpret_cast<uint4 *>(bt + pm_sw(16, 8 + t, kx)) = make_uint4(bl[0], bl[1], bl[2], bl[3]);
            // per 32-column block: the factor of 2^24 sum(a b) (a the biased quant);
            // per 16 columns: the bias term BIAS sum(b) times the factor
            constexpr float BIAS = KIND == 8 ? 128.f : (KIND == 14 ? 32.f : 0.f);
            if ((ib & 3) == 0) {
                const int q = (st * PM_T + t) * 4 + (kx >> 5);
                fs[q] = t < a.T ? fac * 16777216.f : 0.f;
                xs[q] = t < a.T ? xsum : 0.f;
            }
            if ((ib & 1) == 0) bs[(st * PM_T + t) * 8 + (kx >> 4)] = t < a.T ? BIAS * bsum * fac : 0.f;
            // ---- this row's quants of the stage into the A tile as fp16
            //      subnormals (bits = the small integer k: value k 2^-24, exact),
            //      unsigned (Q8_0: q + 128, Q6_K: q + 32; the readback removes the
            //      bias through the block sums), and its scales
            const int slot = c % R;
            if (!pm_wait_warp(raw_full + slot, (c / R) & 1, abort_flag)) { ok = false; break; }
            const uintptr_t s0 = reinterpret_cast<uintptr_t>(a.w) + (size_t)(row0 + r) * row_bytes + (size_t)c * F::CB;
            const uint8_t *p = smem + L::SM_RAW + slot * PM_ROWS * RS + r * RS + (a.tma ? 0 : (s0 & 15));
            uint8_t *at = smem + L::SM_A + st * PM_A_BYTES;
            float *swr = sw + (st * PM_ROWS + r) * L::NG;
            if (r < nrows) {
                if (KIND == 8) {
                    for (int b = 0; b < ng; ++b) {                                 // 32-column blocks of the stage
                        const uint8_t *blk = p + (h * 4 + b) * 34;
                        swr[b] = pm_half(blk);
#pragma unroll
                        for (int q8 = 0; q8 < 4; ++q8) {
                            const uint32_t w0 = pm_word(blk + 2 + 8 * q8) ^ 0x80808080u;
                            const uint32_t w1 = pm_word(blk + 6 + 8 * q8) ^ 0x80808080u;
                            *reinterpret_cast<uint4 *>(at + pm_sw(PM_ROWS, r, b * 32 + 8 * q8)) =
                                make_uint4(__byte_perm(w0, 0, 0x4140), __byte_perm(w0, 0, 0x4342),
                                           __byte_perm(w1, 0, 0x4140), __byte_perm(w1, 0, 0x4342));
                        }
                    }
                } else if (KIND == 12) {
                    const float d = pm_half(p), dmin = pm_half(p + 2);
                    const uint8_t *sc = p + 4;
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) {
                        const int j = 4 * h + jj;                                  // sub-block of the super-block
                        const int s6 = j < 4 ? (sc[j] & 63) : ((sc[j + 4] & 15) | ((sc[j - 4] >> 6) << 4));
                        const int m6 = j < 4 ? (sc[j + 4] & 63) : ((sc[j + 4] >> 4) | ((sc[j] >> 6) << 4));
                        swr[jj] = d * (float)s6;
                        mn[(st * PM_ROWS + r) * 4 + jj] = dmin * (float)m6;
                    }
                    // the half's 64 quant bytes (16-byte aligned): byte 32 p + l holds
                    // column l of sub-blocks 2p (low nibble) and 2p + 1 (high)
                    const uint4 *qv = reinterpret_cast<const uint4 *>(p + 16 + 64 * h);
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        const uint4 q4 = qv[v];
                        const uint32_t ws[4] = {q4.x, q4.y, q4.z, q4.w};
                        uint32_t lo[8], hi[8];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const uint32_t t0 = __byte_perm(ws[e], 0, 0x4140), t1 = __byte_perm(ws[e], 0, 0x4342);
                            lo[2 * e] = t0 & 0x000F000Fu; lo[2 * e + 1] = t1 & 0x000F000Fu;
                            hi[2 * e] = (t0 >> 4) & 0x000F000Fu; hi[2 * e + 1] = (t1 >> 4) & 0x000F000Fu;
                        }
                        const int c0 = (v >> 1) * 64 + (v & 1) * 16;             // sub-block 2p, columns l0..l0+15
                        *reinterpret_cast<uint4 *>(at + pm_sw(PM_ROWS, r, c0)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                        *reinterpret_cast<uint4 *>(at + pm_sw(PM_ROWS, r, c0 + 8)) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
                        *reinterpret_cast<uint4 *>(at + pm_sw(PM_ROWS, r, c0 + 32)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                        *reinterpret_cast<uint4 *>(at + pm_sw(PM_ROWS, r, c0 + 40)) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
                    }
                } else {
                    const float d = pm_half(p + 208);
#pragma unroll
                    for (int g = 0; g < 8; ++g) swr[g] = d * (float)(int8_t)p[192 + 8 * h + g];
                    const uint8_t *ql = p + 64 * h, *qh = p + 128 + 32 * h;
#pragma unroll
                    for (int l0 = 0; l0 < 32; l0 += 8) {
                        uint32_t wa[2], wb[2], wh[2];
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            wa[e] = pm_word(ql + l0 + 4 * e);                      // quarters 0 (low) and 2 (high)
                            wb[e] = pm_word(ql + 32 + l0 + 4 * e);                 // quarters 1 and 3
                            wh[e] = pm_word(qh + l0 + 4 * e);
                        }
#pragma unroll
                        for (int qu = 0; qu < 4; ++qu) {
                            uint32_t v[4];
#pragma unroll
                            for (int e = 0; e < 2; ++e) {
                                const uint32_t lw = ((qu & 1) ? wb[e] : wa[e]) >> (4 * (qu >> 1));
                                const int sh = 2 * qu;                              // high bits to bits 4-5 of each byte
                                const uint32_t hw = sh <= 4 ? (wh[e] << (4 - sh)) : (wh[e] >> (sh - 4));
                                const uint32_t q6 = (lw & 0x0F0F0F0Fu) | (hw & 0x30303030u);
                                v[2 * e] = __byte_perm(q6, 0, 0x4140);
                                v[2 * e + 1] = __byte_perm(q6, 0, 0x4342);
                            }
                            *reinterpret_cast<uint4 *>(at + pm_sw(PM_ROWS, r, qu * 32 + l0)) = make_uint4(v[0], v[1], v[2], v[3]);
                        }
                    }
                }
            }
            // generic-proxy writes of A / B -> visible to the tensor core (async proxy)
            fence_async_shared();
            __syncwarp();
            if (lane == 0) { mbar_arrive(a_full + st); mbar_arrive(raw_empty + slot); }
        }
    } else {
        // ------------------------------------------------ readback: thread = (row, 4 tokens)
        // D holds 2^-24 sum_k a_k b_k (a the biased integer quant, b the scaled
        // activations); per token v = (c D_hi + D_lo) F - B is the block's dot
        // product of the quants with the activations (F = 2^24 times the block's
        // activation factor, B its bias term), then acc += v s_row (- m_row xsum
        // for Q4_K); the stages' sums are added compensated (Kahan).
        const int r = (warp & 3) * 32 + lane, t0 = 4 * (warp >> 2);
        const uint32_t t_lane = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        float acc[4], cmp[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) { acc[k] = 0.f; cmp[k] = 0.f; }
        int gseq = 0;
        bool ok = true;
        for (int u = 0; u < nstages && ok; ++u) {
            const int st = u % NA;
            if (!pm_wait_warp(a_full + st, (u / NA) & 1, abort_flag)) { ok = false; break; }
            const int ng = stage_groups(u);
            const float *swr = sw + (st * PM_ROWS + r) * L::NG;
            const float *fst = fs + st * PM_T * 4, *xst = xs + st * PM_T * 4, *bst = bs + st * PM_T * 8;
            // up to four groups together: their accumulators are read at once, so
            // one TMEM round trip serves them
            constexpr int NB = NGH < 4 ? NGH : 4;
            float part[4] = {0.f, 0.f, 0.f, 0.f};
            for (int g0 = 0; g0 < ng && ok; g0 += NB) {
                float dh[NB][4], dl[NB][4];
#pragma unroll
                for (int gg = 0; gg < NB; ++gg) {
                    if (g0 + gg >= ng) break;
                    const int q = gseq + g0 + gg, slot = q % PM_NS;
                    if (!pm_wait_warp(d_full + slot, (q / PM_NS) & 1, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    pm_tmem_ld4(t_lane + slot * 16 + t0, dh[gg]);
                    pm_tmem_ld4(t_lane + slot * 16 + 8 + t0, dl[gg]);
                }
                tmem_wait_ld();                                  // also before leaving on a timeout
                if (!ok) break;
                tc_fence_before();
                __syncwarp();
                if (lane == 0)
                    for (int gg = 0; gg < NB && g0 + gg < ng; ++gg) mbar_arrive(d_empty + (gseq + g0 + gg) % PM_NS);
#pragma unroll
                for (int gg = 0; gg < NB; ++gg) {
                    const int g = g0 + gg;
                    if (g >= ng) break;
                    const int blk = G == 32 ? g : (g >> 1);
                    const float s = swr[g], mnr = KIND == 12 ? mn[(st * PM_ROWS + r) * 4 + g] : 0.f;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int t = t0 + k;
                        const float uv = FAST ? fmaf(256.f, dh[gg][k], dl[gg][k]) : dh[gg][k] + dl[gg][k];
                        float bt = 0.f;
                        if (KIND != 12) bt = G == 32 ? bst[t * 8 + 2 * g] + bst[t * 8 + 2 * g + 1] : bst[t * 8 + g];
                        part[k] = fmaf(fmaf(uv, fst[t * 4 + blk], -bt), s, part[k]);
                        if (KIND == 12) part[k] = fmaf(-mnr, xst[t * 4 + blk], part[k]);
                    }
                }
            }
            if (!ok) break;
            gseq += ng;
            __syncwarp();
            if (lane == 0) mbar_arrive(s_empty + st);
#pragma unroll
            for (int k = 0; k < 4; ++k) {                      // compensated sum over the stages
                const float y = part[k] - cmp[k], tt = acc[k] + y;
                cmp[k] = (tt - acc[k]) - y;
                acc[k] = tt;
            }
        }
        if (ok && r < nrows) {
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (t0 + k < a.T) a.out[(size_t)(t0 + k) * a.rows + row0 + r] = acc[k];
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 18) tmem_dealloc(tmem, PM_NS * 16);
}

// 3-D map of the weights as 16-byte pieces: (16 bytes, row_bytes / 16 pieces,
// rows), boxes of one chunk's pieces of 128 rows.
template <int KIND>
CUtensorMap weight_map(const PmArgs &a) {
    using F = PmFormat<KIND>;
    CUtensorMap m;
    const size_t row_bytes = (size_t)(a.width / F::SB) * F::BB;
    cuuint64_t dims[3] = {16, (cuuint64_t)(row_bytes / 16), (cuuint64_t)a.rows};
    cuuint64_t strides[2] = {16, (cuuint64_t)row_bytes};
    cuuint32_t box[3] = {16, (cuuint32_t)(F::CB / 16), (cuuint32_t)PM_ROWS};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t *>(a.w), dims, strides,
                                            box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return m;
}

template <int KIND>
cudaError_t launch_kind(PmArgs a, bool fast, cudaStream_t st) {
    static PerDeviceOnce configured;
    configured.run([] {
        if (cudaFuncSetAttribute(qmm_tc_kernel<KIND, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, PmLayout<KIND>::SMEM) !=
                cudaSuccess ||
            cudaFuncSetAttribute(qmm_tc_kernel<KIND, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, PmLayout<KIND>::SMEM) !=
                cudaSuccess)
            throw std::runtime_error("cannot reserve shared memory for the projection kernel");
    });
    using F = PmFormat<KIND>;
    const size_t row_bytes = (size_t)(a.width / F::SB) * F::BB;
    a.tma = row_bytes % 16 == 0 && F::CB % 16 == 0 && F::CB / 16 <= 256;
    CUtensorMap m{};
    if (a.tma) m = weight_map<KIND>(a);
    const dim3 grid((a.rows + PM_ROWS - 1) / PM_ROWS), block(PM_THREADS);
    return fast ? launch_chained(qmm_tc_kernel<KIND, true>, grid, block, PmLayout<KIND>::SMEM, st, m, a)
                : launch_chained(qmm_tc_kernel<KIND, false>, grid, block, PmLayout<KIND>::SMEM, st, m, a);
}

}  // namespace

size_t projection_weight_bytes(int kind, int width, int rows) {
    const int sb = kind == 8 ? 32 : 256, bb = kind == 8 ? 34 : (kind == 12 ? 144 : 210);
    return (size_t)(width / sb) * bb * rows;
}

void projection_run(float *out, const void *weights, const float *x, int kind, int T, int width, int rows,
                    bool fast, cudaStream_t st) {
    if (T < 1 || T > PM_T) throw std::invalid_argument("projection batch must be between 1 and 8");
    if (reinterpret_cast<uintptr_t>(weights) & 15) throw std::invalid_argument("projection weights must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(x) & 15) throw std::invalid_argument("projection activations must be 16-byte aligned");
    PmArgs a{out, static_cast<const uint8_t *>(weights), x, projection_weight_bytes(kind, width, rows), T, width, rows, 0};
    cudaError_t e;
    if (kind == 8) e = launch_kind<8>(a, fast, st);
    else if (kind == 12) e = launch_kind<12>(a, fast, st);
    else if (kind == 14) e = launch_kind<14>(a, fast, st);
    else throw std::invalid_argument("unsupported quantization type");
    if (e != cudaSuccess) throw std::runtime_error(std::string("projection: ") + cudaGetErrorString(e));
}

}  // namespace qv
