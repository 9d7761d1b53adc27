// Gated DeltaNet recurrent path for sm_100a: one fused kernel per layer call.
//
// The reference runs conv -> gdn_prep -> gdn_scan -> delta_out as four
// launches (src/kernels.cu:275-354, 409-414, 557-566).  Here a cluster of
// CPH CTAs owns one value head; each CTA owns D/CPH rows of the head's
// [Dv][Dk] fp32 state, held in registers.  The cluster filters (causal conv
// + SiLU) the q/k channels of its key head (h % Hk) and its v rows, forms the
// L2 norms, the decay a = exp(A softplus(alpha+bias)) and beta = sigmoid(beta),
// and runs the delta rule over the tokens.  The gated RMSNorm needs the whole
// head's readout: the per-CTA sums of squares are exchanged through
// distributed shared memory.  The state is read and written exactly once.
#include "common.cuh"
#include "hotpath.h"

#include <cooperative_groups.h>
#include <stdexcept>
#include <string>

namespace cg = cooperative_groups;

namespace qv {

constexpr int CHUNK = 8;   // tokens staged in shared memory at a time

struct DeltaArgs {
    float *out, *state, *history;
    const float *qkv, *gate, *alpha, *beta, *conv, *decay, *bias, *norm;
    // core mode (no conv / no gated norm): fp16 inputs
    const __half *q16, *k16, *v16;
    // verify recording (layer mode, T <= 8): start state / history copies and
    // the transition trace; null when not recording
    float *saved_state, *saved_history, *trace;
    int T, Hk, Hv;
    float eps;
};

// Transition trace of one recorded verify call (the layout of the reference's
// transitions buffer, src/runtime.cu:369 with src/kernels.cu:356-360): per
// token t < 8, the raw qkv row [t][C], the prepared row [8 + t][C] (q and k
// L2-normalised, q also scaled by 1/sqrt(D), v filtered), then the decays
// [16 C + t Hv + h] and the betas [16 C + 8 Hv + t Hv + h].
__host__ __device__ constexpr size_t delta_trace_floats(int C, int Hv) { return 8 * (2 * (size_t)C + 2 * (size_t)Hv); }

// CORE = false: reference layer semantics (conv, SiLU, gated RMSNorm).
// CORE = true : prepared-input recurrence (raw fp16 q/k/v are L2-normalised
//               here; the output is the state readout before the gated norm).
//
// Grid: CPH CTAs per value head (a cluster); every CTA must own an SM, since
// an SM holding two CTAs would double the time of its whole cluster.
// Thread layout: every thread filters one conv channel; the token loop runs
// TPP threads per PAIR of state rows (16 for D = 128: every thread of the
// CTA; 8 for D = 32), each holding D/TPP columns of both rows (columns
// 4 TPP i + 4j + e), so every k/q value read from shared memory serves two
// rows, and the four dot products of a token (S_a.k, S_b.k, S_a.q, S_b.q,
// all against the state before the token's update) reduce together in one
// transposing butterfly (5 shuffles over 16 lanes, 4 over 8).  Per chunk of
// <= 8 tokens:
//  * the chunk's inputs are loaded one chunk ahead (chunk 0 with the
//    prologue), so their latency overlaps the previous chunk's scan;
//  * each CTA filters (conv + SiLU) all q/k channels of its key head and its
//    own v rows, so the q/k L2 norms need no cross-CTA exchange; the norms
//    are applied as scalars inside the dot products (u = sk*(S.k),
//    o = sq*(S.q), the rank-1 update uses sk*delta);
//  * the gated RMSNorm's per-token sum of squares is the only cross-CTA
//    value: every CTA pushes its partial into each peer's shared memory and
//    arrives on the peer's mbarrier (one-way, no cluster-wide barrier).
// D=128 uses CPH=2 (64 rows, 512 threads): clusters must fit inside one GPC,
// and 48 clusters of 3 do not all fit at once on B200, which then runs a
// second wave; clusters of 2 always fit (one CTA per SM, 96 SMs).
template <int D, int CPH> struct DeltaShape {
    static constexpr int MAXR = (D + CPH - 1) / CPH;              // most rows of a rank
    static constexpr int TPP = D >= 128 ? 16 : 8;                  // token-loop threads per pair of rows
    static constexpr int LOOP = (MAXR + 1) / 2 * TPP;              // token-loop threads
    static constexpr int NEED = LOOP > CHUNK * MAXR ? (LOOP > 2 * D + MAXR ? LOOP : 2 * D + MAXR)
                                                    : (CHUNK * MAXR > 2 * D + MAXR ? CHUNK * MAXR : 2 * D + MAXR);
    static constexpr int NT = ((NEED > 8 * MAXR ? NEED : 8 * MAXR) + 31) / 32 * 32;   // threads per CTA
};

template <int D, int CPH, bool CORE, bool RECORD = false>
__global__ void __cluster_dims__(CPH, 1, 1) __launch_bounds__(DeltaShape<D, CPH>::NT)
delta_kernel(const DeltaArgs a) {
    static_assert(!(CORE && RECORD), "only the layer mode records a verify");
    constexpr int MAXR = DeltaShape<D, CPH>::MAXR, NT = DeltaShape<D, CPH>::NT, TPP = DeltaShape<D, CPH>::TPP;
    constexpr int COLS = D / TPP, NV4 = COLS / 4, CSTRIDE = 4 * TPP, NW = NT / 32;
    static_assert(NV4 >= 1 && COLS % 4 == 0, "a thread holds whole float4 groups of its rows");
    static_assert(2 * D + MAXR <= NT, "one conv channel per thread");
    static_assert(CHUNK * MAXR <= NT, "one output per thread per chunk");
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = CPH > 1 ? (int)cluster.block_rank() : 0;
    const int h = blockIdx.x / CPH, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int Hk = a.Hk, Hv = a.Hv, kh = h % Hk;
    const int C = (2 * Hk + Hv) * D;
    const int row0 = rank * D / CPH, rows = (rank + 1) * D / CPH - row0;   // this CTA's head rows
    // token loop: TPP threads per PAIR of state rows (rows ra, rb), D/TPP
    // columns of each; every k/q value read from shared memory serves both rows
    const int j = tid % TPP, ra = 2 * (tid / TPP), rb = ra + 1;
    const bool has_a = ra < rows, has_b = rb < rows, scans = tid < DeltaShape<D, CPH>::LOOP;

    __shared__ __align__(16) float Fq[CHUNK][D], Fk[CHUNK][D], Fv[CHUNK][MAXR];
    __shared__ __align__(16) float O[CHUNK][MAXR];
    __shared__ float wsum[NW][CHUNK];             // per-warp sums of q^2 or k^2
    __shared__ __align__(16) float scal[CHUNK][8];  // sq, sk, decay, beta, k.q
    __shared__ float osum[2][CPH][CHUNK];         // sums of o^2 pushed by each rank, by chunk parity
    __shared__ __align__(8) uint64_t osum_bar[2];
    __shared__ bool norm_ok;

    if (tid == 0) QV_STAMP(0);
    // Conv channel of this thread: e < D -> q, e < 2D -> k, e < 2D + rows -> v row.
    const int e = tid;
    int c = -1;
    if (e < D) c = kh * D + e;
    else if (e < 2 * D) c = (Hk + kh) * D + (e - D);
    else if (e < 2 * D + rows) c = (2 * Hk + h) * D + row0 + (e - 2 * D);
#ifndef QV_DELTA_PREFETCH
#define QV_DELTA_PREFETCH 1
#endif
    if (!CORE && QV_DELTA_PREFETCH) {
        // L2 prefetch hints, issued before the dependency wait so that their
        // HBM latency overlaps the previous kernel: this CTA's state block
        // (rows row0.. of head h, contiguous), and per warp the lines of its
        // channels' raw inputs, history and conv taps, and of its outputs' gates.
        const float *sblk = a.state + ((size_t)h * D + row0) * D;
        for (int i = tid; i < rows * D / 32; i += NT) prefetch_l2(sblk + 32 * i);
        if (c >= 0 && lane == 0) {
            for (int t = 0; t < a.T && t < CHUNK; ++t) prefetch_l2(a.qkv + (size_t)t * C + c);
            for (int r = 0; r < 3; ++r) prefetch_l2(a.history + (size_t)r * C + c);
        }
        if (c >= 0 && lane < 4) prefetch_l2(a.conv + (size_t)(c + 7 * lane) * 4);   // channels c0 + 8 lane..
        if (lane == 0 && tid < CHUNK * rows && tid / rows < a.T)
            prefetch_l2(a.gate + ((size_t)(tid / rows) * Hv + h) * D + row0 + tid % rows);
        if (tid < a.T && tid < CHUNK) {
            prefetch_l2(a.alpha + (size_t)tid * Hv + h);
            prefetch_l2(a.beta + (size_t)tid * Hv + h);
        }
    }
    if (!CORE && tid == 0) {
        // each rank's CHUNK token-warps arrive once per chunk
        mbar_init(&osum_bar[0], CPH * CHUNK);
        mbar_init(&osum_bar[1], CPH * CHUNK);
        fence_barrier_init();
    }
    // Peers arrive on osum_bar only after it is initialised everywhere (this
    // needs no memory written by another kernel, so it overlaps the previous one).
    if (!CORE && CPH > 1) cluster.sync();
    if (tid == 0) QV_STAMP(1);
    // State, history and inputs may have been written by the previous kernel.
    grid_dependency_wait();
    if (tid == 0) { launch_dependents(); QV_STAMP(2); }

    // ---- loads that do not depend on the chunk
    float w0 = 0.f, w1 = 0.f, w2 = 0.f, w3 = 0.f, h0 = 0.f, h1 = 0.f, h2 = 0.f;
    if (!CORE && c >= 0) {
        const float4 w = *reinterpret_cast<const float4 *>(a.conv + (size_t)c * 4);
        w0 = w.x; w1 = w.y; w2 = w.z; w3 = w.w;
        h0 = a.history[c]; h1 = a.history[(size_t)C + c]; h2 = a.history[2 * (size_t)C + c];
    }
    // One CTA owns each channel's history (and trace) entries: v channels
    // their rows' CTA, the q/k channels of key head kh rank 0 of value head kh.
    const bool owns_channel = c >= 0 && (e >= 2 * D || (h < Hk && rank == 0));
    if (RECORD && owns_channel) {
        a.saved_history[c] = h0; a.saved_history[(size_t)C + c] = h1; a.saved_history[2 * (size_t)C + c] = h2;
    }
    const float decay_h = a.decay[h], bias_h = a.bias[h];
    // Output of this thread in each chunk: token tid / rows, row tid % rows.
    const bool has_out = tid < CHUNK * rows;
    const int out_t = has_out ? tid / rows : 0, out_i = has_out ? tid % rows : 0;
    const float nw = (!CORE && has_out) ? a.norm[row0 + out_i] : 1.f;

    // Chunk inputs are prefetched one chunk ahead (chunk 0 with the prologue).
    float raw_n[CHUNK], al_n = 0.f, be_n = 0.f, gz_n = 0.f;
    auto load_chunk = [&](int c0) {
        const int m = min(CHUNK, a.T - c0);
#pragma unroll
        for (int tt = 0; tt < CHUNK; ++tt) {
            raw_n[tt] = 0.f;
            if (c >= 0 && tt < m) {
                const int t = c0 + tt;
                if (!CORE) raw_n[tt] = a.qkv[(size_t)t * C + c];
                else if (e < D) raw_n[tt] = __half2float(a.q16[((size_t)t * Hk + kh) * D + e]);
                else if (e < 2 * D) raw_n[tt] = __half2float(a.k16[((size_t)t * Hk + kh) * D + e - D]);
                else raw_n[tt] = __half2float(a.v16[((size_t)t * Hv + h) * D + row0 + e - 2 * D]);
            }
        }
        if (tid < m) {
            const size_t idx = (size_t)(c0 + tid) * Hv + h;
            al_n = a.alpha[idx];
            be_n = a.beta[idx];
        }
        gz_n = (!CORE && has_out && out_t < m) ? a.gate[((size_t)(c0 + out_t) * Hv + h) * D + row0 + out_i] : 0.f;
    };
    load_chunk(0);
    // The state is first needed in the token loop: its loads go out after the
    // inputs of the conv, which is needed first.
    float2 Sa[COLS / 2], Sb[COLS / 2];       // column pairs (4i, 4i+1), (4i+2, 4i+3) of float4 group i
    float *srow_a = a.state + ((size_t)h * D + row0 + (has_a ? ra : 0)) * D;
    float *srow_b = a.state + ((size_t)h * D + row0 + (has_b ? rb : 0)) * D;
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
        float4 va = make_float4(0.f, 0.f, 0.f, 0.f), vb = va;
        if (has_a) va = *reinterpret_cast<const float4 *>(srow_a + CSTRIDE * i + 4 * j);
        if (has_b) vb = *reinterpret_cast<const float4 *>(srow_b + CSTRIDE * i + 4 * j);
        Sa[2 * i] = make_float2(va.x, va.y); Sa[2 * i + 1] = make_float2(va.z, va.w);
        Sb[2 * i] = make_float2(vb.x, vb.y); Sb[2 * i + 1] = make_float2(vb.z, vb.w);
        if (RECORD && has_a)
            *reinterpret_cast<float4 *>(a.saved_state + (srow_a - a.state) + CSTRIDE * i + 4 * j) = va;
        if (RECORD && has_b)
            *reinterpret_cast<float4 *>(a.saved_state + (srow_b - a.state) + CSTRIDE * i + 4 * j) = vb;
    }

    for (int t0 = 0, chunk = 0; t0 < a.T; t0 += CHUNK, ++chunk) {
        const int n = min(CHUNK, a.T - t0);
        // ---- this chunk's inputs were prefetched; start the next chunk's loads
        float raw[CHUNK];
#pragma unroll
        for (int tt = 0; tt < CHUNK; ++tt) raw[tt] = raw_n[tt];
        const float al = al_n, be = be_n, gz = gz_n;
        if (t0 + CHUNK < a.T) load_chunk(t0 + CHUNK);
        // ---- conv + SiLU in registers; per-warp sums of squares of q (warps
        //      [0, D/32)) and k (warps [D/32, 2D/32))
        float sq2[CHUNK];
#pragma unroll
        for (int tt = 0; tt < CHUNK; ++tt) {
            float f = raw[tt];
            if (!CORE && tt < n) {
                float v = w3 * f;
                v += w0 * h0; v += w1 * h1; v += w2 * h2;
                h0 = h1; h1 = h2; h2 = f;
                f = silu_fast(v);
            }
            sq2[tt] = 0.f;
            if (c >= 0 && tt < n) {
                if (e < D) { Fq[tt][e] = f; sq2[tt] = f * f; }
                else if (e < 2 * D) { Fk[tt][e - D] = f; sq2[tt] = f * f; }
                else Fv[tt][e - 2 * D] = f;
            }
        }
        if (warp < 2 * D / 32) {
#pragma unroll
            for (int tt = 0; tt < CHUNK; ++tt) {
                const float sum = warp_sum(sq2[tt]);
                if (lane == 0) wsum[warp][tt] = sum;
            }
        }
        __syncthreads();
        if (tid == 0 && chunk == 0) QV_STAMP(3);
        if (tid < n) {
            float qs = 0.f, ks = 0.f;
#pragma unroll
            for (int w = 0; w < D / 32; ++w) { qs += wsum[w][tid]; ks += wsum[D / 32 + w][tid]; }
            scal[tid][0] = rsqrtf(qs + 1e-6f) * rsqrtf((float)D);
            scal[tid][1] = rsqrtf(ks + 1e-6f);
            scal[tid][2] = expf(decay_h * softplusf_(al + bias_h));
            scal[tid][3] = sigmoid_fast(be);
        }
        // k.q of each token (filtered, not normalised), one warp per token
        for (int tt = warp; tt < n; tt += NW) {
            float x = 0.f;
#pragma unroll
            for (int i = 0; i < D / 32; ++i) x = fmaf(Fq[tt][lane + 32 * i], Fk[tt][lane + 32 * i], x);
            x = warp_sum(x);
            if (lane == 0) scal[tt][4] = x;
        }
        __syncthreads();
        if (tid == 0 && chunk == 0) QV_STAMP(4);
        if (RECORD) {
            // transition trace (recorded calls have a single chunk)
            if (owns_channel) {
#pragma unroll
                for (int tt = 0; tt < CHUNK; ++tt) {
                    if (tt >= n) break;
                    const float prep = e < D ? Fq[tt][e] * scal[tt][0]
                                     : e < 2 * D ? Fk[tt][e - D] * scal[tt][1] : Fv[tt][e - 2 * D];
                    a.trace[(size_t)tt * C + c] = raw[tt];
                    a.trace[(size_t)(CHUNK + tt) * C + c] = prep;
                }
            }
            if (rank == 0 && tid < n) {
                a.trace[16 * (size_t)C + (size_t)tid * Hv + h] = scal[tid][2];
                a.trace[16 * (size_t)C + 8 * (size_t)Hv + (size_t)tid * Hv + h] = scal[tid][3];
            }
        }
        // ---- delta rule over the chunk: S = a S; u = S k; delta = beta (v - u);
        //      S += delta k^T; o = S q   (k, q normalised through sk, sq).  The
        //      decay is applied inside the update: u = a (S k), S = a S + delta k,
        //      and the readout is o = a (S q) + delta (k.q): both dot products are
        //      taken against the state before the token's update and reduced
        //      together across the pair's 8 lanes by a transposing butterfly
        //      (lanes j = 0,1: S_a.k, 2,3: S_b.k, 4,5: S_a.q, 6,7: S_b.q).
        if (scans) {
#pragma unroll
            for (int tt = 0; tt < CHUNK; ++tt) {
                if (tt >= n) break;
                const float4 sc = *reinterpret_cast<const float4 *>(scal[tt]);
                const float sqn = sc.x, skn = sc.y, decay = sc.z, beta = sc.w, kq = scal[tt][4];
                const float4 *kk = reinterpret_cast<const float4 *>(Fk[tt]);
                const float4 *qq = reinterpret_cast<const float4 *>(Fq[tt]);
                float4 k4[NV4];
                float2 ua2 = make_float2(0.f, 0.f), ub2 = ua2, wa2 = ua2, wb2 = ua2;
#pragma unroll
                for (int i = 0; i < NV4; ++i) {
                    k4[i] = kk[TPP * i + j];
                    const float4 q4 = qq[TPP * i + j];
                    const float2 kl = make_float2(k4[i].x, k4[i].y), kh = make_float2(k4[i].z, k4[i].w);
                    const float2 ql = make_float2(q4.x, q4.y), qh = make_float2(q4.z, q4.w);
                    ua2 = ffma2(Sa[2 * i], kl, ua2); ua2 = ffma2(Sa[2 * i + 1], kh, ua2);
                    ub2 = ffma2(Sb[2 * i], kl, ub2); ub2 = ffma2(Sb[2 * i + 1], kh, ub2);
                    wa2 = ffma2(Sa[2 * i], ql, wa2); wa2 = ffma2(Sa[2 * i + 1], qh, wa2);
                    wb2 = ffma2(Sb[2 * i], ql, wb2); wb2 = ffma2(Sb[2 * i + 1], qh, wb2);
                }
                const float ua0 = ua2.x, ua1 = ua2.y, ub0 = ub2.x, ub1 = ub2.y;
                const float wa0 = wa2.x, wa1 = wa2.y, wb0 = wb2.x, wb1 = wb2.y;
                const float ua = ua0 + ua1, ub = ub0 + ub1, wa = wa0 + wa1, wb = wb0 + wb1;
                // Transposing butterfly over the pair's TPP lanes: afterwards the
                // lanes of the first quarter hold S_a.k, the second S_b.k, the
                // third S_a.q, the fourth S_b.q (each the full 128-column sum).
                float m;
                bool hq;                                   // this lane's sum is of row b
                if (TPP == 16) {
                    const bool h8 = (j & 8) != 0;
                    hq = (j & 4) != 0;
                    float x0 = h8 ? wa : ua, x1 = h8 ? wb : ub;
                    x0 += __shfl_xor_sync(0xffffffffu, h8 ? ua : wa, 8);
                    x1 += __shfl_xor_sync(0xffffffffu, h8 ? ub : wb, 8);
                    m = hq ? x1 : x0;
                    m += __shfl_xor_sync(0xffffffffu, hq ? x0 : x1, 4);
                    m += __shfl_xor_sync(0xffffffffu, m, 2);
                    m += __shfl_xor_sync(0xffffffffu, m, 1);
                } else {
                    const bool hi4 = (j & 4) != 0;
                    hq = (j & 2) != 0;
                    float m0 = hi4 ? wa : ua, m1 = hi4 ? wb : ub;
                    m0 += __shfl_xor_sync(0xffffffffu, hi4 ? ua : wa, 4);
                    m1 += __shfl_xor_sync(0xffffffffu, hi4 ? ub : wb, 4);
                    m = hq ? m1 : m0;
                    m += __shfl_xor_sync(0xffffffffu, hq ? m0 : m1, 2);
                    m += __shfl_xor_sync(0xffffffffu, m, 1);
                }
                // delta of row a on the first quarter's lanes, of row b on the
                // second's; broadcast to the pair
                const int rl = hq ? rb : ra;
                const float vrow = rl < rows ? Fv[tt][rl] : 0.f;
                const float dl = (vrow - decay * m * skn) * beta * skn;
                const int base = lane & ~(TPP - 1);
                const float da = __shfl_sync(0xffffffffu, dl, base), db = __shfl_sync(0xffffffffu, dl, base + TPP / 4);
                // readout of row a / b on the first lane of the third / fourth quarter
                if ((j == TPP / 2 || j == 3 * TPP / 4) && rl < rows) O[tt][rl] = sqn * fmaf(decay, m, (hq ? db : da) * kq);
                const float2 dec2 = make_float2(decay, decay), da2 = make_float2(da, da), db2 = make_float2(db, db);
#pragma unroll
                for (int i = 0; i < NV4; ++i) {
                    const float2 kl = make_float2(k4[i].x, k4[i].y), kh = make_float2(k4[i].z, k4[i].w);
                    Sa[2 * i] = ffma2(kl, da2, fmul2(Sa[2 * i], dec2));
                    Sa[2 * i + 1] = ffma2(kh, da2, fmul2(Sa[2 * i + 1], dec2));
                    Sb[2 * i] = ffma2(kl, db2, fmul2(Sb[2 * i], dec2));
                    Sb[2 * i + 1] = ffma2(kh, db2, fmul2(Sb[2 * i + 1], dec2));
                }
            }
        }
        __syncthreads();
        if (tid == 0 && chunk == 0) QV_STAMP(5);
        if (t0 + CHUNK >= a.T) {
            // the state is final: its store (this CTA's rows only) overlaps the
            // gated-norm exchange below
#pragma unroll
            for (int i = 0; i < NV4; ++i) {
                if (has_a)
                    *reinterpret_cast<float4 *>(srow_a + CSTRIDE * i + 4 * j) =
                        make_float4(Sa[2 * i].x, Sa[2 * i].y, Sa[2 * i + 1].x, Sa[2 * i + 1].y);
                if (has_b)
                    *reinterpret_cast<float4 *>(srow_b + CSTRIDE * i + 4 * j) =
                        make_float4(Sb[2 * i].x, Sb[2 * i].y, Sb[2 * i + 1].x, Sb[2 * i + 1].y);
            }
        }
        if (CORE) {
            if (has_out && out_t < n) a.out[((size_t)(t0 + out_t) * Hv + h) * D + row0 + out_i] = O[out_t][out_i];
        } else {
            // ---- gated RMSNorm over the whole head: warp tt reduces token tt's sum
            //      of squares over this CTA's rows and pushes it to every rank;
            //      one thread waits for all partials, the block barrier then
            //      orders them for the other threads.
            const int par = chunk & 1;
            if (warp < CHUNK) {
                float x = 0.f;
                for (int i = lane; i < rows; i += 32) x += O[warp][i] * O[warp][i];
                x = warp_sum(x);
                if (lane < CPH) {
                    st_cluster_f32(cluster_map(&osum[par][rank][warp], lane), x);
                    mbar_arrive_cluster(cluster_map(&osum_bar[par], lane));
                }
            }
            if (tid == 0) norm_ok = mbar_wait_cluster(&osum_bar[par], (uint32_t)(chunk >> 1) & 1);
            __syncthreads();
            if (tid == 0 && chunk == 0) QV_STAMP(6);
            if (norm_ok && has_out && out_t < n) {
                float total = 0.f;
#pragma unroll
                for (int q = 0; q < CPH; ++q) total += osum[par][q][out_t];
                const float scale = rsqrtf(total / D + a.eps);
                a.out[((size_t)(t0 + out_t) * Hv + h) * D + row0 + out_i] =
                    O[out_t][out_i] * scale * nw * silu_fast(gz);
            }
        }
        __syncthreads();
    }

    // History: v channels belong to their rows' CTA; the q/k channels of key
    // head kh are written by rank 0 of value head kh (h < Hk) only, at the end:
    // the other value heads of key head kh read these channels' old history
    // after their dependency wait.
    if (!CORE && c >= 0 && (e >= 2 * D || (h < Hk && rank == 0))) {
        a.history[c] = h0; a.history[(size_t)C + c] = h1; a.history[2 * (size_t)C + c] = h2;
    }
    if (tid == 0) QV_STAMP(7);
}

// Commit of a recorded verify call after `accepted` of its tokens were kept
// (the reference's commit, src/runtime.cu:432-454: copy the start state and
// history back, then k_delta_commit = commit_history + a state-only scan over
// the accepted tokens, src/kernels.cu:362-369, 567-574).  Fused here into one
// pass per (value head, row half): the start state is read once from its
// saved copy, the accepted tokens' prepared rows and gates are replayed from
// the trace, and the state and the conv history are written once.
template <int D, int CPH>
__global__ void __launch_bounds__(DeltaShape<D, CPH>::NT)
delta_commit_kernel(float *state, float *history, const float *saved_state, const float *saved_history,
                    const float *trace, int accepted, int Hk, int Hv) {
    constexpr int MAXR = DeltaShape<D, CPH>::MAXR, NV4 = D / 32, COLS = D / 8;
    const int rank = blockIdx.x % CPH, h = blockIdx.x / CPH, tid = threadIdx.x, kh = h % Hk;
    const int C = (2 * Hk + Hv) * D;
    const int row0 = rank * D / CPH, rows = (rank + 1) * D / CPH - row0;
    const int r = tid >> 3, j = tid & 7;
    const bool has_row = r < rows;
    __shared__ __align__(16) float Fk[CHUNK][D], Fv[CHUNK][MAXR];
    __shared__ float gat[CHUNK][2];                    // decay, beta
    grid_dependency_wait();
    if (tid == 0) launch_dependents();
    const float *prep = trace + (size_t)CHUNK * C;
    const float *decays = trace + 16 * (size_t)C, *betas = decays + 8 * (size_t)Hv;
    for (int i = tid; i < accepted * D; i += blockDim.x)
        Fk[i / D][i % D] = prep[(size_t)(i / D) * C + (Hk + kh) * D + i % D];
    for (int i = tid; i < accepted * rows; i += blockDim.x)
        Fv[i / rows][i % rows] = prep[(size_t)(i / rows) * C + (2 * Hk + h) * D + row0 + i % rows];
    if (tid < accepted) {
        gat[tid][0] = decays[(size_t)tid * Hv + h];
        gat[tid][1] = betas[(size_t)tid * Hv + h];
    }
    float S[COLS];
    const size_t srow = ((size_t)h * D + row0 + (has_row ? r : 0)) * D;
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (has_row) v = *reinterpret_cast<const float4 *>(saved_state + srow + 32 * i + 4 * j);
        S[4 * i] = v.x; S[4 * i + 1] = v.y; S[4 * i + 2] = v.z; S[4 * i + 3] = v.w;
    }
    __syncthreads();
    // the reference row update per token: S = a S; delta = b (v - S k); S += delta k
    for (int t = 0; t < accepted; ++t) {
        const float decay = gat[t][0], beta = gat[t][1];
        float4 k4[NV4];
        float u0 = 0.f, u1 = 0.f;
#pragma unroll
        for (int i = 0; i < NV4; ++i) {
            k4[i] = *reinterpret_cast<const float4 *>(&Fk[t][32 * i + 4 * j]);
            u0 += S[4 * i] * k4[i].x; u1 += S[4 * i + 1] * k4[i].y;
            u0 += S[4 * i + 2] * k4[i].z; u1 += S[4 * i + 3] * k4[i].w;
        }
        float u = u0 + u1;
        u += __shfl_xor_sync(0xffffffffu, u, 1);
        u += __shfl_xor_sync(0xffffffffu, u, 2);
        u += __shfl_xor_sync(0xffffffffu, u, 4);
        const float delta = ((has_row ? Fv[t][r] : 0.f) - decay * u) * beta;
#pragma unroll
        for (int i = 0; i < NV4; ++i) {
            S[4 * i] = fmaf(S[4 * i], decay, k4[i].x * delta);
            S[4 * i + 1] = fmaf(S[4 * i + 1], decay, k4[i].y * delta);
            S[4 * i + 2] = fmaf(S[4 * i + 2], decay, k4[i].z * delta);
            S[4 * i + 3] = fmaf(S[4 * i + 3], decay, k4[i].w * delta);
        }
    }
    if (has_row) {
#pragma unroll
        for (int i = 0; i < NV4; ++i)
            *reinterpret_cast<float4 *>(state + srow + 32 * i + 4 * j) =
                make_float4(S[4 * i], S[4 * i + 1], S[4 * i + 2], S[4 * i + 3]);
    }
    // conv history: the saved window shifted by the accepted raw rows (one
    // owner per channel, as in the layer kernel)
    const int e = tid;
    int c = -1;
    if (e < D) c = kh * D + e;
    else if (e < 2 * D) c = (Hk + kh) * D + (e - D);
    else if (e < 2 * D + rows) c = (2 * Hk + h) * D + row0 + (e - 2 * D);
    if (c >= 0 && (e >= 2 * D || (h < Hk && rank == 0))) {
        float w0 = saved_history[c], w1 = saved_history[(size_t)C + c], w2 = saved_history[2 * (size_t)C + c];
        for (int t = 0; t < accepted; ++t) { w0 = w1; w1 = w2; w2 = trace[(size_t)t * C + c]; }
        history[c] = w0; history[(size_t)C + c] = w1; history[2 * (size_t)C + c] = w2;
    }
}

namespace {
void check_launch(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
}  // namespace

// D = 128: 2-CTA clusters per value head (64 rows each); D = 32: one CTA.
void delta_run(float *out, float *state, float *history, const float *qkv, const float *gate,
               const float *alpha, const float *beta, const float *conv, const float *decay,
               const float *bias, const float *norm, int T, int Hk, int Hv, int D, float eps,
               cudaStream_t st) {
    DeltaArgs a{};
    a.out = out; a.state = state; a.history = history; a.qkv = qkv; a.gate = gate;
    a.alpha = alpha; a.beta = beta; a.conv = conv; a.decay = decay; a.bias = bias; a.norm = norm;
    a.T = T; a.Hk = Hk; a.Hv = Hv; a.eps = eps;
    cudaError_t e;
    if (D == 128) e = launch_chained(delta_kernel<128, 2, false>, dim3(Hv * 2), dim3(DeltaShape<128, 2>::NT), 0, st, a);
    else if (D == 32) e = launch_chained(delta_kernel<32, 1, false>, dim3(Hv), dim3(DeltaShape<32, 1>::NT), 0, st, a);
    else throw std::invalid_argument("unsupported DeltaNet dimension");
    check_launch(e, "delta");
}

// Recorded verify: delta_run plus the start-state/history copies and the
// transition trace (T <= 8).
void delta_verify(float *out, float *state, float *history, const float *qkv, const float *gate,
                  const float *alpha, const float *beta, const float *conv, const float *decay,
                  const float *bias, const float *norm, int T, int Hk, int Hv, int D, float eps,
                  float *saved_state, float *saved_history, float *trace, cudaStream_t st) {
    if (T < 1 || T > CHUNK) throw std::invalid_argument("a recorded verify holds 1..8 tokens");
    DeltaArgs a{};
    a.out = out; a.state = state; a.history = history; a.qkv = qkv; a.gate = gate;
    a.alpha = alpha; a.beta = beta; a.conv = conv; a.decay = decay; a.bias = bias; a.norm = norm;
    a.saved_state = saved_state; a.saved_history = saved_history; a.trace = trace;
    a.T = T; a.Hk = Hk; a.Hv = Hv; a.eps = eps;
    cudaError_t e;
    if (D == 128)
        e = launch_chained(delta_kernel<128, 2, false, true>, dim3(Hv * 2), dim3(DeltaShape<128, 2>::NT), 0, st, a);
    else if (D == 32)
        e = launch_chained(delta_kernel<32, 1, false, true>, dim3(Hv), dim3(DeltaShape<32, 1>::NT), 0, st, a);
    else throw std::invalid_argument("unsupported DeltaNet dimension");
    check_launch(e, "delta verify");
}

void delta_commit(float *state, float *history, const float *saved_state, const float *saved_history,
                  const float *trace, int accepted, int Hk, int Hv, int D, cudaStream_t st) {
    if (accepted < 0 || accepted > CHUNK) throw std::invalid_argument("accepted must be between 0 and 8");
    cudaError_t e;
    if (D == 128)
        e = launch_chained(delta_commit_kernel<128, 2>, dim3(Hv * 2), dim3(DeltaShape<128, 2>::NT), 0, st, state,
                           history, saved_state, saved_history, trace, accepted, Hk, Hv);
    else if (D == 32)
        e = launch_chained(delta_commit_kernel<32, 1>, dim3(Hv), dim3(DeltaShape<32, 1>::NT), 0, st, state, history,
                           saved_state, saved_history, trace, accepted, Hk, Hv);
    else throw std::invalid_argument("unsupported DeltaNet dimension");
    check_launch(e, "delta commit");
}

void delta_core_recurrent(float *out, float *state, const __half *q, const __half *k, const __half *v,
                          const float *alpha, const float *beta, const float *decay, const float *bias,
                          int T, int Hk, int Hv, int D, cudaStream_t st) {
    DeltaArgs a{};
    a.out = out; a.state = state; a.q16 = q; a.k16 = k; a.v16 = v;
    a.alpha = alpha; a.beta = beta; a.decay = decay; a.bias = bias;
    a.T = T; a.Hk = Hk; a.Hv = Hv;
    cudaError_t e;
    if (D == 128) e = launch_chained(delta_kernel<128, 2, true>, dim3(Hv * 2), dim3(DeltaShape<128, 2>::NT), 0, st, a);
    else if (D == 32) e = launch_chained(delta_kernel<32, 1, true>, dim3(Hv), dim3(DeltaShape<32, 1>::NT), 0, st, a);
    else throw std::invalid_argument("unsupported DeltaNet dimension");
    check_launch(e, "delta core");
}

}  // namespace qv
