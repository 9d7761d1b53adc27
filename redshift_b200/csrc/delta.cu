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
    int T, Hk, Hv;
    float eps;
};

// CORE = false: reference layer semantics (conv, SiLU, gated RMSNorm).
// CORE = true : prepared-input recurrence (raw fp16 q/k/v are L2-normalised
//               here; the output is the state readout before the gated norm).
//
// Grid: CPH CTAs per value head (a cluster); every CTA must own an SM, since
// an SM holding two CTAs would double the time of its whole cluster.
// Thread layout: 8 threads per PAIR of state rows, D/8 columns of each row per
// thread (columns 32i + 4j + e); every key/query value read from shared
// memory serves both rows.  Each thread filters one or two conv channels.
//
// The tokens of a chunk (<= 8) are solved together in the chunk form of the
// delta rule instead of one after another, so no token waits on the previous
// token's shuffle reductions.  With raw (filtered, unnormalised) k, q, the
// norms sk, sq, decays d_t = exp(l_t), G_t = prod_{r<=t} d_r and
// c_t = beta_t sk_t^2 d_t, the reference recurrence (per row)
//     u_t = d_t sk_t (S_{t-1}.k_t),  x_t = beta_t sk_t (v_t - u_t),
//     S_t = d_t S_{t-1} + x_t k_t,   o_t = sq_t (S_t.q_t)
// becomes, against the chunk's starting state S_0,
//     (I + L) x = b,  b_t = beta_t sk_t v_t - c_t G_{t-1} (S_0.k_t),
//     L[t][s] = c_t (G_{t-1}/G_s) (k_s.k_t)                       (s < t)
//     o_t = sq_t G_t (S_0.q_t) + sum_{s<=t} sq_t (G_t/G_s) (k_s.q_t) x_s
//     S_n = G_n S_0 + sum_s (G_n/G_s) x_s k_s.
// L and the readout matrix are shared by all rows (one warp per token builds
// them from the chunk's Gram products); every row pair does 4 x 8 dot
// products against S_0 (reduced across its 8 lanes by a transposing
// butterfly that leaves token j's sums on lane j), an 8-step forward
// substitution and one rank-8 update.  Decay ratios are exp of differences of
// log-decay prefix sums, so they never overflow.
//  * the state rows and the first chunk's inputs are prefetched into L2
//    before the dependency wait; the chunk's inputs are loaded one chunk
//    ahead (chunk 0 with the prologue, before the state);
//  * each CTA filters (conv + SiLU) all q/k channels of its key head and its
//    own v rows, so the q/k L2 norms need no cross-CTA exchange;
//  * the gated RMSNorm's per-token sum of squares is the only cross-CTA
//    value: every CTA pushes its partial into each peer's shared memory and
//    arrives on the peer's mbarrier (one-way, no cluster-wide barrier).
// D=128 uses CPH=2 (64 rows, 256 threads): clusters must fit inside one GPC,
// and 48 clusters of 3 do not all fit at once on B200, which then runs a
// second wave; clusters of 2 always fit (one CTA per SM, 96 SMs).
template <int D, int CPH> struct DeltaShape {
    static constexpr int MAXR = (D + CPH - 1) / CPH;              // most rows of a rank
    static constexpr int PAIRS = (MAXR + 1) / 2;                   // row pairs of a rank
    static constexpr int NT = ((PAIRS * 8 + 31) / 32) * 32;        // threads per CTA
    static constexpr int NCONV = (2 * D + MAXR + NT - 1) / NT;     // conv channels per thread
    static constexpr int NOUT = (CHUNK * MAXR + NT - 1) / NT;      // outputs per thread per chunk
};

// Sum of K4 x 8 per-lane values over the 8 lanes of a row pair, transposed: on
// return v[k * 8] of lane j holds the total of v[k * 8 + j] (k < K4).
template <int K4> __device__ __forceinline__ void pair_butterfly(float (&v)[K4 * 8], int j) {
    constexpr unsigned FULL = 0xffffffffu;
#pragma unroll
    for (int half = 4; half >= 1; half >>= 1) {
        const bool up = (j & half) != 0;
#pragma unroll
        for (int k = 0; k < K4; ++k) {
#pragma unroll
            for (int t = 0; t < half; ++t) {
                const float lo = v[k * 8 + t], hi = v[k * 8 + t + half];
                v[k * 8 + t] = (up ? hi : lo) + __shfl_xor_sync(FULL, up ? lo : hi, half);
            }
        }
    }
}

template <int D, int CPH, bool CORE>
__global__ void __cluster_dims__(CPH, 1, 1) __launch_bounds__(DeltaShape<D, CPH>::NT)
delta_kernel(const DeltaArgs a) {
    using Shape = DeltaShape<D, CPH>;
    constexpr int MAXR = Shape::MAXR, NT = Shape::NT, NCONV = Shape::NCONV, NOUT = Shape::NOUT;
    constexpr int NV4 = D / 32, COLS = D / 8, NW = NT / 32;
    constexpr unsigned FULL = 0xffffffffu;
    static_assert(2 * D <= NT, "the q/k channels take the first conv channel of threads [0, 2D)");
    static_assert(MAXR % 2 == 0 && CHUNK == 8, "whole row pairs, 8-token chunks");
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = CPH > 1 ? (int)cluster.block_rank() : 0;
    const int h = blockIdx.x / CPH, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int Hk = a.Hk, Hv = a.Hv, kh = h % Hk;
    const int C = (2 * Hk + Hv) * D;
    const int row0 = rank * D / CPH, rows = (rank + 1) * D / CPH - row0;   // this CTA's head rows
    const int j = tid & 7, ra = 2 * (tid >> 3), rb = ra + 1;               // column group / token, row pair
    const bool has_a = ra < rows, has_b = rb < rows;

    __shared__ __align__(16) float Fq[CHUNK][D], Fk[CHUNK][D], Fv[CHUNK][MAXR];
    __shared__ __align__(16) float O[CHUNK][MAXR];
    __shared__ __align__(16) float Lm[CHUNK][CHUNK], Mm[CHUNK][CHUNK];   // substitution / readout matrices
    __shared__ __align__(16) float vec[CHUNK][4];     // per token: beta sk, c G_{t-1}, sq G_t, G_n/G_t
    __shared__ float gnext;                           // G_n of the chunk
    __shared__ float wsum[NW][CHUNK];                 // per-warp sums of q^2 or k^2
    __shared__ float osum[2][CPH][CHUNK];             // sums of o^2 pushed by each rank, by chunk parity
    __shared__ __align__(8) uint64_t osum_bar[2];
    __shared__ bool norm_ok;

    if (!CORE && tid == 0) {
        // each rank's CHUNK token-warps arrive once per chunk
        mbar_init(&osum_bar[0], CPH * CHUNK);
        mbar_init(&osum_bar[1], CPH * CHUNK);
        fence_barrier_init();
    }
    // Peers arrive on osum_bar only after it is initialised everywhere (this
    // needs no memory written by another kernel, so it overlaps the previous one).
    if (!CORE && CPH > 1) cluster.sync();
    // L2 prefetch (before the dependency wait) of this CTA's state rows and of
    // the first chunk's inputs: q/k channels of the key head, v rows, gates and
    // conv history.
    prefetch_l2_range(a.state + ((size_t)h * D + row0) * D, (size_t)rows * D * 4, tid, NT);
    if (!CORE) {
        const int m0 = min(CHUNK, a.T);
        for (int t = 0; t < m0; ++t) {
            const float *x = a.qkv + (size_t)t * C;
            prefetch_l2_range(x + kh * D, D * 4, (tid + 37 * t) % NT, NT);
            prefetch_l2_range(x + (Hk + kh) * D, D * 4, (tid + 37 * t + 11) % NT, NT);
            prefetch_l2_range(x + (2 * Hk + h) * D + row0, rows * 4, (tid + 37 * t + 23) % NT, NT);
            prefetch_l2_range(a.gate + ((size_t)t * Hv + h) * D + row0, rows * 4, (tid + 37 * t + 29) % NT, NT);
        }
        for (int r = 0; r < 3; ++r) {
            const float *x = a.history + (size_t)r * C;
            prefetch_l2_range(x + kh * D, D * 4, (tid + 101 * r + 5) % NT, NT);
            prefetch_l2_range(x + (Hk + kh) * D, D * 4, (tid + 101 * r + 17) % NT, NT);
            prefetch_l2_range(x + (2 * Hk + h) * D + row0, rows * 4, (tid + 101 * r + 31) % NT, NT);
        }
    }
    // State, history and inputs may have been written by the previous kernel.
    grid_dependency_wait();
    if (tid == 0) launch_dependents();

    // Conv channels of this thread: e < D -> q, e < 2D -> k, e < 2D + rows -> v row.
    int c[NCONV], e[NCONV];
#pragma unroll
    for (int u = 0; u < NCONV; ++u) {
        e[u] = tid + u * NT;
        c[u] = -1;
        if (e[u] < D) c[u] = kh * D + e[u];
        else if (e[u] < 2 * D) c[u] = (Hk + kh) * D + (e[u] - D);
        else if (e[u] < 2 * D + rows) c[u] = (2 * Hk + h) * D + row0 + (e[u] - 2 * D);
    }
    // Outputs of this thread in each chunk: index o = tid + u NT -> token o / rows, row o % rows.
    bool has_out[NOUT];
    int out_t[NOUT], out_i[NOUT];
#pragma unroll
    for (int u = 0; u < NOUT; ++u) {
        const int o = tid + u * NT;
        has_out[u] = o < CHUNK * rows;
        out_t[u] = has_out[u] ? o / rows : 0;
        out_i[u] = has_out[u] ? o % rows : 0;
    }

    // Chunk inputs are prefetched one chunk ahead; chunk 0 is issued first.
    // Lanes 0-7 of every warp hold alpha/beta of the chunk's token `lane`.
    float raw_n[NCONV][CHUNK], al_n = 0.f, be_n = 0.f, gz_n[NOUT];
    auto load_chunk = [&](int c0) {
        const int m = min(CHUNK, a.T - c0);
#pragma unroll
        for (int u = 0; u < NCONV; ++u) {
#pragma unroll
            for (int tt = 0; tt < CHUNK; ++tt) {
                raw_n[u][tt] = 0.f;
                if (c[u] >= 0 && tt < m) {
                    const int t = c0 + tt, x = e[u];
                    if (!CORE) raw_n[u][tt] = a.qkv[(size_t)t * C + c[u]];
                    else if (x < D) raw_n[u][tt] = __half2float(a.q16[((size_t)t * Hk + kh) * D + x]);
                    else if (x < 2 * D) raw_n[u][tt] = __half2float(a.k16[((size_t)t * Hk + kh) * D + x - D]);
                    else raw_n[u][tt] = __half2float(a.v16[((size_t)t * Hv + h) * D + row0 + x - 2 * D]);
                }
            }
        }
        al_n = be_n = 0.f;
        if (lane < m) {
            const size_t idx = (size_t)(c0 + lane) * Hv + h;
            al_n = a.alpha[idx];
            be_n = a.beta[idx];
        }
#pragma unroll
        for (int u = 0; u < NOUT; ++u)
            gz_n[u] = (!CORE && has_out[u] && out_t[u] < m)
                          ? a.gate[((size_t)(c0 + out_t[u]) * Hv + h) * D + row0 + out_i[u]] : 0.f;
    };
    load_chunk(0);

    float w[NCONV][4], hs[NCONV][3];
#pragma unroll
    for (int u = 0; u < NCONV; ++u) {
        w[u][0] = w[u][1] = w[u][2] = w[u][3] = 0.f;
        hs[u][0] = hs[u][1] = hs[u][2] = 0.f;
        if (!CORE && c[u] >= 0) {
            const float4 wv = *reinterpret_cast<const float4 *>(a.conv + (size_t)c[u] * 4);
            w[u][0] = wv.x; w[u][1] = wv.y; w[u][2] = wv.z; w[u][3] = wv.w;
            hs[u][0] = a.history[c[u]]; hs[u][1] = a.history[(size_t)C + c[u]];
            hs[u][2] = a.history[2 * (size_t)C + c[u]];
        }
    }
    const float decay_h = a.decay[h], bias_h = a.bias[h];
    float nw[NOUT];
#pragma unroll
    for (int u = 0; u < NOUT; ++u) nw[u] = (!CORE && has_out[u]) ? a.norm[row0 + out_i[u]] : 1.f;

    // ---- the state rows of this thread (needed only by the chunk solve)
    float Sa[COLS], Sb[COLS];
    float *srow_a = a.state + ((size_t)h * D + row0 + (has_a ? ra : 0)) * D;
    float *srow_b = a.state + ((size_t)h * D + row0 + (has_b ? rb : 0)) * D;
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
        float4 va = make_float4(0.f, 0.f, 0.f, 0.f), vb = va;
        if (has_a) va = *reinterpret_cast<const float4 *>(srow_a + 32 * i + 4 * j);
        if (has_b) vb = *reinterpret_cast<const float4 *>(srow_b + 32 * i + 4 * j);
        Sa[4 * i] = va.x; Sa[4 * i + 1] = va.y; Sa[4 * i + 2] = va.z; Sa[4 * i + 3] = va.w;
        Sb[4 * i] = vb.x; Sb[4 * i + 1] = vb.y; Sb[4 * i + 2] = vb.z; Sb[4 * i + 3] = vb.w;
    }

    for (int t0 = 0, chunk = 0; t0 < a.T; t0 += CHUNK, ++chunk) {
        const int n = min(CHUNK, a.T - t0);
        // ---- this chunk's inputs were prefetched; start the next chunk's loads
        float raw[NCONV][CHUNK], gz[NOUT];
#pragma unroll
        for (int u = 0; u < NCONV; ++u)
#pragma unroll
            for (int tt = 0; tt < CHUNK; ++tt) raw[u][tt] = raw_n[u][tt];
#pragma unroll
        for (int u = 0; u < NOUT; ++u) gz[u] = gz_n[u];
        const float al = al_n, be = be_n;
        if (t0 + CHUNK < a.T) load_chunk(t0 + CHUNK);
        // ---- conv + SiLU in registers (rows of tokens >= n are written as
        //      zeros); per-warp sums of squares of q (warps [0, D/32)) and k
        //      (warps [D/32, 2D/32)), from the first channel
        float sq2[CHUNK];
#pragma unroll
        for (int u = 0; u < NCONV; ++u) {
#pragma unroll
            for (int tt = 0; tt < CHUNK; ++tt) {
                float f = raw[u][tt];
                if (!CORE && tt < n) {
                    float v = w[u][3] * f;
                    v += w[u][0] * hs[u][0]; v += w[u][1] * hs[u][1]; v += w[u][2] * hs[u][2];
                    hs[u][0] = hs[u][1]; hs[u][1] = hs[u][2]; hs[u][2] = f;
                    f = siluf_(v);
                }
                if (u == 0) sq2[tt] = 0.f;
                if (c[u] >= 0) {
                    const int x = e[u];
                    if (x < D) { Fq[tt][x] = f; sq2[tt] = f * f; }
                    else if (x < 2 * D) { Fk[tt][x - D] = f; sq2[tt] = f * f; }
                    else Fv[tt][x - 2 * D] = f;
                }
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

        // ---- per-token scalars, on lanes 0-7 of every warp (token = lane);
        //      tokens >= n get zero norms / gates and no decay
        float sqn = 0.f, skn = 0.f, lam = 0.f, beta = 0.f;
        if (lane < n) {
            float qs = 0.f, ks = 0.f;
#pragma unroll
            for (int x = 0; x < D / 32; ++x) { qs += wsum[x][lane]; ks += wsum[D / 32 + x][lane]; }
            sqn = rsqrtf(qs + 1e-6f) * rsqrtf((float)D);
            skn = rsqrtf(ks + 1e-6f);
            lam = decay_h * softplusf_(al + bias_h);          // log of the decay
            beta = sigmoidf_(be);
        }
        float Lam = lam;                                       // inclusive prefix over tokens
#pragma unroll
        for (int off = 1; off < CHUNK; off <<= 1) {
            const float y = __shfl_up_sync(FULL, Lam, off);
            if (lane >= off) Lam += y;
        }
        float Lprev = __shfl_up_sync(FULL, Lam, 1);
        if (lane == 0) Lprev = 0.f;
        const float Lend = __shfl_sync(FULL, Lam, n - 1);
        const float cdec = beta * skn * skn * expf(lam);       // c_t
        // ---- Gram products of the chunk and rows t of L and of the readout
        //      matrix, one warp per token t
        for (int t = warp; t < CHUNK; t += NW) {
            float g16[16];
            if constexpr (D == 128) {
                const float4 kt = reinterpret_cast<const float4 *>(Fk[t])[lane];
                const float4 qt = reinterpret_cast<const float4 *>(Fq[t])[lane];
#pragma unroll
                for (int s = 0; s < CHUNK; ++s) {
                    const float4 ks4 = reinterpret_cast<const float4 *>(Fk[s])[lane];
                    g16[s] = ks4.x * kt.x + ks4.y * kt.y + ks4.z * kt.z + ks4.w * kt.w;
                    g16[8 + s] = ks4.x * qt.x + ks4.y * qt.y + ks4.z * qt.z + ks4.w * qt.w;
                }
            } else {
#pragma unroll
                for (int s = 0; s < CHUNK; ++s) { g16[s] = 0.f; g16[8 + s] = 0.f; }
#pragma unroll
                for (int x = lane; x < D; x += 32) {
                    const float kt = Fk[t][x], qt = Fq[t][x];
#pragma unroll
                    for (int s = 0; s < CHUNK; ++s) { g16[s] += Fk[s][x] * kt; g16[8 + s] += Fk[s][x] * qt; }
                }
            }
            // transposing reduction over the warp: lane l ends with value l >> 1
#pragma unroll
            for (int half = 8; half >= 1; half >>= 1) {
                const bool up = (lane & (2 * half)) != 0;
#pragma unroll
                for (int x = 0; x < half; ++x) {
                    const float lo = g16[x], hi = g16[x + half];
                    g16[x] = (up ? hi : lo) + __shfl_xor_sync(FULL, up ? lo : hi, 2 * half);
                }
            }
            g16[0] += __shfl_xor_sync(FULL, g16[0], 1);
            const int idx = lane >> 1, s = idx & 7;
            const float Ls = __shfl_sync(FULL, Lam, s);
            const float ct = __shfl_sync(FULL, cdec, t), Lpt = __shfl_sync(FULL, Lprev, t);
            const float Lt = __shfl_sync(FULL, Lam, t), sqt = __shfl_sync(FULL, sqn, t);
            if ((lane & 1) == 0) {
                if (idx < 8) Lm[t][s] = s < t ? ct * expf(Lpt - Ls) * g16[0] : 0.f;
                else Mm[t][s] = s <= t ? sqt * expf(Lt - Ls) * g16[0] : 0.f;
            }
        }
        if (warp == 0 && lane < CHUNK) {
            *reinterpret_cast<float4 *>(vec[lane]) =
                make_float4(beta * skn, cdec * expf(Lprev), sqn * expf(Lam), lane < n ? expf(Lend - Lam) : 0.f);
            if (lane == 0) gnext = expf(Lend);
        }

        // ---- dot products of both rows with every token's k and q against the
        //      chunk's starting state
        float dots[32];                                   // [k.a | k.b | q.a | q.b] x token
#pragma unroll
        for (int x = 0; x < 32; ++x) dots[x] = 0.f;
#pragma unroll
        for (int i = 0; i < NV4; ++i) {
#pragma unroll
            for (int t = 0; t < CHUNK; ++t) {
                const float4 k4 = reinterpret_cast<const float4 *>(Fk[t])[8 * i + j];
                const float4 q4 = reinterpret_cast<const float4 *>(Fq[t])[8 * i + j];
                dots[t] = fmaf(Sa[4 * i], k4.x, dots[t]);
                dots[t] = fmaf(Sa[4 * i + 1], k4.y, dots[t]);
                dots[t] = fmaf(Sa[4 * i + 2], k4.z, dots[t]);
                dots[t] = fmaf(Sa[4 * i + 3], k4.w, dots[t]);
                dots[8 + t] = fmaf(Sb[4 * i], k4.x, dots[8 + t]);
                dots[8 + t] = fmaf(Sb[4 * i + 1], k4.y, dots[8 + t]);
                dots[8 + t] = fmaf(Sb[4 * i + 2], k4.z, dots[8 + t]);
                dots[8 + t] = fmaf(Sb[4 * i + 3], k4.w, dots[8 + t]);
                dots[16 + t] = fmaf(Sa[4 * i], q4.x, dots[16 + t]);
                dots[16 + t] = fmaf(Sa[4 * i + 1], q4.y, dots[16 + t]);
                dots[16 + t] = fmaf(Sa[4 * i + 2], q4.z, dots[16 + t]);
                dots[16 + t] = fmaf(Sa[4 * i + 3], q4.w, dots[16 + t]);
                dots[24 + t] = fmaf(Sb[4 * i], q4.x, dots[24 + t]);
                dots[24 + t] = fmaf(Sb[4 * i + 1], q4.y, dots[24 + t]);
                dots[24 + t] = fmaf(Sb[4 * i + 2], q4.z, dots[24 + t]);
                dots[24 + t] = fmaf(Sb[4 * i + 3], q4.w, dots[24 + t]);
            }
        }
        pair_butterfly<4>(dots, j);                       // lane j: token j's four sums
        __syncthreads();                                  // Lm, Mm, vec, gnext

        // ---- right-hand sides on lane j (token j), gathered to the pair
        const float4 vj = *reinterpret_cast<const float4 *>(vec[j]);
        const float bja = vj.x * (has_a ? Fv[j][ra] : 0.f) - vj.y * dots[0];
        const float bjb = vj.x * (has_b ? Fv[j][rb] : 0.f) - vj.y * dots[8];
        const int base = lane & ~7;
        float xa[CHUNK], xb[CHUNK];
#pragma unroll
        for (int s = 0; s < CHUNK; ++s) {
            xa[s] = __shfl_sync(FULL, bja, base + s);
            xb[s] = __shfl_sync(FULL, bjb, base + s);
        }
        // forward substitution (I + L) x = b, L strictly lower triangular
#pragma unroll
        for (int t = 1; t < CHUNK; ++t) {
            const float4 l0 = *reinterpret_cast<const float4 *>(&Lm[t][0]);
            const float4 l1 = *reinterpret_cast<const float4 *>(&Lm[t][4]);
            const float lt[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
            float sa = 0.f, sb = 0.f;
#pragma unroll
            for (int s = 0; s < t; ++s) { sa = fmaf(lt[s], xa[s], sa); sb = fmaf(lt[s], xb[s], sb); }
            xa[t] -= sa;
            xb[t] -= sb;
        }
        // readout of token j for both rows
        {
            const float4 m0 = *reinterpret_cast<const float4 *>(&Mm[j][0]);
            const float4 m1 = *reinterpret_cast<const float4 *>(&Mm[j][4]);
            const float mj[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
            float oa = vj.z * dots[16], ob = vj.z * dots[24];
#pragma unroll
            for (int s = 0; s < CHUNK; ++s) { oa = fmaf(mj[s], xa[s], oa); ob = fmaf(mj[s], xb[s], ob); }
            if (j < n) {
                if (has_a) O[j][ra] = oa;
                if (has_b) O[j][rb] = ob;
            }
        }
        // state at the end of the chunk: S = G_n S + sum_s (G_n / G_s) x_s k_s
        {
            const float gn = gnext;
#pragma unroll
            for (int s = 0; s < CHUNK; ++s) {
                const float es = vec[s][3];
                xa[s] *= es;
                xb[s] *= es;
            }
#pragma unroll
            for (int x = 0; x < COLS; ++x) { Sa[x] *= gn; Sb[x] *= gn; }
#pragma unroll
            for (int i = 0; i < NV4; ++i) {
#pragma unroll
                for (int s = 0; s < CHUNK; ++s) {
                    const float4 k4 = reinterpret_cast<const float4 *>(Fk[s])[8 * i + j];
                    Sa[4 * i] = fmaf(k4.x, xa[s], Sa[4 * i]);
                    Sa[4 * i + 1] = fmaf(k4.y, xa[s], Sa[4 * i + 1]);
                    Sa[4 * i + 2] = fmaf(k4.z, xa[s], Sa[4 * i + 2]);
                    Sa[4 * i + 3] = fmaf(k4.w, xa[s], Sa[4 * i + 3]);
                    Sb[4 * i] = fmaf(k4.x, xb[s], Sb[4 * i]);
                    Sb[4 * i + 1] = fmaf(k4.y, xb[s], Sb[4 * i + 1]);
                    Sb[4 * i + 2] = fmaf(k4.z, xb[s], Sb[4 * i + 2]);
                    Sb[4 * i + 3] = fmaf(k4.w, xb[s], Sb[4 * i + 3]);
                }
            }
        }
        __syncthreads();
        if (CORE) {
#pragma unroll
            for (int u = 0; u < NOUT; ++u)
                if (has_out[u] && out_t[u] < n)
                    a.out[((size_t)(t0 + out_t[u]) * Hv + h) * D + row0 + out_i[u]] = O[out_t[u]][out_i[u]];
        } else {
            // ---- gated RMSNorm over the whole head: warp tt reduces token tt's sum
            //      of squares over this CTA's rows and pushes it to every rank;
            //      one thread waits for all partials, the block barrier then
            //      orders them for the other threads.
            const int par = chunk & 1;
            for (int tt = warp; tt < CHUNK; tt += NW) {
                float x = 0.f;
                if (tt < n)
                    for (int i = lane; i < rows; i += 32) x += O[tt][i] * O[tt][i];
                x = warp_sum(x);
                if (lane < CPH) {
                    st_cluster_f32(cluster_map(&osum[par][rank][tt], lane), x);
                    mbar_arrive_cluster(cluster_map(&osum_bar[par], lane));
                }
            }
            if (tid == 0) norm_ok = mbar_wait_cluster(&osum_bar[par], (uint32_t)(chunk >> 1) & 1);
            __syncthreads();
#pragma unroll
            for (int u = 0; u < NOUT; ++u) {
                if (norm_ok && has_out[u] && out_t[u] < n) {
                    float total = 0.f;
#pragma unroll
                    for (int q = 0; q < CPH; ++q) total += osum[par][q][out_t[u]];
                    const float scale = rsqrtf(total / D + a.eps);
                    a.out[((size_t)(t0 + out_t[u]) * Hv + h) * D + row0 + out_i[u]] =
                        O[out_t[u]][out_i[u]] * scale * nw[u] * siluf_(gz[u]);
                }
            }
        }
        __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < NV4; ++i) {
        if (has_a)
            *reinterpret_cast<float4 *>(srow_a + 32 * i + 4 * j) =
                make_float4(Sa[4 * i], Sa[4 * i + 1], Sa[4 * i + 2], Sa[4 * i + 3]);
        if (has_b)
            *reinterpret_cast<float4 *>(srow_b + 32 * i + 4 * j) =
                make_float4(Sb[4 * i], Sb[4 * i + 1], Sb[4 * i + 2], Sb[4 * i + 3]);
    }
    // History: v channels belong to their rows' CTA; the q/k channels of key
    // head kh are written by rank 0 of value head kh (h < Hk) only.
#pragma unroll
    for (int u = 0; u < NCONV; ++u) {
        if (!CORE && c[u] >= 0 && (e[u] >= 2 * D || (h < Hk && rank == 0))) {
            a.history[c[u]] = hs[u][0]; a.history[(size_t)C + c[u]] = hs[u][1];
            a.history[2 * (size_t)C + c[u]] = hs[u][2];
        }
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
