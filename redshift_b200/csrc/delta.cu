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
// on the first 4 * rows threads, 8 per PAIR of state rows and D/8 columns of
// each (columns 32i + 4j + e), so every k/q value read from shared memory
// serves two rows (the loop is bound by shared-memory bandwidth) and the four
// dot products of a token (S_a.k, S_b.k, S_a.q, S_b.q, all against the state
// before the token's update) reduce together in 4 shuffles.  Per chunk of
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
    static constexpr int NT = ((MAXR * 8 + 31) / 32) * 32;         // threads per CTA
};

template <int D, int CPH, bool CORE, bool RECORD = false>
__global__ void __cluster_dims__(CPH, 1, 1) __launch_bounds__(DeltaShape<D, CPH>::NT)
delta_kernel(const DeltaArgs a) {
    static_assert(!(CORE && RECORD), "only the layer mode records a verify");
    constexpr int MAXR = DeltaShape<D, CPH>::MAXR, NT = DeltaShape<D, CPH>::NT;
    constexpr int NV4 = D / 32, COLS = D / 8, NW = NT / 32;
    static_assert(2 * D + MAXR <= NT, "one conv channel per thread");
    static_assert(CHUNK * MAXR <= NT, "one output per thread per chunk");
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = CPH > 1 ? (int)cluster.block_rank() : 0;
    const int h = blockIdx.x / CPH, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int Hk = a.Hk, Hv = a.Hv, kh = h % Hk;
    const int C = (2 * Hk + Hv) * D;
    const int row0 = rank * D / CPH, rows = (rank + 1) * D / CPH - row0;   // this CTA's head rows
    // token loop: the first 4 * rows threads, 8 per PAIR of state rows (rows
    // ra, rb), D/8 columns of each; every k/q value read from shared memory
    // serves both rows
    const int j = tid & 7, ra = 2 * (tid >> 3), rb = ra + 1;
    const bool has_a = ra < rows, has_b = rb < rows, scans = tid < 4 * MAXR;

    __shared__ __align__(16) float Fq[CHUNK][D], Fk[CHUNK][D], Fv[CHUNK][MAXR];
    __shared__ __align__(16) float O[CHUNK][MAXR];
    __shared__ float wsum[NW][CHUNK];             // per-warp sums of q^2 or k^2
    __shared__ __align__(16) float scal[CHUNK][8];  // sq, sk, decay, beta, k.q
    __shared__ float osum[2][CPH][CHUNK];         // sums of o^2 pushed by each rank, by chunk parity
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
    // State, history and inputs may have been written by the previous kernel.
    grid_dependency_wait();
    if (tid == 0) launch_dependents();

    // ---- loads that do not depend on the chunk
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
        if (RECORD && has_a)
            *reinterpret_cast<float4 *>(a.saved_state + (srow_a - a.state) + 32 * i + 4 * j) = va;
        if (RECORD && has_b)
            *reinterpret_cast<float4 *>(a.saved_state + (srow_b - a.state) + 32 * i + 4 * j) = vb;
    }
    // Conv channel of this thread: e < D -> q, e < 2D -> k, e < 2D + rows -> v row.
    const int e = tid;
    int c = -1;
    if (e < D) c = kh * D + e;
    else if (e < 2 * D) c = (Hk + kh) * D + (e - D);
    else if (e < 2 * D + rows) c = (2 * Hk + h) * D + row0 + (e - 2 * D);
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
                f = siluf_(v);
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
        if (tid < n) {
            float qs = 0.f, ks = 0.f;
#pragma unroll
            for (int w = 0; w < D / 32; ++w) { qs += wsum[w][tid]; ks += wsum[D / 32 + w][tid]; }
            scal[tid][0] = rsqrtf(qs + 1e-6f) * rsqrtf((float)D);
            scal[tid][1] = rsqrtf(ks + 1e-6f);
            scal[tid][2] = expf(decay_h * softplusf_(al + bias_h));
            scal[tid][3] = sigmoidf_(be);
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
                float ua0 = 0.f, ua1 = 0.f, ub0 = 0.f, ub1 = 0.f, wa0 = 0.f, wa1 = 0.f, wb0 = 0.f, wb1 = 0.f;
#pragma unroll
                for (int i = 0; i < NV4; ++i) {
                    k4[i] = kk[8 * i + j];
                    const float4 q4 = qq[8 * i + j];
                    ua0 = fmaf(Sa[4 * i], k4[i].x, ua0); ua1 = fmaf(Sa[4 * i + 1], k4[i].y, ua1);
                    ua0 = fmaf(Sa[4 * i + 2], k4[i].z, ua0); ua1 = fmaf(Sa[4 * i + 3], k4[i].w, ua1);
                    ub0 = fmaf(Sb[4 * i], k4[i].x, ub0); ub1 = fmaf(Sb[4 * i + 1], k4[i].y, ub1);
                    ub0 = fmaf(Sb[4 * i + 2], k4[i].z, ub0); ub1 = fmaf(Sb[4 * i + 3], k4[i].w, ub1);
                    wa0 = fmaf(Sa[4 * i], q4.x, wa0); wa1 = fmaf(Sa[4 * i + 1], q4.y, wa1);
                    wa0 = fmaf(Sa[4 * i + 2], q4.z, wa0); wa1 = fmaf(Sa[4 * i + 3], q4.w, wa1);
                    wb0 = fmaf(Sb[4 * i], q4.x, wb0); wb1 = fmaf(Sb[4 * i + 1], q4.y, wb1);
                    wb0 = fmaf(Sb[4 * i + 2], q4.z, wb0); wb1 = fmaf(Sb[4 * i + 3], q4.w, wb1);
                }
                const float ua = ua0 + ua1, ub = ub0 + ub1, wa = wa0 + wa1, wb = wb0 + wb1;
                const bool hi4 = (j & 4) != 0, hi2 = (j & 2) != 0;
                float m0 = hi4 ? wa : ua, m1 = hi4 ? wb : ub;
                m0 += __shfl_xor_sync(0xffffffffu, hi4 ? ua : wa, 4);
                m1 += __shfl_xor_sync(0xffffffffu, hi4 ? ub : wb, 4);
                float m = hi2 ? m1 : m0;
                m += __shfl_xor_sync(0xffffffffu, hi2 ? m0 : m1, 2);
                m += __shfl_xor_sync(0xffffffffu, m, 1);
                // delta of row a on lanes 0-1, of row b on lanes 2-3; broadcast to the pair
                const int rl = hi2 ? rb : ra;
                const float vrow = rl < rows ? Fv[tt][rl] : 0.f;
                const float dl = (vrow - decay * m * skn) * beta * skn;
                const int base = lane & ~7;
                const float da = __shfl_sync(0xffffffffu, dl, base), db = __shfl_sync(0xffffffffu, dl, base + 2);
                // readout of row a on lane 4, of row b on lane 6
                if ((j == 4 || j == 6) && rl < rows) O[tt][rl] = sqn * fmaf(decay, m, (hi2 ? db : da) * kq);
#pragma unroll
                for (int i = 0; i < NV4; ++i) {
                    Sa[4 * i] = fmaf(Sa[4 * i], decay, k4[i].x * da);
                    Sa[4 * i + 1] = fmaf(Sa[4 * i + 1], decay, k4[i].y * da);
                    Sa[4 * i + 2] = fmaf(Sa[4 * i + 2], decay, k4[i].z * da);
                    Sa[4 * i + 3] = fmaf(Sa[4 * i + 3], decay, k4[i].w * da);
                    Sb[4 * i] = fmaf(Sb[4 * i], decay, k4[i].x * db);
                    Sb[4 * i + 1] = fmaf(Sb[4 * i + 1], decay, k4[i].y * db);
                    Sb[4 * i + 2] = fmaf(Sb[4 * i + 2], decay, k4[i].z * db);
                    Sb[4 * i + 3] = fmaf(Sb[4 * i + 3], decay, k4[i].w * db);
                }
            }
        }
        __syncthreads();
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
            if (norm_ok && has_out && out_t < n) {
                float total = 0.f;
#pragma unroll
                for (int q = 0; q < CPH; ++q) total += osum[par][q][out_t];
                const float scale = rsqrtf(total / D + a.eps);
                a.out[((size_t)(t0 + out_t) * Hv + h) * D + row0 + out_i] =
                    O[out_t][out_i] * scale * nw * siluf_(gz);
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
    if (!CORE && c >= 0 && (e >= 2 * D || (h < Hk && rank == 0))) {
        a.history[c] = h0; a.history[(size_t)C + c] = h1; a.history[2 * (size_t)C + c] = h2;
    }
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
