// Gated DeltaNet recurrent path for sm_100a: one fused kernel per layer call.
//
// The reference runs conv -> gdn_prep -> gdn_scan -> delta_out as four
// launches (src/kernels.cu:275-354, 409-414, 557-566).  Here a cluster of
// CPH CTAs owns one value head; each CTA owns D/CPH rows of the head's
// [Dv][Dk] fp32 state (4 threads per row, D/4 columns each, in registers).
// Every CTA recomputes the causal conv + SiLU of the q/k channels of its key
// head (h % Hk) and of its own v rows, L2-normalises q and k, forms the decay
// a = exp(A softplus(alpha+bias)) and beta = sigmoid(beta), and runs the delta
// rule over the tokens.  The gated RMSNorm needs the whole head's readout:
// the per-CTA sums of squares are exchanged through distributed shared
// memory.  The state is read and written exactly once per call.
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
template <int D, int CPH, bool CORE>
__global__ void __cluster_dims__(CPH, 1, 1) __launch_bounds__(128)
delta_kernel(const DeltaArgs a) {
    constexpr int ROWS = D / CPH;                 // state rows of this CTA
    constexpr int NT = ROWS * 4;                  // 4 threads per row
    static_assert(NT == 128, "one 128-thread CTA per cluster rank");
    constexpr int COLS = D / 4, NV4 = D / 16, NW = NT / 32;
    constexpr int NCH = 2 * D + ROWS;             // q, k channels of the key head + own v rows
    constexpr int CPT = (NCH + NT - 1) / NT;      // conv channels per thread
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = CPH > 1 ? (int)cluster.block_rank() : 0;
    const int h = blockIdx.x / CPH, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int Hk = a.Hk, Hv = a.Hv, kh = h % Hk;
    const int C = (2 * Hk + Hv) * D;
    const int r = tid >> 2, j = tid & 3;          // local row, column quarter
    const int row0 = rank * ROWS;                 // first head row of this CTA

    __shared__ __align__(16) float Fq[CHUNK][D], Fk[CHUNK][D], Fv[CHUNK][ROWS];
    __shared__ __align__(16) float O[CHUNK][ROWS];
    __shared__ float sa[CHUNK], sb[CHUNK], sq[CHUNK], sk[CHUNK];
    __shared__ float psum[2][CHUNK];              // per-CTA sum of squares, double-buffered by chunk

    // State row fragment: columns 16*i + 4*j + e.
    float S[COLS];
    float *srow = a.state + ((size_t)h * D + row0 + r) * D;
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
        const float4 v = *reinterpret_cast<const float4 *>(srow + 16 * i + 4 * j);
        S[4 * i] = v.x; S[4 * i + 1] = v.y; S[4 * i + 2] = v.z; S[4 * i + 3] = v.w;
    }

    // Conv channels of this thread: index e < 2D -> q/k channel of key head kh,
    // else v channel of row row0 + (e - 2D).  Window registers persist across chunks.
    int ch[CPT];
    float w0[CPT], w1[CPT], w2[CPT], w3[CPT], h0[CPT], h1[CPT], h2[CPT];
#pragma unroll
    for (int u = 0; u < CPT; ++u) {
        const int e = tid + u * NT;
        int c = -1;
        if (e < D) c = kh * D + e;
        else if (e < 2 * D) c = (Hk + kh) * D + (e - D);
        else if (e < NCH) c = (2 * Hk + h) * D + row0 + (e - 2 * D);
        ch[u] = c;
        w0[u] = w1[u] = w2[u] = w3[u] = h0[u] = h1[u] = h2[u] = 0.f;
        if (!CORE && c >= 0) {
            const float4 w = *reinterpret_cast<const float4 *>(a.conv + (size_t)c * 4);
            w0[u] = w.x; w1[u] = w.y; w2[u] = w.z; w3[u] = w.w;
            h0[u] = a.history[c]; h1[u] = a.history[(size_t)C + c]; h2[u] = a.history[2 * (size_t)C + c];
        }
    }

    for (int t0 = 0, chunk = 0; t0 < a.T; t0 += CHUNK, ++chunk) {
        const int n = min(CHUNK, a.T - t0);
        // -------- conv + SiLU (all loads of the chunk issued before use)
#pragma unroll
        for (int u = 0; u < CPT; ++u) {
            const int e = tid + u * NT, c = ch[u];
            if (c < 0) continue;
            float raw[CHUNK];
#pragma unroll
            for (int tt = 0; tt < CHUNK; ++tt) {
                raw[tt] = 0.f;
                if (tt < n) {
                    const int t = t0 + tt;
                    if (!CORE) raw[tt] = a.qkv[(size_t)t * C + c];
                    else if (e < D) raw[tt] = __half2float(a.q16[((size_t)t * Hk + kh) * D + e]);
                    else if (e < 2 * D) raw[tt] = __half2float(a.k16[((size_t)t * Hk + kh) * D + e - D]);
                    else raw[tt] = __half2float(a.v16[((size_t)t * Hv + h) * D + row0 + e - 2 * D]);
                }
            }
#pragma unroll
            for (int tt = 0; tt < CHUNK; ++tt) {
                if (tt >= n) break;
                float f = raw[tt];
                if (!CORE) {
                    float v = w3[u] * raw[tt];
                    v += w0[u] * h0[u]; v += w1[u] * h1[u]; v += w2[u] * h2[u];
                    h0[u] = h1[u]; h1[u] = h2[u]; h2[u] = raw[tt];
                    f = siluf_(v);
                }
                if (e < D) Fq[tt][e] = f;
                else if (e < 2 * D) Fk[tt][e - D] = f;
                else Fv[tt][e - 2 * D] = f;
            }
        }
        if (tid < n) {
            const size_t idx = (size_t)(t0 + tid) * Hv + h;
            sa[tid] = expf(a.decay[h] * softplusf_(a.alpha[idx] + a.bias[h]));
            sb[tid] = sigmoidf_(a.beta[idx]);
        }
        __syncthreads();
        // -------- L2 norms of q and k (q also by 1/sqrt(D))
        for (int task = warp; task < 2 * n; task += NW) {
            const int tt = task >> 1;
            const float *src = (task & 1) ? Fk[tt] : Fq[tt];
            float s = 0.f;
#pragma unroll
            for (int i = lane; i < D; i += 32) s += src[i] * src[i];
            s = warp_sum(s);
            if (lane == 0) {
                if (task & 1) sk[tt] = rsqrtf(s + 1e-6f);
                else sq[tt] = rsqrtf(s + 1e-6f) * rsqrtf((float)D);
            }
        }
        __syncthreads();
        for (int e = tid; e < n * D; e += NT) {
            const int tt = e / D, i = e % D;
            Fq[tt][i] *= sq[tt];
            Fk[tt][i] *= sk[tt];
        }
        __syncthreads();
        // -------- delta rule: S = a S; u = S k; delta = beta (v - u); S += delta k^T; o = S q
        for (int tt = 0; tt < n; ++tt) {
            const float decay = sa[tt], beta = sb[tt];
            const float *kk = Fk[tt], *qq = Fq[tt];
            float u0 = 0.f, u1 = 0.f;
#pragma unroll
            for (int i = 0; i < NV4; ++i) {
                const float4 k4 = *reinterpret_cast<const float4 *>(kk + 16 * i + 4 * j);
                S[4 * i] *= decay; S[4 * i + 1] *= decay; S[4 * i + 2] *= decay; S[4 * i + 3] *= decay;
                u0 += S[4 * i] * k4.x; u1 += S[4 * i + 1] * k4.y;
                u0 += S[4 * i + 2] * k4.z; u1 += S[4 * i + 3] * k4.w;
            }
            float u = u0 + u1;
            u += __shfl_xor_sync(0xffffffffu, u, 1);
            u += __shfl_xor_sync(0xffffffffu, u, 2);
            const float delta = (Fv[tt][r] - u) * beta;
            float o0 = 0.f, o1 = 0.f;
#pragma unroll
            for (int i = 0; i < NV4; ++i) {
                const float4 k4 = *reinterpret_cast<const float4 *>(kk + 16 * i + 4 * j);
                const float4 q4 = *reinterpret_cast<const float4 *>(qq + 16 * i + 4 * j);
                S[4 * i] += k4.x * delta; S[4 * i + 1] += k4.y * delta;
                S[4 * i + 2] += k4.z * delta; S[4 * i + 3] += k4.w * delta;
                o0 += S[4 * i] * q4.x; o1 += S[4 * i + 1] * q4.y;
                o0 += S[4 * i + 2] * q4.z; o1 += S[4 * i + 3] * q4.w;
            }
            float o = o0 + o1;
            o += __shfl_xor_sync(0xffffffffu, o, 1);
            o += __shfl_xor_sync(0xffffffffu, o, 2);
            if (j == 0) O[tt][r] = o;
        }
        __syncthreads();
        if (CORE) {
            for (int e = tid; e < n * ROWS; e += NT) {
                const int tt = e / ROWS, i = e % ROWS;
                a.out[((size_t)(t0 + tt) * Hv + h) * D + row0 + i] = O[tt][i];
            }
        } else {
            // -------- gated RMSNorm over the whole head (cluster-wide sum of squares)
            float *ps = psum[chunk & 1];
            for (int tt = warp; tt < n; tt += NW) {
                float s = 0.f;
                for (int i = lane; i < ROWS; i += 32) s += O[tt][i] * O[tt][i];
                s = warp_sum(s);
                if (lane == 0) ps[tt] = s;
            }
            if (CPH > 1) cluster.sync(); else __syncthreads();
            for (int e = tid; e < n * ROWS; e += NT) {
                const int tt = e / ROWS, i = e % ROWS;
                float total = 0.f;
#pragma unroll
                for (int q = 0; q < CPH; ++q)
                    total += CPH > 1 ? cluster.map_shared_rank(ps, q)[tt] : ps[tt];
                const float scale = rsqrtf(total / D + a.eps);
                const size_t o = ((size_t)(t0 + tt) * Hv + h) * D + row0 + i;
                a.out[o] = O[tt][i] * scale * a.norm[row0 + i] * siluf_(a.gate[o]);
            }
        }
        __syncthreads();
    }
    // No CTA may leave while a peer can still read its psum.
    if (!CORE && CPH > 1) cluster.sync();

#pragma unroll
    for (int i = 0; i < NV4; ++i)
        *reinterpret_cast<float4 *>(srow + 16 * i + 4 * j) =
            make_float4(S[4 * i], S[4 * i + 1], S[4 * i + 2], S[4 * i + 3]);
    // History rows: v channels belong to their rows' CTA; the q/k channels of
    // key head kh are written by rank 0 of value head kh (h < Hk) only.
    if (!CORE) {
#pragma unroll
        for (int u = 0; u < CPT; ++u) {
            const int e = tid + u * NT, c = ch[u];
            if (c < 0 || (e < 2 * D && !(h < Hk && rank == 0))) continue;
            a.history[c] = h0[u]; a.history[(size_t)C + c] = h1[u]; a.history[2 * (size_t)C + c] = h2[u];
        }
    }
}

namespace {
void check_launch(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
}  // namespace

// D = 128: 4-CTA clusters per value head (32 state rows per CTA); D = 32: one CTA.
void delta_run(float *out, float *state, float *history, const float *qkv, const float *gate,
               const float *alpha, const float *beta, const float *conv, const float *decay,
               const float *bias, const float *norm, int T, int Hk, int Hv, int D, float eps,
               cudaStream_t st) {
    DeltaArgs a{};
    a.out = out; a.state = state; a.history = history; a.qkv = qkv; a.gate = gate;
    a.alpha = alpha; a.beta = beta; a.conv = conv; a.decay = decay; a.bias = bias; a.norm = norm;
    a.T = T; a.Hk = Hk; a.Hv = Hv; a.eps = eps;
    if (D == 128) delta_kernel<128, 4, false><<<Hv * 4, 128, 0, st>>>(a);
    else if (D == 32) delta_kernel<32, 1, false><<<Hv, 128, 0, st>>>(a);
    else throw std::invalid_argument("unsupported DeltaNet dimension");
    check_launch("delta");
}

void delta_core_recurrent(float *out, float *state, const __half *q, const __half *k, const __half *v,
                          const float *alpha, const float *beta, const float *decay, const float *bias,
                          int T, int Hk, int Hv, int D, cudaStream_t st) {
    DeltaArgs a{};
    a.out = out; a.state = state; a.q16 = q; a.k16 = k; a.v16 = v;
    a.alpha = alpha; a.beta = beta; a.decay = decay; a.bias = bias;
    a.T = T; a.Hk = Hk; a.Hv = Hv;
    if (D == 128) delta_kernel<128, 4, true><<<Hv * 4, 128, 0, st>>>(a);
    else if (D == 32) delta_kernel<32, 1, true><<<Hv, 128, 0, st>>>(a);
    else throw std::invalid_argument("unsupported DeltaNet dimension");
    check_launch("delta core");
}

}  // namespace qv
