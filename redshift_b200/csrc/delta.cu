// Gated DeltaNet recurrent path for sm_100a: one fused kernel per layer call.
//
// The reference runs conv -> gdn_prep -> gdn_scan -> delta_out as four
// launches (src/kernels.cu:275-354, 409-414, 557-566).  Here one CTA owns one
// value head: it recomputes the causal conv + SiLU of the q/k channels of its
// key head (h % Hk) and of its own v channels, L2-normalises q and k, forms
// the decay a = exp(A softplus(alpha+bias)) and beta = sigmoid(beta), runs the
// delta rule over the tokens with the head's 128x128 fp32 state held in
// registers (4 threads per state row, 32 columns each), and applies the gated
// RMSNorm before writing the output.  The state is read and written exactly
// once per call.
#include "common.cuh"
#include "hotpath.h"

#include <stdexcept>
#include <string>

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
// CORE = true : prepared-input recurrence used by the chunked-prefill path
//               (raw fp16 q/k/v are L2-normalised here; output is the state
//               readout before the gated norm).
template <int D, bool CORE>
__global__ void __launch_bounds__(D * 4)
delta_kernel(const DeltaArgs a) {
    constexpr int NT = D * 4, COLS = D / 4, NV4 = D / 16, NW = NT / 32;
    const int h = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int Hk = a.Hk, Hv = a.Hv, kh = h % Hk;
    const int C = (2 * Hk + Hv) * D;
    const int r = tid >> 2, j = tid & 3;

    __shared__ __align__(16) float F[3][CHUNK][D];   // q, k, v (filtered)
    __shared__ __align__(16) float O[CHUNK][D];
    __shared__ float sa[CHUNK], sb[CHUNK], sq[CHUNK], sk[CHUNK];

    // State row fragment: columns 16*i + 4*j + e.
    float S[COLS];
    float *srow = a.state + ((size_t)h * D + r) * D;
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
        const float4 v = *reinterpret_cast<const float4 *>(srow + 16 * i + 4 * j);
        S[4 * i] = v.x; S[4 * i + 1] = v.y; S[4 * i + 2] = v.z; S[4 * i + 3] = v.w;
    }

    // Conv channel owned by this thread (tid < 3D): 0 = q, 1 = k, 2 = v.
    const int ctype = tid / D, cidx = tid % D;
    int c = -1;
    if (ctype == 0) c = kh * D + cidx;
    else if (ctype == 1) c = (Hk + kh) * D + cidx;
    else if (ctype == 2) c = (2 * Hk + h) * D + cidx;
    float w0 = 0, w1 = 0, w2 = 0, w3 = 0, h0 = 0, h1 = 0, h2 = 0;
    if (!CORE && c >= 0) {
        w0 = a.conv[(size_t)c * 4]; w1 = a.conv[(size_t)c * 4 + 1];
        w2 = a.conv[(size_t)c * 4 + 2]; w3 = a.conv[(size_t)c * 4 + 3];
        h0 = a.history[c]; h1 = a.history[(size_t)C + c]; h2 = a.history[2 * (size_t)C + c];
    }

    for (int t0 = 0; t0 < a.T; t0 += CHUNK) {
        const int n = min(CHUNK, a.T - t0);
        if (c >= 0) {
            for (int tt = 0; tt < n; ++tt) {
                float f;
                if (!CORE) {
                    const float raw = a.qkv[(size_t)(t0 + tt) * C + c];
                    float v = w3 * raw;
                    v += w0 * h0; v += w1 * h1; v += w2 * h2;
                    h0 = h1; h1 = h2; h2 = raw;
                    f = siluf_(v);
                } else {
                    const int t = t0 + tt;
                    f = ctype == 0 ? __half2float(a.q16[((size_t)t * Hk + kh) * D + cidx])
                      : ctype == 1 ? __half2float(a.k16[((size_t)t * Hk + kh) * D + cidx])
                                   : __half2float(a.v16[((size_t)t * Hv + h) * D + cidx]);
                }
                F[ctype][tt][cidx] = f;
            }
        }
        if (tid < n) {
            const size_t idx = (size_t)(t0 + tid) * Hv + h;
            sa[tid] = expf(a.decay[h] * softplusf_(a.alpha[idx] + a.bias[h]));
            sb[tid] = sigmoidf_(a.beta[idx]);
        }
        __syncthreads();
        for (int task = warp; task < 2 * n; task += NW) {
            const int tt = task >> 1, which = task & 1;
            float s = 0.f;
            for (int i = lane; i < D; i += 32) { const float x = F[which][tt][i]; s += x * x; }
            s = warp_sum(s);
            if (lane == 0) {
                if (which == 0) sq[tt] = rsqrtf(s + 1e-6f) * rsqrtf((float)D);
                else sk[tt] = rsqrtf(s + 1e-6f);
            }
        }
        __syncthreads();
        for (int e = tid; e < n * D; e += NT) {
            const int tt = e / D, i = e % D;
            F[0][tt][i] *= sq[tt];
            F[1][tt][i] *= sk[tt];
        }
        __syncthreads();
        for (int tt = 0; tt < n; ++tt) {
            const float decay = sa[tt], beta = sb[tt];
            const float *kk = F[1][tt], *qq = F[0][tt];
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
            const float delta = (F[2][tt][r] - u) * beta;
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
            for (int e = tid; e < n * D; e += NT) {
                const int tt = e / D, i = e % D;
                a.out[((size_t)(t0 + tt) * Hv + h) * D + i] = O[tt][i];
            }
        } else {
            for (int tt = warp; tt < n; tt += NW) {
                float s = 0.f;
                for (int i = lane; i < D; i += 32) s += O[tt][i] * O[tt][i];
                const float scale = rsqrtf(warp_sum(s) / D + a.eps);
                const size_t base = ((size_t)(t0 + tt) * Hv + h) * D;
                for (int i = lane; i < D; i += 32)
                    a.out[base + i] = O[tt][i] * scale * a.norm[i] * siluf_(a.gate[base + i]);
            }
        }
        __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < NV4; ++i)
        *reinterpret_cast<float4 *>(srow + 16 * i + 4 * j) =
            make_float4(S[4 * i], S[4 * i + 1], S[4 * i + 2], S[4 * i + 3]);
    // History rows: v channels belong to this head; the q/k channels of key
    // head kh are written by value head kh (h < Hk) only.
    if (!CORE && c >= 0 && (ctype == 2 || h < Hk)) {
        a.history[c] = h0; a.history[(size_t)C + c] = h1; a.history[2 * (size_t)C + c] = h2;
    }
}

namespace {
void check_launch(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
}  // namespace

void delta_run(float *out, float *state, float *history, const float *qkv, const float *gate,
               const float *alpha, const float *beta, const float *conv, const float *decay,
               const float *bias, const float *norm, int T, int Hk, int Hv, int D, float eps,
               cudaStream_t st) {
    DeltaArgs a{};
    a.out = out; a.state = state; a.history = history; a.qkv = qkv; a.gate = gate;
    a.alpha = alpha; a.beta = beta; a.conv = conv; a.decay = decay; a.bias = bias; a.norm = norm;
    a.T = T; a.Hk = Hk; a.Hv = Hv; a.eps = eps;
    if (D == 128) delta_kernel<128, false><<<Hv, 512, 0, st>>>(a);
    else if (D == 32) delta_kernel<32, false><<<Hv, 128, 0, st>>>(a);
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
    if (D == 128) delta_kernel<128, true><<<Hv, 512, 0, st>>>(a);
    else if (D == 32) delta_kernel<32, true><<<Hv, 128, 0, st>>>(a);
    else throw std::invalid_argument("unsupported DeltaNet dimension");
    check_launch("delta core");
}

}  // namespace qv
