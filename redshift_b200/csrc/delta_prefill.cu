// Gated-DeltaNet layer prefill in the chunked form: the reference layer's
// semantics (conv + SiLU with the conv history, q / k L2 norms, the delta
// rule, gated RMSNorm; src/kernels.cu:275-312, 314-354, 409-414 and
// tests/cpu_reference.py:18-52) over a long block of tokens, with the delta
// rule evaluated chunk by chunk on the tensor cores (gdn_chunk.cu).
//
// Three launches:
//  * delta_conv_kernel: causal depthwise conv over [history; raw rows] and
//    SiLU for every (token, channel), written as the fp16 operands of the
//    chunked core (q, k of the key heads, v of the value heads); the last
//    three raw rows become the new conv history;
//  * delta_chunked (gdn_prep_kernel + gdn_scan_kernel): the L2 norms, decays,
//    betas and the recurrence; the state readout goes into `out`;
//  * delta_gated_norm_kernel: out = o rsqrt(mean(o^2) + eps) norm silu(z), in
//    place, one warp per (token, value head).
// Precision: the filtered q, k, v enter the tensor cores as fp16 (the
// chunked core's operand format), which keeps the state within ~1e-3
// relative of the float64 recurrence over thousands of tokens rather than at
// the recurrent kernel's float32 level. The gated RMSNorm rescales each
// output row to unit RMS, so a row whose readout is small carries a larger
// error (up to a few 1e-2 absolute on 4096 random tokens, 1e-2 at the
// 99.99th percentile). qv_delta keeps the exact float32 recurrence.
#include "common.cuh"
#include "hotpath.h"

#include <stdexcept>
#include <string>

namespace qv {

namespace {
constexpr int CONV_TOKENS = 16;           // tokens of one conv thread (a running window)

// One thread per (channel, block of CONV_TOKENS tokens): the window of the
// three raw rows before the block comes from the history or from qkv.
__global__ void __launch_bounds__(256)
delta_conv_kernel(const float *qkv, const float *history, const float *conv, __half *q16, __half *k16,
                  __half *v16, int T, int Hk, int Hv, int D) {
    const int C = (2 * Hk + Hv) * D;
    const int c = blockIdx.x * blockDim.x + threadIdx.x, t0 = blockIdx.y * CONV_TOKENS;
    grid_dependency_wait();
    if (threadIdx.x == 0) launch_dependents();
    if (c >= C) return;
    const float4 w = *reinterpret_cast<const float4 *>(conv + (size_t)c * 4);
    // raw row at token t (t < 0: history row 3 + t)
    auto raw = [&](int t) { return t < 0 ? history[(size_t)(3 + t) * C + c] : qkv[(size_t)t * C + c]; };
    float h0 = raw(t0 - 3), h1 = raw(t0 - 2), h2 = raw(t0 - 1);
    float x[CONV_TOKENS];                      // the block's raw rows, all loads in flight at once
#pragma unroll
    for (int i = 0; i < CONV_TOKENS; ++i) x[i] = t0 + i < T ? qkv[(size_t)(t0 + i) * C + c] : 0.f;
    __half *dst;
    size_t stride;
    if (c < Hk * D) { dst = q16 + c; stride = (size_t)Hk * D; }
    else if (c < 2 * Hk * D) { dst = k16 + (c - Hk * D); stride = (size_t)Hk * D; }
    else { dst = v16 + (c - 2 * Hk * D); stride = (size_t)Hv * D; }
#pragma unroll
    for (int i = 0; i < CONV_TOKENS; ++i) {
        if (t0 + i >= T) break;
        // the reference's order: the three history taps summed, then the new row
        // (cpu_reference.py:25-26)
        const float f = siluf_(((w.x * h0 + w.y * h1) + w.z * h2) + w.w * x[i]);
        h0 = h1; h1 = h2; h2 = x[i];
        dst[(size_t)(t0 + i) * stride] = __float2half_rn(f);
    }
}

// New conv history: the last three raw rows of [history; qkv].
__global__ void __launch_bounds__(256)
delta_history_kernel(const float *qkv, float *history, int T, int C) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    grid_dependency_wait();
    if (threadIdx.x == 0) launch_dependents();
    if (c >= C) return;
    float r[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        const int t = T - 3 + j;                   // raw row index in [history; qkv] terms
        r[j] = t < 0 ? history[(size_t)(3 + t) * C + c] : qkv[(size_t)t * C + c];
    }
#pragma unroll
    for (int j = 0; j < 3; ++j) history[(size_t)j * C + c] = r[j];
}

// Gated RMSNorm over each (token, value head) row of D = 128, in place: one
// warp per row, four values per lane (cpu_reference.py:49-51).
__global__ void __launch_bounds__(256)
delta_gated_norm_kernel(float *out, const float *gate, const float *norm, int rows, float eps) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    grid_dependency_wait();
    if (threadIdx.x == 0) launch_dependents();
    if (row >= rows) return;
    float4 o = reinterpret_cast<float4 *>(out + (size_t)row * 128)[lane];
    const float4 z = reinterpret_cast<const float4 *>(gate + (size_t)row * 128)[lane];
    const float4 n = reinterpret_cast<const float4 *>(norm)[lane];
    const float ss = warp_sum(o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w);
    const float scale = rsqrtf(ss / 128.f + eps);
    o.x *= scale * n.x * siluf_(z.x);
    o.y *= scale * n.y * siluf_(z.y);
    o.z *= scale * n.z * siluf_(z.z);
    o.w *= scale * n.w * siluf_(z.w);
    reinterpret_cast<float4 *>(out + (size_t)row * 128)[lane] = o;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
}  // namespace

size_t delta_prefill_workspace_bytes(int T, int Hk, int Hv) {
    constexpr int D = 128;
    return align256((size_t)T * Hk * D * 2) * 2 + align256((size_t)T * Hv * D * 2) + delta_chunked_workspace_bytes(T, Hv);
}

void delta_prefill(float *out, float *state, float *history, const float *qkv, const float *gate, const float *alpha,
                   const float *beta, const float *conv, const float *decay, const float *bias, const float *norm, int T,
                   int Hk, int Hv, int D, float eps, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (D != 128) throw std::invalid_argument("the chunked DeltaNet prefill needs head dimension 128");
    if (T < 1) throw std::invalid_argument("empty prefill block");
    if (ws_bytes < delta_prefill_workspace_bytes(T, Hk, Hv)) throw std::invalid_argument("DeltaNet prefill workspace too small");
    uint8_t *w = static_cast<uint8_t *>(ws);
    __half *q16 = reinterpret_cast<__half *>(w);
    __half *k16 = reinterpret_cast<__half *>(w + align256((size_t)T * Hk * D * 2));
    __half *v16 = reinterpret_cast<__half *>(w + 2 * align256((size_t)T * Hk * D * 2));
    uint8_t *core_ws = w + 2 * align256((size_t)T * Hk * D * 2) + align256((size_t)T * Hv * D * 2);
    const size_t core_bytes = ws_bytes - (size_t)(core_ws - w);
    const int C = (2 * Hk + Hv) * D;
    cudaError_t e = launch_chained(delta_conv_kernel, dim3((C + 255) / 256, (T + CONV_TOKENS - 1) / CONV_TOKENS),
                                   dim3(256), 0, st, qkv, history, conv, q16, k16, v16, T, Hk, Hv, D);
    if (e != cudaSuccess) throw std::runtime_error(std::string("DeltaNet prefill conv: ") + cudaGetErrorString(e));
    // The history is rewritten only after the conv launch has read it (the
    // next launch in the stream starts its memory accesses after this one
    // completed).
    e = launch_chained(delta_history_kernel, dim3((C + 255) / 256), dim3(256), 0, st, qkv, history, T, C);
    if (e != cudaSuccess) throw std::runtime_error(std::string("DeltaNet prefill history: ") + cudaGetErrorString(e));
    delta_chunked(out, state, q16, k16, v16, alpha, beta, decay, bias, T, Hk, Hv, D, core_ws, core_bytes, st);
    e = launch_chained(delta_gated_norm_kernel, dim3((T * Hv + 7) / 8), dim3(256), 0, st, out, gate, norm, T * Hv, eps);
    if (e != cudaSuccess) throw std::runtime_error(std::string("DeltaNet prefill norm: ") + cudaGetErrorString(e));
}

}  // namespace qv
