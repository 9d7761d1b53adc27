// Quantized projections for verify batches (T <= 8): out[t][row] = sum_k W[row][k] x[t][k]
// with W in the GGUF block formats the reference model uses (src/kernels.cu:31-273,
// 506-552; kinds 8 = Q8_0, 12 = Q4_K, 14 = Q6_K).
//
// Design (HBM-bound GEMV with a small batch):
//  * a CTA of 8 warps owns 32 consecutive rows, 4 per warp; every activation
//    value a lane loads from shared memory serves the warp's 4 rows;
//  * the columns are processed in chunks of 256: the activations of a chunk
//    are staged in shared memory token-major (conflict-free, coalesced), and
//    the chunk's block bytes of the CTA's 32 rows are staged next to them with
//    coalesced, independent 16-bit loads (every block size and row length is
//    even, so 2-byte alignment is all the formats guarantee), unrolled so
//    that many loads are in flight per thread;
//  * lane l then takes 4 consecutive columns of a 32-column group (8 lanes
//    per group, 4 groups per step): one 32-bit load of its quants per row,
//    the group's scale decoded once for the 4 columns, one 128-bit load of
//    the activations per token shared by the warp's 4 rows;
//  * the 4 x 8 per-lane sums are reduced across the warp with a transposing
//    butterfly (31 shuffles) that leaves sum v on lane v.
// FAST = true is the reference's dp4a path semantics (runtime.h:17-20): the
// activations are quantised per 32-column block to 16-bit integers (scale
// max|x| / 32639, round half away from zero) and the weights' scale part
// multiplies the quantised activations while the Q4_K minimum part multiplies
// the exact activations (FP32 scales, sums and accumulation).
#include "common.cuh"
#include "hotpath.h"

#include <stdexcept>
#include <string>

namespace qv {
namespace {

constexpr int QM_WARPS = 8, QM_RW = 4, QM_ROWS = QM_WARPS * QM_RW, QM_KC = 256, QM_T = 8;

__device__ __forceinline__ float ld_half(const uint8_t *p) {
    return __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(p)));
}

template <int KIND, bool FAST>
__global__ void __launch_bounds__(QM_WARPS * 32)
qmm_kernel(float *out, const uint8_t *w, const float *x, int T, int width, int rows) {
    constexpr int SB = KIND == 8 ? 32 : 256;                    // columns per block
    constexpr int BB = KIND == 8 ? 34 : (KIND == 12 ? 144 : 210); // bytes per block
    constexpr int CB = (QM_KC / SB) * BB;                        // bytes of one row in a full chunk
    constexpr int CBP = (CB + 15) / 16 * 16;                     // its shared-memory stride (16-byte rows)
    __shared__ __align__(16) float xs[QM_T][QM_KC];
    __shared__ __align__(16) float qs[FAST ? QM_T : 1][FAST ? QM_KC : 4];
    __shared__ __align__(16) uint16_t wbuf[QM_ROWS * CBP / 2];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row0 = blockIdx.x * QM_ROWS + warp * QM_RW;
    const size_t row_bytes = (size_t)(width / SB) * BB;
    grid_dependency_wait();
    if (tid == 0) launch_dependents();

    float acc[QM_RW][QM_T];
#pragma unroll
    for (int r = 0; r < QM_RW; ++r)
#pragma unroll
        for (int t = 0; t < QM_T; ++t) acc[r][t] = 0.f;

    for (int k0 = 0; k0 < width; k0 += QM_KC) {
        const int len = min(QM_KC, width - k0);                  // a multiple of 32
        __syncthreads();                                         // the previous chunk is consumed
#pragma unroll
        for (int t = 0; t < QM_T; ++t)
            for (int kk = tid; kk < len; kk += QM_WARPS * 32)
                xs[t][kk] = t < T ? x[(size_t)t * width + k0 + kk] : 0.f;
        {
            // the chunk's 16-bit words of the CTA's rows; divisions by the
            // compile-time row stride, a partial last chunk (Q8_0 only) masked
            constexpr int HW = CB / 2;
            const int half_words = (len / SB) * BB / 2;
            const size_t col_off = (size_t)(k0 / SB) * BB;
            const uint8_t *rows0 = w + (size_t)blockIdx.x * QM_ROWS * row_bytes + col_off;
            const int nrows = min(QM_ROWS, rows - (int)blockIdx.x * QM_ROWS);
#pragma unroll 4
            for (int i = tid; i < QM_ROWS * HW; i += QM_WARPS * 32) {
                const int r = i / HW, j = i - r * HW;
                wbuf[r * (CBP / 2) + j] = (r < nrows && j < half_words)
                              ? reinterpret_cast<const uint16_t *>(rows0 + (size_t)r * row_bytes)[j] : 0;
            }
        }
        if (FAST) {
            __syncthreads();
            // 16-bit block quantisation of the activations: one warp per (token, 32-block)
            for (int b = warp; b < QM_T * (len / 32); b += QM_WARPS) {
                const int t = b / (len / 32), kk = (b % (len / 32)) * 32 + lane;
                const float v = xs[t][kk];
                float m = fabsf(v);
#pragma unroll
                for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                const float scale = m / 32639.f;
                float q = 0.f;
                if (scale != 0.f) {
                    const float ratio = v / scale;
                    q = copysignf(floorf(fabsf(ratio) + 0.5f), ratio);
                }
                qs[t][kk] = scale * q;
            }
        }
        __syncthreads();
        const uint8_t *wb = reinterpret_cast<const uint8_t *>(wbuf);
        // lane l covers 4 consecutive columns of a 32-column group: group
        // 4 step + l / 8 of the chunk, columns 4 (l % 8) .. + 3 within it
        const int lg = lane >> 3, lc = (lane & 7) * 4;
        for (int step = 0; step * 128 < len; ++step) {
            const int c = step * 128 + lg * 32 + lc;             // first column (within the chunk)
            if (c >= len) continue;                              // a partial Q8_0 chunk
            float4 x4[QM_T], q4[QM_T];
            float xsum[QM_T];
#pragma unroll
            for (int t = 0; t < QM_T; ++t) {
                x4[t] = *reinterpret_cast<const float4 *>(&xs[t][c]);
                q4[t] = FAST ? *reinterpret_cast<const float4 *>(&qs[FAST ? t : 0][FAST ? c : 0]) : x4[t];
                xsum[t] = (x4[t].x + x4[t].y) + (x4[t].z + x4[t].w);
            }
#pragma unroll
            for (int r = 0; r < QM_RW; ++r) {
                if (row0 + r >= rows) continue;
                const uint8_t *rb = wb + (warp * QM_RW + r) * CBP;
                float wq[4], off = 0.f;                           // weight e = wq[e] - off
                if (KIND == 8) {
                    const uint8_t *b = rb + (c >> 5) * BB;          // 34-byte block of this group
                    const float d = ld_half(b);
                    const uint32_t lo = *reinterpret_cast<const uint16_t *>(b + 2 + lc);
                    const uint32_t hi = *reinterpret_cast<const uint16_t *>(b + 4 + lc);
                    const uint32_t q = lo | (hi << 16);
#pragma unroll
                    for (int e = 0; e < 4; ++e) wq[e] = d * (float)(int8_t)(q >> (8 * e));
                } else if (KIND == 12) {
                    // 6-bit scale and minimum of group g from the 12 packed bytes
                    const int g = c >> 5;                         // group within the 256-column block
                    const uint8_t *sc = rb + 4;
                    const int lo6 = g < 4 ? sc[g] : sc[g + 4];
                    const int hi2s = g < 4 ? 0 : (sc[g - 4] >> 6) << 4;
                    const int zlo = g < 4 ? sc[g + 4] : (sc[g + 4] >> 4);
                    const int hi2z = g < 4 ? 0 : (sc[g] >> 6) << 4;
                    const float s6 = (float)(g < 4 ? (lo6 & 63) : ((lo6 & 15) | hi2s));
                    const float z6 = (float)(g < 4 ? (zlo & 63) : (zlo | hi2z));
                    const float ds = ld_half(rb) * s6;
                    off = ld_half(rb + 2) * z6;
                    const uint32_t q = *reinterpret_cast<const uint32_t *>(rb + 16 + (g >> 1) * 32 + lc) >> (4 * (g & 1));
#pragma unroll
                    for (int e = 0; e < 4; ++e) wq[e] = ds * (float)((q >> (8 * e)) & 15);
                } else {
                    const int half = c >> 7, quarter = (c >> 5) & 3;
                    const uint32_t low = *reinterpret_cast<const uint32_t *>(rb + half * 64 + (quarter & 1) * 32 + lc)
                                         >> (4 * (quarter >> 1));
                    const uint32_t high = *reinterpret_cast<const uint32_t *>(rb + 128 + half * 32 + lc) >> (2 * quarter);
                    const float ds = (float)(int8_t)rb[192 + (c >> 4)] * ld_half(rb + 208);
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        wq[e] = (float)((int)(((high >> (8 * e)) & 3) * 16 + ((low >> (8 * e)) & 15)) - 32) * ds;
                }
#pragma unroll
                for (int t = 0; t < QM_T; ++t) {
                    float a = fmaf(-off, xsum[t], acc[r][t]);
                    a = fmaf(wq[0], q4[t].x, a);
                    a = fmaf(wq[1], q4[t].y, a);
                    a = fmaf(wq[2], q4[t].z, a);
                    acc[r][t] = fmaf(wq[3], q4[t].w, a);
                }
            }
        }
    }
    // transposing butterfly: lane l ends with the sum of value l = r * 8 + t
    float v[QM_RW * QM_T];
#pragma unroll
    for (int r = 0; r < QM_RW; ++r)
#pragma unroll
        for (int t = 0; t < QM_T; ++t) v[r * QM_T + t] = acc[r][t];
#pragma unroll
    for (int half = 16; half >= 1; half >>= 1) {
        const bool up = (lane & half) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float lo = v[i], hi = v[i + half];
            v[i] = (up ? hi : lo) + __shfl_xor_sync(0xffffffffu, up ? lo : hi, half);
        }
    }
    const int r = lane / QM_T, t = lane % QM_T, row = row0 + r;
    if (row < rows && t < T) out[(size_t)t * rows + row] = v[0];
}

template <int KIND>
cudaError_t launch_kind(float *out, const uint8_t *w, const float *x, int T, int width, int rows, bool fast,
                        cudaStream_t st) {
    const dim3 grid((rows + QM_ROWS - 1) / QM_ROWS), block(QM_WARPS * 32);
    return fast ? launch_chained(qmm_kernel<KIND, true>, grid, block, 0, st, out, w, x, T, width, rows)
                : launch_chained(qmm_kernel<KIND, false>, grid, block, 0, st, out, w, x, T, width, rows);
}

}  // namespace

size_t projection_weight_bytes(int kind, int width, int rows) {
    const int sb = kind == 8 ? 32 : 256, bb = kind == 8 ? 34 : (kind == 12 ? 144 : 210);
    return (size_t)(width / sb) * bb * rows;
}

void projection_run(float *out, const void *weights, const float *x, int kind, int T, int width, int rows,
                    bool fast, cudaStream_t st) {
    if (T < 1 || T > QM_T) throw std::invalid_argument("projection batch must be between 1 and 8");
    const uint8_t *w = static_cast<const uint8_t *>(weights);
    cudaError_t e;
    if (kind == 8) e = launch_kind<8>(out, w, x, T, width, rows, fast, st);
    else if (kind == 12) e = launch_kind<12>(out, w, x, T, width, rows, fast, st);
    else if (kind == 14) e = launch_kind<14>(out, w, x, T, width, rows, fast, st);
    else throw std::invalid_argument("unsupported quantization type");
    if (e != cudaSuccess) throw std::runtime_error(std::string("projection: ") + cudaGetErrorString(e));
}

}  // namespace qv
