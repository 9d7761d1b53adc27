// Full-attention hot path for sm_100a: prepare (RMSNorm + partial RoPE + fp16
// KV append), a tcgen05/TMEM FlashAttention kernel that serves both the
// decode/verify regime (split-KV, all 6 GQA heads x T tokens of one KV head
// share every K/V tile) and causal prefill (128 query positions of one head
// per CTA), and the split/shard combine kernels.
//
// Semantics follow the reference's attn_prepare / attention / attention_tiled
// (src/kernels.cu:415-503) and the CPU oracle tests/cpu_reference.py:55-89:
// scores q.k/16 over cache rows [0, position+t], softmax, P.V, times
// sigmoid(gate).
#include "common.cuh"
#include "hotpath.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdexcept>
#include <string>

namespace qv {

constexpr int NQ = 24, NKV = 4, HD = 256, GROUP = NQ / NKV;
constexpr int BM = 128;          // rows per CTA (TMEM lanes)
constexpr int BN = 64;           // cache positions per K/V tile
constexpr int STAGES = 2;        // K/V tile pipeline depth
constexpr float SCORE_LOG2 = 0.0625f * 1.4426950408889634f;   // (1/16) * log2(e)
constexpr float RESCALE_THRESHOLD = 8.f;                      // lazy O rescale, log2 units

// Shared-memory map of fa_kernel (offsets from a 1024-byte aligned base).
constexpr int SM_Q = 0;                                   // 4 x [128 rows][64 d] fp16, 16 KB each
constexpr int SM_KV = SM_Q + 4 * BM * 128;                 // per stage: K 4 x 8 KB, V 4 x 8 KB
constexpr int SM_KV_STAGE = 2 * 4 * BN * 128;
constexpr int SM_P = SM_KV + STAGES * SM_KV_STAGE;         // 2 x [128 rows][64 pos] fp16
constexpr int SM_BAR = SM_P + 2 * BM * 128;
constexpr int SM_TOTAL = SM_BAR + 256;
constexpr int SMEM_BYTES = SM_TOTAL + 1024;                // slack for manual alignment

struct FaParams {
    const __half *q;        // prepared queries [T][24][256]
    const float *q_gate;    // [T][24][512], gate = [256:512) (direct mode), may be null
    float *out;             // [T][24][256] (direct mode)
    float *lse;             // optional natural-log LSE [T][24] (direct mode)
    float *part_o;          // [4][splits][128][256] unnormalised partial O (split mode)
    float *part_ml;         // [4][splits][128][2]  (running max in log2 units, sum)
    int T, position;        // tokens and absolute position of token 0
    int kv_begin;           // absolute position of cache row 0
    int kv_rows;            // valid cache rows
    int mode;               // 0 = decode (GQA-packed rows), 1 = prefill (head-major rows)
    int split_tiles, splits;
    int direct;             // 1: write final output; 0: write split partials
};

__device__ __forceinline__ void row_token_head(const FaParams &p, int r, int &t, int &h) {
    if (p.mode == 0) { t = r / GROUP; h = blockIdx.y * GROUP + r % GROUP; }
    else { t = (gridDim.y - 1 - blockIdx.y) * BM + r; h = blockIdx.x; }
}

__global__ void __launch_bounds__(256, 1)
fa_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
          const FaParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + SM_BAR);
    uint64_t *k_full = bars, *v_full = bars + 2, *kv_empty = bars + 4, *s_full = bars + 6,
             *s_free = bars + 8, *p_full = bars + 10, *p_free = bars + 12, *mma_done = bars + 14;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + SM_BAR + 128);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + SM_BAR + 132);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kv_head = p.mode == 0 ? blockIdx.y : blockIdx.x / GROUP;

    // KV tile range of this CTA (tile = 64 cache rows, local numbering).
    int tile0, ntiles;
    if (p.mode == 0) {
        const int total = (p.kv_rows + BN - 1) / BN;
        tile0 = blockIdx.x * p.split_tiles;
        ntiles = min(p.split_tiles, total - tile0);
    } else {
        const int qtile = gridDim.y - 1 - blockIdx.y;
        const int last_tok = min(p.T, (qtile + 1) * BM) - 1;
        const int limit = min(p.kv_rows, p.position + last_tok - p.kv_begin + 1);
        tile0 = 0;
        ntiles = (limit + BN - 1) / BN;
    }

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(k_full + i, 1); mbar_init(v_full + i, 1); mbar_init(kv_empty + i, 1);
            mbar_init(s_full + i, 1); mbar_init(s_free + i, 4);
            mbar_init(p_full + i, 4); mbar_init(p_free + i, 1);
        }
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) { prefetch_tmap(&tmK); prefetch_tmap(&tmV); }
    if (warp == 1) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }

    // Stage the query rows into the 128B-swizzled K-major layout of operand A.
    // Rows without a (token, head) are zero.
    for (int u = threadIdx.x; u < BM * 32; u += blockDim.x) {
        const int r = u >> 5, unit = u & 31, chunk = unit >> 3, w = unit & 7;
        int t, h;
        row_token_head(p, r, t, h);
        const bool valid = (p.mode == 0 ? r < p.T * GROUP : true) && t < p.T;
        uint4 val = make_uint4(0, 0, 0, 0);
        if (valid) val = *reinterpret_cast<const uint4 *>(p.q + ((size_t)t * NQ + h) * HD + unit * 8);
        *reinterpret_cast<uint4 *>(smem + SM_Q + chunk * (BM * 128) + r * 128 + ((w ^ (r & 7)) << 4)) = val;
    }
    fence_async_shared();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            int issued = 0;
            for (int j = 0; j < ntiles; ++j) {
                const int s = j & 1;
                if (j >= STAGES && !mbar_wait(kv_empty + s, ((j >> 1) - 1) & 1, abort_flag)) break;
                const int y = (tile0 + j) * BN;
                uint8_t *kd = smem + SM_KV + s * SM_KV_STAGE, *vd = kd + 4 * BN * 128;
                mbar_expect_tx(k_full + s, 4 * BN * 128);
                for (int c = 0; c < 4; ++c) tma_load_2d(kd + c * BN * 128, &tmK, k_full + s, kv_head * HD + c * 64, y);
                mbar_expect_tx(v_full + s, 4 * BN * 128);
                for (int c = 0; c < 4; ++c) tma_load_2d(vd + c * BN * 128, &tmV, v_full + s, kv_head * HD + c * 64, y);
                issued = j + 1;
            }
            // Drain: every issued load must land before the CTA may exit.
            for (int j = max(0, issued - 2); j < issued; ++j) {
                const long long t0 = clock64();
                while (!mbar_try_wait(v_full + (j & 1), (j >> 1) & 1) && clock64() - t0 < WAIT_LIMIT_CYCLES) {}
                while (!mbar_try_wait(k_full + (j & 1), (j >> 1) & 1) && clock64() - t0 < WAIT_LIMIT_CYCLES) {}
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc_qk = idesc_f16(BM, BN, false, false);
            const uint32_t idesc_pv = idesc_f16(BM, HD, false, true);
            const uint32_t q_base = smem_addr(smem + SM_Q);
            auto issue_pv = [&](int i) -> bool {
                const int s = i & 1;
                if (!mbar_wait(p_full + s, (i >> 1) & 1, abort_flag)) return false;
                if (!mbar_wait(v_full + s, (i >> 1) & 1, abort_flag)) return false;
                tc_fence_after();
                const uint32_t pa = smem_addr(smem + SM_P + s * BM * 128);
                const uint32_t vb = smem_addr(smem + SM_KV + s * SM_KV_STAGE + 4 * BN * 128);
#pragma unroll
                for (int k = 0; k < BN / 16; ++k)
                    mma_f16_ss(tmem + 128, sw128_desc(pa + k * 32, 16, 1024),
                               sw128_desc(vb + k * 16 * 128, BN * 128, 1024), idesc_pv,
                               (i > 0 || k > 0) ? 1u : 0u);
                mma_commit(p_free + s);
                mma_commit(kv_empty + s);
                return true;
            };
            bool ok = true;
            for (int j = 0; j < ntiles && ok; ++j) {
                const int s = j & 1;
                if (!mbar_wait(k_full + s, (j >> 1) & 1, abort_flag)) { ok = false; break; }
                if (j >= 2 && !mbar_wait(s_free + s, ((j >> 1) - 1) & 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t kb = smem_addr(smem + SM_KV + s * SM_KV_STAGE);
#pragma unroll
                for (int k = 0; k < HD / 16; ++k)
                    mma_f16_ss(tmem + s * BN, sw128_desc(q_base + (k >> 2) * (BM * 128) + (k & 3) * 32, 16, 1024),
                               sw128_desc(kb + (k >> 2) * (BN * 128) + (k & 3) * 32, 16, 1024),
                               idesc_qk, k > 0 ? 1u : 0u);
                mma_commit(s_full + s);
                if (j >= 1) ok = issue_pv(j - 1);
            }
            if (ok && ntiles > 0) issue_pv(ntiles - 1);
            // All MMAs of this thread must finish before TMEM is released.
            mma_commit(mma_done);
            const long long t0 = clock64();
            while (!mbar_try_wait(mma_done, 0) && clock64() - t0 < WAIT_LIMIT_CYCLES) {}
        }
    } else if (warp >= 4) {
        // ------------------------------------------------ softmax + epilogue
        const int wq = warp - 4, r = wq * 32 + lane;
        const uint32_t t_lane = tmem + ((uint32_t)(wq * 32) << 16);
        int t, h;
        row_token_head(p, r, t, h);
        const bool valid = (p.mode == 0 ? r < p.T * GROUP : true) && t < p.T;
        const int pos_limit = valid ? p.position + t - p.kv_begin : -1;   // last visible local row
        float m_use = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < ntiles; ++j) {
            const int s = j & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(s_full + s, (j >> 1) & 1, abort_flag))) { ok = false; break; }
            tc_fence_after();
            float x[BN];
#pragma unroll
            for (int c = 0; c < BN / 16; ++c) tmem_ld16(t_lane + s * BN + c * 16, *reinterpret_cast<float(*)[16]>(x + c * 16));
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free + s);
            const int key0 = (tile0 + j) * BN;
            const int lim = min(pos_limit, p.kv_rows - 1) - key0;     // columns <= lim are visible
            float m_tile = -INFINITY;
#pragma unroll
            for (int c = 0; c < BN; ++c) {
                x[c] = c <= lim ? x[c] * SCORE_LOG2 : -INFINITY;
                m_tile = fmaxf(m_tile, x[c]);
            }
            float factor = 1.f;
            const bool need = m_tile > m_use + RESCALE_THRESHOLD;
            if (need) { factor = exp2f(m_use - m_tile); m_use = m_tile; l *= factor; }
            if (j > 0 && __any_sync(0xffffffffu, need)) {
                // O already holds tiles < j: wait for PV(j-1), then rescale rows in TMEM.
                if (!__all_sync(0xffffffffu, mbar_wait(p_free + ((j - 1) & 1), ((j - 1) >> 1) & 1, abort_flag))) { ok = false; break; }
                tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < HD / 16; ++c) {
                    float o[16];
                    tmem_ld16(t_lane + 128 + c * 16, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 16; ++e) o[e] *= factor;
                    tmem_st16(t_lane + 128 + c * 16, o);
                }
                tmem_wait_st();
            }
            const float mref = m_use == -INFINITY ? 0.f : m_use;
            uint32_t packed[BN / 2];
            float sum = 0.f;
#pragma unroll
            for (int c = 0; c < BN; c += 2) {
                const __half2 hp = __floats2half2_rn(exp2f(x[c] - mref), exp2f(x[c + 1] - mref));
                const float2 back = __half22float2(hp);
                sum += back.x + back.y;
                packed[c / 2] = *reinterpret_cast<const uint32_t *>(&hp);
            }
            l += sum;
            if (j >= 2 && !__all_sync(0xffffffffu, mbar_wait(p_free + s, ((j - 2) >> 1) & 1, abort_flag))) { ok = false; break; }
            uint8_t *prow = smem + SM_P + s * BM * 128 + r * 128;
#pragma unroll
            for (int w = 0; w < 8; ++w)
                *reinterpret_cast<uint4 *>(prow + ((w ^ (r & 7)) << 4)) =
                    make_uint4(packed[4 * w], packed[4 * w + 1], packed[4 * w + 2], packed[4 * w + 3]);
            fence_async_shared();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full + s);
        }
        // Epilogue: the final PV's commit on p_free marks O complete.
        if (ok && ntiles > 0 &&
            __all_sync(0xffffffffu, mbar_wait(p_free + ((ntiles - 1) & 1), ((ntiles - 1) >> 1) & 1, abort_flag))) {
            tc_fence_after();
            if (p.direct) {
                const float inv = valid && l > 0.f ? 1.f / l : 0.f;
                float *dst = valid ? p.out + ((size_t)t * NQ + h) * HD : nullptr;
                const float *gate = valid && p.q_gate ? p.q_gate + ((size_t)t * NQ + h) * 2 * HD + HD : nullptr;
#pragma unroll 1
                for (int c = 0; c < HD / 16; ++c) {
                    float o[16];
                    tmem_ld16(t_lane + 128 + c * 16, o);
                    tmem_wait_ld();
                    if (dst) {
#pragma unroll
                        for (int e = 0; e < 16; e += 4) {
                            float4 v = make_float4(o[e] * inv, o[e + 1] * inv, o[e + 2] * inv, o[e + 3] * inv);
                            if (gate) {
                                const float4 g = *reinterpret_cast<const float4 *>(gate + c * 16 + e);
                                v.x *= sigmoidf_(g.x); v.y *= sigmoidf_(g.y);
                                v.z *= sigmoidf_(g.z); v.w *= sigmoidf_(g.w);
                            }
                            *reinterpret_cast<float4 *>(dst + c * 16 + e) = v;
                        }
                    }
                }
                if (valid && p.lse) p.lse[(size_t)t * NQ + h] = l > 0.f ? (m_use + log2f(l)) * 0.6931471805599453f : -INFINITY;
            } else {
                const size_t slot = ((size_t)kv_head * p.splits + blockIdx.x) * BM + r;
                float *dst = p.part_o + slot * HD;
#pragma unroll 1
                for (int c = 0; c < HD / 16; ++c) {
                    float o[16];
                    tmem_ld16(t_lane + 128 + c * 16, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 16; e += 4)
                        *reinterpret_cast<float4 *>(dst + c * 16 + e) = make_float4(o[e], o[e + 1], o[e + 2], o[e + 3]);
                }
                p.part_ml[slot * 2] = m_use;
                p.part_ml[slot * 2 + 1] = l;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------- prepare
// One block per (head, token): 24 query heads then 4 key heads.  RMSNorm with
// weight, rotary embedding on dims [0,64) as pairs (i, i+32) with angle
// (position+t) * 1e7^(-i/32) evaluated in double precision, queries written
// as fp16 operand rows, keys/values rounded to fp16 into the cache.
__global__ void __launch_bounds__(256)
attn_prepare_kernel(const float *q_gate, const float *key, const float *value, const float *qn,
                    const float *kn, __half *qw, __half *kc, __half *vc, int position,
                    int append_row0, float eps) {
    const int t = blockIdx.x, h = blockIdx.y, i = threadIdx.x;
    const bool isq = h < NQ;
    const int kh = h - NQ;
    const float *src = isq ? q_gate + ((size_t)t * NQ + h) * 2 * HD : key + ((size_t)t * NKV + kh) * HD;
    __shared__ float row[HD], red[8];
    const float x = src[i];
    float ss = warp_sum(x * x);
    if ((i & 31) == 0) red[i >> 5] = ss;
    __syncthreads();
    ss = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) ss += red[w];
    const float inv = rsqrtf(ss / HD + eps);
    row[i] = x * inv * (isq ? qn : kn)[i];
    __syncthreads();
    if (i < 32) {
        const double theta = (double)(position + t) * exp(-(double)i / 32.0 * 16.11809565095832);  // ln(1e7)
        double sd, cd;
        sincos(theta, &sd, &cd);
        const float c = (float)cd, s = (float)sd, a = row[i], b = row[i + 32];
        row[i] = a * c - b * s;
        row[i + 32] = a * s + b * c;
    }
    __syncthreads();
    if (isq) {
        qw[((size_t)t * NQ + h) * HD + i] = __float2half_rn(row[i]);
    } else if (append_row0 >= 0) {
        const size_t o = ((size_t)(append_row0 + t) * NKV + kh) * HD + i;
        kc[o] = __float2half_rn(row[i]);
        vc[o] = __float2half_rn(value[((size_t)t * NKV + kh) * HD + i]);
    }
}

// ---------------------------------------------------------------- combine
// Merge the split partials of one (token, head) row.  mode_out 0: final
// gated output; 1: normalised shard partial + natural-log LSE.
__global__ void __launch_bounds__(256)
attn_combine_kernel(float *out, float *out_lse, const float *part_o, const float *part_ml,
                    const float *q_gate, int splits, int final_gate) {
    const int t = blockIdx.x / NQ, h = blockIdx.x % NQ, d = threadIdx.x;
    const int g = h / GROUP, r = t * GROUP + h % GROUP;
    float M = -INFINITY;
    for (int s = 0; s < splits; ++s) M = fmaxf(M, part_ml[(((size_t)g * splits + s) * BM + r) * 2]);
    float num = 0.f, den = 0.f;
    if (M != -INFINITY) {
        for (int s = 0; s < splits; ++s) {
            const size_t slot = ((size_t)g * splits + s) * BM + r;
            const float m = part_ml[slot * 2];
            if (m == -INFINITY) continue;
            const float w = exp2f(m - M);
            den += w * part_ml[slot * 2 + 1];
            num += w * part_o[slot * HD + d];
        }
    }
    const size_t o = ((size_t)t * NQ + h) * HD + d;
    if (final_gate) {
        out[o] = (den > 0.f ? num / den : 0.f) * sigmoidf_(q_gate[((size_t)t * NQ + h) * 2 * HD + HD + d]);
    } else {
        out[o] = den > 0.f ? num / den : 0.f;
        if (d == 0) out_lse[(size_t)t * NQ + h] = den > 0.f ? (M + log2f(den)) * 0.6931471805599453f : -INFINITY;
    }
}

// Merge per-GPU shard partials (normalised O, natural-log LSE) into the gated
// output: O = sum_g exp(lse_g - LSE) O_g, times sigmoid(gate).
__global__ void __launch_bounds__(256)
attn_merge_kernel(float *out, const float *parts, const float *lses, int shards, int T,
                  const float *q_gate) {
    const int t = blockIdx.x / NQ, h = blockIdx.x % NQ, d = threadIdx.x;
    const size_t row = (size_t)t * NQ + h, stride_o = (size_t)T * NQ * HD, stride_l = (size_t)T * NQ;
    float M = -INFINITY;
    for (int g = 0; g < shards; ++g) M = fmaxf(M, lses[g * stride_l + row]);
    float num = 0.f, den = 0.f;
    if (M != -INFINITY)
        for (int g = 0; g < shards; ++g) {
            const float L = lses[g * stride_l + row];
            if (L == -INFINITY) continue;
            const float w = expf(L - M);
            den += w;
            num += w * parts[g * stride_o + row * HD + d];
        }
    out[row * HD + d] = (den > 0.f ? num / den : 0.f) * sigmoidf_(q_gate[row * 2 * HD + HD + d]);
}

// ======================================================================= host
namespace {
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

// 2-D map over a [rows][4*256] fp16 cache: box = 64 dims x 64 rows, 128B swizzle.
CUtensorMap cache_map(const void *base, int rows) {
    CUtensorMap m;
    cuuint64_t dims[2] = {(cuuint64_t)NKV * HD, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)NKV * HD * sizeof(__half)};
    cuuint32_t box[2] = {64, (cuuint32_t)BN};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims,
                                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return m;
}

void check_launch(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

bool configured = false;
void configure() {
    if (configured) return;
    if (cudaFuncSetAttribute(fa_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess)
        throw std::runtime_error("cannot reserve shared memory for the attention kernel");
    configured = true;
}

struct Split { int tiles, splits; };
// Split-KV plan: about 37 CTAs per KV head (148 SMs / 4 heads), whole tiles
// per split.  The plan depends only on the cache length.
Split decode_split(int kv_rows) {
    const int total = (kv_rows + BN - 1) / BN;
    const int per = (total + 36) / 37;
    return {per, (total + per - 1) / per};
}
size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
}  // namespace

size_t attention_workspace_bytes(int T, int kv_rows) {
    size_t q = align256((size_t)T * NQ * HD * sizeof(__half));
    if (T * GROUP > BM) return q;                        // prefill regime: direct output
    const Split sp = decode_split(kv_rows);
    return q + align256((size_t)NKV * sp.splits * BM * HD * sizeof(float)) +
           align256((size_t)NKV * sp.splits * BM * 2 * sizeof(float));
}

// Core of one attention layer over a device cache holding absolute positions
// [kv_begin, kv_begin + kv_rows).  New rows are appended at local row
// position - kv_begin when append is true.  Writes either the final gated
// output (shard_out == nullptr) or a normalised partial + LSE (shard mode).
void attention_run(float *out, float *shard_lse, __half *kc, __half *vc, const float *q_gate,
                   const float *key, const float *value, const float *qn, const float *kn, int T,
                   int position, int kv_begin, int kv_rows, bool append, float eps, void *ws,
                   size_t ws_bytes, cudaStream_t st) {
    if (ws_bytes < attention_workspace_bytes(T, kv_rows)) throw std::invalid_argument("attention workspace too small");
    configure();
    uint8_t *w = static_cast<uint8_t *>(ws);
    __half *qw = reinterpret_cast<__half *>(w);
    attn_prepare_kernel<<<dim3(T, NQ + NKV), 256, 0, st>>>(q_gate, key, value, qn, kn, qw, kc, vc, position,
                                                           append ? position - kv_begin : -1, eps);
    check_launch("attention prepare");
    const CUtensorMap mk = cache_map(kc, kv_rows), mv = cache_map(vc, kv_rows);
    FaParams p{};
    p.q = qw; p.q_gate = q_gate; p.T = T; p.position = position;
    p.kv_begin = kv_begin; p.kv_rows = kv_rows;
    if (T * GROUP <= BM) {
        const Split sp = decode_split(kv_rows);
        p.mode = 0; p.split_tiles = sp.tiles; p.splits = sp.splits; p.direct = 0;
        p.part_o = reinterpret_cast<float *>(w + align256((size_t)T * NQ * HD * sizeof(__half)));
        p.part_ml = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(p.part_o) +
                                              align256((size_t)NKV * sp.splits * BM * HD * sizeof(float)));
        fa_kernel<<<dim3(sp.splits, NKV), 256, SMEM_BYTES, st>>>(mk, mv, p);
        check_launch("attention decode");
        attn_combine_kernel<<<T * NQ, 256, 0, st>>>(out, shard_lse, p.part_o, p.part_ml, q_gate, sp.splits,
                                                    shard_lse ? 0 : 1);
        check_launch("attention combine");
    } else {
        if (shard_lse) throw std::invalid_argument("shard partials are limited to decode batches");
        p.mode = 1; p.direct = 1; p.out = out; p.splits = 1;
        fa_kernel<<<dim3(NQ, (T + BM - 1) / BM), 256, SMEM_BYTES, st>>>(mk, mv, p);
        check_launch("attention prefill");
    }
}

void attention_merge(float *out, const float *parts, const float *lses, int shards, int T,
                     const float *q_gate, cudaStream_t st) {
    attn_merge_kernel<<<T * NQ, 256, 0, st>>>(out, parts, lses, shards, T, q_gate);
    check_launch("attention merge");
}

// Core-level causal prefill on already-prepared fp16 queries (no norm, RoPE
// or gate): out [T][24][256] = softmax(q.k/16, causal) v, optional LSE.
void prefill_core(float *out, float *lse, const __half *q, const __half *kc, const __half *vc, int T,
                  int position, cudaStream_t st) {
    configure();
    const int kv_rows = position + T;
    const CUtensorMap mk = cache_map(kc, kv_rows), mv = cache_map(vc, kv_rows);
    FaParams p{};
    p.q = q; p.T = T; p.position = position; p.kv_begin = 0; p.kv_rows = kv_rows;
    p.mode = 1; p.direct = 1; p.out = out; p.lse = lse; p.splits = 1;
    fa_kernel<<<dim3(NQ, (T + BM - 1) / BM), 256, SMEM_BYTES, st>>>(mk, mv, p);
    check_launch("prefill attention");
}

}  // namespace qv
