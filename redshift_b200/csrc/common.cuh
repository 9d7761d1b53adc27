// Device-side building blocks for the sm_100a hot-path kernels: mbarriers with
// bounded waits, TMA tile loads, tcgen05 (TMEM alloc / MMA / ld / st) and the
// shared-memory matrix descriptors of the 5th-generation tensor core.
//
// Every wait in this file is bounded: a wait that runs past its limit sets the
// library's device error word and returns false, so no kernel can spin
// forever on a barrier that is never completed.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>
#include <stdexcept>
#include <utility>

namespace qv {

// Status word written by kernels when a bounded wait gives up (see status.cu).
extern __device__ int g_status;
enum : int { STATUS_OK = 0, STATUS_TIMEOUT = 1, STATUS_BAD_ARGUMENT = 2 };

constexpr long long WAIT_LIMIT_CYCLES = 4000000000LL;   // ~2 s at 1.9 GHz

__device__ __forceinline__ void raise_status(int code) { atomicCAS(&g_status, 0, code); }

// Phase timestamps for latency studies.  Compiled in only when the library is
// built with QV_TIMELINE defined (never in the product build): the calling
// thread stores %globaltimer into slot `i` of its CTA's row of g_timeline
// ([QV_TIMELINE_CTAS][QV_TIMELINE_SLOTS], read back by qv_timeline_read).
#ifdef QV_TIMELINE
constexpr int QV_TIMELINE_CTAS = 1024, QV_TIMELINE_SLOTS = 16;
extern __device__ unsigned long long g_timeline[QV_TIMELINE_CTAS * QV_TIMELINE_SLOTS];
__device__ __forceinline__ void qv_stamp(int i) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    const unsigned cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    if (cta < (unsigned)QV_TIMELINE_CTAS) g_timeline[cta * QV_TIMELINE_SLOTS + i] = t;
}
#define QV_STAMP(i) qv_stamp(i)
#else
#define QV_STAMP(i) ((void)0)
#endif

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_addr(bar)), "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}"
                 :: "r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
                 :: "r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Wait for the phase with the given parity to complete.  Gives up after
// WAIT_LIMIT_CYCLES (or at once when *abort is already set), records the
// timeout and sets *abort so that the other roles of the CTA wind down.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = clock64();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (clock64() - start > WAIT_LIMIT_CYCLES) {
            raise_status(STATUS_TIMEOUT);
            *abort = 1;
            return false;
        }
    }
}

// Cluster (DSMEM) helpers: address of the same shared variable in CTA `rank`
// of the cluster, a store there, and a release-arrive on a peer's mbarrier.
__device__ __forceinline__ uint32_t cluster_map(const void *p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" :: "r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t remote_bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" :: "r"(remote_bar) : "memory");
}
// Bounded acquire-wait (cluster scope) on a local mbarrier that peers arrive on.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity) {
    const long long start = clock64();
    while (true) {
        uint32_t ok;
        asm volatile("{\n\t.reg .pred p;\n\t"
                     "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
                     "selp.u32 %0, 1, 0, p;\n\t}"
                     : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
        if (ok) return true;
        if (clock64() - start > WAIT_LIMIT_CYCLES) { raise_status(STATUS_TIMEOUT); return false; }
    }
}

// System-scope flag access for signalling across GPUs (peer memory).
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// 64-bit words that carry a value and its ready flag together (low 32 bits:
// the value's bits, high 32 bits: the flag).  An aligned 64-bit access is
// single-copy atomic, so a reader that sees the flag also sees the value and
// no fence is needed between data and flag.
__device__ __forceinline__ void st_word_sys(uint64_t *p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_word_sys(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// ---------------------------------------------------------------- proxies
__device__ __forceinline__ void fence_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Orders this thread's generic-proxy global writes before later async-proxy
// (TMA) reads of the same memory issued after a CTA-level synchronisation.
__device__ __forceinline__ void fence_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---------------------------------------------------------------- launch chaining
// Programmatic dependent launch: a kernel launched with the programmatic
// stream-serialisation attribute may start while its predecessor in the
// stream is still running.  grid_dependency_wait() blocks until that
// predecessor has completed and its memory is visible (a no-op without the
// attribute); every kernel calls it before touching memory another kernel
// wrote, and signals its own dependents only after it (so a kernel two
// launches back has always completed when a kernel starts).
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Named barrier over a subset of the CTA's warps (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------- TMA
// 2-D tiled bulk tensor load global -> shared, completion via the mbarrier's
// transaction count, into this CTA only.  Coordinates are in elements; the
// innermost one must be a multiple of 8 for 16-bit data.
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, uint64_t *bar,
                                            int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];"
        :: "r"(smem_addr(dst)), "l"(tmap), "r"(smem_addr(bar)), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void *tmap) {
    asm volatile("prefetch.tensormap [%0];" :: "l"(tmap) : "memory");
}
// L2 prefetch hint: it moves nothing into the CTA and leaves no copy that a
// later write could make stale (L2 is the device's point of coherence), so it
// may be issued before the grid-dependency wait, while the previous kernel
// still runs.
__device__ __forceinline__ void prefetch_l2(const void *p) {
    asm volatile("prefetch.global.L2 [%0];" :: "l"(p));
}

// Device-scope acquire load (for a word written by other CTAs of a grid).
__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_addr(dst_smem)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                 :: "r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (fp16 inputs, fp32 accumulate).
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
                 : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16: A is read from TMEM (M rows in
// lanes, two fp16 per 32-bit column, K=16 per instruction = 8 columns).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
                 :: "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
                 : "memory");
}
// Arrive on an mbarrier once every previously issued tcgen05.mma of this
// thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// 32 lanes x 32 bit, 16 consecutive columns: thread i of the warp gets
// columns [col, col+16) of TMEM lane (warp's lane base + i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                   "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
                 "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
                 :: "r"(taddr),
                    "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])),
                    "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
                    "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
                    "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
                    "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])),
                    "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
                    "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
                    "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
                 : "memory");
}

// Shared-memory matrix descriptor (tcgen05 "version 1" format):
//   bits  0-13  start address >> 4
//   bits 16-29  leading-dimension byte offset >> 4
//   bits 32-45  stride-dimension byte offset >> 4
//   bits 46-47  version = 1
//   bits 49-51  base offset (0: swizzle atoms are 1024-byte aligned)
//   bits 61-63  layout: 2 = 128-byte swizzle
// K-major, 128B swizzle: rows of 128 bytes, 8-row groups `sbo` bytes apart.
// MN-major, 128B swizzle: 64-element atoms along M/N `lbo` bytes apart,
// 8-deep K groups `sbo` bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor for kind::f16 with fp16 A/B and fp32 accumulator.
//   bits 4-5 D format (1 = f32), 7-9 A format (0 = f16), 10-12 B format,
//   15 A major (1 = MN), 16 B major, 17-22 N >> 3, 24-28 M >> 4.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool a_mn, bool b_mn) {
    return (1u << 4) | (0u << 7) | (0u << 10) | ((a_mn ? 1u : 0u) << 15) |
           ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------- packed fp32
// Two-wide fp32 arithmetic of sm_100 (fma / mul on a float2 in one
// instruction, each lane rounded as the scalar operation would be).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// ---------------------------------------------------------------- misc math
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int d = 16; d; d >>= 1) x += __shfl_xor_sync(0xffffffffu, x, d);
    return x;
}
// 2^x with the SFU's approximate exp2 (flushes subnormal results to zero).
__device__ __forceinline__ float exp2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }
__device__ __forceinline__ float siluf_(float x) { return x * sigmoidf_(x); }
// Fast forms for the DeltaNet path: sigmoid(x) = 1 / (1 + 2^(-x log2 e)) with
// the SFU's approximate 2^x and reciprocal (a few float ulp; a huge negative
// x gives 1/inf = 0).
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float sigmoid_fast(float x) { return rcp_approx(1.f + exp2_approx(-1.4426950408889634f * x)); }
__device__ __forceinline__ float silu_fast(float x) { return x * sigmoid_fast(x); }
__device__ __forceinline__ float softplusf_(float x) { return x > 20.f ? x : log1pf(expf(x)); }

// ---------------------------------------------------------------- host set-up
// cuTensorMapEncodeTiled from the driver, looked up once per process.
inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        cudaDriverEntryPointQueryResult q;
        void *ptr = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !ptr)
            throw std::runtime_error("cuTensorMapEncodeTiled is unavailable");
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }();
    return fn;
}


// Runs a set-up step once per CUDA device, with that device current.  Kernel
// attributes such as the dynamic shared-memory limit are kept per device by
// the runtime, so a process that drives several GPUs must set them on each;
// concurrent first calls from several host threads run the step once.
class PerDeviceOnce {
  public:
    template <class F> void run(F &&setup) {
        int dev = -1;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
            throw std::runtime_error("no usable current CUDA device");
        if (done_[dev].load(std::memory_order_acquire)) return;
        std::lock_guard<std::mutex> guard(lock_);
        if (done_[dev].load(std::memory_order_relaxed)) return;
        setup();
        done_[dev].store(true, std::memory_order_release);
    }

  private:
    static constexpr int kMaxDevices = 64;
    std::mutex lock_;
    std::atomic<bool> done_[kMaxDevices] = {};
};

// ---------------------------------------------------------------- host launch
// Launch `kernel` on `stream` with programmatic stream serialisation: its CTAs
// may be scheduled (and run up to grid_dependency_wait()) while the previous
// kernel of the stream drains, which hides the launch gap between the
// kernels of one layer and between layers.
template <typename... Params, typename... Args>
inline cudaError_t launch_chained(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                                  cudaStream_t stream, Args &&...args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace qv
