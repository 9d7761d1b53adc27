// Checkpoint / restore of layer state in one launch.
//
// The reference's Model::copy_state (src/runtime.cu:455-485) snapshots or
// restores, per layer, the attention KV cache's valid prefix (prefix x 4 heads
// x 256 x fp16, for K and for V) and the DeltaNet state and conv history, as
// one cudaMemcpy each: 128 copies for the 64-layer model.  Here the whole list
// of (destination, source, bytes) spans is one kernel launch: the span table
// travels in the kernel parameters, every CTA walks the spans and copies its
// grid-stride share of each with 16-byte loads and stores (4 in flight per
// thread), so the copy runs at the HBM copy rate however many spans there are.
// The table (at most 160 spans) stays within the classic 4 KB parameter space.
// Spans whose addresses or length are not 16-byte multiples take a byte loop.
#include "common.cuh"
#include "hotpath.h"

#include <algorithm>
#include <stdexcept>
#include <string>

namespace qv {
namespace {

struct SpanTable {
    char *dst[MAX_COPY_SPANS];
    const char *src[MAX_COPY_SPANS];
    size_t bytes[MAX_COPY_SPANS];
    int count;
};

__global__ void __launch_bounds__(256) copy_spans_kernel(const SpanTable t) {
    grid_dependency_wait();
    if (threadIdx.x == 0) launch_dependents();
    const size_t nthreads = (size_t)gridDim.x * blockDim.x;
    const size_t me = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (int s = 0; s < t.count; ++s) {
        char *d = t.dst[s];
        const char *src = t.src[s];
        const size_t n = t.bytes[s];
        const bool vec = ((reinterpret_cast<uintptr_t>(d) | reinterpret_cast<uintptr_t>(src) | n) & 15) == 0;
        if (vec) {
            const size_t words = n / 16;
            int4 *dw = reinterpret_cast<int4 *>(d);
            const int4 *sw = reinterpret_cast<const int4 *>(src);
            size_t i = me;
            for (; i + 3 * nthreads < words; i += 4 * nthreads) {
                const int4 a = __ldg(sw + i), b = __ldg(sw + i + nthreads);
                const int4 c = __ldg(sw + i + 2 * nthreads), e = __ldg(sw + i + 3 * nthreads);
                dw[i] = a; dw[i + nthreads] = b; dw[i + 2 * nthreads] = c; dw[i + 3 * nthreads] = e;
            }
            for (; i < words; i += nthreads) dw[i] = __ldg(sw + i);
        } else {
            for (size_t i = me; i < n; i += nthreads) d[i] = src[i];
        }
    }
}

}  // namespace

void copy_spans(void *const *dst, const void *const *src, const size_t *bytes, int count, cudaStream_t st) {
    if (count < 1 || count > MAX_COPY_SPANS) throw std::invalid_argument("span count must be 1..160");
    SpanTable t{};
    size_t total = 0;
    for (int i = 0; i < count; ++i) {
        t.dst[i] = static_cast<char *>(dst[i]);
        t.src[i] = static_cast<const char *>(src[i]);
        t.bytes[i] = bytes[i];
        total += bytes[i];
    }
    t.count = count;
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // 4 CTAs of 256 threads per SM cover the copy; tiny copies use fewer CTAs
    const size_t want = (total / 16 + 1023) / 1024;
    const int grid = (int)std::max<size_t>(1, std::min<size_t>((size_t)sms * 4, want));
    const cudaError_t e = launch_chained(copy_spans_kernel, dim3(grid), dim3(256), 0, st, t);
    if (e != cudaSuccess) throw std::runtime_error(std::string("copy spans: ") + cudaGetErrorString(e));
}

}  // namespace qv
