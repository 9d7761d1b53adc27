// Device-side status word shared by all kernels of the library.  A kernel
// whose bounded wait gives up writes a non-zero code here instead of
// spinning forever; the synchronous entry points read and clear it.
#include "common.cuh"
#include "hotpath.h"

#include <stdexcept>

namespace qv {

__device__ int g_status = 0;

int read_and_clear_status() {
    int value = 0;
    if (cudaMemcpyFromSymbol(&value, g_status, sizeof(int)) != cudaSuccess)
        throw std::runtime_error("cannot read the device status word");
    if (value) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_status, &zero, sizeof(int)) != cudaSuccess)
            throw std::runtime_error("cannot clear the device status word");
    }
    return value;
}

#ifdef QV_TIMELINE
__device__ unsigned long long g_timeline[QV_TIMELINE_CTAS * QV_TIMELINE_SLOTS];
#endif

}  // namespace qv

#ifdef QV_TIMELINE
// Latency-study builds only: copy the phase timestamps of the last launches
// ([1024 CTAs][16 slots] of %globaltimer nanoseconds) to the host and clear them.
extern "C" int qv_timeline_read(unsigned long long *dst) {
    const size_t bytes = sizeof(qv::g_timeline);
    void *addr = nullptr;
    if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpyFromSymbol(dst, qv::g_timeline, bytes) != cudaSuccess ||
        cudaGetSymbolAddress(&addr, qv::g_timeline) != cudaSuccess || cudaMemset(addr, 0, bytes) != cudaSuccess)
        return -1;
    return 0;
}
#endif
