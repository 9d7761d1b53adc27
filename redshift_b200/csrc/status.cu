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

}  // namespace qv
