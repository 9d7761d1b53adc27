// qv_attention_noalloc: the verify/decode attention layer for callers that
// cannot allocate device memory.
//
// Some callers have no way to obtain device memory: a serving runtime that
// handed all of HBM to its own pools (KV cache, activations) at start-up and
// treats any later allocation as a failure, or a plugin host that owns every
// allocation and gives its plugins only the tensors of the call.  This entry
// point needs nothing from them but the inputs and outputs: its scratch space
// (the split-KV partials: each split's unnormalised output rows and their
// running max and sum) lives in a fixed array in device memory that every GPU
// holds from the moment the library is loaded until the process exits.
#include "../../include/runtime.h"
#include "hotpath.h"

#include <cmath>
#include <cstdio>
#include <mutex>
#include <stdexcept>
#include <string>

namespace {

// Fixed scratch: large enough for every decode/verify call of up to 8 tokens
// at any context up to 139,264 (the largest needs 9,775,360 bytes).  It is
// zero at load; its first 256 bytes are the attention launch's barrier
// counters, which must start at zero and which every call leaves at zero.
constexpr size_t kScratchBytes = 10u << 20;   // 10 MiB per GPU
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_lock;
void *g_scratch_addr[kMaxDevices] = {};       // device address of the array, per device

// Device address of the scratch array on the current device.  The symbol's
// name in host code is only a host-side handle, so the address is looked up
// (once per device, with that device current) and handed to the kernels.
void *scratch_on_current_device() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        throw std::runtime_error("no usable current CUDA device");
    std::lock_guard<std::mutex> guard(g_setup_lock);
    if (!g_scratch_addr[dev]) {
        void *ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || !ptr)
            throw std::runtime_error(std::string("cannot resolve the fixed scratch array: ") + cudaGetErrorString(e));
        g_scratch_addr[dev] = ptr;
    }
    return g_scratch_addr[dev];
}

void require(bool ok, const char *message) {
    if (!ok) throw std::invalid_argument(message);
}

}  // namespace

extern "C" int qv_attention_noalloc(float *out, void *key_cache, void *value_cache, const float *q_gate,
                                    const float *key, const float *value, const float *q_norm,
                                    const float *k_norm, int batch, int position, float epsilon, void *stream) {
    qv::clear_error();
    try {
        require(batch >= 1 && batch <= 8, "batch must be between 1 and 8");
        require(std::isfinite(epsilon) && epsilon > 0.f, "epsilon must be finite and positive");
        require(position >= 0 && position <= 139264 - batch, "attention context exceeds 139264");
        require(out && key_cache && value_cache && q_gate && key && value && q_norm && k_norm,
                "null attention buffer");
        const size_t need = qv::attention_workspace_bytes(batch, position + batch);
        if (need > kScratchBytes)
            throw std::invalid_argument("call needs " + std::to_string(need) + " bytes of scratch; the fixed array holds " +
                                        std::to_string(kScratchBytes));
        void *scratch = scratch_on_current_device();
        qv::attention_run(out, nullptr, static_cast<__half *>(key_cache), static_cast<__half *>(value_cache), q_gate,
                          key, value, q_norm, k_norm, batch, position, 0, position + batch, true, epsilon, scratch,
                          kScratchBytes, static_cast<cudaStream_t>(stream));
        return 0;
    } catch (const std::exception &e) {
        qv::record_error(e.what());
    } catch (...) {
        qv::record_error("unknown native error");
    }
    return -1;
}
