// C ABI of libqvelox.so (declared in include/runtime.h).
//
// Error convention of the reference (src/runtime.cu:9-79): every entry point
// clears a thread-local message, validates all arguments before touching a
// caller buffer, returns 0 on success and -1 with the message set on failure.
#include "../../include/runtime.h"
#include "common.cuh"
#include "hotpath.h"

#include <cmath>
#include <cstdio>
#include <limits>
#include <stdexcept>
#include <string>

namespace {

thread_local char g_message[512] = {};

struct Failure : std::runtime_error { using std::runtime_error::runtime_error; };

void require(bool ok, const char *message) {
    if (!ok) throw std::invalid_argument(message);
}
void cuda_ok(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw Failure(std::string(what) + ": " + cudaGetErrorString(e));
}

template <class F>
int guarded(F &&body) noexcept {
    g_message[0] = '\0';
    try {
        body();
        return 0;
    } catch (const std::exception &e) {
        std::snprintf(g_message, sizeof(g_message), "%s", e.what());
    } catch (...) {
        std::snprintf(g_message, sizeof(g_message), "unknown native error");
    }
    return -1;
}

size_t checked_bytes(size_t count, size_t elem) {
    require(elem == 0 || count <= std::numeric_limits<size_t>::max() / elem, "buffer size overflow");
    return count * elem;
}

// Device allocation owned for the duration of one synchronous call.
class DeviceBuffer {
  public:
    explicit DeviceBuffer(size_t bytes) : bytes_(bytes) {
        if (bytes) cuda_ok(cudaMalloc(&ptr_, bytes), "device allocation");
    }
    ~DeviceBuffer() { if (ptr_) cudaFree(ptr_); }
    DeviceBuffer(const DeviceBuffer &) = delete;
    DeviceBuffer &operator=(const DeviceBuffer &) = delete;
    template <class T = void> T *get() const { return static_cast<T *>(ptr_); }
    void upload(const void *src, size_t bytes, size_t offset = 0) {
        if (bytes) cuda_ok(cudaMemcpy(static_cast<char *>(ptr_) + offset, src, bytes, cudaMemcpyHostToDevice), "upload");
    }
    void zero() {
        if (ptr_) cuda_ok(cudaMemset(ptr_, 0, bytes_), "workspace clear");
    }
    void download(void *dst, size_t bytes, size_t offset = 0) const {
        if (bytes) cuda_ok(cudaMemcpy(dst, static_cast<const char *>(ptr_) + offset, bytes, cudaMemcpyDeviceToHost), "download");
    }
  private:
    void *ptr_ = nullptr;
    size_t bytes_ = 0;
};

// Wait for the device and surface both CUDA errors and kernel status codes.
void finish() {
    cuda_ok(cudaGetLastError(), "kernel launch");
    cuda_ok(cudaDeviceSynchronize(), "kernel execution");
    const int status = qv::read_and_clear_status();
    if (status)
        throw Failure("a kernel gave up waiting on an internal barrier (status " + std::to_string(status) + ")");
}

constexpr int kMaxContext = 139264;      // position+batch <= 139264 (reference runtime.h:42)
constexpr int kAttnHeads = 24, kKvHeads = 4, kHeadDim = 256;
constexpr size_t kCacheRow = (size_t)kKvHeads * kHeadDim * sizeof(uint16_t);

void check_epsilon(float eps) { require(std::isfinite(eps) && eps > 0.f, "epsilon must be finite and positive"); }
void check_delta_dims(int key_heads, int value_heads, int dim) {
    require((dim == 32 || dim == 128) && key_heads > 0 && value_heads >= key_heads &&
            value_heads <= 48 && value_heads % key_heads == 0, "unsupported DeltaNet dimensions");
}
cudaStream_t as_stream(void *s) { return static_cast<cudaStream_t>(s); }

// ------------------------------------------------------------------ attention
void attention_host(float *out, void *key_cache, void *value_cache, const float *q_gate,
                    const float *key, const float *value, const float *q_norm, const float *k_norm,
                    int batch, int position, float eps) {
    const int n = position + batch;
    DeviceBuffer kc(checked_bytes(n, kCacheRow)), vc(checked_bytes(n, kCacheRow));
    kc.upload(key_cache, (size_t)position * kCacheRow);
    vc.upload(value_cache, (size_t)position * kCacheRow);
    const size_t out_elems = (size_t)batch * kAttnHeads * kHeadDim;
    const size_t kv_elems = (size_t)batch * kKvHeads * kHeadDim;
    DeviceBuffer qg(2 * out_elems * sizeof(float)), k(kv_elems * sizeof(float)), v(kv_elems * sizeof(float));
    DeviceBuffer qn(kHeadDim * sizeof(float)), kn(kHeadDim * sizeof(float)), o(out_elems * sizeof(float));
    qg.upload(q_gate, 2 * out_elems * sizeof(float));
    k.upload(key, kv_elems * sizeof(float));
    v.upload(value, kv_elems * sizeof(float));
    qn.upload(q_norm, kHeadDim * sizeof(float));
    kn.upload(k_norm, kHeadDim * sizeof(float));
    const size_t ws_bytes = qv::attention_workspace_bytes(batch, n);
    DeviceBuffer ws(ws_bytes);
    ws.zero();                          // the decode tail's barrier words start at zero
    qv::attention_run(o.get<float>(), nullptr, kc.get<__half>(), vc.get<__half>(), qg.get<float>(),
                      k.get<float>(), v.get<float>(), qn.get<float>(), kn.get<float>(), batch, position,
                      0, n, true, eps, ws.get(), ws_bytes, nullptr);
    finish();
    o.download(out, out_elems * sizeof(float));
    // The prefix is never modified: only the appended rows travel back.
    kc.download(static_cast<char *>(key_cache) + (size_t)position * kCacheRow, (size_t)batch * kCacheRow,
                (size_t)position * kCacheRow);
    vc.download(static_cast<char *>(value_cache) + (size_t)position * kCacheRow, (size_t)batch * kCacheRow,
                (size_t)position * kCacheRow);
}

int test_attention(float *out, void *key_cache, void *value_cache, const float *q_gate,
                   const float *key, const float *value, const float *q_norm, const float *k_norm,
                   int batch, int position, float epsilon, int max_batch) {
    return guarded([&] {
        require(batch >= 1 && batch <= max_batch,
                max_batch == 8 ? "batch must be between 1 and 8" : "batch must be between 1 and 139264");
        check_epsilon(epsilon);
        require(position >= 0 && position <= kMaxContext - batch, "attention context exceeds 139264");
        require(out && key_cache && value_cache && q_gate && key && value && q_norm && k_norm,
                "null attention buffer");
        attention_host(out, key_cache, value_cache, q_gate, key, value, q_norm, k_norm, batch, position, epsilon);
    });
}

// ------------------------------------------------------------------ DeltaNet
int test_delta(float *out, float *state, float *history, const float *qkv, const float *gate,
               const float *alpha, const float *beta, const float *conv, const float *decay,
               const float *bias, const float *norm, int batch, int key_heads, int value_heads, int dim,
               float epsilon, int max_batch) {
    return guarded([&] {
        require(batch >= 1 && batch <= max_batch,
                max_batch == 8 ? "batch must be between 1 and 8" : "batch must be between 1 and 139264");
        check_epsilon(epsilon);
        require(out && state && history && qkv && gate && alpha && beta && conv && decay && bias && norm,
                "null DeltaNet buffer");
        check_delta_dims(key_heads, value_heads, dim);
        const size_t C = (size_t)(2 * key_heads + value_heads) * dim;
        const size_t out_b = checked_bytes((size_t)batch * value_heads * dim, sizeof(float));
        const size_t head_b = (size_t)batch * value_heads * sizeof(float);
        const size_t state_b = (size_t)value_heads * dim * dim * sizeof(float);
        DeviceBuffer s(state_b), h(3 * C * sizeof(float)), q(checked_bytes(batch * C, sizeof(float)));
        DeviceBuffer z(out_b), a(head_b), b(head_b), c(4 * C * sizeof(float));
        DeviceBuffer d(value_heads * sizeof(float)), bi(value_heads * sizeof(float)), n(dim * sizeof(float));
        DeviceBuffer o(out_b);
        s.upload(state, state_b); h.upload(history, 3 * C * sizeof(float));
        q.upload(qkv, batch * C * sizeof(float)); z.upload(gate, out_b);
        a.upload(alpha, head_b); b.upload(beta, head_b); c.upload(conv, 4 * C * sizeof(float));
        d.upload(decay, value_heads * sizeof(float)); bi.upload(bias, value_heads * sizeof(float));
        n.upload(norm, dim * sizeof(float));
        qv::delta_run(o.get<float>(), s.get<float>(), h.get<float>(), q.get<float>(), z.get<float>(),
                      a.get<float>(), b.get<float>(), c.get<float>(), d.get<float>(), bi.get<float>(),
                      n.get<float>(), batch, key_heads, value_heads, dim, epsilon, nullptr);
        finish();
        o.download(out, out_b);
        s.download(state, state_b);
        h.download(history, 3 * C * sizeof(float));
    });
}

// ------------------------------------------------------------------ RMSNorm
__global__ void rms_norm_kernel(float *out, const float *x, const float *w, int width, float eps) {
    const size_t row = (size_t)blockIdx.x * width;
    __shared__ float red[8];
    float s = 0.f;
    for (int i = threadIdx.x; i < width; i += blockDim.x) s += x[row + i] * x[row + i];
    s = qv::warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    s = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += red[i];
    const float inv = rsqrtf(s / width + eps);
    for (int i = threadIdx.x; i < width; i += blockDim.x) out[row + i] = x[row + i] * inv * w[i];
}

}  // namespace

namespace qv {
// Access to the thread-local message of qv_error() for entry points defined
// in other files of the library.
void clear_error() { g_message[0] = '\0'; }
void record_error(const char *message) { std::snprintf(g_message, sizeof(g_message), "%s", message); }
}  // namespace qv

extern "C" {

const char *qv_error(void) { return g_message; }

// ------------------------------------------------------------------ projections
// Quantized projection through host buffers (the reference's test_projection,
// src/runtime.cu:80-113): allocate, upload, run, download, synchronously.
static int test_projection(float *out, const void *weights, const float *x, int kind, int batch, int width,
                           int rows, bool fast) {
    return guarded([&] {
        require(batch >= 1 && batch <= 8, "batch must be between 1 and 8");
        require(out && weights && x, "null projection buffer");
        require(kind == 8 || kind == 12 || kind == 14, "unsupported quantization type");
        const int block = kind == 8 ? 32 : 256;
        require(width > 0 && width % block == 0 && rows > 0 && rows <= 248320, "invalid projection dimensions");
        const size_t wbytes = qv::projection_weight_bytes(kind, width, rows);
        const size_t xbytes = (size_t)batch * width * sizeof(float), obytes = (size_t)batch * rows * sizeof(float);
        DeviceBuffer w(wbytes), in(xbytes), o(obytes);
        w.upload(weights, wbytes);
        in.upload(x, xbytes);
        qv::projection_run(o.get<float>(), w.get(), in.get<float>(), kind, batch, width, rows, fast, nullptr);
        finish();
        o.download(out, obytes);
    });
}
int qv_test_mm(float *out, const void *weights, const float *x, int kind, int batch, int width, int rows) {
    return test_projection(out, weights, x, kind, batch, width, rows, false);
}
int qv_test_mm_fast(float *out, const void *weights, const float *x, int kind, int batch, int width, int rows) {
    return test_projection(out, weights, x, kind, batch, width, rows, true);
}

int qv_test_norm(float *out, const float *x, const float *weights, int batch, int width, float epsilon) {
    return guarded([&] {
        require(batch >= 1 && batch <= 8, "batch must be between 1 and 8");
        check_epsilon(epsilon);
        require(out && x && weights, "null normalization buffer");
        require(width > 0 && width <= 17408, "invalid normalization width");
        const size_t bytes = (size_t)batch * width * sizeof(float);
        DeviceBuffer in(bytes), w(width * sizeof(float)), o(bytes);
        in.upload(x, bytes);
        w.upload(weights, width * sizeof(float));
        rms_norm_kernel<<<batch, 256>>>(o.get<float>(), in.get<float>(), w.get<float>(), width, epsilon);
        finish();
        o.download(out, bytes);
    });
}

int qv_test_delta(float *out, float *state, float *history, const float *qkv, const float *gate,
                  const float *alpha, const float *beta, const float *conv, const float *decay,
                  const float *bias, const float *norm, int batch, int key_heads, int value_heads, int dim,
                  float epsilon) {
    return test_delta(out, state, history, qkv, gate, alpha, beta, conv, decay, bias, norm, batch, key_heads,
                      value_heads, dim, epsilon, 8);
}

int qv_test_attention(float *out, void *key_cache, void *value_cache, const float *q_gate, const float *key,
                      const float *value, const float *q_norm, const float *k_norm, int batch, int position,
                      float epsilon) {
    return test_attention(out, key_cache, value_cache, q_gate, key, value, q_norm, k_norm, batch, position,
                          epsilon, 8);
}

// ------------------------------------------------------------------ model ABI
int qv_create(void **handle, const char *path, int context, float epsilon) {
    return guarded([&] {
        require(handle != nullptr, "null handle output");
        *handle = nullptr;
        require(path != nullptr, "null model path");
        require(context >= 1 && context <= kMaxContext, "context capacity must be 1..139264");
        check_epsilon(epsilon);
        throw Failure("full-model evaluation (GGUF weights and loader) is not part of this build");
    });
}
static int no_model(void *handle) {
    return guarded([&] {
        require(handle != nullptr, "null model handle");
        throw Failure("invalid model handle: this build creates no model sessions");
    });
}
int qv_upload(void *handle, int, uint64_t, uint64_t) { return no_model(handle); }
int qv_evaluate(void *handle, const int *, int, float *) { return no_model(handle); }
int qv_verify(void *handle, const int *, int, float *) { return no_model(handle); }
int qv_commit(void *handle, int) { return no_model(handle); }
int qv_advance(void *handle, const int *, int, int *) { return no_model(handle); }
int qv_reset(void *handle) { return no_model(handle); }
int qv_checkpoint(void *handle) { return no_model(handle); }
int qv_restore(void *handle) { return no_model(handle); }
int qv_position(void *handle, int *position) {
    return guarded([&] {
        require(position != nullptr, "null position output");
        require(handle != nullptr, "null model handle");
        throw Failure("invalid model handle: this build creates no model sessions");
    });
}
void qv_destroy(void *) {}

// ------------------------------------------------------------------ additive
int qv_test_attention_prefill(float *out, void *key_cache, void *value_cache, const float *q_gate,
                              const float *key, const float *value, const float *q_norm, const float *k_norm,
                              int batch, int position, float epsilon) {
    return test_attention(out, key_cache, value_cache, q_gate, key, value, q_norm, k_norm, batch, position,
                          epsilon, kMaxContext);
}

int qv_test_delta_prefill(float *out, float *state, float *history, const float *qkv, const float *gate,
                          const float *alpha, const float *beta, const float *conv, const float *decay,
                          const float *bias, const float *norm, int batch, int key_heads, int value_heads,
                          int dim, float epsilon) {
    return test_delta(out, state, history, qkv, gate, alpha, beta, conv, decay, bias, norm, batch, key_heads,
                      value_heads, dim, epsilon, kMaxContext);
}

size_t qv_attention_workspace(int batch, int position) {
    if (batch < 1 || position < 0 || position > kMaxContext - batch) return 0;
    return qv::attention_workspace_bytes(batch, position + batch);
}

int qv_attention(float *out, void *key_cache, void *value_cache, const float *q_gate, const float *key,
                 const float *value, const float *q_norm, const float *k_norm, int batch, int position,
                 float epsilon, void *workspace, size_t workspace_bytes, void *stream) {
    return guarded([&] {
        require(batch >= 1, "batch must be positive");
        check_epsilon(epsilon);
        require(position >= 0 && position <= kMaxContext - batch, "attention context exceeds 139264");
        require(out && key_cache && value_cache && q_gate && key && value && q_norm && k_norm && workspace,
                "null attention buffer");
        qv::attention_run(out, nullptr, static_cast<__half *>(key_cache), static_cast<__half *>(value_cache),
                          q_gate, key, value, q_norm, k_norm, batch, position, 0, position + batch, true,
                          epsilon, workspace, workspace_bytes, as_stream(stream));
    });
}

int qv_delta(float *out, float *state, float *history, const float *qkv, const float *gate, const float *alpha,
             const float *beta, const float *conv, const float *decay, const float *bias, const float *norm,
             int batch, int key_heads, int value_heads, int dim, float epsilon, void *stream) {
    return guarded([&] {
        require(batch >= 1 && batch <= kMaxContext, "batch must be between 1 and 139264");
        check_epsilon(epsilon);
        require(out && state && history && qkv && gate && alpha && beta && conv && decay && bias && norm,
                "null DeltaNet buffer");
        check_delta_dims(key_heads, value_heads, dim);
        qv::delta_run(out, state, history, qkv, gate, alpha, beta, conv, decay, bias, norm, batch, key_heads,
                      value_heads, dim, epsilon, as_stream(stream));
    });
}

int qv_copy_spans(void *const *dst, const void *const *src, const size_t *bytes, int count, void *stream) {
    return guarded([&] {
        require(count >= 1 && count <= qv::MAX_COPY_SPANS, "span count must be 1..160");
        require(dst && src && bytes, "null span table");
        for (int i = 0; i < count; ++i) require(bytes[i] == 0 || (dst[i] && src[i]), "null span address");
        qv::copy_spans(dst, src, bytes, count, as_stream(stream));
    });
}

size_t qv_mm_weight_bytes(int kind, int width, int rows) {
    if (!(kind == 8 || kind == 12 || kind == 14) || width <= 0 || rows <= 0 || width % (kind == 8 ? 32 : 256))
        return 0;
    return qv::projection_weight_bytes(kind, width, rows);
}

int qv_mm(float *out, const void *weights, const float *x, int kind, int batch, int width, int rows, int fast,
          void *stream) {
    return guarded([&] {
        require(batch >= 1 && batch <= 8, "batch must be between 1 and 8");
        require(out && weights && x, "null projection buffer");
        require(kind == 8 || kind == 12 || kind == 14, "unsupported quantization type");
        const int block = kind == 8 ? 32 : 256;
        require(width > 0 && width % block == 0 && rows > 0 && rows <= 248320, "invalid projection dimensions");
        qv::projection_run(out, weights, x, kind, batch, width, rows, fast != 0, as_stream(stream));
    });
}

size_t qv_delta_trace_floats(int key_heads, int value_heads, int dim) {
    if (!(dim == 32 || dim == 128) || key_heads < 1 || value_heads < key_heads || value_heads > 48 ||
        value_heads % key_heads != 0)
        return 0;
    return 8 * (2 * (size_t)(2 * key_heads + value_heads) * dim + 2 * (size_t)value_heads);
}

int qv_delta_verify(float *out, float *state, float *history, const float *qkv, const float *gate,
                    const float *alpha, const float *beta, const float *conv, const float *decay,
                    const float *bias, const float *norm, int batch, int key_heads, int value_heads, int dim,
                    float epsilon, float *saved_state, float *saved_history, float *trace, void *stream) {
    return guarded([&] {
        require(batch >= 1 && batch <= 8, "a recorded verify holds 1..8 tokens");
        check_epsilon(epsilon);
        require(out && state && history && qkv && gate && alpha && beta && conv && decay && bias && norm,
                "null DeltaNet buffer");
        require(saved_state && saved_history && trace, "null verify record buffer");
        check_delta_dims(key_heads, value_heads, dim);
        qv::delta_verify(out, state, history, qkv, gate, alpha, beta, conv, decay, bias, norm, batch, key_heads,
                         value_heads, dim, epsilon, saved_state, saved_history, trace, as_stream(stream));
    });
}

int qv_delta_commit(float *state, float *history, const float *saved_state, const float *saved_history,
                    const float *trace, int accepted, int batch, int key_heads, int value_heads, int dim,
                    void *stream) {
    return guarded([&] {
        require(batch >= 1 && batch <= 8, "a recorded verify holds 1..8 tokens");
        require(accepted >= 0 && accepted <= batch, "acceptance outside verified batch");
        require(state && history && saved_state && saved_history && trace, "null commit buffer");
        check_delta_dims(key_heads, value_heads, dim);
        if (accepted == batch) return;          // the verify already left this state
        qv::delta_commit(state, history, saved_state, saved_history, trace, accepted, key_heads, value_heads, dim,
                         as_stream(stream));
    });
}

size_t qv_attention_shard_workspace(int batch, int shard_rows) {
    if (batch < 1 || batch > qv::attention_max_shard_batch() || shard_rows < 0) return 0;
    // The split plan is not monotone in the row count: cover both cases.
    const size_t a = qv::attention_workspace_bytes(batch, shard_rows + batch);
    const size_t b = shard_rows ? qv::attention_workspace_bytes(batch, shard_rows) : 0;
    return a > b ? a : b;
}

int qv_attention_shard(float *partial, float *lse, void *key_cache, void *value_cache, int shard_begin,
                       int shard_rows, const float *q_gate, const float *key, const float *value,
                       const float *q_norm, const float *k_norm, int batch, int position, float epsilon,
                       void *workspace, size_t workspace_bytes, void *stream) {
    return guarded([&] {
        require(batch >= 1 && batch <= qv::attention_max_shard_batch(), "shard batch must be between 1 and 10");
        check_epsilon(epsilon);
        require(position >= 0 && position <= kMaxContext - batch, "attention context exceeds 139264");
        require(shard_begin >= 0 && shard_rows >= 0, "invalid shard range");
        const bool append = shard_begin + shard_rows == position;
        require(append || shard_begin + shard_rows < position, "shard extends past the verify position");
        require(partial && lse && key_cache && value_cache && q_gate && key && value && q_norm && k_norm &&
                workspace, "null attention buffer");
        const int rows = shard_rows + (append ? batch : 0);
        require(rows > 0, "empty shard");
        qv::attention_run(partial, lse, static_cast<__half *>(key_cache), static_cast<__half *>(value_cache),
                          q_gate, key, value, q_norm, k_norm, batch, position, shard_begin, rows, append,
                          epsilon, workspace, workspace_bytes, as_stream(stream));
    });
}

int qv_attention_merge(float *out, const float *partials, const float *lses, int shards, int batch,
                       const float *q_gate, void *stream) {
    return guarded([&] {
        require(shards >= 1 && shards <= 64, "shards must be between 1 and 64");
        require(batch >= 1 && batch <= kMaxContext, "invalid batch");
        require(out && partials && lses && q_gate, "null merge buffer");
        qv::attention_merge(out, partials, lses, shards, batch, q_gate, as_stream(stream));
    });
}

size_t qv_attention_exchange_bytes(int world) {
    if (world < 1 || world > qv::attention_exchange_max_world()) return 0;
    return qv::attention_exchange_bytes(world);
}

int qv_attention_shard_exchange(float *out, void *key_cache, void *value_cache, int shard_begin, int shard_rows,
                                const float *q_gate, const float *key, const float *value, const float *q_norm,
                                const float *k_norm, int batch, int position, float epsilon,
                                const void *peer_buffers, int world, int rank, int sequence, void *workspace,
                                size_t workspace_bytes, void *stream) {
    return guarded([&] {
        require(batch >= 1 && batch <= qv::attention_max_shard_batch(), "shard batch must be between 1 and 10");
        check_epsilon(epsilon);
        require(position >= 0 && position <= kMaxContext - batch, "attention context exceeds 139264");
        require(shard_begin >= 0 && shard_rows >= 0, "invalid shard range");
        const bool append = shard_begin + shard_rows == position;
        require(append || shard_begin + shard_rows < position, "shard extends past the verify position");
        require(world >= 1 && world <= qv::attention_exchange_max_world() && rank >= 0 && rank < world,
                "invalid exchange group");
        require(sequence >= 0, "the exchange sequence number must not be negative");
        require(out && key_cache && value_cache && q_gate && key && value && q_norm && k_norm && peer_buffers &&
                workspace, "null attention buffer");
        const int rows = shard_rows + (append ? batch : 0);
        require(rows > 0, "empty shard");
        qv::attention_shard_exchange(out, static_cast<__half *>(key_cache), static_cast<__half *>(value_cache),
                                     q_gate, key, value, q_norm, k_norm, batch, position, shard_begin, rows, append,
                                     epsilon, static_cast<const uint64_t *>(peer_buffers), world, rank, sequence,
                                     workspace, workspace_bytes, as_stream(stream));
    });
}

int qv_prefill_attention(float *out, float *lse, const void *q, const void *key_cache, const void *value_cache,
                         int tokens, int position, void *stream) {
    return guarded([&] {
        require(tokens >= 1 && position >= 0 && position <= kMaxContext - tokens, "invalid prefill range");
        require(out && q && key_cache && value_cache, "null prefill buffer");
        qv::prefill_core(out, lse, static_cast<const __half *>(q), static_cast<const __half *>(key_cache),
                         static_cast<const __half *>(value_cache), tokens, position, as_stream(stream));
    });
}

int qv_delta_core(float *out, float *state, const void *q, const void *k, const void *v, const float *alpha,
                  const float *beta, const float *decay, const float *bias, int tokens, int key_heads,
                  int value_heads, int dim, void *stream) {
    return guarded([&] {
        require(tokens >= 1 && tokens <= kMaxContext, "tokens must be between 1 and 139264");
        check_delta_dims(key_heads, value_heads, dim);
        require(out && state && q && k && v && alpha && beta && decay && bias, "null DeltaNet buffer");
        qv::delta_core_recurrent(out, state, static_cast<const __half *>(q), static_cast<const __half *>(k),
                                 static_cast<const __half *>(v), alpha, beta, decay, bias, tokens, key_heads,
                                 value_heads, dim, as_stream(stream));
    });
}

size_t qv_delta_prefill_workspace(int tokens, int key_heads, int value_heads) {
    if (tokens < 1 || tokens > kMaxContext || key_heads < 1 || value_heads < key_heads || value_heads > 48 ||
        value_heads % key_heads)
        return 0;
    return qv::delta_prefill_workspace_bytes(tokens, key_heads, value_heads);
}

int qv_delta_prefill(float *out, float *state, float *history, const float *qkv, const float *gate, const float *alpha,
                     const float *beta, const float *conv, const float *decay, const float *bias, const float *norm,
                     int tokens, int key_heads, int value_heads, int dim, float epsilon, void *workspace,
                     size_t workspace_bytes, void *stream) {
    return guarded([&] {
        require(tokens >= 1 && tokens <= kMaxContext, "tokens must be between 1 and 139264");
        check_epsilon(epsilon);
        check_delta_dims(key_heads, value_heads, dim);
        require(dim == 128, "the chunked DeltaNet path needs dim 128");
        require(out && state && history && qkv && gate && alpha && beta && conv && decay && bias && norm && workspace,
                "null DeltaNet buffer");
        require(workspace_bytes >= qv::delta_prefill_workspace_bytes(tokens, key_heads, value_heads),
                "workspace too small");
        qv::delta_prefill(out, state, history, qkv, gate, alpha, beta, conv, decay, bias, norm, tokens, key_heads,
                          value_heads, dim, epsilon, workspace, workspace_bytes, as_stream(stream));
    });
}

size_t qv_delta_chunked_workspace(int tokens, int value_heads) {
    if (tokens < 1 || tokens > kMaxContext || value_heads < 1 || value_heads > 48) return 0;
    return qv::delta_chunked_workspace_bytes(tokens, value_heads);
}

int qv_delta_chunked(float *out, float *state, const void *q, const void *k, const void *v, const float *alpha,
                     const float *beta, const float *decay, const float *bias, int tokens, int key_heads,
                     int value_heads, int dim, void *workspace, size_t workspace_bytes, void *stream) {
    return guarded([&] {
        require(tokens >= 1 && tokens <= kMaxContext, "tokens must be between 1 and 139264");
        check_delta_dims(key_heads, value_heads, dim);
        require(dim == 128, "the chunked DeltaNet path needs dim 128");
        require(out && state && q && k && v && alpha && beta && decay && bias && workspace, "null DeltaNet buffer");
        require(workspace_bytes >= qv::delta_chunked_workspace_bytes(tokens, value_heads), "workspace too small");
        qv::delta_chunked(out, state, static_cast<const __half *>(q), static_cast<const __half *>(k),
                          static_cast<const __half *>(v), alpha, beta, decay, bias, tokens, key_heads, value_heads,
                          dim, workspace, workspace_bytes, as_stream(stream));
    });
}

int qv_status(void) {
    int status = -1;
    const int rc = guarded([&] {
        cuda_ok(cudaDeviceSynchronize(), "device synchronize");
        status = qv::read_and_clear_status();
    });
    return rc ? -1 : status;
}

}  // extern "C"
