#ifndef QVELOX_RUNTIME_H
#define QVELOX_RUNTIME_H
/* C ABI of the B200 (sm_100a) build of the Redshift hot path, libqvelox.so.
 *
 * Part 1 keeps the reference ABI (cristianku/redshift src/runtime.h:14-74)
 * symbol for symbol, so qvelox/runtime.py binds this library unmodified.
 * Part 2 is additive: entry points with no counterpart in the reference,
 * for prefill-length blocks, device-resident (stream-ordered) calls and the
 * multi-GPU split-KV decode.
 *
 * Every int-returning function returns 0 on success and -1 on failure;
 * qv_error() then describes the failure (thread-local, cleared by the next
 * call).  Arguments are validated before any caller buffer is read. */
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ===================== Part 1: the reference ABI ===================== */

/* Replaces src/runtime.h:14 (thread-local message of the last failure). */
const char *qv_error(void);

/* Replace src/runtime.h:15-21 (the reference's test_projection,
 * src/runtime.cu:80-113).  out [batch][rows] = W x for W [rows][width] in
 * block format kind 8 (Q8_0), 12 (Q4_K) or 14 (Q6_K), batch 1..8, width a
 * multiple of the block (32 / 256), 1..248320 rows; host buffers,
 * synchronous.  qv_test_mm_fast quantises the activations per 32-column block
 * to 16-bit integers first (the reference's dp4a path semantics). */
int qv_test_mm(float *out, const void *weights, const float *x,
               int kind, int batch, int width, int rows);
int qv_test_mm_fast(float *out, const void *weights, const float *x,
               int kind, int batch, int width, int rows);

/* Replaces src/runtime.h:22-23.  Weighted RMSNorm of batch rows (1..8) of
 * width 1..17408.  Host buffers. */
int qv_test_norm(float *out, const float *x, const float *weights,
                 int batch, int width, float epsilon);

/* Replaces src/runtime.h:25-36.  One gated-DeltaNet layer over batch 1..8
 * tokens, host buffers.  D = 32 or 128; 1 <= key_heads <= value_heads <= 48;
 * value_heads divisible by key_heads; C = (2*key_heads+value_heads)*D.
 * out/gate: [batch,value_heads,D]; state (in/out): [value_heads,D,D];
 * history (in/out): [3,C]; qkv: [batch,C]; alpha/beta: [batch,value_heads];
 * conv: [C,4]; decay/bias: [value_heads]; norm: [D]. */
int qv_test_delta(float *out, float *state, float *history,
                  const float *qkv, const float *gate,
                  const float *alpha, const float *beta,
                  const float *conv, const float *decay,
                  const float *bias, const float *norm,
                  int batch, int key_heads, int value_heads, int dim,
                  float epsilon);

/* Replaces src/runtime.h:38-46.  Fixed attention: 24 query heads, 4 KV
 * heads, head dimension 256, batch 1..8, host buffers.
 * out: [batch,24,256]; q_gate: [batch,24,512]; key/value: [batch,4,256];
 * q_norm/k_norm: [256].  Caches (in/out) hold IEEE float16 bits as
 * [position+batch,4,256]; only [0,position) is read and only the appended
 * rows [position,position+batch) are written back.
 * 0 <= position and position+batch <= 139264. */
int qv_test_attention(float *out, void *key_cache, void *value_cache,
                      const float *q_gate, const float *key, const float *value,
                      const float *q_norm, const float *k_norm,
                      int batch, int position, float epsilon);

/* Replace src/runtime.h:54-74.  Full-model evaluation needs the quantized
 * weights of the GGUF file and its loader, which are outside this build: qv_create
 * validates its arguments then fails; every call on a handle fails with
 * "null model handle"; qv_destroy(NULL) is a no-op. */
int qv_create(void **handle, const char *path, int context, float epsilon);
int qv_upload(void *handle, int slot, uint64_t offset, uint64_t length);
int qv_evaluate(void *handle, const int *tokens, int batch, float *out);
int qv_verify(void *handle, const int *tokens, int batch, float *out);
int qv_commit(void *handle, int accepted);
int qv_advance(void *handle, const int *tokens, int batch, int *next);
int qv_reset(void *handle);
int qv_checkpoint(void *handle);
int qv_restore(void *handle);
int qv_position(void *handle, int *position);
void qv_destroy(void *handle);

/* ===================== Part 2: additive entry points ===================== */

/* Prefill-length validation entry points: the semantics, layouts and
 * validation of qv_test_attention / qv_test_delta, for batch >= 1
 * (attention: position+batch <= 139264; DeltaNet: batch <= 139264).  The
 * reference reaches these blocks only as 8-token calls (qvelox/server.py:177-193). */
int qv_test_attention_prefill(float *out, void *key_cache, void *value_cache,
                              const float *q_gate, const float *key, const float *value,
                              const float *q_norm, const float *k_norm,
                              int batch, int position, float epsilon);
int qv_test_delta_prefill(float *out, float *state, float *history,
                          const float *qkv, const float *gate,
                          const float *alpha, const float *beta,
                          const float *conv, const float *decay,
                          const float *bias, const float *norm,
                          int batch, int key_heads, int value_heads, int dim,
                          float epsilon);

/* Device-resident attention layer: the operation k_attention performs inside
 * the reference model loop (src/kernels.cu:575-580, called from
 * src/runtime.cu:402-405).  All pointers are device memory; the call is
 * asynchronous on `stream` (a cudaStream_t, NULL = legacy default stream).
 * The caches hold >= position+batch rows.  `workspace` is caller-owned device
 * memory of at least qv_attention_workspace(batch, position) bytes; it must
 * be zero-filled once before its first use (its first 256 bytes hold the
 * counters of the barrier at which a decode launch's CTAs meet before they
 * combine their splits; every call leaves them ready for the next, so later
 * calls need no clearing).  A workspace serves one call at a time. */
size_t qv_attention_workspace(int batch, int position);
int qv_attention(float *out, void *key_cache, void *value_cache,
                 const float *q_gate, const float *key, const float *value,
                 const float *q_norm, const float *k_norm,
                 int batch, int position, float epsilon,
                 void *workspace, size_t workspace_bytes, void *stream);

/* Device-resident DeltaNet layer: the operation k_delta performs in the
 * reference model loop (src/kernels.cu:557-566, src/runtime.cu:384-397).
 * Same layouts as qv_test_delta; batch >= 1; asynchronous on `stream`. */
int qv_delta(float *out, float *state, float *history,
             const float *qkv, const float *gate,
             const float *alpha, const float *beta,
             const float *conv, const float *decay,
             const float *bias, const float *norm,
             int batch, int key_heads, int value_heads, int dim,
             float epsilon, void *stream);

/* Device-resident quantized projection: the operation the reference model's
 * projection() performs (src/runtime.cu:345-354 with src/kernels.cu:506-552):
 * out [batch][rows] = W x for batch 1..8, W [rows][width] in block format
 * `kind` (8 = Q8_0, 12 = Q4_K, 14 = Q6_K; qv_mm_weight_bytes bytes), x
 * [batch][width] f32.  fast != 0 selects the 16-bit activation-block path of
 * qv_test_mm_fast.  All pointers are device memory; weights and x must be
 * 16-byte aligned (as cudaMalloc gives; other addresses are rejected).
 * Asynchronous on `stream`. */
size_t qv_mm_weight_bytes(int kind, int width, int rows);
int qv_mm(float *out, const void *weights, const float *x, int kind, int batch,
          int width, int rows, int fast, void *stream);

/* Checkpoint / restore of the layer state (the reference's Model::copy_state,
 * src/runtime.cu:455-485, which issues one cudaMemcpy per attention KV prefix
 * and per DeltaNet state / history): copies `count` (1..160) spans
 * dst[i] <- src[i] of bytes[i] bytes in one launch.  dst, src and bytes are
 * host arrays of device addresses and sizes (read during the call); the
 * spans must not overlap each other.  Asynchronous on `stream`. */
int qv_copy_spans(void *const *dst, const void *const *src, const size_t *bytes,
                  int count, void *stream);

/* Verify transaction of a DeltaNet layer, the state side of the reference's
 * qv_verify / qv_commit (src/runtime.h:57-68; src/runtime.cu:363-374 saves the
 * start state and history and records the transitions, src/runtime.cu:389-395
 * with src/kernels.cu:356-360 writes the trace, src/runtime.cu:432-454 with
 * src/kernels.cu:362-369, 567-574 commits).  All pointers are device memory,
 * asynchronous on `stream`.
 *
 * qv_delta_verify is qv_delta (batch 1..8) that, in the same pass, copies the
 * start state into saved_state [value_heads][dim][dim] and the start history
 * into saved_history [3][C], and writes the transition trace into `trace`
 * (qv_delta_trace_floats floats, C = (2*key_heads+value_heads)*dim): per
 * token t < 8 the raw qkv row at t*C, the prepared row at (8+t)*C (q and k
 * L2-normalised, q also times 1/sqrt(dim), v filtered), the decay at
 * 16*C + t*value_heads + h and the beta at 16*C + 8*value_heads +
 * t*value_heads + h.
 *
 * qv_delta_commit, after `accepted` of the `batch` verified tokens were kept
 * (0 <= accepted <= batch): accepted == batch keeps the verify's result;
 * otherwise state and history become the start state and history advanced
 * by the first `accepted` tokens, rebuilt from the saved copies and the trace
 * in one kernel (no start-state copy back). */
size_t qv_delta_trace_floats(int key_heads, int value_heads, int dim);
int qv_delta_verify(float *out, float *state, float *history,
                    const float *qkv, const float *gate,
                    const float *alpha, const float *beta,
                    const float *conv, const float *decay,
                    const float *bias, const float *norm,
                    int batch, int key_heads, int value_heads, int dim,
                    float epsilon, float *saved_state, float *saved_history,
                    float *trace, void *stream);
int qv_delta_commit(float *state, float *history, const float *saved_state,
                    const float *saved_history, const float *trace,
                    int accepted, int batch, int key_heads, int value_heads,
                    int dim, void *stream);

/* Sequence-split decode across GPUs.  A shard cache holds the absolute
 * positions [shard_begin, shard_begin+shard_rows) as rows [0,shard_rows).
 * When shard_begin+shard_rows == position the batch's new rows are appended
 * to this shard (capacity >= shard_rows+batch) and attended; otherwise the
 * shard must lie wholly before position.  Writes the shard's normalised
 * partial [batch,24,256] (no gate) and natural-log LSE [batch,24] (-inf for
 * rows that see no key).  batch 1..10.  qv_attention_merge combines `shards`
 * stacked partials [shards,batch,24,256] / LSEs [shards,batch,24] into the
 * gated output [batch,24,256].  The workspace follows qv_attention's rule
 * (zero-filled before its first use). */
size_t qv_attention_shard_workspace(int batch, int shard_rows);
int qv_attention_shard(float *partial, float *lse, void *key_cache, void *value_cache,
                       int shard_begin, int shard_rows,
                       const float *q_gate, const float *key, const float *value,
                       const float *q_norm, const float *k_norm,
                       int batch, int position, float epsilon,
                       void *workspace, size_t workspace_bytes, void *stream);
int qv_attention_merge(float *out, const float *partials, const float *lses, int shards,
                       int batch, const float *q_gate, void *stream);

/* Fused multi-GPU verify: qv_attention_shard, then an all-to-all exchange of
 * the (partial, LSE) pairs through peer memory and the merge, with no
 * collective library on the path.  peer_buffers is a device array of `world`
 * pointers (rank order) to every rank's exchange buffer of
 * qv_attention_exchange_bytes(world) bytes, zero-initialised before the first
 * call and mapped into this process (CUDA IPC / symmetric memory).  Each
 * rank stores its partial into every buffer and raises a flag there, then
 * waits (bounded; on timeout qv_status reports it) for all ranks' flags.
 * `sequence` (>= 0) numbers the calls on the same buffers: the same value on
 * every rank, one more for each call (n, n+1, n+2, ...; after the first call
 * it may restart at any value of the other parity).  Its parity selects one
 * of two buffer slots and its low 24 bits tag every exchanged word, so a word
 * that arrives after its reader timed out is never accepted by a later call;
 * a call that reported a timeout has an undefined `out`, the buffers stay
 * usable.  All ranks must make the same sequence of calls.  world 1..8,
 * batch 1..10; out [batch,24,256] is the gated output, identical on every
 * rank. */
size_t qv_attention_exchange_bytes(int world);
int qv_attention_shard_exchange(float *out, void *key_cache, void *value_cache,
                                int shard_begin, int shard_rows,
                                const float *q_gate, const float *key, const float *value,
                                const float *q_norm, const float *k_norm,
                                int batch, int position, float epsilon,
                                const void *peer_buffers, int world, int rank, int sequence,
                                void *workspace, size_t workspace_bytes, void *stream);

/* Core causal prefill attention (no norm, RoPE or gate), device memory:
 * q [tokens,24,256] fp16 at absolute positions position..position+tokens-1;
 * caches [position+tokens,4,256] fp16; out [tokens,24,256] fp32 =
 * softmax(q.k/16 over keys <= own position) v; lse [tokens,24] natural log
 * (may be NULL).  Asynchronous on `stream`. */
int qv_prefill_attention(float *out, float *lse, const void *q,
                         const void *key_cache, const void *value_cache,
                         int tokens, int position, void *stream);

/* Core gated-DeltaNet recurrence over a prefill block (no conv, no gated
 * norm), device memory: raw q,k [tokens,key_heads,D] fp16 (L2-normalised
 * inside; q also by 1/sqrt(D)), v [tokens,value_heads,D] fp16, alpha/beta
 * raw [tokens,value_heads] (log decay = decay*softplus(alpha+bias), beta =
 * sigmoid(beta)), state [value_heads,D,D] fp32 in/out; out
 * [tokens,value_heads,D] fp32 is the state readout before the gated norm. */
int qv_delta_core(float *out, float *state, const void *q, const void *k, const void *v,
                  const float *alpha, const float *beta, const float *decay, const float *bias,
                  int tokens, int key_heads, int value_heads, int dim, void *stream);

/* The same computation as qv_delta_core in the chunked form (chunks of 64
 * tokens, tensor cores): one parallel pass builds every chunk's triangular
 * (WY) factors, one sequential pass per value head carries the state across
 * chunks.  dim must be 128.  `workspace` is caller-owned device memory of at
 * least qv_delta_chunked_workspace(tokens, value_heads) bytes (0 = invalid
 * arguments); its contents need not be initialised.  Asynchronous on
 * `stream`. */
size_t qv_delta_chunked_workspace(int tokens, int value_heads);
int qv_delta_chunked(float *out, float *state, const void *q, const void *k, const void *v,
                     const float *alpha, const float *beta, const float *decay, const float *bias,
                     int tokens, int key_heads, int value_heads, int dim,
                     void *workspace, size_t workspace_bytes, void *stream);

/* Gated-DeltaNet layer prefill in the chunked form (device memory,
 * asynchronous on `stream`): the layer of qv_delta -- causal conv + SiLU over
 * the conv history and the block, q / k L2 norms, the delta rule, gated
 * RMSNorm, history updated to the block's last three raw rows -- over a long
 * block of tokens, with the recurrence evaluated in chunks of 64 tokens on
 * the tensor cores (qv_delta_chunked).  Same arguments and layouts as
 * qv_delta; dim must be 128.  The filtered q, k, v enter the tensor cores as
 * fp16, which bounds the state at ~1e-3 relative (not qv_delta's float32
 * level) over thousands of tokens; qv_delta stays the exact recurrence.
 * `workspace`: caller-owned device memory of at least
 * qv_delta_prefill_workspace(tokens, key_heads, value_heads) bytes (0 =
 * invalid arguments), contents need not be initialised. */
size_t qv_delta_prefill_workspace(int tokens, int key_heads, int value_heads);
int qv_delta_prefill(float *out, float *state, float *history,
                     const float *qkv, const float *gate,
                     const float *alpha, const float *beta,
                     const float *conv, const float *decay,
                     const float *bias, const float *norm,
                     int tokens, int key_heads, int value_heads, int dim,
                     float epsilon, void *workspace, size_t workspace_bytes, void *stream);

/* qv_attention without a workspace argument, for callers that cannot
 * allocate device memory (no counterpart in the reference ABI).  A serving
 * runtime that gave all of HBM to its own pools at start-up, or a plugin host
 * that owns every allocation, can still run the verify/decode attention
 * layer: the call allocates nothing (no cudaMalloc, no library allocator).
 * Its scratch space is one fixed 10 MiB array in device memory that each GPU
 * holds from library load until process exit; that covers batch 1..8 at any
 * context up to 139264, and larger requests are rejected with an error.
 * Arguments, layouts and results are those of qv_attention (device pointers,
 * asynchronous on `stream`), with batch limited to 1..8.
 * The first call on a device looks up the array's device address (once per
 * device, with that device current); make that first call before any stream
 * capture.  Every call uses the same array and leaves its contents behind.
 * The array is zero when the library loads; its first 256 bytes are the
 * counters of the barrier inside the attention launch, which must start at
 * zero and which every call leaves at zero again, and each call writes every
 * other byte before reading it.  Calls that overlap on the GPU (other
 * streams, other host threads) race on the array: issue them in order on one
 * stream per device. */
int qv_attention_noalloc(float *out, void *key_cache, void *value_cache,
                         const float *q_gate, const float *key, const float *value,
                         const float *q_norm, const float *k_norm,
                         int batch, int position, float epsilon, void *stream);

/* Synchronise the current device and return (then clear) the status word
 * that kernels set when a bounded internal wait gives up: 0 = none. */
int qv_status(void);

#ifdef __cplusplus
}
#endif
#endif
