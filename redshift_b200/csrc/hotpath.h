// Internal C++ launch API of the hot-path kernels (not part of the C ABI).
// All functions are stream-ordered, take device pointers and throw
// std::exception subclasses on invalid arguments or launch failures.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace qv {

// Attention (attention.cu).  Cache layout [rows][4][256] fp16.
size_t attention_workspace_bytes(int T, int kv_rows);
int attention_max_shard_batch();   // largest batch of the split-KV (decode) regime
void attention_run(float *out, float *shard_lse, __half *kc, __half *vc, const float *q_gate,
                   const float *key, const float *value, const float *qn, const float *kn, int T,
                   int position, int kv_begin, int kv_rows, bool append, float eps, void *ws,
                   size_t ws_bytes, cudaStream_t st);
void attention_merge(float *out, const float *parts, const float *lses, int shards, int T,
                     const float *q_gate, cudaStream_t st);
size_t attention_exchange_bytes(int world);
int attention_exchange_max_world();
void attention_shard_exchange(float *out, __half *kc, __half *vc, const float *q_gate, const float *key,
                              const float *value, const float *qn, const float *kn, int T, int position,
                              int kv_begin, int kv_rows, bool append, float eps, const uint64_t *peers,
                              int world, int rank, int seq, void *ws, size_t ws_bytes, cudaStream_t st);
void prefill_core(float *out, float *lse, const __half *q, const __half *kc, const __half *vc, int T,
                  int position, cudaStream_t st);
// Prefill regime of attention_run (prefill.cu): prepared hi / lo query rows,
// cache rows [0, kv_rows), token t sees rows [0, position + t], output times
// sigmoid(gate) when q_gate is given.
void prefill_precise(float *out, const __half *q, const __half *q_lo, const float *q_gate, const __half *kc,
                     const __half *vc, int T, int position, int kv_rows, cudaStream_t st);

// Gated DeltaNet (delta.cu).
void delta_run(float *out, float *state, float *history, const float *qkv, const float *gate,
               const float *alpha, const float *beta, const float *conv, const float *decay,
               const float *bias, const float *norm, int T, int Hk, int Hv, int D, float eps,
               cudaStream_t st);
// Verify transaction: delta_run that also saves the start state / history and
// writes the transition trace (8 (2C + 2Hv) floats, T <= 8); the commit
// rebuilds state and history from those after `accepted` tokens were kept.
void delta_verify(float *out, float *state, float *history, const float *qkv, const float *gate,
                  const float *alpha, const float *beta, const float *conv, const float *decay,
                  const float *bias, const float *norm, int T, int Hk, int Hv, int D, float eps,
                  float *saved_state, float *saved_history, float *trace, cudaStream_t st);
void delta_commit(float *state, float *history, const float *saved_state, const float *saved_history,
                  const float *trace, int accepted, int Hk, int Hv, int D, cudaStream_t st);
void delta_core_recurrent(float *out, float *state, const __half *q, const __half *k, const __half *v,
                          const float *alpha, const float *beta, const float *decay, const float *bias,
                          int T, int Hk, int Hv, int D, cudaStream_t st);

// Quantized projections (projection.cu): kinds 8 = Q8_0, 12 = Q4_K, 14 = Q6_K;
// out [T][rows] = W [rows][width] x [T][width], T <= 8; `fast` = the 16-bit
// activation-block path.
size_t projection_weight_bytes(int kind, int width, int rows);
void projection_run(float *out, const void *weights, const float *x, int kind, int T, int width, int rows,
                    bool fast, cudaStream_t st);

// Checkpoint / restore (copy.cu): copy up to MAX_COPY_SPANS (dst, src, bytes)
// device spans in one launch.
constexpr int MAX_COPY_SPANS = 160;
void copy_spans(void *const *dst, const void *const *src, const size_t *bytes, int count, cudaStream_t st);

// Chunked gated DeltaNet prefill (gdn_chunk.cu): same inputs / outputs as
// delta_core_recurrent, D = 128, chunks of 64 tokens on tcgen05.
size_t delta_chunked_workspace_bytes(int T, int Hv);
void delta_chunked(float *out, float *state, const __half *q, const __half *k, const __half *v, const float *alpha,
                   const float *beta, const float *decay, const float *bias, int T, int Hk, int Hv, int D, void *ws,
                   size_t ws_bytes, cudaStream_t st);

// Gated-DeltaNet layer prefill in the chunked form (delta_prefill.cu): the
// layer of delta_run (conv + SiLU with history, norms, delta rule, gated
// RMSNorm) over T tokens, D = 128, with the recurrence on tcgen05.
size_t delta_prefill_workspace_bytes(int T, int Hk, int Hv);
void delta_prefill(float *out, float *state, float *history, const float *qkv, const float *gate, const float *alpha,
                   const float *beta, const float *conv, const float *decay, const float *bias, const float *norm, int T,
                   int Hk, int Hv, int D, float eps, void *ws, size_t ws_bytes, cudaStream_t st);

// The thread-local message behind qv_error() (runtime.cu).
void clear_error();
void record_error(const char *message);

// Device status word (status.cu): 0 = ok, else the first error a kernel raised.
int read_and_clear_status();

}  // namespace qv
