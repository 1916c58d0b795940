/*
 * b200_engine.h - native batch-1 greedy decode engine for the Qwen2.5
 * architecture on the b200 Linear kernels (C ABI).
 *
 * The reference runs this model in Qwen2Model (reference src/qwen2.cpp,
 * include/infer/qwen2.hpp:41-54); this engine is the GPU-resident
 * counterpart: same weights (qbin archives), same arithmetic at the BF16
 * tensor boundaries, but q/k/v and gate/up weights concatenated, RMSNorm /
 * SiLU*up / residual adds fused into the decode GEMVs, and each decode step
 * one CUDA graph with the token and position kept on the device.
 *
 * All pointers are device pointers the caller owns and keeps alive for the
 * engine's lifetime.  The engine allocates its activations and KV cache once
 * in b200_engine_create.  Returns B200_OK or a B200_ERR_* / cudaError_t.
 */
#ifndef B200_ENGINE_H_
#define B200_ENGINE_H_

#include "b200_linear.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct b200_engine* b200_engine_t;

typedef struct {
  int hidden;        /* 896 */
  int intermediate;  /* 4864 */
  int layers;        /* 24 */
  int heads;         /* 14 (head_dim = hidden / heads must be 64) */
  int kv_heads;      /* 2 */
  int vocab;         /* 151936 (multiple of 8) */
  int max_seq;       /* KV cache length (<= 8192) */
  float eps;         /* RMSNorm epsilon */
  float theta;       /* RoPE base */
  int w8;            /* 1: W8A16 Linear weights (group 64), 0: BF16 */
} b200_engine_config;

/* One layer.  qkv_* are the q, k, v projections concatenated by rows
 * ([q; k; v], (heads + 2 kv_heads) * head_dim rows), gate_up_* the gate and
 * up projections ([gate; up], 2 * intermediate rows).  *_s are the BF16
 * group-64 scales (W8A16 only, else NULL).  Norm gains are BF16. */
typedef struct {
  const void* qkv_w;
  const uint16_t* qkv_s;
  const uint16_t* qkv_b;
  const void* o_w;
  const uint16_t* o_s;
  const void* gate_up_w;
  const uint16_t* gate_up_s;
  const void* down_w;
  const uint16_t* down_s;
  const uint16_t* input_norm;
  const uint16_t* post_norm;
} b200_engine_layer;

/* embed: [vocab, hidden] BF16 (also the tied LM head). */
int b200_engine_create(b200_engine_t* engine, const b200_engine_config* config,
                       const b200_engine_layer* layers, const uint16_t* embed,
                       const uint16_t* final_norm, b200_stream_t stream);
int b200_engine_destroy(b200_engine_t engine);

/* Prefill the prompt (host token ids, n <= max_seq) from position 0; the
 * first generated token becomes output token 0.  Asynchronous. */
int b200_engine_prefill(b200_engine_t engine, const int* prompt, int n);

/* `steps` greedy decode steps, each appending one token to the output list
 * (prompt length + all decoded steps <= max_seq, else B200_ERR_TOO_LARGE).
 * Asynchronous. */
int b200_engine_decode(b200_engine_t engine, int steps);

/* Decode modes.  PERSISTENT (the default where the shapes allow it): all
 * steps of one b200_engine_decode call in one cooperative kernel, one CTA
 * per SM; each CTA streams its share of every weight matrix ahead into
 * shared memory, and activations pass between CTAs as tagged words that are
 * their own synchronisation.  GRAPH: one CUDA graph replay per step (146
 * kernel launches for the 24-layer model). */
#define B200_ENGINE_DECODE_PERSISTENT 0
#define B200_ENGINE_DECODE_GRAPH 1
/* Selects the decode mode (B200_ERR_TOO_LARGE: the persistent kernel does
 * not take this model's shapes / shared-memory needs). */
int b200_engine_set_decode_mode(b200_engine_t engine, int mode);
/* Profiling timeline of the persistent kernel: with phases > 0 the next
 * decode calls record, for their first `phases` phases (5 per layer: q|k|v,
 * attention, o_proj, gate|up, down_proj; then LM head, argmax), each CTA's
 * input-staged, phase-done, first-weight-block-landed and input-arrived
 * times (global timer, ns); 0 turns it off.  Allocates grid x phases x 32
 * bytes. */
int b200_engine_set_trace(b200_engine_t engine, int phases);
/* Copies the timeline ([cta][phase][staged, done, block, arrived]) to host memory when
 * out != NULL (synchronises); returns the CTA count (0: tracing off). */
int b200_engine_read_trace(b200_engine_t engine, unsigned long long* out);
/* Test hook of the failure path (persistent mode): in the next decode call,
 * CTA 0 stops before layer phase `phase` (5 per layer) of the first step and
 * never writes its outputs, so the other CTAs' bounded waits for them expire
 * (2 s): the kernel records B200_DEVICE_TIMEOUT_GRID, every CTA leaves its
 * loops and drains its copies, and the context stays usable.  The decode
 * call's tokens are then undefined; prefill again before decoding.  No GPU
 * fault is involved. */
int b200_engine_test_stall(b200_engine_t engine, int phase);
/* The current decode mode. */
int b200_engine_decode_mode(b200_engine_t engine);
/* Device-side error word of the persistent kernel (B200_DEVICE_*; a bounded
 * wait that expired).  Synchronises the engine's stream; clear != 0 resets
 * it. */
int b200_engine_device_status(b200_engine_t engine, int clear);

/* Replaces the token the next decode step consumes (after a prefill or a
 * decode call): teacher forcing, e.g. to follow another engine's tokens and
 * compare logits step by step.  The output list keeps the engine's own
 * argmax. */
int b200_engine_force_token(b200_engine_t engine, int token);
/* Copies the first `count` output tokens to host memory (synchronises). */
int b200_engine_tokens(b200_engine_t engine, int* out, int count);

/* Copies the BF16 logits of the last step to host memory (synchronises). */
int b200_engine_logits(b200_engine_t engine, uint16_t* out);

/* Causal GQA prefill attention of the engine on the tensor cores (head_dim
 * 64): q rows [tokens][q_stride] BF16 with head h at column h*64 (RoPE
 * applied), K / V caches [kv_heads][max_seq][64] BF16 holding positions
 * [0, pos0 + tokens), out rows [tokens][out_stride] (head h at h*64); query
 * t at position pos0 + t attends positions [0, pos0 + t].  FP32 scores and
 * softmax, P rounded to BF16 for P.V, output BF16.  The reference computes
 * the same attention with one CUDA-core block per (head, token)
 * (src/cuda/kernels.cu:221-283, attention_prefill_bf16_kernel). */
int b200_attention_prefill_bf16(const uint16_t* q, int q_stride, const uint16_t* kcache,
                                const uint16_t* vcache, uint16_t* out, int out_stride,
                                int tokens, int pos0, int heads, int kv_heads, int max_seq,
                                b200_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* B200_ENGINE_H_ */
