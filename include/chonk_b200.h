/*
 * chonk_b200 — C ABI of the B200 (sm_100a) decode engine.
 *
 * Drop-in for the device side of ChonkLM's llama-webgpu runtime
 * (bilalba/ChonkLM src/lib/llama-wgsl-runtime.ts).  A host binding (ctypes
 * here; Node-API / Bun FFI for the TypeScript host) re-exposes the module API
 * loadLlamaWgslModel / generateLlamaWgsl / disposeLlamaWgsl /
 * resetLlamaWgslConversation on top of these calls.
 *
 * Conventions: every call is synchronous with respect to the caller, returns
 * 0 on success and a negative CK_E* code on failure, with the message kept
 * per handle (ck_last_error) or per thread for calls without a handle
 * (ck_global_error).  A handle is not thread-safe; at most one call may be in
 * flight per handle, as the reference allows one runToken per engine
 * (llama-wgsl-runtime.ts:1222, :1238).  No torch or CUDA types cross this
 * boundary: pointers are host pointers unless a name says `dev`.
 */
#ifndef CHONK_B200_H
#define CHONK_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CK_OK 0
#define CK_EINVAL -1      /* bad argument / unsupported configuration          */
#define CK_ECUDA -2       /* CUDA runtime error                                 */
#define CK_ESTATE -3      /* call not valid in the engine's current state       */
#define CK_ECONTEXT -4    /* context exhausted (llama-wgsl-runtime.ts:1030-1033) */
#define CK_EDEVICE -5     /* device-side check failed (bad token id, timeout)   */
#define CK_ENOMEM -6      /* device allocation failed / KV pool exhausted        */
#define CK_EBUSY -7       /* batch: every sequence slot is in use               */

/* GGML tensor types accepted for weights (gguf.ts:5-14). */
#define CK_GGML_F32 0
#define CK_GGML_F16 1
#define CK_GGML_Q5_0 6
#define CK_GGML_Q5_1 7
#define CK_GGML_Q8_0 8
#define CK_GGML_Q4_K 12
#define CK_GGML_Q6_K 14

#define CK_ARCH_LLAMA 0   /* manifest architecture "llama" (covers qwen3)       */
#define CK_ARCH_GEMMA3 1  /* manifest architecture "gemma3"                     */

#define CK_KV_F16 0
#define CK_KV_F32 1

#define CK_MAX_LAYERS 128

/* Mirrors LlamaManifest.model (llama-wgsl-runtime.ts:36-72) for the fields
 * the GGUF path uses, plus the engine's context length (:227). */
typedef struct ck_model_cfg {
  int32_t hidden, intermediate, vocab, layers, heads, kv_heads, head_dim;
  int32_t context_length;          /* min(ModelDef.maxContext, manifest.maxContext) */
  float norm_eps, qk_norm_eps;
  float embedding_scale;           /* sqrt(hidden) for gemma3, else 1 (:405)  */
  int32_t arch;                    /* CK_ARCH_*                                */
  int32_t rope_interleaved;        /* ropeLayout == "interleaved" (:402)       */
  int32_t qk_norm;                 /* q/k norm tensors present (:399)          */
  int32_t kv_dtype;                /* CK_KV_F16 (default) or CK_KV_F32         */
  uint32_t layer_rope_theta[CK_MAX_LAYERS];  /* Math.round(theta) (:1477)      */
  uint32_t layer_window[CK_MAX_LAYERS];      /* 0 = full attention (:413-415)  */
} ck_model_cfg;

/* Sampling options of runToken (sampling.ts:1-7 + the penalty ids of
 * llama-wgsl-runtime.ts:1028) plus the Philox stream that replaces
 * Math.random (sampling.ts:70). */
typedef struct ck_sampling {
  double temperature;              /* default 0 (greedy); JS numbers are doubles */
  double top_p;                    /* default 1                                */
  int32_t top_k;                   /* default 0 (off)                          */
  double repetition_penalty;       /* default 1                                */
  const uint32_t* penalized_ids;   /* NULL: use the engine's token history     */
  int32_t n_penalized;
  uint64_t philox_seed;
  uint64_t philox_offset;          /* draw index of the next sampled token     */
} ck_sampling;

typedef struct ck_engine ck_engine;

/* ---- lifecycle: LlamaWgslEngine.create / dispose (:669-919, :1152-1215) ---- */
int ck_create(const ck_model_cfg* cfg, int device, ck_engine** out);
/* Upload one tensor by its alias-resolved GGUF name ("blk.3.attn_q.weight",
 * "token_embd.weight", "output.weight", "output_norm.weight", ...).
 * shape is the GGUF (ggml) order: shape[0] = row length.  Quantized weights
 * are re-laid into the device's streaming layout; norm weights (F32/F16) are
 * stored as fp32 (TensorLoader.floatBytes, :594-611). */
int ck_upload_tensor(ck_engine* h, const char* name, int ggml_type, const int64_t* shape, int ndim,
                     const void* bytes, size_t nbytes);
/* Checks every tensor the step needs is present, allocates KV + scratch. */
int ck_finalize(ck_engine* h);
int ck_destroy(ck_engine* h);

/* ---- per-token step: LlamaWgslEngine.runToken (:1025-1150) ---- */
/* Runs `token` at the current position; with need_logits computes logits and
 * writes the greedy argmax (or the sampled id when `s` asks for sampling) to
 * *out_id.  Advances the position by one. */
int ck_run_token(ck_engine* h, uint32_t token, int need_logits, const ck_sampling* s, uint32_t* out_id);
/* Prefill `n` prompt tokens without host round trips between tokens; the
 * last one computes logits when need_logits_last (runToken loop at
 * llama-wgsl-runtime.ts:281-288).  Long prompts go through the tensor-core
 * prefill (ck_set_prefill_gemm). */
int ck_prefill(ck_engine* h, const uint32_t* tokens, int n, int need_logits_last, const ck_sampling* s,
               uint32_t* out_id);
/* Decode loop of generateLlamaWgsl (:291-307) kept on the device: feeds
 * `first` (the id produced by the previous step), then each produced id, up
 * to max_new ids written to out_ids (first included, as `generated` holds
 * it), stopping after an id in eos_ids.  *n_out = number of ids written. */
int ck_decode(ck_engine* h, uint32_t first, int max_new, const ck_sampling* s, const uint32_t* eos_ids,
              int n_eos, uint32_t* out_ids, int* n_out);

int ck_get_logits(ck_engine* h, float* out, size_t n);           /* last logits, fp32[vocab]   */
int ck_get_candidates(ck_engine* h, float* val, uint32_t* idx, size_t n); /* ARGMAX_STAGE1 output */
int ck_reset(ck_engine* h);                                       /* reset() (:1011-1019)       */
int ck_position(ck_engine* h, int* pos);                          /* position getter (:1021)    */
/* Rewind to `pos` <= position, keeping the KV prefix [0, pos) (prefix reuse,
 * generateLlamaWgsl :268-280, without re-running the prefix). */
int ck_truncate(ck_engine* h, int pos);
const char* ck_last_error(ck_engine* h);
const char* ck_global_error(void);

/* ---- execution controls ---- */
/* Use the caller's CUDA stream (cudaStream_t passed as void*); NULL = the
 * engine's own stream.  Lets a caller time steps with its own events. */
int ck_set_stream(ck_engine* h, void* stream);
/* Candidate list of the sampler.  0 (default): the reference's, the
 * per-256-logit chunk maxima of ARGMAX_STAGE1_WGSL that
 * sampleFromCandidateBuffer (sampling.ts:23-76) reads.  1: exact over the
 * whole vocabulary, the K largest penalized logits (K = top-k when 1..1024,
 * else 1024; ties to the lower id), found by a block-level radix select on
 * every CTA's slice of the vocabulary and once more over their candidates;
 * temperature, top-k, top-p and the Philox draw then run as in the
 * reference.  Takes effect at the next step call; greedy steps are not
 * affected.  No counterpart in the reference (its candidates are the chunk
 * maxima). */
int ck_set_sampler(ck_engine* h, int exact);

/* Step implementation: 0 = one persistent cooperative kernel per token
 * (default), 1 = per-op kernels replayed from a CUDA graph. */
int ck_set_mode(ck_engine* h, int mode);
/* Tensor-core prefill.  No counterpart in the reference, which feeds a prompt
 * token by token (llama-wgsl-runtime.ts:281-288); ck_prefill keeps that
 * interface.  A ck_prefill of at least min_tokens + 1 ids (llama / qwen3
 * graphs) runs all but the last id through the layers together as tcgen05
 * GEMMs, `chunk` ids per pass (0: 1024, the largest), writing their K/V rows
 * into the cache; the last id takes the single-token step.  Logits then match
 * the token-by-token ones within the decode tolerance, not bit for bit.
 * min_tokens 0 disables it; the default is 64. */
int ck_set_prefill_gemm(ck_engine* h, int min_tokens, int chunk);
/* Enqueue n greedy decode steps on the engine stream without synchronising
 * (benchmark/profiling use).  The first step reads the token already stored
 * at the current position; each step's argmax feeds the next. */
int ck_enqueue_decode_steps(ck_engine* h, int n);
/* Same, each step sampling with `s` (null = greedy), the draws numbered from
 * s->philox_offset as ck_decode numbers them: the sampled configurations'
 * timed steps (benchmark/profiling use; no reference counterpart). */
int ck_enqueue_decode_steps_sampled(ck_engine* h, int n, const ck_sampling* s);
int ck_sync(ck_engine* h);
/* Host<->device bytes copied so far by the step calls (run_token, prefill,
 * decode, reset, truncate): the e2e transfer count. */
int ck_io_bytes(ck_engine* h, uint64_t* h2d_bytes, uint64_t* d2h_bytes);
/* Device timeline: with tracing on, the megakernel stamps %globaltimer (ns)
 * at the start and end of every phase on CTA 0 (slots [2i], [2i+1]) and the
 * per-phase kernels stamp start / after-prefetch / end per CTA (slots
 * 4096 + cta*8 + {0,1,2}).  ck_trace_read copies the first n slots. */
int ck_trace(ck_engine* h, int enable);
int ck_trace_read(ck_engine* h, uint64_t* out, size_t n);
/* Bytes of weights + KV the next decode step reads (roofline numerator). */
int ck_step_bytes(ck_engine* h, double* weight_bytes, double* kv_bytes);

/* ---- parity helpers (no model needed) ---- */
/* Dequantize n rows x k weights through the device layout: raw GGUF block
 * bytes -> device re-layout -> fp32, using the WGSL formulas' rounding. */
int ck_dequant(int ggml_type, const void* bytes, size_t nbytes, int k, int n, float* out, int device);
/* y = W x through the production matvec kernel (x host fp32[k], y fp32[n]). */
int ck_matvec(int ggml_type, const void* bytes, size_t nbytes, int k, int n, const float* x, float* y,
              int device);
/* Y[T x n] = X[T x k] W^T through the batched path (its prologue and the
 * tcgen05 tensor-core GEMM): x host fp32 [T][k], y host fp32 [T][n]. */
int ck_matmul(int ggml_type, const void* bytes, size_t nbytes, int k, int n, const float* x, int T, float* y,
              int device);
/* Time `reps` launches of the matvec kernel on an n x k weight resident on
 * the device; writes mean microseconds per launch (CUDA events). */
int ck_bench_matvec(int ggml_type, const void* bytes, size_t nbytes, int k, int n, int reps, double* us_per,
                    int device);

/* y = W x like ck_matvec, for callers that cannot allocate device memory
 * (their device memory is owned by another caching allocator, or a serving
 * loop cannot afford the device synchronisation of cudaMalloc/cudaFree).  No
 * counterpart in the reference: it has no native code.  w_dev holds the raw
 * GGUF block bytes of n rows x k weights, x_dev fp32[k], y_dev fp32[n], all in
 * caller-owned device memory; stream is a cudaStream_t (NULL = default
 * stream) and the call returns after the result is ready.  Nothing is
 * allocated: the device-layout copy of the weights goes to a static device
 * array of 16 MiB (plus 4.25 KiB of state), held by every GPU that loads the
 * library until exit; larger weights are rejected with CK_EINVAL.  The first
 * call on a device resolves that array's address (one-time set-up, done once
 * even when several host threads call at once) and should come before any
 * stream capture.  Every call waits for its work on `stream` to finish
 * before it returns.  All calls share the array: calls that overlap on the
 * GPU race. */
int ck_matvec_noalloc(int ggml_type, const void* w_dev, size_t nbytes, int k, int n, const float* x_dev,
                      float* y_dev, void* stream);

/* ---- batched decode (continuous batching) ----
 * No counterpart in the reference, whose engine decodes one sequence
 * (llama-wgsl-runtime.ts:619-1150): several sequences share one engine's
 * weights and advance together, one position per step each (a sequence
 * still in its prompt feeds its next prompt token, the others their last
 * generated id), so every sequence gets exactly the ids generateLlamaWgsl
 * (:242-314) would give it with greedy decoding.  Sequences may be added
 * between steps; a finished sequence frees its slot and KV blocks at once.
 * llama / qwen3 architectures; paged fp16 KV cache (16-position blocks).
 * Not thread-safe per batch; the engine must not run single-sequence steps
 * while a batch step is in flight. */
typedef struct ck_batch ck_batch;
/* max_seqs concurrent sequences; kv_blocks 16-position blocks of KV pool
 * (0 = enough for every slot at the full context length). */
int ck_batch_create(ck_engine* h, int max_seqs, int kv_blocks, ck_batch** out);
/* Queue a sequence: prompt of n >= 1 ids, up to max_new >= 1 generated ids
 * (capped at the context left, as generateLlamaWgsl does), stopping after
 * an id in eos_ids (which is kept).  CK_EBUSY when every slot is taken,
 * CK_ENOMEM when the KV pool cannot hold it. */
int ck_batch_add_seq(ck_batch* b, const uint32_t* prompt, int n, int max_new, const uint32_t* eos_ids, int n_eos,
                     int* seq_id);
/* One step of every queued sequence; *n_active = sequences still running. */
int ck_batch_step(ck_batch* b, int* n_active);
/* Ids generated so far (done = 0) or the final ids of a finished sequence
 * (done = 1; the result is released).  Copies min(n, cap) ids. */
int ck_batch_collect(ck_batch* b, int seq_id, uint32_t* out_ids, int cap, int* n_out, int* done);
int ck_batch_stats(ck_batch* b, uint64_t* steps, uint64_t* tokens_fed, uint64_t* tokens_generated);
const char* ck_batch_last_error(ck_batch* b);
int ck_batch_destroy(ck_batch* b);

/* sizeof(ck_model_cfg) and sizeof(ck_sampling) as compiled, so bindings can
 * check their struct mirrors; needs no GPU. */
void ck_abi_info(int* sizeof_cfg, int* sizeof_sampling);

#ifdef __cplusplus
}
#endif
#endif
