/*
 * modelc_cuda.h -- C ABI of the B200 (sm_100a) speculative-decoding step for
 * modelc (yingkitw/modelc).  Plain pointers and sizes only; no CUDA or torch
 * types cross this boundary.  Every entry point cites the reference interface
 * it replaces (paths inside the modelc repository).
 *
 * Ownership and threading (mirrors the reference's Runtime / KvCache split,
 * serve/infer.rs:129 and generate.rs:18-24):
 *   - mc_weights is immutable after mc_weights_load and may be shared by any
 *     number of sessions and host threads (the reference's RwLock<Runtime>).
 *   - mc_session owns one request's KV cache, draft state and stream; it is
 *     not thread-safe: one host thread per session (one KvCache per request).
 * Entry points that touch a device make that device (the handle's, or the
 * one mc_sample_rows' pointers live on) current for the calling thread and
 * leave it current; a host thread that drives several devices selects its
 * own device again afterwards.
 * All functions return MC_OK (0) or a negative mc_status; mc_last_error()
 * returns the calling thread's last error message.  There is no CPU
 * fallback: without a usable sm_100 device every entry point fails with
 * MC_E_CUDA.
 */
#ifndef MODELC_CUDA_H
#define MODELC_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define MC_API __attribute__((visibility("default")))
#else
#define MC_API
#endif

typedef int32_t mc_status;
#define MC_OK 0
#define MC_E_INVALID -1   /* bad argument / null pointer */
#define MC_E_SHAPE -2     /* tensor shape mismatch (reference: transformer.rs:831 panic) */
#define MC_E_DTYPE -3     /* unsupported tensor dtype for the B200 path */
#define MC_E_OOM -4       /* device allocation failed */
#define MC_E_CUDA -5      /* CUDA runtime error / no sm_100 device */
#define MC_E_NCCL -6      /* collective failure (tensor-parallel builds) */
#define MC_E_TIMEOUT -7   /* a bounded device wait expired */
#define MC_E_CANCELLED -8 /* the cancel flag was raised (generate.rs:639) */
#define MC_E_NO_HEAD -9   /* no lm_head and no tied embedding: the reference's None
                             (transformer.rs:94-95) */
#define MC_E_CAPACITY -10 /* context would exceed the session's KV capacity */

/* Tensor dtypes accepted by mc_weights_load (model.rs:6-42 DataType subset). */
#define MC_DTYPE_F32 0       /* f32; matrices must be exactly representable as
                                int8 rows with power-of-two scales */
#define MC_DTYPE_I8_TENSOR 1 /* int8 + one scale (compiler.rs:207-229 format;
                                dequant q as f32 * scale, model.rs:182-185) */
#define MC_DTYPE_I8_ROW 2    /* int8 + one f32 scale per output row */
#define MC_DTYPE_Q4_0 3      /* ggml q4_0 blocks (parsers/gguf/dequant.rs:23-46) */

#define MC_MEM_HOST 0
#define MC_MEM_DEVICE 1

/* Head-geometry modes.  REFERENCE reproduces the reference runtime exactly:
 * n_heads = hidden/64 (metadata is dropped, transformer.rs:1007-1027 +
 * arch.rs:128-137), MHA, RoPE base 10000 (transformer.rs:925), RMSNorm eps
 * 1e-6 (transformer.rs:91, :775, :806).  GENERAL takes the fields below. */
#define MC_MODE_REFERENCE 0
#define MC_MODE_GENERAL 1

typedef struct mc_model_cfg {
  int32_t mode;
  int32_t n_layers;
  int32_t hidden;
  int32_t n_heads;    /* GENERAL only */
  int32_t n_kv_heads; /* GENERAL only */
  int32_t head_dim;   /* GENERAL only */
  int32_t ffn;
  int32_t vocab;
  float rope_theta;   /* GENERAL only */
  float eps;          /* GENERAL only */
  int32_t tp_rank;    /* tensor parallelism (Megatron): this rank's shard of */
  int32_t tp_world;   /* tp_world (0 or 1 = no sharding).  Column-parallel
                         q/k/v (by heads) and gate/up (by FFN rows),
                         row-parallel o and down (one all-reduce each),
                         vocab-parallel LM head; embedding and norms
                         replicated.  Requires n_heads, n_kv_heads, ffn and
                         vocab divisible by tp_world. */
} mc_model_cfg;

/* One tensor, as the reference's TensorData {shape, dtype, data}
 * (model.rs:14-18) plus its name.  Names follow the reference
 * (model.layers.{i}.self_attn.q_proj.weight, model.embed_tokens.weight,
 * lm_head.weight, model.norm.weight, ...). */
typedef struct mc_tensor_desc {
  const char* name;
  int32_t dtype;
  int32_t location;     /* MC_MEM_HOST or MC_MEM_DEVICE (data and scales) */
  int32_t ndim;         /* 1 or 2 */
  int64_t shape[2];     /* [out, in] for matrices (transformer.rs:825) */
  const void* data;
  const float* scales;  /* I8_ROW: shape[0] floats; I8_TENSOR: 1 float */
} mc_tensor_desc;

typedef struct mc_weights mc_weights;
typedef struct mc_session mc_session;
typedef struct mc_linear mc_linear;
typedef struct mc_mlp_drafter mc_mlp_drafter;
typedef struct mc_ngram_drafter mc_ngram_drafter;
typedef struct mc_kv_snapshot mc_kv_snapshot;

/* Speculative session configuration (GenerationConfig, generate.rs:65-167,
 * restricted to the fields the speculative step reads). */
typedef struct mc_spec_cfg {
  int32_t gamma;        /* draft tokens per round (GenerationConfig::gamma) */
  int32_t max_context;  /* KV capacity in tokens (prompt + generated + gamma),
                           at most 4030 per request in this build (64 KV
                           pages of 64 positions, less one prefill chunk);
                           larger values return MC_E_CAPACITY */
  int32_t bonus;        /* 0: reference verify (gamma positions, no bonus
                           token, generate.rs:695-726); 1: gamma+1 positions
                           with the bonus token */
  float temperature;    /* 0 = greedy; > 0 = sampling at this temperature
                           (draft and target) */
  uint64_t seed;
  volatile int32_t* cancel;  /* optional; checked between rounds (generate.rs:639) */
  int32_t accept_mode;  /* temperature > 0 only.  0: accept draft x with
                           probability min(1, p(x)/q(x)), else emit a sample of
                           max(0, p - q) (distribution-preserving); 1: the
                           reference's rule, accept when the target's own
                           sample equals x (generate.rs:695-726).  Random
                           numbers: Philox4x32-10 keyed by seed, counter
                           (slot, round). */
  int32_t n_requests;   /* concurrent requests B (0 or 1: one).  B > 1: B
                           independent greedy requests, each with its own KV
                           capacity max_context, decoded in lock step: every
                           round runs the gamma draft steps over B tokens,
                           one verify forward over B x (gamma or gamma+1)
                           positions, and B acceptances.  B x (gamma +
                           bonus) <= 64. */
  float top_p;          /* temperature > 0: top-p filter on every draft and
                           target distribution when 0 < top_p < 1
                           (generate.rs:961-963), as mc_sample_rows states it */
  float min_p;          /* likewise min-p when 0 < min_p < 1 (generate.rs:964-966) */
  int32_t shift_context;  /* GenerationConfig::max_context (0 = None): after a
                             round or a fallback step whose context exceeds it,
                             the context shift of generate.rs:26-63 on the
                             device (tokens, target KV, draft KV); greedy
                             sessions only.  Must leave room for a round:
                             shift_context + gamma + 2 <= max_context. */
  int32_t anchor_tokens;  /* GenerationConfig::anchor_tokens: tokens kept at the
                             front by the anchored shift */
  int32_t kv_mode;        /* target KV variant (make_kv_cache, generate.rs:17-24):
                             MC_KV_FP32, MC_KV_INT8 (use_int8_kv) or MC_KV_MIXED
                             (use_mixed_kv, window 64).  Values are held as the
                             reference's k_all()/v_all() return them (int8 codes
                             times the token's scale); the storage stays f32.
                             INT8 and MIXED: one-rank sessions.  MIXED: greedy;
                             its forwards (prime and verify) append one token at
                             a time, as the cache ages token by token. */
} mc_spec_cfg;

#define MC_KV_FP32 0
#define MC_KV_INT8 1
#define MC_KV_MIXED 2

/* Load (quantize-free) weights to the device and repack them for the
 * tensor-core GEMV.  Replaces Runtime::from_raw (runtime/serve.rs:121-132),
 * which dequantizes every tensor to f32; here int8 rows stay int8 in HBM. */
MC_API mc_status mc_weights_load(const mc_tensor_desc* tensors, size_t n,
                          const mc_model_cfg* cfg, int32_t device,
                          mc_weights** out);
MC_API mc_status mc_weights_destroy(mc_weights* w);
/* Bytes of packed weights resident on the device. */
MC_API int64_t mc_weights_bytes(const mc_weights* w);

/* A session = one request: target KV (and draft KV when draft != NULL).
 * Replaces make_kv_cache (generate.rs:18-24) + the per-request state of
 * speculative_generate (generate.rs:598-637).  The drafter of its rounds is
 * the transformer draft; with draft == NULL it is the reference's default,
 * the trigram n-gram index of the context (speculative_generate with
 * draft_model None, generate.rs:615, :642-646, :771-841): the prompt's
 * windows, plus after every round or fallback step the window ending at the
 * last token (update_ngram_index), drafts of up to gamma most-frequent
 * continuations (count ties: the earliest window), and when no key matches,
 * one standard generation step (generate.rs:647-693, not counted as a round).
 * Drafters other than the transformer draft decode greedily (temperature 0). */
MC_API mc_status mc_session_create(const mc_weights* target, const mc_weights* draft,
                            const mc_spec_cfg* cfg, mc_session** out);
/* A session whose rounds draft with MlpDraftModel (draft.rs:91-147) on the
 * device, as modelc's server wires it (serve/mod.rs:151-166 ->
 * speculative_generate's draft_model, generate.rs:642-646): gamma greedy
 * steps from the context's last token, then the batched verify and
 * acceptance.  The drafter is borrowed: keep it alive while the session
 * exists.  Greedy only (temperature 0). */
MC_API mc_status mc_session_create_mlp(const mc_weights* target, const mc_mlp_drafter* draft,
                                const mc_spec_cfg* cfg, mc_session** out);
MC_API mc_status mc_session_destroy(mc_session* s);

/* Batched forward_llama_cached (transformer.rs:64-96): forwards n token ids
 * (token_embedding, generate.rs:843-863) at positions kv_len..kv_len+n-1,
 * appends their K/V and writes n x vocab logits to logits_out (host memory,
 * may be NULL).  Equivalent to n sequential single-token calls. */
MC_API mc_status mc_forward(mc_session* s, const uint32_t* ids, int32_t n,
                     float* logits_out);
/* The same forward through the draft model's weights and KV. */
MC_API mc_status mc_draft_forward(mc_session* s, const uint32_t* ids, int32_t n,
                           float* logits_out);
/* KvCache::len (transformer.rs:633-638) and rollback from the end. */
MC_API int32_t mc_kv_len(const mc_session* s);
MC_API mc_status mc_kv_truncate(mc_session* s, int32_t len);

/* DraftModel::draft (draft.rs:18-21) for the transformer draft: greedy
 * decode of gamma tokens after context (KV of the common prefix reused). */
MC_API mc_status mc_draft(mc_session* s, const uint32_t* context, int32_t n,
                   int32_t gamma, uint32_t* out, int32_t* n_out);

/* MlpDraftModel (draft.rs:28-147) on the device: MlpDraftModel::from_runtime's
 * tensors (draft.fc1.weight [dh][d], draft.fc1.bias [dh], draft.fc2.weight
 * [V][dh], draft.fc2.bias [V], and draft.embed.weight or the target's
 * model.embed_tokens.weight / transformer.wte.weight [V][d]), all f32.
 * mc_mlp_draft is DraftModel::draft at temperature 0: gamma <= 16 greedy
 * steps from the context's last token, logits bit-identical to the
 * reference's sequential f32 sums. */
MC_API mc_status mc_mlp_draft_create(const mc_tensor_desc* tensors, size_t n, int32_t device,
                              mc_mlp_drafter** out);
MC_API mc_status mc_mlp_draft(mc_mlp_drafter* d, const uint32_t* context, int32_t n,
                       int32_t gamma, uint32_t* out, int32_t* n_out);
MC_API mc_status mc_mlp_draft_destroy(mc_mlp_drafter* d);

/* The n-gram drafter of speculative_generate (build_ngram_index +
 * draft_tokens + most_frequent, generate.rs:771-841) on the device: the
 * index is the history's windows of `ngram` tokens; up to gamma <= 16 steps,
 * each the most frequent continuation of the current last `ngram` tokens,
 * stopping at the first key without one.  Count ties go to the continuation
 * seen first (the reference leaves them to HashMap iteration order).
 * max_tokens bounds the history length. */
MC_API mc_status mc_ngram_draft_create(int32_t ngram, int32_t max_tokens, int32_t device,
                                mc_ngram_drafter** out);
MC_API mc_status mc_ngram_draft(mc_ngram_drafter* d, const uint32_t* tokens, int32_t n_tokens,
                         int32_t gamma, uint32_t* out, int32_t* n_out);
MC_API mc_status mc_ngram_draft_destroy(mc_ngram_drafter* d);

/* speculative_generate (generate.rs:598-767) with the draft model given at
 * session creation: prime the prompt, then rounds of draft -> batched verify
 * -> acceptance, all on the device, until >= max_tokens tokens exist (the
 * reference may overshoot by up to gamma-1, generate.rs:638,751).
 * out receives up to cap generated ids; accepted (may be NULL) receives the
 * accepted-draft count of each round (up to accepted_cap). */
MC_API mc_status mc_speculative_generate(mc_session* s, const uint32_t* prompt,
                                  int32_t n_prompt, int32_t max_tokens,
                                  uint32_t* out, int32_t cap, int32_t* n_out,
                                  int32_t* accepted, int32_t accepted_cap,
                                  int32_t* n_rounds);

/* Batched speculative_generate: n_requests (= the session's B) prompts,
 * concatenated in `prompts` with lengths `lens`.  Request z's generated ids go
 * to out + z * out_stride (up to out_stride ids, count in n_out[z]), its
 * per-round accepted counts to accepted + z * accepted_stride (NULL: not
 * returned) and its round count to n_rounds[z] (may be NULL).  Every request
 * produces exactly the tokens it would produce alone. */
MC_API mc_status mc_speculative_generate_batch(mc_session* s, const uint32_t* prompts,
                                        const int32_t* lens, int32_t n_requests,
                                        int32_t max_tokens, uint32_t* out,
                                        int32_t out_stride, int32_t* n_out,
                                        int32_t* accepted, int32_t accepted_stride,
                                        int32_t* n_rounds);

/* Device-resident variants for measurement: prompt already primed with
 * mc_spec_prime; mc_spec_decode runs the round loop only (every request
 * until it holds >= max_tokens generated ids; n_generated = their sum). */
MC_API mc_status mc_spec_prime(mc_session* s, const uint32_t* prompt, int32_t n_prompt);
MC_API mc_status mc_spec_prime_batch(mc_session* s, const uint32_t* prompts,
                              const int32_t* lens, int32_t n_requests);
MC_API mc_status mc_spec_decode(mc_session* s, int32_t max_tokens, int32_t* n_generated);

/* Prefix cache (prefix_cache.rs:14-110, used by serve/infer.rs:122-175).
 * mc_kv_snapshot_take copies request z's context tokens and target K/V as
 * they stand (after mc_spec_prime or decoding: the reference inserts the
 * prompt plus generated ids with the KvCache speculative_generate returns)
 * into a device allocation of its own; mc_kv_snapshot_tokens returns its
 * token count and copies up to cap of them.  mc_spec_prime_cached is
 * mc_spec_prime for a prompt that starts with the snapshot's tokens
 * (speculative_generate with a CacheLookup, generate.rs:617-636): the K/V
 * of the matched tokens are restored and only the rest are forwarded; the
 * n-gram index still covers the whole prompt, the transformer draft primes
 * the whole prompt.  Same target model, device and kv_mode; one-request
 * sessions.  The longest-prefix LRU lookup itself is host logic
 * (modelc_b200.PrefixCache). */
MC_API mc_status mc_kv_snapshot_take(mc_session* s, int32_t request, mc_kv_snapshot** out);
MC_API int32_t mc_kv_snapshot_tokens(const mc_kv_snapshot* snap, uint32_t* out, int32_t cap);
MC_API mc_status mc_kv_snapshot_destroy(mc_kv_snapshot* snap);
MC_API mc_status mc_spec_prime_cached(mc_session* s, const mc_kv_snapshot* snap,
                                      const uint32_t* prompt, int32_t n_prompt);
/* mc_spec_decode (and mc_speculative_generate) look at the cancel flag of
 * mc_spec_cfg before every batch of at most 64 rounds (generate.rs:639 looks
 * before every round) and return MC_E_CANCELLED with the rounds run so far
 * kept: mc_spec_read returns them, and after the flag is lowered the session
 * continues or rewinds as usual. */
MC_API mc_status mc_spec_read(mc_session* s, uint32_t* out, int32_t cap, int32_t* n_out,
                       int32_t* accepted, int32_t accepted_cap, int32_t* n_rounds);
/* mc_spec_read for request z of a batched session. */
MC_API mc_status mc_spec_read_request(mc_session* s, int32_t z, uint32_t* out, int32_t cap,
                               int32_t* n_out, int32_t* accepted, int32_t accepted_cap,
                               int32_t* n_rounds);
/* Restart decoding from the primed prompt: the prompt's KV is kept, the
 * generated tokens and round log are dropped. */
MC_API mc_status mc_spec_rewind(mc_session* s);
/* Tensor parallelism.  mc_tp_unique_id creates the communicator id on one
 * rank (the host distributes its 128 bytes to all ranks); every rank then
 * calls mc_session_tp_init on a session whose target weights were loaded
 * with tp_world > 1 (the draft stays replicated: tp_world 0 or 1).  The
 * all-reduces run on the session stream, inside its CUDA graphs.  Greedy
 * decoding only; every rank computes the same tokens.  NCCL (libnccl.so.2)
 * is loaded when first needed. */
MC_API mc_status mc_tp_unique_id(char id_out[128]);
MC_API mc_status mc_session_tp_init(mc_session* s, const char id[128], int32_t rank,
                             int32_t world);
/* Fused tensor-parallel reduction over NVLink (instead of NCCL all-reduces):
 * every rank exports its exchange buffer (64-byte CUDA IPC handle), the host
 * gathers the handles of all ranks in rank order (world x 64 bytes) and each
 * rank opens its peers before its first decode (a handle exported by another
 * session of the same process is opened directly, so ranks may also be one
 * host thread per GPU).  The row-parallel GEMV then stores its partial rows
 * into every rank's buffer and a reduce kernel adds them in rank order; the
 * vocab-parallel LM head exchanges its per-token argmax keys the same way.
 * Every cross-rank wait is bounded (mc_session_set_wait_timeout); an expired
 * wait returns MC_E_TIMEOUT.  With open peers an int8 target needs no NCCL
 * (mc_session_tp_init is then optional); q4_0 forwards of more than 16
 * tokens still reduce through NCCL.  All ranks must reach the host barrier
 * before any destroys its session. */
MC_API mc_status mc_session_tp_ipc_handle(mc_session* s, char handle_out[64]);
MC_API mc_status mc_session_tp_open_peers(mc_session* s, const char* handles);
/* Limit, in milliseconds, of every bounded device wait of this session (a
 * tensor-parallel peer's flag in the fused reduction and the vocab-parallel
 * head; default 5000).  A wait that expires raises the session's error word:
 * the call returns MC_E_TIMEOUT, every later wait of the session gives up at
 * once, and the session stays failed (its ranks' epochs are out of step):
 * destroy it.  The CUDA context stays usable.  The reference has no device
 * waits; this stands in for a peer that failed in the middle of a request. */
MC_API mc_status mc_session_set_wait_timeout(mc_session* s, int32_t ms);
/* Reseed the stochastic rounds (GenerationConfig::seed per request,
 * generate.rs:146-167); applies from the next round. */
MC_API mc_status mc_spec_set_seed(mc_session* s, uint64_t seed);
/* Enqueue n verify forwards (gamma or gamma+1 positions at the current
 * target length, no acceptance, no state change) on the session stream and
 * return immediately: for timing the verify forward with stream events. */
MC_API mc_status mc_spec_verify_launch(mc_session* s, int32_t n);
/* The session's CUDA stream (a cudaStream_t) for stream-ordered timing. */
MC_API void* mc_session_stream(mc_session* s);
/* Kernel launches one speculative round enqueues (draft steps, verify,
 * acceptance): the kernel nodes of the round's CUDA graph, captured at the
 * first decode (0 before it). */
MC_API int32_t mc_session_round_launches(const mc_session* s);

/* Standalone quantized projection y = x . dequant(W)^T (linear_with,
 * transformer.rs:825-843) on device buffers: x is m x in (f32, row-major),
 * y is m x out.  `stream` is a cudaStream_t passed as void* (NULL = legacy
 * default stream). */
MC_API mc_status mc_linear_create(const mc_tensor_desc* w, int32_t device,
                           mc_linear** out);
MC_API mc_status mc_linear_destroy(mc_linear* l);
MC_API mc_status mc_linear_run(mc_linear* l, const float* x_dev, int32_t m,
                        float* y_dev, void* stream);
MC_API int64_t mc_linear_weight_bytes(const mc_linear* l);

/* Allocation-free variant of mc_linear_run.  It has no counterpart in the
 * reference, which has no device path at all.  Same arguments as
 * mc_linear_run, but the activation scratch (the packed digit operand and
 * the per-token exponents) lives in one fixed device array compiled into
 * this library, 768 KiB + 256 B per device, instead of in buffers owned by
 * the handle, and the call itself allocates no device or host memory.
 *
 * It exists for callers that may allocate at start-up (mc_linear_create
 * packs the weights then) but not when they run a projection. One example
 * is a serving process whose HBM is already divided between weights and KV
 * pages under a hard budget, where a new allocation can fail or fragment
 * the pool. Another is a latency-critical decode loop sharing the GPU with
 * other streams, where cudaMalloc/cudaFree may synchronise the whole device
 * and stall them.
 *
 * Route: the encoder computes each token's statistics itself and the GEMV
 * runs once per group of up to 16 tokens, streaming the weights once per
 * group; it never takes the tcgen05 GEMM that mc_linear_run uses for more
 * than 16 tokens (or 9-16 tokens on matrices of 8192+ rows).  Both routes sum
 * exactly in int32, so the results agree with mc_linear_run's; for m > 16
 * the static call is slower.
 *
 * Limit: in_features <= 16384; a larger matrix returns MC_E_CAPACITY and
 * launches nothing.  The first call on each device looks up the array's
 * device address (a host-side lookup; no clear, no launch), so make that
 * first call before any stream capture.  The address is kept for the life
 * of the process: cudaDeviceReset on that device is not supported while the
 * library is in use.  All calls on one device share the array: calls that
 * overlap in time (different streams or threads with no ordering between
 * them) race on it and corrupt each other's results; issue them on one
 * stream or synchronise between them. */
MC_API mc_status mc_linear_run_static(mc_linear* l, const float* x_dev, int32_t m,
                               float* y_dev, void* stream);

/* One token per row of logits (device memory, n_rows x vocab, f32), written
 * to tokens_dev (device, n_rows) on `stream` (a cudaStream_t as void*).
 * Replaces sample (generate.rs:948-969, the penalty- and constraint-free path
 * of sample_constrained, :982-1027):
 *   temperature <= 0: argmax (generate.rs:1088-1098): the first strict
 *     maximum; NaN and -inf never win; 0 when no entry does;
 *   temperature > 0: softmax(l / T), then top-p (generate.rs:1034-1063) when
 *     0 < top_p < 1, then min-p (generate.rs:1071-1086) when 0 < min_p < 1,
 *     then an inverse-CDF draw.  The filters are restated on the exact
 *     weights e_v = exp((l_v - max) / T): top-p keeps the shortest prefix of
 *     (e desc, index asc) whose integer mass sum floor(e_v 2^32) reaches
 *     ceil(top_p x total); min-p drops e_v < min_p.  The uniform of row r is
 *     Philox4x32-10 keyed by seed with counter (slot r, round), the stream
 *     of the stochastic sessions, in place of the reference's
 *     StdRng::seed_from_u64(seed + step).
 * vocab <= 262144. */
MC_API mc_status mc_sample_rows(const float* logits_dev, int32_t n_rows, int32_t vocab,
                                float temperature, float top_p, float min_p, uint64_t seed,
                                uint32_t round, uint32_t* tokens_dev, void* stream);

MC_API size_t mc_last_error(char* buf, size_t cap);
MC_API const char* mc_version(void);

#ifdef __cplusplus
}
#endif
#endif /* MODELC_CUDA_H */
