/*
 * mc_oracle.h -- CPU restatement of modelc's speculative-decoding path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity oracle: only the
 * tests, the smoke check and bench.py's cpu_baseline / reference arm may load
 * it, and only as the checker.  The CUDA product path never links or calls it.
 *
 * The reference (yingkitw/modelc) is Rust; no Rust toolchain exists here, so
 * this is a C restatement of the reference functions, kept in the reference's
 * operation order (separate f32 multiply and add, sequential sums, division
 * where the reference divides, glibc expf/powf/sinf/cosf).  Every function
 * cites the reference file:line it follows.
 *
 * Two model modes:
 *   ORACLE_MODE_REFERENCE  -- exactly the reference's semantics:
 *       n_heads = hidden/64 (min 1), head_dim = hidden/n_heads, MHA only,
 *       RoPE base 10000, RMSNorm eps 1e-6  (transformer.rs:70-96, :775, :806,
 *       :925; arch.rs:128-137).
 *   ORACLE_MODE_GENERAL    -- the same algorithm with GQA, head_dim, RoPE
 *       base and eps as parameters (needed by the 8B/70B/TinyLlama shapes,
 *       which lie outside the reference's hard-coded semantics).
 */
#ifndef MC_ORACLE_H
#define MC_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORACLE_MODE_REFERENCE 0
#define ORACLE_MODE_GENERAL 1

/* ---------------- numeric helpers (transformer.rs:825-1000) ---------------- */
void oracle_linear(const float* w, int rows, int cols, const float* bias,
                   const float* x, float* out);
void oracle_linear_par(const float* w, int rows, int cols, const float* x,
                       float* out, int n_threads);
void oracle_rms_norm(const float* x, int n, const float* w, int wlen, float eps,
                     float* out);
void oracle_silu(const float* x, int n, float* out);
void oracle_add(const float* a, int na, const float* b, int nb, float* out);
void oracle_rope(const float* x, int n, int pos, int n_heads, float base,
                 float* out);
void oracle_rope_table(int max_pos, int head_dim, float base, float* cos_out,
                       float* sin_out);
void oracle_attention_kv(const float* q, int q_len, const float* k_all,
                         const float* v_all, int seq_len, int n_heads,
                         int n_kv_heads, float* out);
void oracle_softmax_inplace(float* xs, int n);

/* ---------------- sampling (generate.rs:948-1124) ---------------- */
int oracle_argmax(const float* xs, int n);
void oracle_softmax(const float* xs, int n, float* out);
void oracle_apply_top_p(float* probs, int n, float top_p);
void oracle_apply_min_p(float* probs, int n, float min_p);
float oracle_rand_f32(uint64_t seed);
uint32_t oracle_multinomial(const float* probs, int n, uint64_t step,
                            uint64_t seed);
void oracle_chacha_block(const uint32_t key[8], uint64_t counter,
                         uint64_t nonce, int rounds, uint32_t out[16]);
uint32_t oracle_sample(const float* logits, int n, float temperature,
                       float top_p, float min_p, uint64_t step, uint64_t seed);

/* ---------------- weight materialisation ---------------- */
void oracle_quantize_int8_tensor(const float* x, size_t n, int8_t* q,
                                 float* scale);
void oracle_quantize_int8_rows(const float* x, int rows, int cols, int8_t* q,
                               float* scales);
void oracle_dequant_int8_rows(const int8_t* q, const float* scales, int rows,
                              int cols, float* out);
void oracle_dequant_int8_tensor(const int8_t* q, float scale, size_t n,
                                float* out);
int oracle_quantize_q4_0(const float* x, size_t n, uint8_t* blocks);
int oracle_dequant_q4_0(const uint8_t* blocks, size_t n, float* out);
float oracle_f16_to_f32(uint16_t h);
uint16_t oracle_f32_to_f16(float f);

/* ---------------- model + KV cache ---------------- */
typedef struct {
  const float* attn_norm; /* [hidden] or NULL */
  const float* wq;        /* [n_heads*head_dim, hidden] */
  const float* wk;        /* [n_kv*head_dim, hidden] */
  const float* wv;        /* [n_kv*head_dim, hidden] */
  const float* wo;        /* [hidden, n_heads*head_dim] */
  const float* mlp_norm;  /* [hidden] or NULL */
  const float* wg;        /* [ffn, hidden] */
  const float* wu;        /* [ffn, hidden] */
  const float* wd;        /* [hidden, ffn] */
} oracle_layer;

typedef struct {
  int mode;
  int n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab;
  float rope_base, eps;
  const float* embed;      /* [vocab, hidden] */
  const float* final_norm; /* [hidden] or NULL */
  const float* lm_head;    /* [vocab, hidden] or NULL (tied to embed) */
  const oracle_layer* layers;
  int n_threads;           /* 1 = reference-faithful sequential linear */
} oracle_model;

/* KvLayer variants (transformer.rs:167-193).  The cache holds f32 values
 * as k_all()/v_all() return them: INT8 tokens and MIXED cold tokens hold
 * their dequantized int8 codes (q * scale). */
#define ORACLE_KV_FP32 0
#define ORACLE_KV_INT8 1
#define ORACLE_KV_MIXED 2

typedef struct {
  int n_layers, kv_dim, len, cap;
  float* k; /* [n_layers][cap][kv_dim] */
  float* v;
  int mode;   /* ORACLE_KV_* */
  int window; /* MIXED: f32 ("hot") tokens kept */
  int hot;    /* MIXED: tokens now in the hot window (the last `hot` positions) */
} oracle_kv;

int oracle_model_resolve(oracle_model* m);
oracle_kv* oracle_kv_new(int n_layers, int kv_dim, int cap);
void oracle_kv_free(oracle_kv* kv);
void oracle_kv_truncate(oracle_kv* kv, int len);
int oracle_kv_len(const oracle_kv* kv);
void oracle_kv_set_mode(oracle_kv* kv, int mode, int window);
void oracle_kv_qdq(float* x, int n);
void oracle_kv_shift(oracle_kv* kv, int n, int anchor);
int oracle_context_shift(uint32_t* tok, int* len, int* prompt_len, oracle_kv* kv, int max_ctx,
                         int anchor, int* removed_at);

void oracle_token_embedding(const oracle_model* m, uint32_t id, float* out);
int oracle_forward(const oracle_model* m, const float* input, oracle_kv* kv,
                   float* logits);
int oracle_forward_ids(const oracle_model* m, const uint32_t* ids, int n,
                       oracle_kv* kv, float* logits);

/* ---------------- drafters ---------------- */
#define ORACLE_DRAFT_NGRAM 0
#define ORACLE_DRAFT_LLAMA 1
#define ORACLE_DRAFT_MLP 2
#define ORACLE_DRAFT_NONE 3

typedef struct {
  int vocab, hidden, draft_hidden;
  const float *embed, *w1, *b1, *w2, *b2;
  float temperature, top_p;
} oracle_mlp_draft;

typedef struct oracle_llama_draft oracle_llama_draft;
oracle_llama_draft* oracle_llama_draft_new(const oracle_model* m, int cap);
void oracle_llama_draft_free(oracle_llama_draft* d);
int oracle_llama_draft_run(oracle_llama_draft* d, const uint32_t* ctx, int n,
                       int gamma, uint32_t* out);
void oracle_llama_draft_shift(oracle_llama_draft* d, int at, int n);
int oracle_mlp_draft_run(const oracle_mlp_draft* d, const uint32_t* ctx, int n,
                         int gamma, uint32_t* out);
int oracle_ngram_draft(const uint32_t* tokens, int n_tokens,
                       const uint32_t* ctx, int n_ctx, int ngram, int gamma,
                       uint32_t* out);

/* ---------------- generation (generate.rs:399-767) ---------------- */
typedef struct {
  int max_tokens;
  float temperature, top_p, min_p;
  int gamma;
  uint64_t seed;
  int tok_vocab;   /* tokenizer vocab for the OOV stop; 0 disables */
  int bonus;       /* 0: reference verify (k forwards, no bonus); 1: k+1 */
  volatile int* cancel;
  int max_context;   /* GenerationConfig::max_context (0 = None) */
  int anchor_tokens; /* GenerationConfig::anchor_tokens */
  int kv_mode;       /* ORACLE_KV_*: use_int8_kv / use_mixed_kv (window 64) */
} oracle_gen_cfg;

int oracle_generate_core(const oracle_model* m, const uint32_t* prompt,
                         int n_prompt, const oracle_gen_cfg* cfg,
                         uint32_t* out, int cap);
int oracle_speculative_generate(const oracle_model* m, int draft_kind,
                                void* drafter, const uint32_t* prompt,
                                int n_prompt, const oracle_gen_cfg* cfg,
                                uint32_t* out, int cap, int* accepted,
                                int* n_rounds, int rounds_cap);
int oracle_speculative_generate_kv(const oracle_model* m, int draft_kind,
                                   void* drafter, const uint32_t* prompt,
                                   int n_prompt, const oracle_gen_cfg* cfg,
                                   uint32_t* out, int cap, int* accepted,
                                   int* n_rounds, int rounds_cap, oracle_kv* kv_io,
                                   int matched_len);

/* ---------------- stochastic speculative sampling (not in the reference) */
void oracle_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);
float oracle_philox_uniform(uint64_t seed, uint32_t round, uint32_t slot);
float oracle_filtered_weights(const float* l, int n, float t, float top_p, float min_p,
                              float* w);
uint32_t oracle_sample_philox(const float* l, int n, float t, float top_p, float min_p,
                              uint64_t seed, uint32_t round, uint32_t slot);
int oracle_llama_draft_sample(oracle_llama_draft* d, const uint32_t* ctx, int n, int gamma,
                              float t, float top_p, float min_p, uint64_t seed, uint32_t round,
                              uint32_t* out, float* qlog);
int oracle_speculative_sample(const oracle_model* m, oracle_llama_draft* drafter,
                              const uint32_t* prompt, int n_prompt, const oracle_gen_cfg* cfg,
                              int accept_mode, uint32_t* out, int cap, int* accepted,
                              int* n_rounds, int rounds_cap);

#ifdef __cplusplus
}
#endif
#endif
