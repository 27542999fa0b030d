/*
 * mc_oracle.c -- CPU restatement of modelc's speculative-decoding path.
 *
 * TEST INFRASTRUCTURE ONLY (the parity oracle).  See mc_oracle.h.
 * Compiled with -O2 -fno-fast-math -ffp-contract=off so
 * every f32 multiply and add is rounded separately, in the reference's order.
 * All reference citations are paths inside the yingkitw/modelc repository.
 */
#include "mc_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>

/* ======================= numeric helpers ======================= */

/* transformer.rs:825-843 linear_with: y[r] = bias[r] + sum_c W[r,c]*x[c],
 * c ascending, multiply then add (Rust does not contract to FMA). */
void oracle_linear(const float* w, int rows, int cols, const float* bias,
                   const float* x, float* out) {
  for (int r = 0; r < rows; ++r) {
    float acc = bias ? bias[r] : 0.0f;
    const float* row = w + (size_t)r * cols;
    for (int c = 0; c < cols; ++c) acc += row[c] * x[c];
    out[r] = acc;
  }
}

/* Bit-identical parallel variant of linear_with: output rows are split over
 * pthreads and eight rows are interleaved per thread; every row keeps its own
 * sequential c-ascending f32 sum, so each output equals oracle_linear's. */
typedef struct {
  const float* w;
  const float* x;
  float* out;
  int cols, b0, b1, rows;
} lin_job;

static void* lin_worker(void* arg) {
  lin_job* j = (lin_job*)arg;
  int cols = j->cols;
  const float* x = j->x;
  for (int b = j->b0; b < j->b1; ++b) {
    int r0 = b * 8;
    int nr = j->rows - r0 < 8 ? j->rows - r0 : 8;
    if (nr == 8) {
      const float* p0 = j->w + (size_t)r0 * cols;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f, a4 = 0.f, a5 = 0.f,
            a6 = 0.f, a7 = 0.f;
      for (int c = 0; c < cols; ++c) {
        float xc = x[c];
        a0 += p0[c] * xc;
        a1 += p0[(size_t)cols + c] * xc;
        a2 += p0[(size_t)2 * cols + c] * xc;
        a3 += p0[(size_t)3 * cols + c] * xc;
        a4 += p0[(size_t)4 * cols + c] * xc;
        a5 += p0[(size_t)5 * cols + c] * xc;
        a6 += p0[(size_t)6 * cols + c] * xc;
        a7 += p0[(size_t)7 * cols + c] * xc;
      }
      float* o = j->out + r0;
      o[0] = a0; o[1] = a1; o[2] = a2; o[3] = a3;
      o[4] = a4; o[5] = a5; o[6] = a6; o[7] = a7;
    } else {
      for (int r = r0; r < r0 + nr; ++r) {
        float acc = 0.0f;
        const float* row = j->w + (size_t)r * cols;
        for (int c = 0; c < cols; ++c) acc += row[c] * x[c];
        j->out[r] = acc;
      }
    }
  }
  return NULL;
}

void oracle_linear_par(const float* w, int rows, int cols, const float* x,
                       float* out, int n_threads) {
  int nblk = (rows + 7) / 8;
  if (n_threads < 1) n_threads = 1;
  if (n_threads > 256) n_threads = 256;
  if (n_threads > nblk) n_threads = nblk > 0 ? nblk : 1;
  pthread_t th[256];
  lin_job jobs[256];
  for (int t = 0; t < n_threads; ++t) {
    jobs[t].w = w;
    jobs[t].x = x;
    jobs[t].out = out;
    jobs[t].cols = cols;
    jobs[t].rows = rows;
    jobs[t].b0 = (int)((long long)nblk * t / n_threads);
    jobs[t].b1 = (int)((long long)nblk * (t + 1) / n_threads);
  }
  for (int t = 1; t < n_threads; ++t) pthread_create(&th[t], NULL, lin_worker, &jobs[t]);
  lin_worker(&jobs[0]);
  for (int t = 1; t < n_threads; ++t) pthread_join(th[t], NULL);
}

/* transformer.rs:888-896 rms_norm: ms = sum(v*v)/n; rms = sqrt(ms+eps);
 * out = v / rms * w  (w defaults to 1.0 past its length). */
void oracle_rms_norm(const float* x, int n, const float* w, int wlen, float eps,
                     float* out) {
  float nf = (float)(n > 1 ? n : 1);
  float ss = 0.0f;
  for (int i = 0; i < n; ++i) ss += x[i] * x[i];
  float ms = ss / nf;
  float rms = sqrtf(ms + eps);
  for (int i = 0; i < n; ++i) {
    float wi = (w && i < wlen) ? w[i] : 1.0f;
    out[i] = x[i] / rms * wi;
  }
}

/* transformer.rs:907-909 silu: v / (1 + e^-v). */
void oracle_silu(const float* x, int n, float* out) {
  for (int i = 0; i < n; ++i) out[i] = x[i] / (1.0f + expf(-x[i]));
}

/* transformer.rs:911-916 add: elementwise, missing entries read as 0. */
void oracle_add(const float* a, int na, const float* b, int nb, float* out) {
  int n = na > nb ? na : nb;
  for (int i = 0; i < n; ++i) {
    float av = i < na ? a[i] : 0.0f;
    float bv = i < nb ? b[i] : 0.0f;
    out[i] = av + bv;
  }
}

/* transformer.rs:921-938 rope: rotate-half pairs (i, i+half) of each head,
 * theta = pos * base^(-i/half) in f32, sin/cos from libm. */
void oracle_rope(const float* x, int n, int pos, int n_heads, float base,
                 float* out) {
  int nh = n_heads > 1 ? n_heads : 1;
  int head_dim = n / nh;
  if (head_dim < 1) head_dim = 1;
  int half = head_dim / 2;
  if (out != x) memcpy(out, x, sizeof(float) * (size_t)n);
  for (int h = 0; h < n_heads; ++h) {
    int off = h * head_dim;
    for (int i = 0; i < half; ++i) {
      float expo = -(float)i / (float)half;
      float theta = (float)pos * powf(base, expo);
      float s = sinf(theta), c = cosf(theta);
      float x0 = x[off + i];
      float x1 = x[off + i + half];
      out[off + i] = x0 * c - x1 * s;
      out[off + i + half] = x0 * s + x1 * c;
    }
  }
}

/* The per-(pos, i) cos/sin factors oracle_rope uses, laid out [pos][half]. */
void oracle_rope_table(int max_pos, int head_dim, float base, float* cos_out,
                       float* sin_out) {
  int half = head_dim / 2;
  for (int p = 0; p < max_pos; ++p)
    for (int i = 0; i < half; ++i) {
      float expo = -(float)i / (float)half;
      float theta = (float)p * powf(base, expo);
      cos_out[(size_t)p * half + i] = cosf(theta);
      sin_out[(size_t)p * half + i] = sinf(theta);
    }
}

/* transformer.rs:985-1000 softmax_inplace: max fold from -inf, exp(x-max),
 * sequential sum, divide when the sum is positive. */
void oracle_softmax_inplace(float* xs, int n) {
  if (n <= 0) return;
  float mx = -INFINITY;
  for (int i = 0; i < n; ++i) mx = fmaxf(mx, xs[i]);
  float sum = 0.0f;
  for (int i = 0; i < n; ++i) {
    xs[i] = expf(xs[i] - mx);
    sum += xs[i];
  }
  if (sum > 0.0f)
    for (int i = 0; i < n; ++i) xs[i] /= sum;
}

/* transformer.rs:944-982 attention_kv.  k_all/v_all hold seq_len positions of
 * n_kv_heads*head_dim floats.  With n_kv_heads == n_heads this is exactly the
 * reference (MHA); with fewer KV heads query head h reads KV head
 * h / (n_heads/n_kv_heads) (grouped-query generalisation). */
void oracle_attention_kv(const float* q, int q_len, const float* k_all,
                         const float* v_all, int seq_len, int n_heads,
                         int n_kv_heads, float* out) {
  int nh = n_heads > 1 ? n_heads : 1;
  int head_dim = q_len / nh;
  if (head_dim < 1) head_dim = 1;
  int group = n_heads / (n_kv_heads > 0 ? n_kv_heads : 1);
  if (group < 1) group = 1;
  int kv_stride = n_kv_heads * head_dim;
  float* scores = (float*)malloc(sizeof(float) * (size_t)(seq_len > 0 ? seq_len : 1));
  float scale = sqrtf((float)head_dim);
  for (int h = 0; h < n_heads; ++h) {
    const float* qh = q + (size_t)h * head_dim;
    int kvh = h / group;
    for (int t = 0; t < seq_len; ++t) {
      const float* kh = k_all + (size_t)t * kv_stride + (size_t)kvh * head_dim;
      float dot = 0.0f;
      for (int i = 0; i < head_dim; ++i) dot += qh[i] * kh[i];
      scores[t] = dot / scale;
    }
    oracle_softmax_inplace(scores, seq_len);
    float* oh = out + (size_t)h * head_dim;
    for (int i = 0; i < head_dim; ++i) oh[i] = 0.0f;
    for (int t = 0; t < seq_len; ++t) {
      const float* vh = v_all + (size_t)t * kv_stride + (size_t)kvh * head_dim;
      float wgt = scores[t];
      for (int i = 0; i < head_dim; ++i) oh[i] += wgt * vh[i];
    }
  }
  free(scores);
}

/* ======================= sampling ======================= */

/* generate.rs:1088-1098 argmax: first strict maximum, NaN never wins. */
int oracle_argmax(const float* xs, int n) {
  int best = 0;
  float best_val = -INFINITY;
  for (int i = 0; i < n; ++i)
    if (xs[i] > best_val) {
      best = i;
      best_val = xs[i];
    }
  return best;
}

/* generate.rs:1100-1105 softmax (no zero-sum guard). */
void oracle_softmax(const float* xs, int n, float* out) {
  float mx = -INFINITY;
  for (int i = 0; i < n; ++i) mx = fmaxf(mx, xs[i]);
  float sum = 0.0f;
  for (int i = 0; i < n; ++i) {
    out[i] = expf(xs[i] - mx);
    sum += out[i];
  }
  for (int i = 0; i < n; ++i) out[i] = out[i] / sum;
}

typedef struct {
  float p;
  int i;
} prob_idx;

static int cmp_prob_desc(const void* a, const void* b) {
  const prob_idx* x = (const prob_idx*)a;
  const prob_idx* y = (const prob_idx*)b;
  if (x->p > y->p) return -1;
  if (x->p < y->p) return 1;
  return x->i - y->i; /* stable: equal probabilities keep index order */
}

/* generate.rs:1034-1063 apply_top_p. */
void oracle_apply_top_p(float* probs, int n, float top_p) {
  prob_idx* idx = (prob_idx*)malloc(sizeof(prob_idx) * (size_t)(n > 0 ? n : 1));
  for (int i = 0; i < n; ++i) {
    idx[i].p = probs[i];
    idx[i].i = i;
  }
  qsort(idx, (size_t)n, sizeof(prob_idx), cmp_prob_desc);
  float cum = 0.0f;
  int keep = 0;
  for (int j = 0; j < n; ++j) {
    cum += idx[j].p;
    keep += 1;
    if (cum >= top_p) break;
  }
  char* kept = (char*)calloc((size_t)(n > 0 ? n : 1), 1);
  for (int j = 0; j < keep; ++j) kept[idx[j].i] = 1;
  for (int i = 0; i < n; ++i)
    if (!kept[i]) probs[i] = 0.0f;
  float sum = 0.0f;
  for (int i = 0; i < n; ++i) sum += probs[i];
  if (sum > 0.0f)
    for (int i = 0; i < n; ++i) probs[i] /= sum;
  free(kept);
  free(idx);
}

/* generate.rs:1071-1086 apply_min_p. */
void oracle_apply_min_p(float* probs, int n, float min_p) {
  float mx = 0.0f;
  for (int i = 0; i < n; ++i) mx = fmaxf(mx, probs[i]);
  float threshold = mx * min_p;
  for (int i = 0; i < n; ++i)
    if (probs[i] < threshold) probs[i] = 0.0f;
  float sum = 0.0f;
  for (int i = 0; i < n; ++i) sum += probs[i];
  if (sum > 0.0f)
    for (int i = 0; i < n; ++i) probs[i] /= sum;
}

/* ChaCha block function (D. J. Bernstein, "ChaCha, a variant of Salsa20",
 * 2008): 64-bit block counter in words 12-13, 64-bit nonce in words 14-15,
 * `rounds` rounds (rand_chacha's ChaCha12Rng uses 12). */
#define ROTL32(v, c) (((v) << (c)) | ((v) >> (32 - (c))))
#define QR(a, b, c, d)              \
  a += b; d ^= a; d = ROTL32(d, 16); \
  c += d; b ^= c; b = ROTL32(b, 12); \
  a += b; d ^= a; d = ROTL32(d, 8);  \
  c += d; b ^= c; b = ROTL32(b, 7);

void oracle_chacha_block(const uint32_t key[8], uint64_t counter,
                         uint64_t nonce, int rounds, uint32_t out[16]) {
  uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,
                    key[0], key[1], key[2], key[3], key[4], key[5], key[6],
                    key[7], (uint32_t)counter, (uint32_t)(counter >> 32),
                    (uint32_t)nonce, (uint32_t)(nonce >> 32)};
  uint32_t x[16];
  memcpy(x, s, sizeof(x));
  for (int r = 0; r < rounds; r += 2) {
    QR(x[0], x[4], x[8], x[12]);
    QR(x[1], x[5], x[9], x[13]);
    QR(x[2], x[6], x[10], x[14]);
    QR(x[3], x[7], x[11], x[15]);
    QR(x[0], x[5], x[10], x[15]);
    QR(x[1], x[6], x[11], x[12]);
    QR(x[2], x[7], x[8], x[13]);
    QR(x[3], x[4], x[9], x[14]);
  }
  for (int i = 0; i < 16; ++i) out[i] = x[i] + s[i];
}

/* rand_core 0.6.4 SeedableRng::seed_from_u64: a PCG32 stream (M. O'Neill,
 * PCG, 2014: LCG multiplier 6364136223846793005, increment
 * 11634580027462260723, XSH-RR output) fills the 32-byte seed little-endian. */
static void seed_from_u64(uint64_t state, uint32_t key[8]) {
  const uint64_t MUL = 6364136223846793005ull;
  const uint64_t INC = 11634580027462260723ull;
  for (int i = 0; i < 8; ++i) {
    state = state * MUL + INC;
    uint32_t xorshifted = (uint32_t)(((state >> 18) ^ state) >> 27);
    uint32_t rot = (uint32_t)(state >> 59);
    key[i] = (xorshifted >> rot) | (xorshifted << ((32 - rot) & 31));
  }
}

/* rand 0.8.6: StdRng (= rand_chacha 0.3.1 ChaCha12Rng, key = seed, counter 0,
 * stream 0) seeded by seed_from_u64, then Standard's f32: the top 24 bits of
 * next_u32() times 2^-24.  Used by generate.rs:1107-1124 multinomial. */
float oracle_rand_f32(uint64_t seed) {
  uint32_t key[8], blk[16];
  seed_from_u64(seed, key);
  oracle_chacha_block(key, 0, 0, 12, blk);
  return (float)(blk[0] >> 8) * (1.0f / 16777216.0f);
}

/* generate.rs:1107-1124 multinomial with a seed (seed + step). */
uint32_t oracle_multinomial(const float* probs, int n, uint64_t step,
                            uint64_t seed) {
  float r = oracle_rand_f32(seed + step);
  float cum = 0.0f;
  for (int i = 0; i < n; ++i) {
    cum += probs[i];
    if (r < cum) return (uint32_t)i;
  }
  return n > 0 ? (uint32_t)(n - 1) : 0u;
}

/* generate.rs:948-969 sample (the penalty/constraint-free fast path of
 * sample_constrained, generate.rs:982-1027). */
uint32_t oracle_sample(const float* logits, int n, float temperature,
                       float top_p, float min_p, uint64_t step, uint64_t seed) {
  if (!logits || n <= 0) return 0;
  if (temperature <= 0.0f) return (uint32_t)oracle_argmax(logits, n);
  float* scaled = (float*)malloc(sizeof(float) * (size_t)n);
  float* probs = (float*)malloc(sizeof(float) * (size_t)n);
  for (int i = 0; i < n; ++i) scaled[i] = logits[i] / temperature;
  oracle_softmax(scaled, n, probs);
  if (top_p > 0.0f && top_p < 1.0f) oracle_apply_top_p(probs, n, top_p);
  if (min_p > 0.0f && min_p < 1.0f) oracle_apply_min_p(probs, n, min_p);
  uint32_t t = oracle_multinomial(probs, n, step, seed);
  free(scaled);
  free(probs);
  return t;
}

/* ======================= weight materialisation ======================= */

/* compiler.rs:207-229 int8 per-tensor quantiser: scale = max|x|/127,
 * q = round(clamp(x/scale, -127, 127)).  A zero tensor is left unquantised;
 * *scale = 0 reports that case. */
void oracle_quantize_int8_tensor(const float* x, size_t n, int8_t* q,
                                 float* scale) {
  float max_abs = 0.0f;
  for (size_t i = 0; i < n; ++i) max_abs = fmaxf(max_abs, fabsf(x[i]));
  if (!(max_abs > 0.0f)) {
    *scale = 0.0f;
    memset(q, 0, n);
    return;
  }
  float s = max_abs / 127.0f;
  for (size_t i = 0; i < n; ++i) {
    float v = x[i] / s;
    v = v < -127.0f ? -127.0f : (v > 127.0f ? 127.0f : v);
    q[i] = (int8_t)roundf(v);
  }
  *scale = s;
}

/* The same rule applied to each output row of an [out, in] matrix (the
 * per-row int8 format the B200 kernels stream).  An all-zero row gets scale
 * 1.0 and zero codes, as transformer.rs:195-197 does for KV rows. */
void oracle_quantize_int8_rows(const float* x, int rows, int cols, int8_t* q,
                               float* scales) {
  for (int r = 0; r < rows; ++r) {
    float s;
    oracle_quantize_int8_tensor(x + (size_t)r * cols, (size_t)cols,
                                q + (size_t)r * cols, &s);
    scales[r] = s > 0.0f ? s : 1.0f;
  }
}

/* model.rs:182-185 int8 dequantisation: (q as f32) * scale, per row. */
void oracle_dequant_int8_rows(const int8_t* q, const float* scales, int rows,
                              int cols, float* out) {
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < cols; ++c)
      out[(size_t)r * cols + c] = (float)q[(size_t)r * cols + c] * scales[r];
}

void oracle_dequant_int8_tensor(const int8_t* q, float scale, size_t n,
                                float* out) {
  for (size_t i = 0; i < n; ++i) out[i] = (float)q[i] * scale;
}

float oracle_f16_to_f32(uint16_t h) {
  _Float16 f;
  memcpy(&f, &h, 2);
  return (float)f;
}

uint16_t oracle_f32_to_f16(float f) {
  _Float16 h = (_Float16)f;
  uint16_t b;
  memcpy(&b, &h, 2);
  return b;
}

/* q4_0 block quantiser, restating the published ggml reference quantiser
 * (quantize_row_q4_0_reference, ggml MIT): per 32-element block the value of
 * largest magnitude m gives d = m / -8, codes = min(15, (int)(x/d + 8.5)),
 * element j in the low nibble of byte j, element j+16 in the high nibble.
 * Block = fp16 d (little-endian) + 16 code bytes = 18 bytes. */
int oracle_quantize_q4_0(const float* x, size_t n, uint8_t* blocks) {
  if (n % 32) return -1;
  for (size_t b = 0; b < n / 32; ++b) {
    const float* xb = x + b * 32;
    float amax = 0.0f, mx = 0.0f;
    for (int j = 0; j < 32; ++j)
      if (amax < fabsf(xb[j])) {
        amax = fabsf(xb[j]);
        mx = xb[j];
      }
    float d = mx / -8.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint16_t dh = oracle_f32_to_f16(d);
    uint8_t* out = blocks + b * 18;
    out[0] = (uint8_t)(dh & 0xff);
    out[1] = (uint8_t)(dh >> 8);
    for (int j = 0; j < 16; ++j) {
      float x0 = xb[j] * id, x1 = xb[16 + j] * id;
      int q0 = (int)(int8_t)(x0 + 8.5f), q1 = (int)(int8_t)(x1 + 8.5f);
      if (q0 > 15) q0 = 15;
      if (q1 > 15) q1 = 15;
      out[2 + j] = (uint8_t)(q0 | (q1 << 4));
    }
  }
  return 0;
}

/* parsers/gguf/dequant.rs:23-46 dequantize_q4_0: y[j] = (lo-8)*d,
 * y[j+16] = (hi-8)*d with d the block's fp16 scale widened to f32. */
int oracle_dequant_q4_0(const uint8_t* blocks, size_t n, float* out) {
  if (n % 32) return -1;
  for (size_t b = 0; b < n / 32; ++b) {
    const uint8_t* blk = blocks + b * 18;
    float d = oracle_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
    for (int j = 0; j < 16; ++j) {
      int x0 = (blk[2 + j] & 0x0F) - 8;
      int x1 = (blk[2 + j] >> 4) - 8;
      out[b * 32 + j] = (float)x0 * d;
      out[b * 32 + j + 16] = (float)x1 * d;
    }
  }
  return 0;
}

/* ======================= model + KV cache ======================= */

/* Resolve the head geometry.  Reference mode follows arch.rs:128-137 (the
 * runtime view drops metadata, transformer.rs:1007-1027, so heads = hidden/64)
 * and the hard-coded constants at transformer.rs:91, :775, :806 and :925. */
int oracle_model_resolve(oracle_model* m) {
  if (m->mode == ORACLE_MODE_REFERENCE) {
    int nh = m->hidden == 0 ? 1 : m->hidden / 64;
    if (nh < 1) nh = 1;
    m->n_heads = nh;
    m->head_dim = m->hidden / nh;
    if (m->head_dim < 1) m->head_dim = 1;
    if (m->n_kv_heads != 0 && m->n_kv_heads != nh) return -1; /* MHA only */
    m->n_kv_heads = nh;
    m->rope_base = 10000.0f;
    m->eps = 1e-6f;
  }
  if (m->n_heads <= 0 || m->n_kv_heads <= 0 || m->head_dim <= 0) return -1;
  if (m->n_heads % m->n_kv_heads) return -1;
  return 0;
}

oracle_kv* oracle_kv_new(int n_layers, int kv_dim, int cap) {
  oracle_kv* kv = (oracle_kv*)calloc(1, sizeof(oracle_kv));
  kv->n_layers = n_layers;
  kv->kv_dim = kv_dim;
  kv->cap = cap;
  kv->len = 0;
  size_t n = (size_t)n_layers * (size_t)cap * (size_t)kv_dim;
  kv->k = (float*)calloc(n > 0 ? n : 1, sizeof(float));
  kv->v = (float*)calloc(n > 0 ? n : 1, sizeof(float));
  return kv;
}

void oracle_kv_free(oracle_kv* kv) {
  if (!kv) return;
  free(kv->k);
  free(kv->v);
  free(kv);
}

/* Dropping positions from the end (speculative rollback).  The reference has
 * only front eviction (transformer.rs:424-583); its sequential verify never
 * forwards a rejected draft, and truncation reproduces exactly that state. */
void oracle_kv_truncate(oracle_kv* kv, int len) {
  if (len < kv->len) {
    if (len < 0) len = 0;
    if (kv->mode == ORACLE_KV_MIXED) {
      kv->hot -= kv->len - len;
      if (kv->hot < 0) kv->hot = 0;
    }
    kv->len = len;
  }
}

/* make_kv_cache (generate.rs:17-24): the KvLayer variant of every layer;
 * MIXED keeps `window` tokens in f32 (the reference passes 64). */
void oracle_kv_set_mode(oracle_kv* kv, int mode, int window) {
  kv->mode = mode;
  kv->window = window;
  kv->hot = 0;
}

/* transformer.rs:196-206 quantize_scale + quantize, then the dequantization
 * k_all()/v_all() apply (q as f32 * scale, :287-297): x becomes the values
 * an int8 layer returns for it.  scale = max|x| / 127 (1 when the max is 0);
 * q = round(x / scale) (halves away from zero) clamped to +-127, and a NaN
 * quotient casts to 0 (Rust's saturating `as i8`).  f32::max ignores NaN, as
 * fmaxf does. */
void oracle_kv_qdq(float* x, int n) {
  float mx = 0.0f;
  for (int i = 0; i < n; ++i) mx = fmaxf(mx, fabsf(x[i]));
  const float scale = mx > 0.0f ? mx / 127.0f : 1.0f;
  for (int i = 0; i < n; ++i) {
    const float r = roundf(x[i] / scale);
    const float q = isnan(r) ? 0.0f : (r < -127.0f ? -127.0f : (r > 127.0f ? 127.0f : r));
    x[i] = q * scale;
  }
}

/* One position's K and V in every layer through oracle_kv_qdq. */
static void kv_qdq_pos(oracle_kv* kv, int pos) {
  for (int l = 0; l < kv->n_layers; ++l) {
    const size_t off = ((size_t)l * kv->cap + (size_t)pos) * kv->kv_dim;
    oracle_kv_qdq(kv->k + off, kv->kv_dim);
    oracle_kv_qdq(kv->v + off, kv->kv_dim);
  }
}

/* Positions [from + n, len) move to [from, len - n) in every layer. */
static void kv_remove(oracle_kv* kv, int from, int n) {
  const size_t row = (size_t)kv->kv_dim;
  const int tail = kv->len - from - n;
  for (int l = 0; l < kv->n_layers; ++l) {
    float* k = kv->k + (size_t)l * kv->cap * row;
    float* v = kv->v + (size_t)l * kv->cap * row;
    if (tail > 0) {
      memmove(k + (size_t)from * row, k + (size_t)(from + n) * row, sizeof(float) * (size_t)tail * row);
      memmove(v + (size_t)from * row, v + (size_t)(from + n) * row, sizeof(float) * (size_t)tail * row);
    }
  }
  kv->len -= n;
}

/* KvCache::shift_anchored -> KvLayer::shift_anchored (transformer.rs:495-583),
 * which falls back to KvLayer::shift (:427-493) when anchor is 0, n is 0,
 * n >= len or len - n <= anchor.  shift drops the oldest min(n, len) tokens
 * (a MIXED layer from its cold tokens first).  The anchored form keeps the
 * first `anchor` tokens, drops the next n and re-appends the kept ones to a
 * cleared layer: an INT8 layer re-quantizes every kept token from its
 * dequantized values, a MIXED layer re-quantizes all but the last `window`
 * (they reach the cold part again), an FP32 layer is unchanged. */
void oracle_kv_shift(oracle_kv* kv, int n, int anchor) {
  const int len = kv->len;
  if (anchor == 0 || n == 0 || n >= len || len - n <= anchor) {
    const int remove = n < len ? n : len;
    if (kv->mode == ORACLE_KV_MIXED) {
      const int cold = len - kv->hot;
      if (remove > cold) kv->hot -= remove - cold;
    }
    kv_remove(kv, 0, remove);
    return;
  }
  const int keep = len - n;
  kv_remove(kv, anchor, n);
  if (kv->mode == ORACLE_KV_INT8) {
    for (int p = 0; p < keep; ++p) kv_qdq_pos(kv, p);
  } else if (kv->mode == ORACLE_KV_MIXED) {
    for (int p = 0; p + kv->window < keep; ++p) kv_qdq_pos(kv, p);
    kv->hot = keep < kv->window ? keep : kv->window;
  }
}

/* generate.rs:26-63 context_shift: with overflow = len - max_ctx + max_ctx/4,
 * either the anchored eviction (anchor > 0 and len > anchor + overflow: the
 * tokens [anchor, anchor + overflow) leave the list and the cache) or the
 * oldest `overflow` tokens leave.  prompt_len shrinks by the prompt tokens
 * removed.  *removed_at: where the removed range started.  Returns overflow. */
int oracle_context_shift(uint32_t* tok, int* len, int* prompt_len, oracle_kv* kv, int max_ctx,
                         int anchor, int* removed_at) {
  const int L = *len;
  const int overflow = L - max_ctx + max_ctx / 4;
  if (anchor > 0 && overflow > 0 && L > anchor + overflow) {
    if (kv) oracle_kv_shift(kv, overflow, anchor);
    const int suffix_start = anchor + overflow, suffix_len = L - suffix_start;
    memmove(tok + anchor, tok + suffix_start, sizeof(uint32_t) * (size_t)suffix_len);
    *len = anchor + suffix_len;
    if (*prompt_len > anchor) {
      const int non_anchor = *prompt_len - anchor;
      const int removed = overflow < non_anchor ? overflow : non_anchor;
      *prompt_len = anchor + non_anchor - removed;
    }
    if (removed_at) *removed_at = anchor;
  } else {
    if (kv) oracle_kv_shift(kv, overflow, 0);
    const int new_len = L - overflow;
    memmove(tok, tok + overflow, sizeof(uint32_t) * (size_t)new_len);
    *len = new_len;
    *prompt_len = *prompt_len > overflow ? *prompt_len - overflow : 0;
    if (removed_at) *removed_at = 0;
  }
  return overflow;
}

int oracle_kv_len(const oracle_kv* kv) { return kv ? kv->len : 0; }

/* generate.rs:843-863 token_embedding: the id's row, zeros when out of range. */
void oracle_token_embedding(const oracle_model* m, uint32_t id, float* out) {
  if (m->embed && (size_t)id < (size_t)m->vocab) {
    memcpy(out, m->embed + (size_t)id * m->hidden, sizeof(float) * (size_t)m->hidden);
  } else {
    memset(out, 0, sizeof(float) * (size_t)m->hidden);
  }
}

static void lin(const oracle_model* m, const float* w, int rows, int cols,
                const float* x, float* out) {
  if (m->n_threads > 1)
    oracle_linear_par(w, rows, cols, x, out, m->n_threads);
  else
    oracle_linear(w, rows, cols, NULL, x, out);
}

/* transformer.rs:64-96 forward_llama_cached with llama_step (:739-760),
 * llama_attention (:762-798) and llama_mlp (:800-817).  Returns 1 when logits
 * were produced, 0 when the model has no output head (the reference's None). */
int oracle_forward(const oracle_model* m, const float* input, oracle_kv* kv,
                   float* logits) {
  int d = m->hidden, hd = m->head_dim;
  int qd = m->n_heads * hd, kvd = m->n_kv_heads * hd, f = m->ffn;
  float* h = (float*)malloc(sizeof(float) * (size_t)d);
  float* normed = (float*)malloc(sizeof(float) * (size_t)d);
  float* tmp = (float*)malloc(sizeof(float) * (size_t)d);
  float* q = (float*)malloc(sizeof(float) * (size_t)qd);
  float* k = (float*)malloc(sizeof(float) * (size_t)kvd);
  float* v = (float*)malloc(sizeof(float) * (size_t)kvd);
  float* attn = (float*)malloc(sizeof(float) * (size_t)qd);
  float* g = (float*)malloc(sizeof(float) * (size_t)(f > 0 ? f : 1));
  float* u = (float*)malloc(sizeof(float) * (size_t)(f > 0 ? f : 1));
  memcpy(h, input, sizeof(float) * (size_t)d);
  int pos = kv ? kv->len : 0;
  /* KvLayer::append (transformer.rs:348-420): an INT8 layer quantizes the
   * new token; a MIXED layer whose hot part would exceed its window moves
   * the oldest hot token to the cold part (quantized) */
  const int stored = kv && pos < kv->cap;
  const int cold = (stored && kv->mode == ORACLE_KV_MIXED && kv->hot + 1 > kv->window)
                       ? pos - kv->window : -1;

  for (int l = 0; l < m->n_layers; ++l) {
    const oracle_layer* L = &m->layers[l];
    if (L->wq && L->wk && L->wv && L->wo) {
      if (L->attn_norm)
        oracle_rms_norm(h, d, L->attn_norm, d, m->eps, normed);
      else
        memcpy(normed, h, sizeof(float) * (size_t)d);
      lin(m, L->wq, qd, d, normed, q);
      lin(m, L->wk, kvd, d, normed, k);
      lin(m, L->wv, kvd, d, normed, v);
      oracle_rope(q, qd, pos, m->n_heads, m->rope_base, q);
      oracle_rope(k, kvd, pos, m->n_kv_heads, m->rope_base, k);
      const float *k_all = k, *v_all = v;
      int seq = 1;
      if (kv && pos < kv->cap) {
        float* kl = kv->k + ((size_t)l * kv->cap) * kvd;
        float* vl = kv->v + ((size_t)l * kv->cap) * kvd;
        memcpy(kl + (size_t)pos * kvd, k, sizeof(float) * (size_t)kvd);
        memcpy(vl + (size_t)pos * kvd, v, sizeof(float) * (size_t)kvd);
        if (kv->mode == ORACLE_KV_INT8) {
          oracle_kv_qdq(kl + (size_t)pos * kvd, kvd);
          oracle_kv_qdq(vl + (size_t)pos * kvd, kvd);
        } else if (cold >= 0) {
          oracle_kv_qdq(kl + (size_t)cold * kvd, kvd);
          oracle_kv_qdq(vl + (size_t)cold * kvd, kvd);
        }
        k_all = kl;
        v_all = vl;
        seq = pos + 1;
      }
      oracle_attention_kv(q, qd, k_all, v_all, seq, m->n_heads, m->n_kv_heads,
                          attn);
      lin(m, L->wo, d, qd, attn, tmp);
      oracle_add(h, d, tmp, d, h);
    }
    if (L->wg && L->wu && L->wd) {
      if (L->mlp_norm)
        oracle_rms_norm(h, d, L->mlp_norm, d, m->eps, normed);
      else
        memcpy(normed, h, sizeof(float) * (size_t)d);
      lin(m, L->wg, f, d, normed, g);
      lin(m, L->wu, f, d, normed, u);
      oracle_silu(g, f, g);
      for (int i = 0; i < f; ++i) g[i] = g[i] * u[i];
      lin(m, L->wd, d, f, g, tmp);
      oracle_add(h, d, tmp, d, h);
    }
  }
  if (stored) {
    kv->len = pos + 1;
    if (kv->mode == ORACLE_KV_MIXED && kv->hot < kv->window) kv->hot++;
  }

  if (m->final_norm) oracle_rms_norm(h, d, m->final_norm, d, m->eps, h);
  int have = 0;
  const float* head = m->lm_head ? m->lm_head : m->embed;
  if (head && logits) {
    lin(m, head, m->vocab, d, h, logits);
    have = 1;
  } else if (head) {
    have = 1;
  }
  free(h); free(normed); free(tmp); free(q); free(k); free(v); free(attn);
  free(g); free(u);
  return have;
}

/* Batched form of forward_llama_cached: n single-token forwards in order, one
 * logits row per position (the per-position math is unchanged). */
int oracle_forward_ids(const oracle_model* m, const uint32_t* ids, int n,
                       oracle_kv* kv, float* logits) {
  float* e = (float*)malloc(sizeof(float) * (size_t)m->hidden);
  int have = 1;
  for (int i = 0; i < n; ++i) {
    oracle_token_embedding(m, ids[i], e);
    have = oracle_forward(m, e, kv,
                          logits ? logits + (size_t)i * m->vocab : NULL);
  }
  free(e);
  return have;
}

/* ======================= drafters ======================= */

struct oracle_llama_draft {
  const oracle_model* m;
  oracle_kv* kv;
  uint32_t* cached; /* token at each KV position */
  float* logits;
  float* emb;
};

/* A transformer draft behind the DraftModel trait (draft.rs:18-21).  The
 * reference ships no transformer drafter; this one is defined as: greedily
 * decode `gamma` tokens after `ctx` with the draft model.  The KV of the
 * longest common prefix with the previous call is reused, which gives the same
 * result as a fresh forward over ctx because each position's math only reads
 * earlier positions. */
oracle_llama_draft* oracle_llama_draft_new(const oracle_model* m, int cap) {
  oracle_llama_draft* d = (oracle_llama_draft*)calloc(1, sizeof(*d));
  d->m = m;
  d->kv = oracle_kv_new(m->n_layers, m->n_kv_heads * m->head_dim, cap);
  d->cached = (uint32_t*)calloc((size_t)cap, sizeof(uint32_t));
  d->logits = (float*)malloc(sizeof(float) * (size_t)m->vocab);
  d->emb = (float*)malloc(sizeof(float) * (size_t)m->hidden);
  return d;
}

void oracle_llama_draft_free(oracle_llama_draft* d) {
  if (!d) return;
  oracle_kv_free(d->kv);
  free(d->cached);
  free(d->logits);
  free(d->emb);
  free(d);
}

static void draft_step(oracle_llama_draft* d, uint32_t tok) {
  int pos = d->kv->len;
  oracle_token_embedding(d->m, tok, d->emb);
  oracle_forward(d->m, d->emb, d->kv, d->logits);
  if (pos < d->kv->cap) d->cached[pos] = tok;
}

int oracle_llama_draft_run(oracle_llama_draft* d, const uint32_t* ctx, int n,
                       int gamma, uint32_t* out) {
  if (n <= 0 || gamma <= 0) return 0;
  if (n + gamma > d->kv->cap) return 0;
  int p = 0;
  while (p < d->kv->len && p < n && d->cached[p] == ctx[p]) ++p;
  if (p > n - 1) p = n - 1;
  oracle_kv_truncate(d->kv, p);
  for (int i = p; i < n; ++i) draft_step(d, ctx[i]);
  for (int j = 0; j < gamma; ++j) {
    out[j] = (uint32_t)oracle_argmax(d->logits, d->m->vocab);
    if (j + 1 < gamma) draft_step(d, out[j]);
  }
  return gamma;
}

/* The transformer draft's side of a context shift (the reference has no
 * transformer drafter; this is the definition the device follows): the
 * positions [at, at + n) leave its cache and its token list, so both keep
 * matching the shifted context. */
void oracle_llama_draft_shift(oracle_llama_draft* d, int at, int n) {
  const int len = d->kv->len;
  if (len <= at || n <= 0) return;
  const int rm = len - at < n ? len - at : n;
  kv_remove(d->kv, at, rm);
  memmove(d->cached + at, d->cached + at + rm, sizeof(uint32_t) * (size_t)(len - at - rm));
}

/* draft.rs:91-147 MlpDraftModel::{forward, draft}: embed -> FC1+ReLU -> FC2
 * -> argmax (temperature <= 0).  The reference samples with an unseeded
 * thread_rng when temperature > 0; the restatement draws from seed 0. */
int oracle_mlp_draft_run(const oracle_mlp_draft* d, const uint32_t* ctx, int n,
                         int gamma, uint32_t* out) {
  uint32_t cur = n > 0 ? ctx[n - 1] : 0u;
  float* hid = (float*)malloc(sizeof(float) * (size_t)(d->draft_hidden > 0 ? d->draft_hidden : 1));
  float* logits = (float*)malloc(sizeof(float) * (size_t)(d->vocab > 0 ? d->vocab : 1));
  for (int s = 0; s < gamma; ++s) {
    size_t idx = (size_t)cur * d->hidden;
    if (idx + d->hidden <= (size_t)d->vocab * d->hidden) {
      const float* e = d->embed + idx;
      for (int i = 0; i < d->draft_hidden; ++i) {
        float sum = d->b1[i];
        const float* row = d->w1 + (size_t)i * d->hidden;
        for (int j = 0; j < d->hidden; ++j) sum += row[j] * e[j];
        hid[i] = fmaxf(sum, 0.0f);
      }
      for (int i = 0; i < d->vocab; ++i) {
        float sum = d->b2[i];
        const float* row = d->w2 + (size_t)i * d->draft_hidden;
        for (int j = 0; j < d->draft_hidden; ++j) sum += row[j] * hid[j];
        logits[i] = sum;
      }
    } else {
      memset(logits, 0, sizeof(float) * (size_t)d->vocab);
    }
    uint32_t next = d->temperature <= 0.0f
                        ? (uint32_t)oracle_argmax(logits, d->vocab)
                        : oracle_sample(logits, d->vocab, d->temperature,
                                        d->top_p, 0.0f, 0, 0);
    out[s] = next;
    cur = next;
  }
  free(hid);
  free(logits);
  return gamma;
}

/* generate.rs:771-841 n-gram drafter.  `tokens` holds the (key, next) pairs
 * the index was built from, as a flat token sequence per window; here the
 * index is rebuilt from the window list passed in (see ngram_* below). */
typedef struct {
  uint32_t* keys; /* n per entry */
  uint32_t* next;
  int len, cap, n;
} ngram_index;

static void ngram_push(ngram_index* ix, const uint32_t* key, uint32_t next) {
  if (ix->len == ix->cap) {
    ix->cap = ix->cap ? ix->cap * 2 : 64;
    ix->keys = (uint32_t*)realloc(ix->keys, sizeof(uint32_t) * (size_t)ix->cap * ix->n);
    ix->next = (uint32_t*)realloc(ix->next, sizeof(uint32_t) * (size_t)ix->cap);
  }
  memcpy(ix->keys + (size_t)ix->len * ix->n, key, sizeof(uint32_t) * (size_t)ix->n);
  ix->next[ix->len++] = next;
}

/* generate.rs:771-784 build_ngram_index. */
static void ngram_build(ngram_index* ix, const uint32_t* t, int len) {
  if (len < ix->n + 1) return;
  for (int s = 0; s + ix->n < len; ++s) ngram_push(ix, t + s, t[s + ix->n]);
}

/* generate.rs:787-801 update_ngram_index: adds only the window ending at the
 * last token. */
static void ngram_update(ngram_index* ix, const uint32_t* t, int len) {
  if (len < ix->n + 1) return;
  int s = len - (ix->n + 1);
  ngram_push(ix, t + s, t[s + ix->n]);
}

/* generate.rs:804-841 draft_tokens + most_frequent.  The reference breaks
 * count ties by HashMap iteration order (unspecified); the restatement takes
 * the candidate seen first. */
static int ngram_draft(const ngram_index* ix, const uint32_t* ctx, int n_ctx,
                       int gamma, uint32_t* out) {
  int n = ix->n, cnt = 0;
  uint32_t* c = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(n_ctx + gamma + 1));
  memcpy(c, ctx, sizeof(uint32_t) * (size_t)n_ctx);
  int clen = n_ctx;
  uint32_t* cands = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(ix->len + 1));
  for (int g = 0; g < gamma; ++g) {
    if (clen < n) break; /* a short key never equals an n-token key */
    const uint32_t* key = c + clen - n;
    int nc = 0;
    for (int e = 0; e < ix->len; ++e)
      if (!memcmp(ix->keys + (size_t)e * n, key, sizeof(uint32_t) * (size_t)n))
        cands[nc++] = ix->next[e];
    if (nc == 0) break;
    uint32_t best = cands[0];
    int best_count = 0;
    for (int i = 0; i < nc; ++i) {
      int seen_before = 0;
      for (int j = 0; j < i; ++j)
        if (cands[j] == cands[i]) { seen_before = 1; break; }
      if (seen_before) continue;
      int count = 0;
      for (int j = i; j < nc; ++j) count += cands[j] == cands[i];
      if (count > best_count) {
        best_count = count;
        best = cands[i];
      }
    }
    out[cnt++] = best;
    c[clen++] = best;
  }
  free(cands);
  free(c);
  return cnt;
}

int oracle_ngram_draft(const uint32_t* tokens, int n_tokens,
                       const uint32_t* ctx, int n_ctx, int ngram, int gamma,
                       uint32_t* out) {
  ngram_index ix = {0};
  ix.n = ngram;
  ngram_build(&ix, tokens, n_tokens);
  int r = ngram_draft(&ix, ctx, n_ctx, gamma, out);
  free(ix.keys);
  free(ix.next);
  return r;
}

/* ======================= generation ======================= */

/* generate.rs:19: KvCache::new_mixed(n_layers, hidden, 64) */
static const int kMixedWindow = 64;

static int is_cancelled(const oracle_gen_cfg* cfg) {
  return cfg->cancel && *cfg->cancel;
}

/* generate.rs:399-525 generate_core (penalties, constraints, stop strings and
 * context shifting are off at the default config and are not restated). */
int oracle_generate_core(const oracle_model* m, const uint32_t* prompt,
                         int n_prompt, const oracle_gen_cfg* cfg,
                         uint32_t* out, int cap) {
  if (n_prompt <= 0) return 0;
  oracle_kv* kv = oracle_kv_new(m->n_layers, m->n_kv_heads * m->head_dim,
                                n_prompt + cfg->max_tokens + 1);
  float* logits = (float*)malloc(sizeof(float) * (size_t)m->vocab);
  float* e = (float*)malloc(sizeof(float) * (size_t)m->hidden);
  int have = 0;
  for (int i = 0; i < n_prompt; ++i) {
    oracle_token_embedding(m, prompt[i], e);
    have = oracle_forward(m, e, kv, logits);
  }
  int generated = 0;
  if (have) {
    for (;;) {
      if (generated >= cfg->max_tokens || is_cancelled(cfg)) break;
      uint32_t next = oracle_sample(logits, m->vocab, cfg->temperature,
                                    cfg->top_p, cfg->min_p,
                                    (uint64_t)generated, cfg->seed);
      if (generated < cap) out[generated] = next;
      generated++;
      if (cfg->tok_vocab > 0 && (int)next >= cfg->tok_vocab) break;
      oracle_token_embedding(m, next, e);
      if (!oracle_forward(m, e, kv, logits)) break;
    }
  }
  oracle_kv_free(kv);
  free(logits);
  free(e);
  return generated < cap ? generated : cap;
}

/* generate.rs:598-767 speculative_generate, restated in order: prime every
 * prompt token (logits discarded), then per round draft `gamma` tokens and
 * verify them one forward at a time starting from the last context token
 * (which re-forwards the last prompt token once), accepting while the
 * target's sample equals the draft and pushing the target's token at the
 * first mismatch.  No bonus token unless cfg->bonus (then a fully accepted
 * round forwards the last draft and pushes the target's next token, the
 * k+1-position verify).  Returns the number of generated tokens; accepted[]
 * receives each round's accepted-draft count. */
int oracle_speculative_generate(const oracle_model* m, int draft_kind,
                                void* drafter, const uint32_t* prompt,
                                int n_prompt, const oracle_gen_cfg* cfg,
                                uint32_t* out, int cap, int* accepted,
                                int* n_rounds, int rounds_cap) {
  return oracle_speculative_generate_kv(m, draft_kind, drafter, prompt, n_prompt, cfg, out, cap,
                                        accepted, n_rounds, rounds_cap, NULL, 0);
}

/* speculative_generate with a CacheLookup (generate.rs:617-636): kv_io
 * (when not NULL) holds the K/V of the first matched_len prompt tokens and
 * receives the cache the run ends with (the KvCache speculative_generate
 * returns); only prompt tokens [matched_len, n_prompt) are primed. */
int oracle_speculative_generate_kv(const oracle_model* m, int draft_kind,
                                   void* drafter, const uint32_t* prompt,
                                   int n_prompt, const oracle_gen_cfg* cfg,
                                   uint32_t* out, int cap, int* accepted,
                                   int* n_rounds, int rounds_cap, oracle_kv* kv_io,
                                   int matched_len) {
  if (n_rounds) *n_rounds = 0;
  if (n_prompt <= 0) return 0;
  int gamma = cfg->gamma;
  int tcap = (n_prompt > cfg->max_context ? n_prompt : cfg->max_context) + cfg->max_tokens +
             gamma + 2;
  uint32_t* tok = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)tcap);
  memcpy(tok, prompt, sizeof(uint32_t) * (size_t)n_prompt);
  int len = n_prompt, prompt_len = n_prompt;
  oracle_kv* kv = kv_io;
  if (!kv) {
    kv = oracle_kv_new(m->n_layers, m->n_kv_heads * m->head_dim, tcap + 1);
    oracle_kv_set_mode(kv, cfg->kv_mode, kMixedWindow);
    matched_len = 0;
  }
  /* generate.rs:671-681, :738-748: the context shift after a step or a round */
  #define SHIFT_CONTEXT()                                                                  \
    if (cfg->max_context > 0 && len > cfg->max_context) {                                 \
      int at_ = 0;                                                                         \
      const int ov_ = oracle_context_shift(tok, &len, &prompt_len, kv, cfg->max_context,   \
                                           cfg->anchor_tokens, &at_);                      \
      if (draft_kind == ORACLE_DRAFT_LLAMA)                                                \
        oracle_llama_draft_shift((oracle_llama_draft*)drafter, at_, ov_);                  \
    }
  float* logits = (float*)malloc(sizeof(float) * (size_t)m->vocab);
  float* e = (float*)malloc(sizeof(float) * (size_t)m->hidden);
  uint32_t* draft = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(gamma + 1));
  ngram_index ix = {0};
  ix.n = 3;
  ngram_build(&ix, tok, len);

  for (int i = matched_len; i < n_prompt; ++i) {
    oracle_token_embedding(m, prompt[i], e);
    oracle_forward(m, e, kv, logits);
  }
  int rounds = 0;
  while (len - prompt_len < cfg->max_tokens) {
    if (is_cancelled(cfg)) break;
    int nd = 0;
    if (draft_kind == ORACLE_DRAFT_LLAMA)
      nd = oracle_llama_draft_run((oracle_llama_draft*)drafter, tok, len, gamma, draft);
    else if (draft_kind == ORACLE_DRAFT_MLP)
      nd = oracle_mlp_draft_run((const oracle_mlp_draft*)drafter, tok, len, gamma, draft);
    else if (draft_kind == ORACLE_DRAFT_NGRAM)
      nd = ngram_draft(&ix, tok, len, gamma, draft);
    if (nd == 0) {
      uint32_t last = tok[len - 1];
      oracle_token_embedding(m, last, e);
      int have = oracle_forward(m, e, kv, logits);
      uint32_t next = oracle_sample(have ? logits : NULL, m->vocab,
                                    cfg->temperature, cfg->top_p, cfg->min_p,
                                    (uint64_t)(len - prompt_len), cfg->seed);
      tok[len++] = next;
      ngram_update(&ix, tok, len);
      SHIFT_CONTEXT()
      if (cfg->tok_vocab > 0 && (int)next >= cfg->tok_vocab) break;
      continue;
    }
    int acc = 0;
    for (int j = 0; j < nd; ++j) {
      uint32_t last = tok[len - 1];
      oracle_token_embedding(m, last, e);
      int have = oracle_forward(m, e, kv, logits);
      uint32_t next = oracle_sample(have ? logits : NULL, m->vocab,
                                    cfg->temperature, cfg->top_p, cfg->min_p,
                                    (uint64_t)(len - prompt_len), cfg->seed);
      if (next == draft[j]) {
        tok[len++] = draft[j];
        acc++;
        if (cfg->tok_vocab > 0 && (int)draft[j] >= cfg->tok_vocab) break;
      } else {
        tok[len++] = next;
        break;
      }
    }
    if (cfg->bonus && acc == nd) {
      uint32_t last = tok[len - 1];
      oracle_token_embedding(m, last, e);
      int have = oracle_forward(m, e, kv, logits);
      uint64_t step = (uint64_t)(len - prompt_len);
      uint32_t bonus = oracle_sample(have ? logits : NULL, m->vocab,
                                     cfg->temperature, cfg->top_p, cfg->min_p,
                                     step, cfg->seed);
      tok[len++] = bonus;
    }
    if (accepted && rounds < rounds_cap) accepted[rounds] = acc;
    rounds++;
    ngram_update(&ix, tok, len);
    SHIFT_CONTEXT()
    if (len - prompt_len >= cfg->max_tokens) break;
    if (acc < nd && cfg->tok_vocab > 0 && (int)tok[len - 1] >= cfg->tok_vocab)
      break;
  }
  int gen = len - prompt_len;
  int ncopy = gen < cap ? gen : cap;
  memcpy(out, tok + prompt_len, sizeof(uint32_t) * (size_t)ncopy);
  if (n_rounds) *n_rounds = rounds;
  if (kv != kv_io) oracle_kv_free(kv);
  free(logits); free(e); free(draft); free(tok);
  free(ix.keys); free(ix.next);
  return ncopy;
  #undef SHIFT_CONTEXT
}

/* ---------------- stochastic speculative sampling ----------------
 * Not in the reference (its verify is "target sample == draft", Q4); this is
 * the min(1, p/q) scheme with residual resampling (Leviathan, Kalman, Matias,
 * ICML 2023; Chen et al. 2023) that the device implements, restated here as
 * the statistical reference, plus the reference-compatible sample-and-match
 * rule on the same random stream.
 *
 * Random stream: Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random
 * numbers: as easy as 1, 2, 3", SC 2011): ten rounds of
 *   (hi0, lo0) = M0 * c0, (hi1, lo1) = M1 * c2,
 *   c = (hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0),
 * with the key advanced by the Weyl constants between rounds. */
static void philox_round(uint32_t c[4], const uint32_t k[2]) {
  const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
  const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
  const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
  const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
  const uint32_t n0 = hi1 ^ c[1] ^ k[0], n2 = hi0 ^ c[3] ^ k[1];
  c[0] = n0;
  c[1] = lo1;
  c[2] = n2;
  c[3] = lo0;
}

void oracle_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
  uint32_t c[4] = {ctr[0], ctr[1], ctr[2], ctr[3]};
  uint32_t k[2] = {key[0], key[1]};
  for (int r = 0; r < 10; ++r) {
    if (r > 0) {
      k[0] += 0x9E3779B9u;
      k[1] += 0xBB67AE85u;
    }
    philox_round(c, k);
  }
  memcpy(out, c, sizeof(c));
}

/* Uniform in [0, 1) with 24 random bits for (seed, round, slot).  Slots per
 * round: draft sample j -> j, acceptance test of position j -> 32 + j,
 * residual / target / bonus sample at position j -> 64 + j. */
float oracle_philox_uniform(uint64_t seed, uint32_t round, uint32_t slot) {
  const uint32_t ctr[4] = {slot, round, 0u, 0u};
  const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  uint32_t o[4];
  oracle_philox4x32_10(ctr, key, o);
  return (float)(o[0] >> 8) * (1.0f / 16777216.0f);
}

/* The device sampler's fixed summation order, which this stochastic scheme
 * defines (it is not the reference's): weights in tiles of 1024 elements;
 * in a tile, lane l (0..31) adds elements 32 i + l for i = 0..31 in order,
 * then the 32 lane sums meet in an xor butterfly (offsets 16, 8, 4, 2, 1);
 * the tile sums are added in tile order. */
#define DEV_TILE 1024
static float dev_tile_sum(const float* w, int n, int tile, int* last) {
  float s[32], t[32];
  int lst = -1;
  for (int l = 0; l < 32; ++l) {
    float acc = 0.0f;
    for (int i = 0; i < 32; ++i) {
      const int v = tile * DEV_TILE + i * 32 + l;
      if (v < n) {
        acc += w[v];
        if (w[v] > 0.0f && v > lst) lst = v;
      }
    }
    s[l] = acc;
  }
  for (int o = 16; o; o >>= 1) {
    for (int l = 0; l < 32; ++l) t[l] = s[l] + s[l ^ o];
    memcpy(s, t, sizeof(s));
  }
  *last = lst;
  return s[0];
}

static float dev_sum(const float* w, int n) {
  float tot = 0.0f;
  int last;
  for (int t = 0; t * DEV_TILE < n; ++t) tot += dev_tile_sum(w, n, t, &last);
  return tot;
}

/* Inverse CDF over non-negative weights w with total s (dev_sum), as the
 * device walks it: tau = u * s; the first tile whose running tile sum
 * exceeds tau; inside it, 32-element rows scanned across lanes by the
 * Hillis-Steele inclusive scan (offsets 1, 2, 4, 8, 16), the first positive
 * element whose running sum exceeds the remainder.  If rounding leaves no
 * such element: the last positive element of that tile, else of the row. */
static int inv_cdf(const float* w, int n, float s, float u) {
  const int nt = (n + DEV_TILE - 1) / DEV_TILE;
  float tile[256];
  int tlast[256];
  for (int t = 0; t < nt; ++t) tile[t] = dev_tile_sum(w, n, t, &tlast[t]);
  const float tau = u * s;
  float c = 0.0f;
  int kt = -1, fallback = -1;
  for (int t = 0; t < nt; ++t) {
    if (tlast[t] >= 0) fallback = tlast[t];
    if (kt < 0 && c + tile[t] > tau) {
      kt = t;
    } else if (kt < 0) {
      c += tile[t];
    }
  }
  if (fallback < 0) fallback = 0;
  if (kt < 0) return fallback;
  const float rem = tau - c;
  float run = 0.0f;
  for (int i = 0; i < 32; ++i) {
    float x[32], sc[32], nx[32];
    for (int l = 0; l < 32; ++l) {
      const int v = kt * DEV_TILE + i * 32 + l;
      x[l] = v < n ? w[v] : 0.0f;
      sc[l] = x[l];
    }
    for (int o = 1; o < 32; o <<= 1) {
      for (int l = 0; l < 32; ++l) nx[l] = l >= o ? sc[l] + sc[l - o] : sc[l];
      memcpy(sc, nx, sizeof(sc));
    }
    for (int l = 0; l < 32; ++l)
      if (run + sc[l] > rem && x[l] > 0.0f) return kt * DEV_TILE + i * 32 + l;
    run += sc[31];
  }
  return tlast[kt] >= 0 ? tlast[kt] : fallback;
}

/* Weights of softmax(l / T) after top-p (generate.rs:1034-1063) and min-p
 * (generate.rs:1071-1086), restated on e_v = exp((l_v - max) / T), whose
 * maximum is 1, so that every decision is exact:
 *   top-p (0 < top_p < 1): order v by (e_v descending, v ascending), as the
 *     reference's stable descending sort does; give each v the integer mass
 *     m_v = floor(e_v * 2^32); keep the shortest prefix whose mass sum
 *     reaches T = ceil(top_p * sum_v m_v) (the sum in double, one rounding);
 *   min-p (0 < min_p < 1): drop v with e_v < min_p (p_v < min_p * max_v p_v
 *     with max e = 1), applied after top-p as the reference does.
 * The renormalisations of the reference are left to the sampler, which
 * draws from unnormalised weights.  Returns the sum of the weights in the
 * device sampler's order (dev_sum). */
float oracle_filtered_weights(const float* l, int n, float t, float top_p, float min_p,
                              float* w) {
  float mx = -INFINITY;
  for (int v = 0; v < n; ++v)
    if (l[v] > mx) mx = l[v];
  for (int v = 0; v < n; ++v) w[v] = expf((l[v] - mx) / t);
  if (top_p > 0.0f && top_p < 1.0f && n > 0) {
    prob_idx* idx = (prob_idx*)malloc(sizeof(prob_idx) * (size_t)n);
    unsigned long long total = 0;
    for (int v = 0; v < n; ++v) {
      idx[v].p = w[v];
      idx[v].i = v;
      total += (unsigned long long)(w[v] * 4294967296.0f);
    }
    qsort(idx, (size_t)n, sizeof(prob_idx), cmp_prob_desc);
    const unsigned long long target = (unsigned long long)ceil((double)top_p * (double)total);
    unsigned long long cum = 0;
    int keep = 0;
    while (keep < n) {
      cum += (unsigned long long)(idx[keep].p * 4294967296.0f);
      ++keep;
      if (cum >= target) break;
    }
    for (int j = keep; j < n; ++j) w[idx[j].i] = 0.0f;
    free(idx);
  }
  if (min_p > 0.0f && min_p < 1.0f)
    for (int v = 0; v < n; ++v)
      if (w[v] < min_p) w[v] = 0.0f;
  return dev_sum(w, n);
}

static int sample_filt(const float* l, int n, float t, float top_p, float min_p, float u,
                       float* scratch) {
  const float s = oracle_filtered_weights(l, n, t, top_p, min_p, scratch);
  return inv_cdf(scratch, n, s, u);
}

/* One token from logits at temperature t (> 0) after top-p and min-p, with
 * the uniform of (seed, round, slot); t <= 0 is greedy (generate.rs:948-969). */
uint32_t oracle_sample_philox(const float* l, int n, float t, float top_p, float min_p,
                              uint64_t seed, uint32_t round, uint32_t slot) {
  if (n <= 0) return 0;
  if (!(t > 0.0f)) return (uint32_t)oracle_argmax(l, n);
  float* w = (float*)malloc(sizeof(float) * (size_t)n);
  const int y = sample_filt(l, n, t, top_p, min_p, oracle_philox_uniform(seed, round, slot), w);
  free(w);
  return (uint32_t)y;
}

/* The transformer draft sampling gamma tokens at temperature t; q logits of
 * every step go to qlog[j * vocab]. */
int oracle_llama_draft_sample(oracle_llama_draft* d, const uint32_t* ctx, int n, int gamma,
                              float t, float top_p, float min_p, uint64_t seed, uint32_t round,
                              uint32_t* out, float* qlog) {
  if (n <= 0 || gamma <= 0) return 0;
  if (n + gamma > d->kv->cap) return 0;
  const int V = d->m->vocab;
  float* w = (float*)malloc(sizeof(float) * (size_t)V);
  int p = 0;
  while (p < d->kv->len && p < n && d->cached[p] == ctx[p]) ++p;
  if (p > n - 1) p = n - 1;
  oracle_kv_truncate(d->kv, p);
  for (int i = p; i < n; ++i) draft_step(d, ctx[i]);
  for (int j = 0; j < gamma; ++j) {
    memcpy(qlog + (size_t)j * V, d->logits, sizeof(float) * (size_t)V);
    out[j] = (uint32_t)sample_filt(d->logits, V, t, top_p, min_p,
                                   oracle_philox_uniform(seed, round, (uint32_t)j), w);
    if (j + 1 < gamma) draft_step(d, out[j]);
  }
  free(w);
  return gamma;
}

/* speculative_generate with a sampling transformer draft.  accept_mode 0:
 * accept draft x at position j when u < p_j(x) / q_j(x), else emit a sample
 * of max(0, p_j - q_j) and end the round; accept_mode 1 (the reference's
 * rule, generate.rs:695-726): accept when the target's own sample at j equals
 * x, else emit that sample.  Round structure, prime (quirk Q1), budget check
 * and bonus as oracle_speculative_generate.  Every distribution (draft q,
 * target p, bonus) is softmax(l / T) after cfg->top_p and cfg->min_p as
 * oracle_filtered_weights restates them. */
int oracle_speculative_sample(const oracle_model* m, oracle_llama_draft* drafter,
                              const uint32_t* prompt, int n_prompt, const oracle_gen_cfg* cfg,
                              int accept_mode, uint32_t* out, int cap, int* accepted,
                              int* n_rounds, int rounds_cap) {
  if (n_rounds) *n_rounds = 0;
  if (n_prompt <= 0 || cfg->gamma <= 0 || cfg->temperature <= 0.0f) return 0;
  const int gamma = cfg->gamma, V = m->vocab;
  const float t = cfg->temperature;
  const int tcap = n_prompt + cfg->max_tokens + gamma + 2;
  uint32_t* tok = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)tcap);
  memcpy(tok, prompt, sizeof(uint32_t) * (size_t)n_prompt);
  int len = n_prompt;
  const int prompt_len = n_prompt;
  oracle_kv* kv = oracle_kv_new(m->n_layers, m->n_kv_heads * m->head_dim, tcap + 1);
  float* logits = (float*)malloc(sizeof(float) * (size_t)V);
  float* qlog = (float*)malloc(sizeof(float) * (size_t)V * (size_t)gamma);
  float* w = (float*)malloc(sizeof(float) * (size_t)V);
  float* wp = (float*)malloc(sizeof(float) * (size_t)V);
  float* wq = (float*)malloc(sizeof(float) * (size_t)V);
  float* e = (float*)malloc(sizeof(float) * (size_t)m->hidden);
  uint32_t* draft = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)gamma);
  const float tp = cfg->top_p, mn = cfg->min_p;
  for (int i = 0; i < n_prompt; ++i) {
    oracle_token_embedding(m, prompt[i], e);
    oracle_forward(m, e, kv, logits);
  }
  int rounds = 0;
  while (len - prompt_len < cfg->max_tokens) {
    if (is_cancelled(cfg)) break;
    const uint32_t r = (uint32_t)rounds;
    oracle_llama_draft_sample(drafter, tok, len, gamma, t, tp, mn, cfg->seed, r, draft, qlog);
    int acc = 0;
    for (int j = 0; j < gamma; ++j) {
      oracle_token_embedding(m, tok[len - 1], e);
      oracle_forward(m, e, kv, logits);
      const float u_res = oracle_philox_uniform(cfg->seed, r, 64u + (uint32_t)j);
      if (accept_mode == 1) {
        const int y = sample_filt(logits, V, t, tp, mn, u_res, w);
        if ((uint32_t)y == draft[j]) {
          tok[len++] = draft[j];
          acc++;
          continue;
        }
        tok[len++] = (uint32_t)y;
        break;
      }
      /* p and q after the same filters; the draft sampled x from q */
      const float sp = oracle_filtered_weights(logits, V, t, tp, mn, wp);
      const float sq = oracle_filtered_weights(qlog + (size_t)j * V, V, t, tp, mn, wq);
      const uint32_t x = draft[j];
      const float ep = wp[x], eq = wq[x];
      const float u = oracle_philox_uniform(cfg->seed, r, 32u + (uint32_t)j);
      if (u * eq * sp < ep * sq) {
        tok[len++] = x;
        acc++;
        continue;
      }
      for (int v = 0; v < V; ++v) w[v] = fmaxf(wp[v] / sp - wq[v] / sq, 0.0f);
      const float rs = dev_sum(w, V);
      const int y = rs > 0.0f ? inv_cdf(w, V, rs, u_res) : inv_cdf(wp, V, sp, u_res);
      tok[len++] = (uint32_t)y;
      break;
    }
    if (cfg->bonus && acc == gamma) {
      oracle_token_embedding(m, tok[len - 1], e);
      oracle_forward(m, e, kv, logits);
      const float u = oracle_philox_uniform(cfg->seed, r, 64u + (uint32_t)gamma);
      tok[len++] = (uint32_t)sample_filt(logits, V, t, tp, mn, u, w);
    }
    if (accepted && rounds < rounds_cap) accepted[rounds] = acc;
    rounds++;
  }
  const int gen = len - prompt_len;
  const int ncopy = gen < cap ? gen : cap;
  memcpy(out, tok + prompt_len, sizeof(uint32_t) * (size_t)ncopy);
  if (n_rounds) *n_rounds = rounds;
  oracle_kv_free(kv);
  free(logits); free(qlog); free(w); free(wp); free(wq); free(e); free(draft); free(tok);
  return ncopy;
}
