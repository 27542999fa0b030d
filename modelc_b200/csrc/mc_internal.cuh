// mc_internal.cuh -- shared device helpers and kernel interfaces of the
// modelc B200 speculative-decoding library (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "modelc_b200 is built for sm_100a only"
#endif

namespace mc {

// ---------------------------------------------------------------------------
// Packed-weight geometry.
//
// A quantized [N, K] matrix (reference layout [out, in], transformer.rs:825)
// is stored as 16-row "stripes" x 32-column "k-blocks".  One k-block of one
// stripe is 512 bytes: 32 lanes x 16 bytes, each lane's 16 bytes being exactly
// its A fragment of mma.m16n8k32.s8 (rows g and g+8, columns 4t..4t+3 and
// 16+4t..16+4t+3, g = lane/4, t = lane%4).  Stripes are stored k-block-major,
// so a warp streaming a contiguous range of (stripe, k-block) indices reads
// contiguous, fully coalesced 512-byte runs.
// ---------------------------------------------------------------------------
constexpr int kStripeRows = 16;
constexpr int kKBlock = 32;
constexpr int kFragBytes = 512;

// Activations are fixed-point: per token a power-of-two exponent e with
// X = round(x * 2^e), |X| <= 2^20, held as three balanced base-128 int8
// digits X = d0*2^14 + d1*2^7 + d2.  Column c = 3*token + digit of the B
// operand; NT n8-tiles cover 8*NT columns.
constexpr int kDigits = 3;
constexpr int kGroupTokens = 16;  // tokens per operand group (NT <= 6, 48 columns)
constexpr int kMaxGroups = 4;
constexpr int kMaxTokens = kGroupTokens * kMaxGroups;  // tokens per forward
constexpr int kExpNonFinite = -100000;  // exponent marking a non-finite row

// n8 tiles of one operand group: up to 16 tokens in 1, 2, 3 or 6 tiles;
// larger forwards are cut into groups of 16 tokens of 6 tiles each.
__host__ __device__ inline int nt_for_tokens(int m) {
  if (m > kGroupTokens) return 6;
  int cols = kDigits * m;
  int nt = (cols + 7) / 8;
  if (nt == 4 || nt == 5) nt = 6;
  return nt;  // 1, 2, 3 or 6
}
__host__ __device__ inline int groups_for_tokens(int m) {
  return (m + kGroupTokens - 1) / kGroupTokens;
}

// Token -> sequence map of one forward over n_seq sequences of seq_len
// tokens each (one sequence: seq_len = M, strides unused).  Token m is
// offset i = m % seq_len of sequence z = m / seq_len, at position
// pos_ptr[z * pos_stride] + pos_add + i, with KV pages
// page_table[z * pt_stride + ...]; its argmax key goes to
// keys[z * key_stride + i].
#ifdef __CUDACC__
// Programmatic dependent launch: wait for the preceding grid's completion and
// memory; let the next grid launch.
__device__ __forceinline__ void grid_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
#endif

struct SeqMap {
  int seq_len;
  int pos_stride;   // ints between the sequences' position counters
  int pt_stride;    // page-table entries per sequence
  int key_stride;   // 64-bit keys between the sequences' key arrays
};
__host__ __device__ inline int seq_of(const SeqMap& s, int m) {
  return s.seq_len > 0 ? m / s.seq_len : 0;
}
__host__ __device__ inline int seq_off(const SeqMap& s, int m) {
  return s.seq_len > 0 ? m % s.seq_len : m;
}
__host__ __device__ inline int key_slot(const SeqMap& s, int m) {
  return seq_of(s, m) * s.key_stride + seq_off(s, m);
}

// Packed weight formats.
//   WF_I8: per (stripe, k-block) 512 bytes, one 16-byte A fragment per lane,
//          plus one f32 scale per packed row.
//   WF_Q4: ggml q4_0 (32-weight blocks along K with one fp16 scale,
//          parsers/gguf/dequant.rs:23-46).  Per (stripe, k-block) 256 bytes,
//          8 per lane: word 0 byte b holds the nibbles of A registers a0
//          (low) and a1 (high) byte b, word 1 those of a2 and a3, so
//          (w & 0x0F0F0F0F) and ((w >> 4) & 0x0F0F0F0F) are the unsigned
//          codes.  Block scales: one u32 per (stripe, k-block, g) holding
//          the fp16 scales of rows g (low half) and g + 8.
//   WF_I8R: WF_I8 weights streamed through a shared-memory ring by bulk
//          copies instead of register batches (the GEMV variant for large
//          matrices); same packing.
enum WFmt : int { WF_I8 = 0, WF_Q4 = 1, WF_I8R = 2 };
constexpr int kQ4BlockBytes = 18;  // fp16 scale + 16 bytes of nibbles

// Epilogue kinds of the quantized GEMV.
enum Epi : int {
  EPI_STORE = 0,   // out[m][row] = y
  EPI_RESID = 1,   // out[m][row] += y           (O and down projections)
  EPI_SWIGLU = 2,  // act[m][i] = silu(gate)*up  (gate/up rows interleaved)
  EPI_QKV = 3,     // RoPE(q), RoPE(k) -> q buffer and paged KV, v -> KV
  EPI_LMHEAD = 4,  // logits + first-index argmax keys (row index + row_offset)
  EPI_TP = 5,      // row-parallel partial sums stored into every rank's reduce buffer
};

// Tensor-parallel exchange buffers (one region per rank, opened by the peers
// through CUDA IPC, or directly when the peer lives in the same process):
// partial sums [2 sets][R senders][kMaxTokens][d] floats, then flags [2
// sets][kMaxTP] epochs, then argmax keys [2 sets][kMaxTP senders][kMaxTokens]
// and their flags [2 sets][kMaxTP].  A row-parallel GEMV (EPI_TP) of epoch e
// stores its rows into set e % 2, slot `rank`, of every rank, and its last
// CTA publishes e in every rank's flags; the reduce kernel waits for all R
// flags, adds the slots in rank order (identical bits on every rank), then
// does h += sum and the next encoder's statistics.  The vocab-parallel LM
// head exchanges its per-token argmax keys the same way (k_tp_keys).  Every
// wait is bounded by *wait_ns nanoseconds; an expired wait raises *err, and
// once *err is raised later waits give up at once.
constexpr int kMaxTP = 8;
struct TPArgs {
  float* red[kMaxTP];      // every rank's reduce region (index = rank)
  unsigned* flag[kMaxTP];  // every rank's flags
  unsigned long long* keyx[kMaxTP];  // every rank's key slots
  unsigned* kflag[kMaxTP];           // every rank's key flags
  int rank, world, d;
  const unsigned* epoch;   // this rank's epoch counter
  unsigned* kepoch;        // this rank's key-exchange epoch counter
  int* cnt;                // CTA arrival counter of the GEMV (zeroed)
  int* err;
  const long long* wait_ns;  // limit of each bounded wait (device word)
};

struct QuantArgs {
  const float* h;        // [M][ld]
  int ld;
  int d;                 // logical length
  int M;
  const float* w;        // RMSNorm weight or nullptr
  int wlen;
  float eps;
  int do_norm;
  uint8_t* xq;           // packed digits
  int KB;                // ceil(d/32) (padded k-blocks written)
  int nt;
  int* xexp;
  // Producer-side statistics (use_stats != 0): sum of squares as np partials
  // pss[m * np_stride + j], and max |x * w| as float bits amax[m]; the kernel
  // then zeroes amax_next[0..kMaxTokens) for the following producer.
  int tc_layout;         // write the tcgen05 B-operand layout (see digit_word)
  int use_stats;
  const float* pss;
  int np, np_stride;
  const unsigned* amax;
  unsigned* amax_next;
  const void* pf;        // L2 prefetch of upcoming weights, or nullptr
  long long pf_bytes;
  // The O projection's input straight from the attention's page partials
  // (att_o != nullptr; the partial layout and geometry of AttnArgs): each
  // (token, head) is combined over its pages here -- weights e^(m_p - M)
  // with M a max over the pages, denominator sum_p w_p l_p by a fixed
  // shuffle tree, numerator sum_p w_p o_p in page order, then a division --
  // and h / ld are unused.  amax is then the attention's bound on each
  // token's max |output| (AttnArgs::st_amax).
  const float* att_o;
  const float* att_ml;
  int att_chunks, att_Hkv, att_G, att_hdp, att_qblk, att_page;
  SeqMap att_seq;
  const int* att_pos;
  int att_pos_add;
  int trace_slot;        // MC_TRACE builds: 1 + timeline slot, 0 = untraced
};

struct GemvArgs {
  const int4* w;         // packed weights (WF_Q4: 8 bytes per lane per k-block)
  const float* scale;    // WF_I8: [n_stripes*16] per packed row (0 on padding rows)
  const uint32_t* qscale;// WF_Q4: [n_stripes][KB][8] fp16 pairs (rows g, g+8)
  const uint8_t* x;      // packed activation digits of this launch's group [KB][32][8*NT]
  const int* xexp;       // [M] exponents of this launch's tokens
  int KB;                // k-blocks per stripe
  int n_stripes;
  int M;                 // tokens of this launch (GEMV: <= 16; tcgen05 GEMM: <= 64)
  int m0;                // forward-wide index of this launch's first token
  int* ws;               // split-K partial sums [n_stripes][groups][16][48] (zeroed)
  int* cnt;              // [n_stripes][groups] k-block arrival counters (zeroed)
  int* err;              // set to 1 when a bounded device wait expires
  // Statistics for the next activation encoding, produced by the RESID and
  // SWIGLU epilogues: per-stripe sum of squares st_pss[m * st_np + stripe]
  // (RESID only) and max |value * st_w[row]| folded into st_amax[m] (float
  // bits, atomicMax).  st_amax == nullptr disables both.
  float* st_pss;
  int st_np;
  unsigned* st_amax;
  const float* st_w;
  const void* next_w;    // weights of the next GEMV in the stream (L2 prefetch)
  long long next_bytes;  // its packed size
  long long next_pf_bytes;  // how much of it to prefetch
  // epilogue
  float* out;            // STORE/RESID/SWIGLU/LMHEAD destination
  int ldo;               // row stride (elements) of out per token
  int n_out;             // valid output rows (N) or SwiGLU width (F)
  unsigned long long* keys;  // LMHEAD: per-token argmax keys
  // QKV epilogue
  float* q_out;          // [M][H][hdp]
  float* kc;             // layer K pages [page][Hkv][P][hdp]
  float* vc;
  const int* page_table;
  const int* pos_ptr;    // token positions: SeqMap
  int pos_add;
  SeqMap seq;            // token -> sequence (QKV positions and pages, LMHEAD keys)
  const float* rope_cos; // [pos][half_p]
  const float* rope_sin;
  int half_p, hdp, H, Hkv, page;
  int sq, sk;            // Q and K stripe counts
  int kv_prefetch;       // QKV: warm L2 with this layer's K/V pages for the attention
  int row_offset;        // LMHEAD: global vocabulary index of packed row 0
  const int4* wtc;       // tcgen05 path: weights in the canonical layout (k_gemm_tc)
  TPArgs tp;             // EPI_TP
  // Encoding tail (bar != nullptr; RESID and SWIGLU): after the epilogues
  // the grid meets at a barrier (bar[0] arrivals, bar[1] generation; bounded
  // wait), then every CTA encodes its slice of the next projection's input
  // as k_quant<true> would with enc (its statistics path, k-blocks split
  // over the grid).  The grid is at most one wave of the tail variant
  // (occupancy), so all its CTAs are resident.
  QuantArgs enc;
  unsigned* bar;
  int trace_slot;        // MC_TRACE builds: 1 + timeline slot, 0 = untraced
};


struct AttnArgs {
  const float* q;        // [M][H][hdp]
  const float* kc;       // layer pages
  const float* vc;
  const int* page_table;
  const int* pos_ptr;
  int pos_add;
  SeqMap seq;
  int qblk;              // tokens of one sequence per CTA (query block)
  int kv_pre;            // 1: every K/V position below a sequence's first new
                         // position was written before this launch's graph
                         // began, so those pages may be read before
                         // griddepcontrol.wait (the verify graph: only its
                         // own QKV writes target K/V, at the new positions)
  int M, H, Hkv, hdp, page;
  float inv_scale_den;   // sqrt(head_dim) (divisor, transformer.rs:966)
  int max_chunks;
  float* part_o;         // [blocks][Hkv][max_chunks][G*qblk][hdp]: sum_t e^(s_t - m_p) v_t
  float* part_ml;        // [blocks][Hkv][max_chunks][G*qblk][2]: (m_p, l_p) of each page p
  unsigned* st_amax;     // per token: max over its pages and heads of |o_p| / l_p,
                         // a bound on its max |output| (float bits, atomicMax)
  const void* pf;        // L2 prefetch of upcoming weights while HBM is idle, or nullptr
  long long pf_bytes;
  // Encoding tail (bar != nullptr; attention_tail_fits): after its partials
  // and bound are out the grid meets at a bounded barrier (bar[0] arrivals,
  // bar[1] generation), then every CTA combines and encodes a slice of the O
  // projection's input as k_quant_att would with enc (its att_* fields
  // describing these partials), saving that launch.
  QuantArgs enc;
  unsigned* bar;
  int* err;              // raised when the barrier's bounded wait expires
  int trace_slot;        // MC_TRACE builds: 1 + timeline slot, 0 = untraced
};

// Token m = (sequence z, offset i) by EmbedArgs::seq; each sequence z has
// its context at ctx + z * ctx_stride, its counter at off[z * seq.pos_stride]
// and its keys at keys + z * seq.key_stride.
enum EmbedSrc : int {
  SRC_IDS = 0,     // ids[m]
  SRC_CTX_AT = 1,  // ctx_z[off_z + i]
  SRC_KEYS = 2,    // argmax key keys_z[i]
  SRC_VERIFY = 3,  // i == 0 ? ctx_z[len_z - 1] : key keys_z[i - 1]
};

struct EmbedArgs {
  int src;
  const uint32_t* ids;
  const uint32_t* ctx;
  const int* off;        // SRC_CTX_AT offset / SRC_VERIFY context length
  const unsigned long long* keys;
  SeqMap seq;
  int ctx_stride;
  uint32_t* ids_out;     // optional: resolved ids [M]
  const int8_t* emb_q;   // [vocab][d] int8
  const float* emb_scale;// [vocab]
  const uint8_t* emb_q4; // or q4_0 blocks [vocab][d/32][18] (then emb_q unused)
  int d, vocab, M;
  float* h;              // [M][d]
  unsigned long long* zero_keys;  // keys this forward will produce (key_slot of
  int n_zero;                     // tokens 0..n_zero-1 by seq)
  // statistics of h for the first encoding: st_pss[m * st_np] = sum(h*h),
  // st_amax[m] = max |h * st_w| (plain stores); st_zero[0..n_st_zero) zeroed
  float* st_pss;
  int st_np;
  unsigned* st_amax;
  const float* st_w;
  unsigned* st_zero;
  int n_st_zero;
  int trace_slot;        // MC_TRACE builds: 1 + timeline slot, 0 = untraced
};

// Tensor parallelism: after the all-reduce of a row-parallel projection's
// partial sums, h += y and the next encoder's statistics (as the RESID
// epilogue produces them): pss[m * n_blk + blk] over 1024-element blocks and
// max |h * w| folded into amax[m].
struct ResidArgs {
  float* h;              // [M][d]
  const float* y;        // [M][d] reduced partial sums
  int d, M;
  float* pss;
  unsigned* amax;
  const float* w;        // next RMSNorm weight or nullptr
  int trace_slot;
};
cudaError_t launch_resid_stats(const ResidArgs& a, cudaStream_t s, bool pdl);
// The reduce step of EPI_TP (waits for the peers with a bounded spin, then
// h += sum of the R partials and the statistics as k_resid_stats); advances
// the epoch.
cudaError_t launch_tp_reduce(const ResidArgs& a, const TPArgs& t, unsigned* epoch, int* cnt,
                             cudaStream_t s, bool pdl);
// Vocab-parallel LM head over peer memory: the max over the ranks of the
// argmax keys of n_seq sequences of seq_len tokens (key_stride apart).
cudaError_t launch_tp_keys(const TPArgs& t, unsigned long long* keys, int n_seq, int seq_len,
                           int key_stride, cudaStream_t s, bool pdl);
constexpr int kResidBlock = 1024;

struct SpecState {
  int ctx_len;
  int lt;          // target KV length
  int ld;          // draft KV length
  int generated;
  int prompt_len;
  int max_tokens;
  int gamma;
  int n_rounds;
  int bonus;
  int rounds_cap;
  int accept_mode;     // stochastic: 0 = min(1, p/q) + residual, 1 = sample == draft
  float temperature;   // > 0: stochastic rounds
  uint32_t seed_lo, seed_hi;
  float top_p;         // applied when in (0, 1) (generate.rs:961-963)
  float min_p;         // applied when in (0, 1) (generate.rs:964-966)
  // draft tokens of this round (gamma for the model drafters; the n-gram
  // drafter may find fewer, 0 meaning the reference's one-step fallback,
  // generate.rs:647-693), and the n-gram index: its entry count, the context
  // length its last update saw, the key length n
  int n_draft;
  int ng_len;
  int ng_last_len;
  int ngram;
  // the context shift of the last round (generate.rs:26-63): tokens removed
  // (0: none), where the removed range starts, the target / draft KV
  // lengths before it, whether it was the anchored form; shifts so far
  int sh_n, sh_at, sh_lt, sh_ld, sh_anch, n_shifts;
  // MIXED target cache: tokens in its f32 window (the last kv_hot
  // positions), and the round's first verify position
  int kv_hot, mx_base;
  unsigned long long tkeys[kGroupTokens];
  unsigned long long dkeys[kGroupTokens];
};
// SpecState stride in ints and in keys (sequences of a batched session)
constexpr int kStateInts = (int)(sizeof(SpecState) / sizeof(int));
constexpr int kStateKeys = (int)(sizeof(SpecState) / sizeof(unsigned long long));
static_assert(sizeof(SpecState) % sizeof(unsigned long long) == 0, "SpecState stride");

// Argmax keys: larger key = larger value, ties -> smaller index.
__host__ __device__ inline unsigned long long argmax_key(float v, uint32_t idx) {
  uint32_t b = 0;
#ifdef __CUDA_ARCH__
  b = __float_as_uint(v);
#else
  memcpy(&b, &v, 4);
#endif
  uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)o << 32) | (unsigned long long)(~idx);
}
__host__ __device__ inline uint32_t key_index(unsigned long long k) {
  return k == 0ull ? 0u : ~(uint32_t)(k & 0xffffffffull);
}

// Kernel launchers (mc_kernels.cu).  All kernels are launched with
// programmatic stream serialization allowed: each one issues its
// data-independent loads (weights) before griddepcontrol.wait.
cudaError_t launch_gemv(const GemvArgs& a, int epi, int nt, int wf, int grid,
                        cudaStream_t s, bool pdl);
int gemv_blocks_per_sm(int epi, int nt, int wf, bool tail = false);
// tcgen05 GEMM for 9..64 tokens: grid (128-row tiles, ksplit), 48 digit
// columns per group of 16 tokens; the digits must be encoded with
// QuantArgs::tc_layout; ksplit > 1 merges through ws/cnt.
cudaError_t launch_gemm_tc(const GemvArgs& a, int epi, int ksplit, cudaStream_t s, bool pdl);
cudaError_t launch_pack_tc(const int8_t* src, long long src_ld, const int* row_map,
                           const int* col_map, int n_rows, int n_tiles, int KB, int4* dst,
                           cudaStream_t s);
cudaError_t prepare_tc();  // shared-memory limit of the tcgen05 GEMM (outside capture)
constexpr int kTcTileRows = 128;
constexpr int kTcMaxSplit = 8;  // k-split CTAs of one tile = one cluster (portable size)
// The tcgen05 operands are K-major with the 128-byte swizzle: K runs in atoms
// of 128 bytes (4 k-blocks of 32); the weight copy is [tile][atom][128 rows]
// [128 bytes], the digits [atom][column][128 bytes], 16-byte chunk c of row r
// stored at chunk c ^ (r % 8).  K is padded to whole atoms (zero weights).
__host__ __device__ inline int tc_atoms(int KB) { return (KB + 3) / 4; }
cudaError_t launch_quant(const QuantArgs& a, cudaStream_t s, bool pdl);
// Records msg as the calling thread's error (mc_last_error) and returns st.
int32_t set_error(int32_t st, const char* msg);
// amax[m] = max |x[m][0..d)| as float bits, m < M (the statistics of an
// un-normalised encoding, QuantArgs::use_stats with np = 0)
cudaError_t launch_act_amax(const float* x, int ld, int d, int M, unsigned* amax, cudaStream_t s,
                            bool pdl);
cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl);
// Whether launch_attention runs a with the encoding tail: the tensor-core
// kernel with one m-tile, a grid of at most one wave of it on nsm SMs, and
// the combined slice within its shared memory (a.enc.M / KB set).
bool attention_tail_fits(const AttnArgs& a, int nsm);
cudaError_t launch_embed(const EmbedArgs& a, cudaStream_t s, bool pdl);
// One CTA per sequence z of a batch: st + z, ctx + z * ctx_stride,
// acc_log + z * log_stride.  A sequence whose budget is spent (generated >=
// max_tokens > 0) is left unchanged.
// Target KV variants (mc_spec_cfg::kv_mode).
enum KvMode : int { KV_FP32 = 0, KV_INT8 = 1, KV_MIXED = 2 };

// The new tokens of one forward in one layer's K/V pages: token m =
// (sequence z, offset i) by seq, at position pos_ptr[z * seq.pos_stride] +
// pos_add + i, head h column c at ((page * Hkv + h) * page_len + pos % page_len)
// * hdp + c.
struct KvQArgs {
  float* kc;
  float* vc;
  const int* page_table;
  const int* pos_ptr;
  int pos_add;
  SeqMap seq;
  int M, Hkv, hd, hdp, page;
};
// KvLayer::append of an INT8 layer on those tokens (mc_kvcache.cu).
cudaError_t launch_kv_qdq(const KvQArgs& a, cudaStream_t s, bool pdl);

// The window of a MIXED layer (make_kv_cache, generate.rs:19).
constexpr int kMixedWindow = 64;

// KvLayer::append of a MIXED layer (transformer.rs:389-419) for one token
// per request at position pos_ptr[z * seq.pos_stride] + pos_add in one
// layer: when the f32 window already holds `window` tokens -- min(hot +
// step, window) with hot = hot_ptr[z * hot_stride] (or hot_const) before the
// first of `step` earlier appends -- the token `window` positions back is
// quantized (its originals saved to bak first when bak is set: a verify
// step, which the acceptance may roll back).
struct KvMixArgs {
  float* kc;
  float* vc;
  const int* page_table;
  const int* pos_ptr;
  int pos_add;
  SeqMap seq;            // seq_len 1: one token per request
  int B, Hkv, hdp, page, window;
  const int* hot_ptr;
  int hot_stride;
  int hot_const;
  int step;
  float* bak;            // [B][bak_steps][layers][2][Hkv * hdp] or nullptr
  int bak_steps, layer, layers;
  int* base_out;         // step 0, layer 0: the position into base_out[z * base_stride]
  int base_stride;
};
cudaError_t launch_kv_mixed_age(const KvMixArgs& a, cudaStream_t s, bool pdl);

// One KV cache (target or draft) of every request, for the context shift.
struct KvPlanes {
  float* k;             // [layers][layer_stride floats]: pages [page][Hkv][page_len][hdp]
  float* v;
  size_t layer_stride;
  int layers, Hkv, hd, hdp, page;
  const int* pt;        // request z's page-table row at pt + z * pt_stride
  int pt_stride;
};
struct ShiftArgs {
  SpecState* st;
  uint32_t* ctx;
  int ctx_stride;
  int B;
  int shift_context;    // GenerationConfig::max_context
  int anchor;           // GenerationConfig::anchor_tokens
  int requant;          // re-quantize kept tokens after an anchored shift (INT8, MIXED)
  int window;           // MIXED target: its window (kept f32 tokens); 0 otherwise
  KvPlanes t, d;        // target KV; draft KV (d.layers == 0: none)
};
// generate.rs:26-63 context_shift after a round, on the device: the plan and
// token move, the K/V moves, the re-quantization (three launches).
cudaError_t launch_context_shift(const ShiftArgs& a, int nsm, cudaStream_t s, bool pdl);

// After a MIXED session's acceptance: the window quantizations of verify
// steps the acceptance dropped (steps >= lt - mx_base) are undone from bak,
// then kv_hot advances by the steps kept (two launches).
cudaError_t launch_kv_mixed_commit(SpecState* st, const KvPlanes& t, const float* bak, int B,
                                   int steps, int window, cudaStream_t s, bool pdl);

cudaError_t launch_accept_greedy(SpecState* st, uint32_t* ctx, int* acc_log, int vm, int n_seq,
                                 int ctx_stride, int log_stride, cudaStream_t s, bool pdl);
cudaError_t launch_set_int(int* p, int v, cudaStream_t s);
// The n-gram drafter of speculative_generate inside the round graph
// (generate.rs:642-646 with no draft model; build_ngram_index,
// update_ngram_index, draft_tokens, generate.rs:771-841), one CTA per
// sequence z: first the window ending at the context's last token joins the
// index when the context grew since the last update, then up to gamma draft
// tokens into st->dkeys and their count into st->n_draft.  The index of
// sequence z is ng + z * ng_cap * (n + 1): up to ng_cap entries of n + 1
// tokens (key, continuation) in insertion order; list: ng_cap ints per
// sequence of scratch.
cudaError_t launch_ngram_round(SpecState* st, const uint32_t* ctx, uint32_t* ng, int* list,
                               int ctx_stride, int ng_cap, int n_seq, cudaStream_t s);
}  // namespace mc
typedef struct mc_mlp_drafter mc_mlp_drafter;
namespace mc {
// MlpDraftModel (draft.rs:91-147) inside the round graph: gamma greedy steps
// for each of n_seq sequences from its context's last token, keys into
// st[z].dkeys; hid is scratch of n_seq x mlp_hidden floats.
cudaError_t mlp_round(const mc_mlp_drafter* m, SpecState* st, const uint32_t* ctx, int ctx_stride,
                      int n_seq, int gamma, float* hid, cudaStream_t stream);
int mlp_device(const mc_mlp_drafter* m);
int mlp_vocab(const mc_mlp_drafter* m);
int mlp_hidden(const mc_mlp_drafter* m);
// Stochastic rounds: sample draft step j from softmax(logits / T) into
// *key_out (as an argmax key), and the acceptance of a whole round from the
// verify logits tlog [vm][V] and the draft logits dlog [gamma][V].
cudaError_t launch_sample_rows(const float* logits, int rows, int V, float t, float top_p,
                               float min_p, uint64_t seed, uint32_t rnd, uint32_t* out,
                               cudaStream_t s);
cudaError_t launch_sample_draft(SpecState* st, const float* logits, int V, int j,
                                unsigned long long* key_out, cudaStream_t s, bool pdl);
cudaError_t launch_accept_stochastic(SpecState* st, uint32_t* ctx, int* acc_log, int vm,
                                     const float* tlog, const float* dlog, int V,
                                     cudaStream_t s, bool pdl);
constexpr int kSampleMaxVocab = 256 * 1024;  // tiles of 1024 staged in shared memory

// Timeline of traced launches (MC_TRACE builds only): per slot the earliest
// CTA start, the earliest return from the dependency wait and the latest CTA
// end, in %globaltimer nanoseconds.
constexpr int kTraceSlots = 4096;
cudaError_t trace_reset();
cudaError_t trace_read(unsigned long long* out, int n);  // n slots x 3 values
size_t attention_smem_bytes(int G, int qblk, int hdp, int page);
int attention_qblk(int G, int seq_len);  // tokens per attention CTA
size_t gemv_ws_ints_per_stripe(int nt);
cudaError_t prepare_kernels(size_t quant_smem, size_t attn_smem);
cudaError_t launch_pack_int8(const int8_t* src, long long src_ld,
                             const float* src_scale, const int* row_map,
                             const int* col_map, int n_stripes, int KB,
                             int4* dst, float* dst_scale, cudaStream_t s);
// q4_0 source [rows][src_KB] blocks of 18 bytes -> WF_Q4 stripes of the KB
// blocks starting at block kb_off, rows through row_map (size n_stripes*16,
// -1 = padding row: zero scale, codes 8).
cudaError_t launch_pack_q4(const uint8_t* src, const int* row_map, int n_stripes, int KB,
                           int src_KB, int kb_off, uint2* dst, uint32_t* dst_scale,
                           cudaStream_t s);

}  // namespace mc
