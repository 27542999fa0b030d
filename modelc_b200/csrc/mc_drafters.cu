// mc_drafters.cu -- the reference's two small drafters behind DraftModel
// (draft.rs:18-21), on the device.
//
//  MLP drafter (MlpDraftModel, draft.rs:28-147): embedding row -> FC1 + bias
//  -> ReLU -> FC2 + bias -> argmax, gamma times.  Every output row is summed
//  by one thread in the reference's order (bias first, then j ascending, a
//  separate multiply and add), so logits -- and the greedy draft -- are the
//  reference's bit for bit.  Greedy only: the reference samples with an
//  unseeded generator when temperature > 0.
//
//  n-gram drafter (build_ngram_index / draft_tokens / most_frequent,
//  generate.rs:771-841): the index of a token history is the set of its
//  windows (n-token key -> next token), so one CTA scans the history for the
//  current key and takes the most frequent continuation.  Count ties: the
//  continuation seen first (the reference leaves them to HashMap order).
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "mc_internal.cuh"
#include "modelc_cuda.h"

using mc::argmax_key;
using mc::key_index;

namespace {

mc_status set_err(mc_status st, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return mc::set_error(st, buf);
}

constexpr int kMlpFc1Threads = 128;
constexpr int kMlpFc2Threads = 256;
constexpr int kNgramThreads = 1024;

// Where the drafter's steps take their tokens and leave their keys.  The
// standalone drafter: *first, keys[].  Inside a session's round graph
// (st != nullptr): sequence z = blockIdx.y starts from its context's last
// token, ctx + z * ctx_stride at st[z].ctx_len - 1, and its keys are
// st[z].dkeys; hid holds one row of dh per sequence.
struct MlpIo {
  const uint32_t* first;
  unsigned long long* keys;
  mc::SpecState* st;
  const uint32_t* ctx;
  int ctx_stride;
};
__device__ __forceinline__ unsigned long long* mlp_keys(const MlpIo& io) {
  return io.st ? io.st[blockIdx.y].dkeys : io.keys;
}
// Token of draft step s: the context's last token, then the previous step's
// argmax.
__device__ __forceinline__ uint32_t mlp_token(const MlpIo& io, int s) {
  if (s > 0) return key_index(mlp_keys(io)[s - 1]);
  if (io.st) {
    const mc::SpecState* st = io.st + blockIdx.y;
    return io.ctx[(size_t)blockIdx.y * io.ctx_stride + st->ctx_len - 1];
  }
  return *io.first;
}

// FC1 + ReLU of step s (draft.rs:104-113): hid[i] = max(b1[i] + sum_j
// w1[i][j] * e[j], 0), j ascending; the embedding row is staged in shared
// memory.  A token past the embedding leaves hid untouched (FC2 then emits
// zero logits, draft.rs:97-101).
__global__ void __launch_bounds__(kMlpFc1Threads) k_mlp_fc1(const float* __restrict__ embed,
                                                            const float* __restrict__ w1,
                                                            const float* __restrict__ b1, int V,
                                                            int d, int dh, MlpIo io, int s,
                                                            float* __restrict__ hid) {
  extern __shared__ float se[];
  const uint32_t t = mlp_token(io, s);
  // step s's key collects FC2's atomicMax after this launch: start it at 0
  if (blockIdx.x == 0 && threadIdx.x == 0) mlp_keys(io)[s] = 0ull;
  hid += (size_t)blockIdx.y * dh;
  if ((size_t)t * d + d > (size_t)V * d) return;  // block-uniform
  const float* e = embed + (size_t)t * d;
  for (int j = threadIdx.x; j < d; j += blockDim.x) se[j] = e[j];
  __syncthreads();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= dh) return;
  const float* row = w1 + (size_t)i * d;
  float sum = b1[i];
  int j = 0;
  if ((d & 3) == 0 && (reinterpret_cast<uintptr_t>(row) & 15) == 0)
    for (; j < d; j += 4) {
      const float4 w = *reinterpret_cast<const float4*>(row + j);
      sum = __fadd_rn(sum, __fmul_rn(w.x, se[j]));
      sum = __fadd_rn(sum, __fmul_rn(w.y, se[j + 1]));
      sum = __fadd_rn(sum, __fmul_rn(w.z, se[j + 2]));
      sum = __fadd_rn(sum, __fmul_rn(w.w, se[j + 3]));
    }
  for (; j < d; ++j) sum = __fadd_rn(sum, __fmul_rn(row[j], se[j]));
  hid[i] = fmaxf(sum, 0.0f);  // f32::max: a NaN sum gives 0
}

// FC2 (draft.rs:115-124) and the argmax (first strict maximum, NaN never
// chosen) folded into keys[s]: one thread per vocabulary row.
__global__ void __launch_bounds__(kMlpFc2Threads) k_mlp_fc2(const float* __restrict__ w2,
                                                            const float* __restrict__ b2, int V,
                                                            int d, int dh, MlpIo io, int s,
                                                            const float* __restrict__ hid) {
  extern __shared__ float sh[];
  const uint32_t t = mlp_token(io, s);
  unsigned long long* keys = mlp_keys(io);
  hid += (size_t)blockIdx.y * dh;
  const bool in = (size_t)t * d + d <= (size_t)V * d;
  for (int j = threadIdx.x; j < dh; j += blockDim.x) sh[j] = in ? hid[j] : 0.0f;
  __syncthreads();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  unsigned long long k = 0ull;
  if (i < V) {
    float sum = 0.0f;  // out-of-range token: zero logits
    if (in) {
      const float* row = w2 + (size_t)i * dh;
      sum = b2[i];
      for (int j = 0; j < dh; ++j) sum = __fadd_rn(sum, __fmul_rn(row[j], sh[j]));
    }
    if (sum > -INFINITY) k = argmax_key(__fadd_rn(sum, 0.0f), (uint32_t)i);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, k, o);
    k = k2 > k ? k2 : k;
  }
  if ((threadIdx.x & 31) == 0 && k) atomicMax(keys + s, k);
}

// One step of draft_tokens (generate.rs:804-841) + most_frequent
// (:832-841), block-wide: among the index entries whose n-token key equals
// key[0, n) (shared memory), the continuation with the highest count; count
// ties go to the continuation of the earliest entry (the reference leaves
// them to HashMap order).  Entry e (in insertion order) is row(e): its key
// row(e)[0 .. n), its continuation row(e)[n].  list: scratch of n_ent ints.
// Returns the token, or -1 when no key matches.
template <class Row>
__device__ long long ngram_step(Row row, int n_ent, int n, const uint32_t* key, int* list,
                                int* s_nm, unsigned long long* s_best) {
  if (threadIdx.x == 0) *s_nm = 0;
  __syncthreads();
  for (int e = threadIdx.x; e < n_ent; e += blockDim.x) {
    const uint32_t* r = row(e);
    bool eq = true;
    for (int q = 0; q < n && eq; ++q) eq = r[q] == key[q];
    if (eq) list[atomicAdd(s_nm, 1)] = e;
  }
  __syncthreads();
  const int nm = *s_nm;
  if (nm == 0) return -1;  // block-uniform
  // (count, -first entry) of each match's continuation, packed so that the
  // largest key is the most frequent, earliest-seen continuation
  unsigned long long best = 0ull;
  for (int i = threadIdx.x; i < nm; i += blockDim.x) {
    const uint32_t c = row(list[i])[n];
    unsigned count = 0;
    int first = 0x7fffffff;
    for (int j = 0; j < nm; ++j)
      if (row(list[j])[n] == c) {
        ++count;
        first = min(first, list[j]);
      }
    const unsigned long long k = ((unsigned long long)count << 32) |
                                 (unsigned long long)(0x7fffffffu - (unsigned)first);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long b2 = __shfl_xor_sync(0xffffffffu, best, o);
    best = b2 > best ? b2 : best;
  }
  if ((threadIdx.x & 31) == 0) s_best[threadIdx.x >> 5] = best;
  __syncthreads();
  unsigned long long b = 0ull;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) b = s_best[w] > b ? s_best[w] : b;
  const int first = (int)(0x7fffffffu - (unsigned)(b & 0xffffffffull));
  __syncthreads();  // s_best and list may be reused by the next step
  return (long long)row(first)[n];
}

// draft_tokens over the index of toks[0, n_tok) (build_ngram_index: every
// window): step g looks up the last n tokens of toks[0, n_tok + g) and
// appends the continuation ngram_step picks.  Stops at the first step without
// a match.  list: scratch of n_tok ints.
__global__ void __launch_bounds__(kNgramThreads) k_ngram_draft(uint32_t* toks, int n_tok, int n,
                                                               int gamma, int* list,
                                                               uint32_t* out, int* n_out) {
  __shared__ int s_nm;
  __shared__ unsigned long long s_best[kNgramThreads / 32];
  __shared__ uint32_t s_key[32];
  int produced = 0;
  for (int g = 0; g < gamma; ++g) {
    const int clen = n_tok + g;
    if (clen < n || n < 1 || n > 32) break;  // a short key matches no n-token key (block-uniform)
    if (threadIdx.x < n) s_key[threadIdx.x] = toks[clen - n + threadIdx.x];
    __syncthreads();
    // entry e: the window at toks[e] (windows ascend)
    const long long next = ngram_step([&](int e) { return toks + e; }, max(n_tok - n, 0), n, s_key,
                                      list, &s_nm, s_best);
    if (next < 0) break;  // block-uniform
    if (threadIdx.x == 0) {
      toks[clen] = (uint32_t)next;  // the draft extends the lookup context, not the index
      out[g] = (uint32_t)next;
    }
    ++produced;
    __syncthreads();
  }
  if (threadIdx.x == 0) *n_out = produced;
}

// The n-gram drafter of a session's round (see launch_ngram_round): one CTA
// per sequence.  The index is the prompt's windows plus, per earlier round or
// fallback step, the window ending at the context's last token
// (update_ngram_index adds only that one), each entry a copy of its n + 1
// tokens (the index keeps them when a context shift drops their tokens, as
// the reference's HashMap does).  At most ng_cap entries per sequence; the
// updates past it are dropped.
__global__ void __launch_bounds__(kNgramThreads) k_ngram_round(mc::SpecState* st_all,
                                                               const uint32_t* ctx_all,
                                                               uint32_t* ng_all, int* list_all,
                                                               int ctx_stride, int ng_cap) {
  __shared__ int s_nm, s_len, s_nent, s_stop;
  __shared__ unsigned long long s_best[kNgramThreads / 32];
  __shared__ uint32_t s_tok[32 + mc::kGroupTokens];  // the key window, then the drafts
  const int z = blockIdx.x;
  mc::SpecState* st = st_all + z;
  const uint32_t* ctx = ctx_all + (size_t)z * ctx_stride;
  const int n = st->ngram, gamma = st->gamma;
  uint32_t* ng = ng_all + (size_t)z * ng_cap * (n + 1);
  int* list = list_all + (size_t)z * ng_cap;
  if (threadIdx.x == 0) {
    // a request whose budget is spent takes no more rounds (generate.rs:638)
    s_stop = (st->max_tokens > 0 && st->generated >= st->max_tokens) || n < 1 || n > 32;
    const int len = st->ctx_len;
    if (!s_stop && len > st->ng_last_len) {  // update_ngram_index after the last round
      if (len >= n + 1 && st->ng_len < ng_cap) {
        uint32_t* e = ng + (size_t)st->ng_len * (n + 1);
        for (int q = 0; q <= n; ++q) e[q] = ctx[len - (n + 1) + q];
        st->ng_len += 1;
      }
      st->ng_last_len = len;
    }
    s_len = len;
    s_nent = st->ng_len;
  }
  __syncthreads();
  if (s_stop) return;
  const int len = s_len;
  const int base = len - n;  // s_tok[i] holds context position base + i
  if (threadIdx.x < n) s_tok[threadIdx.x] = base + (int)threadIdx.x >= 0 ? ctx[base + threadIdx.x] : 0u;
  __syncthreads();
  int produced = 0;
  for (int g = 0; g < gamma; ++g) {
    if (len + g < n) break;  // a short key matches no n-token key (block-uniform)
    const long long next = ngram_step([&](int e) { return ng + (size_t)e * (n + 1); }, s_nent, n,
                                      s_tok + g, list, &s_nm, s_best);
    if (next < 0) break;  // block-uniform
    if (threadIdx.x == 0) s_tok[n + g] = (uint32_t)next;
    ++produced;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    st->n_draft = produced;
    for (int j = 0; j < mc::kGroupTokens; ++j)
      st->dkeys[j] = j < produced ? argmax_key(0.0f, s_tok[n + j]) : 0ull;
  }
}

#define CK(expr)                                                                        \
  do {                                                                                  \
    cudaError_t e_ = (expr);                                                            \
    if (e_ != cudaSuccess)                                                              \
      return set_err(MC_E_CUDA, "%s: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, \
                     __LINE__);                                                         \
  } while (0)

const mc_tensor_desc* find_desc(const mc_tensor_desc* t, size_t n, const char* name) {
  for (size_t i = 0; i < n; ++i)
    if (t[i].name && !strcmp(t[i].name, name)) return &t[i];
  return nullptr;
}

}  // namespace

struct mc_mlp_drafter {
  int dev = 0;
  int V = 0, d = 0, dh = 0;
  float *embed = nullptr, *w1 = nullptr, *b1 = nullptr, *w2 = nullptr, *b2 = nullptr;
  float* hid = nullptr;
  uint32_t* first = nullptr;
  unsigned long long* keys = nullptr;  // [kGroupTokens] argmax keys of the steps
  cudaStream_t stream = nullptr;
  std::vector<void*> allocs;
};

struct mc_ngram_drafter {
  int dev = 0;
  int n = 3;
  int cap = 0;  // history tokens
  uint32_t* toks = nullptr;  // [cap + kGroupTokens]
  int* list = nullptr;       // [cap]
  uint32_t* out = nullptr;   // [kGroupTokens]
  int* n_out = nullptr;
  uint32_t* h_buf = nullptr; // pinned staging
  cudaStream_t stream = nullptr;
};

// gamma draft steps (FC1 + ReLU, then FC2 + argmax) for n_seq sequences
static cudaError_t mlp_steps(const mc_mlp_drafter* m, const MlpIo& io, int n_seq, int gamma,
                             float* hid, cudaStream_t stream) {
  const size_t smem1 = (size_t)m->d * sizeof(float), smem2 = (size_t)m->dh * sizeof(float);
  const dim3 g1((m->dh + kMlpFc1Threads - 1) / kMlpFc1Threads, n_seq);
  const dim3 g2((m->V + kMlpFc2Threads - 1) / kMlpFc2Threads, n_seq);
  for (int s = 0; s < gamma; ++s) {
    k_mlp_fc1<<<g1, kMlpFc1Threads, smem1, stream>>>(m->embed, m->w1, m->b1, m->V, m->d, m->dh,
                                                      io, s, hid);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    k_mlp_fc2<<<g2, kMlpFc2Threads, smem2, stream>>>(m->w2, m->b2, m->V, m->d, m->dh, io, s, hid);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

namespace mc {
// The MLP drafter's gamma steps for every sequence of a session's round:
// tokens from the contexts, keys into st[z].dkeys, hid: n_seq x dh floats.
cudaError_t mlp_round(const mc_mlp_drafter* m, SpecState* st, const uint32_t* ctx, int ctx_stride,
                      int n_seq, int gamma, float* hid, cudaStream_t stream) {
  const MlpIo io{nullptr, nullptr, st, ctx, ctx_stride};
  return mlp_steps(m, io, n_seq, gamma, hid, stream);
}
int mlp_device(const mc_mlp_drafter* m) { return m->dev; }
int mlp_vocab(const mc_mlp_drafter* m) { return m->V; }
int mlp_hidden(const mc_mlp_drafter* m) { return m->dh; }

cudaError_t launch_ngram_round(SpecState* st, const uint32_t* ctx, uint32_t* ng, int* list,
                               int ctx_stride, int ng_cap, int n_seq, cudaStream_t s) {
  k_ngram_round<<<n_seq, kNgramThreads, 0, s>>>(st, ctx, ng, list, ctx_stride, ng_cap);
  return cudaGetLastError();
}
}  // namespace mc

static void mlp_free(mc_mlp_drafter* m) {
  cudaSetDevice(m->dev);
  if (m->stream) cudaStreamDestroy(m->stream);
  for (void* p : m->allocs) cudaFree(p);
  delete m;
}

extern "C" mc_status mc_mlp_draft_create(const mc_tensor_desc* tensors, size_t n, int32_t device,
                                         mc_mlp_drafter** out) {
  if (!tensors || !out) return set_err(MC_E_INVALID, "null argument");
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
    return set_err(MC_E_CUDA, "no CUDA device %d", device);
  // draft.rs:48-86: draft.embed.weight, else the target's embedding
  const mc_tensor_desc* te = find_desc(tensors, n, "draft.embed.weight");
  if (!te) te = find_desc(tensors, n, "transformer.wte.weight");
  if (!te) te = find_desc(tensors, n, "model.embed_tokens.weight");
  const mc_tensor_desc* t1 = find_desc(tensors, n, "draft.fc1.weight");
  const mc_tensor_desc* c1 = find_desc(tensors, n, "draft.fc1.bias");
  const mc_tensor_desc* t2 = find_desc(tensors, n, "draft.fc2.weight");
  const mc_tensor_desc* c2 = find_desc(tensors, n, "draft.fc2.bias");
  if (!te || !t1 || !c1 || !t2 || !c2)
    return set_err(MC_E_INVALID, "MLP draft tensors missing (draft.fc1/fc2 weight and bias, an embedding)");
  for (const mc_tensor_desc* t : {te, t1, c1, t2, c2})
    if (t->dtype != MC_DTYPE_F32 || !t->data)
      return set_err(MC_E_DTYPE, "MLP draft tensor %s must be f32", t->name);
  if (te->ndim != 2 || t1->ndim != 2 || t2->ndim != 2)
    return set_err(MC_E_SHAPE, "MLP draft matrices must be 2-D");
  const int V = (int)t2->shape[0], dh = (int)t2->shape[1], d = (int)te->shape[1];
  if (V <= 0 || dh <= 0 || d <= 0 || t1->shape[0] != dh || t1->shape[1] != d ||
      c1->shape[0] != dh || c2->shape[0] != V || te->shape[0] != V)
    return set_err(MC_E_SHAPE, "MLP draft shapes: embed %lldx%lld, fc1 %lldx%lld, fc2 %lldx%lld",
                   (long long)te->shape[0], (long long)te->shape[1], (long long)t1->shape[0],
                   (long long)t1->shape[1], (long long)t2->shape[0], (long long)t2->shape[1]);
  if ((size_t)d * sizeof(float) > 96 * 1024 || (size_t)dh * sizeof(float) > 48 * 1024)
    return set_err(MC_E_SHAPE, "MLP draft widths %d / %d above the staging limit", d, dh);
  mc_mlp_drafter* m = new mc_mlp_drafter();
  m->dev = device;
  m->V = V;
  m->d = d;
  m->dh = dh;
  cudaSetDevice(device);
  auto up = [&](const mc_tensor_desc* t, size_t count, float** dst) -> cudaError_t {
    cudaError_t e = cudaMalloc(dst, count * sizeof(float));
    if (e != cudaSuccess) return e;
    m->allocs.push_back(*dst);
    return cudaMemcpy(*dst, t->data, count * sizeof(float),
                      t->location == MC_MEM_DEVICE ? cudaMemcpyDeviceToDevice
                                                   : cudaMemcpyHostToDevice);
  };
  cudaError_t e = up(te, (size_t)V * d, &m->embed);
  if (e == cudaSuccess) e = up(t1, (size_t)dh * d, &m->w1);
  if (e == cudaSuccess) e = up(c1, (size_t)dh, &m->b1);
  if (e == cudaSuccess) e = up(t2, (size_t)V * dh, &m->w2);
  if (e == cudaSuccess) e = up(c2, (size_t)V, &m->b2);
  if (e == cudaSuccess && (e = cudaMalloc(&m->hid, (size_t)dh * sizeof(float))) == cudaSuccess)
    m->allocs.push_back(m->hid);
  if (e == cudaSuccess && (e = cudaMalloc(&m->first, sizeof(uint32_t))) == cudaSuccess)
    m->allocs.push_back(m->first);
  if (e == cudaSuccess &&
      (e = cudaMalloc(&m->keys, mc::kGroupTokens * sizeof(unsigned long long))) == cudaSuccess)
    m->allocs.push_back(m->keys);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess && d * sizeof(float) > 48 * 1024)
    e = cudaFuncSetAttribute(k_mlp_fc1, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(d * sizeof(float)));
  if (e != cudaSuccess) {
    mlp_free(m);
    return set_err(MC_E_CUDA, "MLP draft set-up: %s", cudaGetErrorString(e));
  }
  *out = m;
  return MC_OK;
}

extern "C" mc_status mc_mlp_draft_destroy(mc_mlp_drafter* m) {
  if (m) mlp_free(m);
  return MC_OK;
}

extern "C" mc_status mc_mlp_draft(mc_mlp_drafter* m, const uint32_t* context, int32_t n,
                                  int32_t gamma, uint32_t* out, int32_t* n_out) {
  if (!m || !out || !n_out || n < 0 || gamma < 0 || (n > 0 && !context))
    return set_err(MC_E_INVALID, "bad arguments");
  if (gamma > mc::kGroupTokens)
    return set_err(MC_E_INVALID, "gamma %d above %d", gamma, mc::kGroupTokens);
  *n_out = 0;
  if (gamma == 0) return MC_OK;
  CK(cudaSetDevice(m->dev));
  const uint32_t cur = n > 0 ? context[n - 1] : 0u;  // draft.rs:130
  CK(cudaMemcpyAsync(m->first, &cur, sizeof(cur), cudaMemcpyHostToDevice, m->stream));
  CK(cudaMemsetAsync(m->keys, 0, (size_t)gamma * sizeof(unsigned long long), m->stream));
  const MlpIo io{m->first, m->keys, nullptr, nullptr, 0};
  CK(mlp_steps(m, io, 1, gamma, m->hid, m->stream));
  unsigned long long keys[mc::kGroupTokens];
  CK(cudaMemcpyAsync(keys, m->keys, (size_t)gamma * sizeof(unsigned long long),
                     cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  for (int s = 0; s < gamma; ++s) out[s] = key_index(keys[s]);
  *n_out = gamma;
  return MC_OK;
}

extern "C" mc_status mc_ngram_draft_create(int32_t ngram, int32_t max_tokens, int32_t device,
                                           mc_ngram_drafter** out) {
  if (!out || ngram < 1 || max_tokens < 1) return set_err(MC_E_INVALID, "bad arguments");
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
    return set_err(MC_E_CUDA, "no CUDA device %d", device);
  mc_ngram_drafter* g = new mc_ngram_drafter();
  g->dev = device;
  g->n = ngram;
  g->cap = max_tokens;
  cudaSetDevice(device);
  cudaError_t e = cudaMalloc(&g->toks, ((size_t)max_tokens + mc::kGroupTokens) * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMalloc(&g->list, (size_t)max_tokens * sizeof(int));
  if (e == cudaSuccess) e = cudaMalloc(&g->out, mc::kGroupTokens * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMalloc(&g->n_out, sizeof(int));
  if (e == cudaSuccess) e = cudaMallocHost(&g->h_buf, (size_t)max_tokens * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&g->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    mc_ngram_draft_destroy(g);
    return set_err(MC_E_OOM, "n-gram draft set-up: %s", cudaGetErrorString(e));
  }
  *out = g;
  return MC_OK;
}

extern "C" mc_status mc_ngram_draft_destroy(mc_ngram_drafter* g) {
  if (!g) return MC_OK;
  cudaSetDevice(g->dev);
  if (g->stream) cudaStreamDestroy(g->stream);
  cudaFree(g->toks);
  cudaFree(g->list);
  cudaFree(g->out);
  cudaFree(g->n_out);
  if (g->h_buf) cudaFreeHost(g->h_buf);
  delete g;
  return MC_OK;
}

extern "C" mc_status mc_ngram_draft(mc_ngram_drafter* g, const uint32_t* tokens, int32_t n_tokens,
                                    int32_t gamma, uint32_t* out, int32_t* n_out) {
  if (!g || !out || !n_out || n_tokens < 0 || gamma < 0 || (n_tokens > 0 && !tokens))
    return set_err(MC_E_INVALID, "bad arguments");
  if (gamma > mc::kGroupTokens)
    return set_err(MC_E_INVALID, "gamma %d above %d", gamma, mc::kGroupTokens);
  if (n_tokens > g->cap)
    return set_err(MC_E_CAPACITY, "history of %d tokens above the drafter's %d", n_tokens, g->cap);
  *n_out = 0;
  if (gamma == 0 || n_tokens == 0) return MC_OK;
  CK(cudaSetDevice(g->dev));
  memcpy(g->h_buf, tokens, (size_t)n_tokens * sizeof(uint32_t));
  CK(cudaMemcpyAsync(g->toks, g->h_buf, (size_t)n_tokens * sizeof(uint32_t),
                     cudaMemcpyHostToDevice, g->stream));
  k_ngram_draft<<<1, kNgramThreads, 0, g->stream>>>(g->toks, n_tokens, g->n, gamma, g->list,
                                                    g->out, g->n_out);
  CK(cudaGetLastError());
  int produced = 0;
  CK(cudaMemcpyAsync(&produced, g->n_out, sizeof(int), cudaMemcpyDeviceToHost, g->stream));
  uint32_t buf[mc::kGroupTokens];
  CK(cudaMemcpyAsync(buf, g->out, (size_t)gamma * sizeof(uint32_t), cudaMemcpyDeviceToHost,
                     g->stream));
  CK(cudaStreamSynchronize(g->stream));
  for (int i = 0; i < produced; ++i) out[i] = buf[i];
  *n_out = produced;
  return MC_OK;
}
