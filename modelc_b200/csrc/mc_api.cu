// mc_api.cu -- host side of the C ABI (include/modelc_cuda.h): weight
// loading and repacking, per-request sessions (paged KV, device-resident
// speculative state), forward enqueue, and the CUDA-graph speculative round.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <dlfcn.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "mc_internal.cuh"
#include "modelc_cuda.h"

using namespace mc;

// ------------------------------------------------------------------ errors
static thread_local std::string g_err;

static mc_status set_err(mc_status st, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return st;
}

namespace mc {
// The calling thread's error message, for the library's other sources.
mc_status set_error(mc_status st, const char* msg) {
  g_err = msg;
  return st;
}
}  // namespace mc

#define CK(call)                                                                    \
  do {                                                                              \
    cudaError_t e_ = (call);                                                        \
    if (e_ != cudaSuccess)                                                          \
      return set_err(e_ == cudaErrorMemoryAllocation ? MC_E_OOM : MC_E_CUDA,        \
                     "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__,     \
                     __LINE__);                                                     \
  } while (0)

#define CKS(expr)                  \
  do {                             \
    mc_status s_ = (expr);         \
    if (s_ != MC_OK) return s_;    \
  } while (0)

extern "C" size_t mc_last_error(char* buf, size_t cap) {
  if (buf && cap) {
    size_t n = std::min(cap - 1, g_err.size());
    memcpy(buf, g_err.data(), n);
    buf[n] = 0;
  }
  return g_err.size();
}

extern "C" const char* mc_version(void) { return "modelc_b200 0.1 (sm_100a)"; }

static mc_status check_device(int device) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0)
    return set_err(MC_E_CUDA, "no CUDA device available (%s)", cudaGetErrorString(e));
  if (device < 0 || device >= n) return set_err(MC_E_INVALID, "device %d out of range", device);
  cudaDeviceProp p;
  CK(cudaGetDeviceProperties(&p, device));
  if (p.major != 10)
    return set_err(MC_E_CUDA, "device %d is sm_%d%d; this library is built for sm_100a", device,
                   p.major, p.minor);
  CK(cudaSetDevice(device));
  return MC_OK;
}

// ------------------------------------------------------------------ memory
struct Allocs {
  std::vector<void*> ptrs;
  size_t bytes = 0;
  template <class T>
  mc_status alloc(T** p, size_t n) {
    void* q = nullptr;
    size_t b = std::max<size_t>(n * sizeof(T), 16);
    cudaError_t e = cudaMalloc(&q, b);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return set_err(MC_E_OOM, "cudaMalloc(%zu) failed: %s", b, cudaGetErrorString(e));
    }
    ptrs.push_back(q);
    bytes += b;
    *p = (T*)q;
    return MC_OK;
  }
  void free_all() {
    for (void* p : ptrs) cudaFree(p);
    ptrs.clear();
    bytes = 0;
  }
};

static inline int round_up(int x, int m) { return (x + m - 1) / m * m; }

// ------------------------------------------------------------------ NCCL
// Loaded on first use (tensor parallelism only) from the process's
// libnccl.so.2, so single-GPU users need no NCCL.  Types restated from the
// NCCL API: an opaque communicator, a 128-byte unique id, int enums.
namespace nccl {
typedef void* Comm;
struct UniqueId {
  char internal[128];
};
constexpr int kFloat32 = 7, kUint64 = 5, kSum = 0, kMax = 2;
typedef int (*GetUniqueIdFn)(UniqueId*);
typedef int (*CommInitRankFn)(Comm*, int, UniqueId, int);
typedef int (*AllReduceFn)(const void*, void*, size_t, int, int, Comm, cudaStream_t);
typedef int (*CommDestroyFn)(Comm);
typedef const char* (*ErrorStringFn)(int);
struct Api {
  GetUniqueIdFn get_unique_id = nullptr;
  CommInitRankFn comm_init_rank = nullptr;
  AllReduceFn all_reduce = nullptr;
  CommDestroyFn comm_destroy = nullptr;
  ErrorStringFn error_string = nullptr;
};
static Api g_api;
static std::mutex g_mu;

static mc_status load() {
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_api.all_reduce) return MC_OK;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the one torch loaded
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!h) return set_err(MC_E_NCCL, "libnccl.so.2 not found: %s", dlerror());
  Api a;
  a.get_unique_id = (GetUniqueIdFn)dlsym(h, "ncclGetUniqueId");
  a.comm_init_rank = (CommInitRankFn)dlsym(h, "ncclCommInitRank");
  a.all_reduce = (AllReduceFn)dlsym(h, "ncclAllReduce");
  a.comm_destroy = (CommDestroyFn)dlsym(h, "ncclCommDestroy");
  a.error_string = (ErrorStringFn)dlsym(h, "ncclGetErrorString");
  if (!a.get_unique_id || !a.comm_init_rank || !a.all_reduce || !a.comm_destroy)
    return set_err(MC_E_NCCL, "libnccl.so.2 lacks the expected entry points");
  g_api = a;
  return MC_OK;
}

static mc_status check(int r, const char* what) {
  if (r == 0) return MC_OK;
  return set_err(MC_E_NCCL, "%s: %s", what,
                 g_api.error_string ? g_api.error_string(r) : "nccl error");
}
}  // namespace nccl

// ------------------------------------------------------------------ packed matrices
struct PMat {
  int N = 0, K = 0;  // logical rows / cols
  int n_stripes = 0, KB = 0;
  int fmt = WF_I8;
  int4* w = nullptr;
  float* scale = nullptr;      // WF_I8 row scales
  uint32_t* qscale = nullptr;  // WF_Q4 block scales
  int4* wtc = nullptr;         // WF_I8: copy in the tcgen05 operand layout (9..16 tokens)
  long long algo_bytes = 0;  // codes + scales actually used
};

// k-split of a tcgen05 GEMM: enough CTAs to fill the SMs, each with at least
// 16 k-steps; the splits of a tile form one cluster (at most 8 CTAs).
static int tc_ksplit(const PMat& W, int nsm) {
  const int tiles = (W.n_stripes + 7) / 8;
  int k = std::max(1, nsm / std::max(tiles, 1));
  return std::max(1, std::min({k, W.KB / 16, kTcMaxSplit}));
}

// Projections run on the tcgen05 tensor cores when the matrix has the
// canonical-layout copy (int8 weights) and either more than 16 tokens (the
// GEMV would stream the weights once per 16) or 9..16 tokens and at least
// 8192 rows (64 tiles of 128): below that the few tiles and their k-split
// merges are latency-bound and the GEMV is faster (measured 27 vs 34 us at
// 4096x4096).
static bool use_tc(const PMat& W, int M) {
  if (!W.wtc || M > kMaxTokens) return false;
  if (M > kGroupTokens) return true;
  return M > 8 && W.n_stripes >= 512;
}

// The GEMV variant of a matrix: int8 matrices of at least 96 MiB (the
// 8B-shape gate/up projection and LM head) stream their weights through the
// shared-memory ring, where a deeper stream pays; smaller ones keep register
// batches, whose first batch before the dependency wait costs the producing
// encoder less.
#ifndef MC_RING_MIN_MB
#define MC_RING_MIN_MB 96
#endif
constexpr long long kRingMinBytes = (long long)MC_RING_MIN_MB << 20;
static int gemv_wf(const PMat& W) {
  if (W.fmt == WF_I8 && (long long)W.n_stripes * W.KB * kFragBytes >= kRingMinBytes)
    return WF_I8R;
  return W.fmt;
}

// CTAs per GEMV launch.  q4_0 partial sums are f32 and the grid sets their
// k-split, so a q4_0 grid must not depend on the token count: it uses the
// smallest occupancy over all token tiles.
#ifndef MC_GEMV_MAX_BPS
#define MC_GEMV_MAX_BPS 0  // 0: as many CTAs per SM as occupancy allows
#endif
template <class BpsFn>
static int gemv_grid(const PMat& W, int nsm, int nt, BpsFn bps) {
  int b = bps(nt);
  if (W.fmt == WF_Q4)
    for (int t : {1, 2, 3, 6}) b = std::min(b, bps(t));
  if (MC_GEMV_MAX_BPS > 0) b = std::min(b, MC_GEMV_MAX_BPS);
  return std::min(W.n_stripes, nsm * std::max(b, 1));
}

// One projection of M <= kMaxTokens tokens whose digits the encoder wrote
// for it: the tcgen05 GEMM, or the GEMV once per group of 16 tokens (each
// group's digits are their own operand block).  a carries the epilogue, the
// workspace and the next-matrix prefetch; the prefetch goes with the last
// group.
template <class BpsFn>
static cudaError_t run_projection(const PMat& W, int epi, int M, GemvArgs a, int nsm,
                                  cudaStream_t st, BpsFn bps) {
  a.w = W.w;
  a.scale = W.scale;
  a.qscale = W.qscale;
  a.KB = W.KB;
  a.n_stripes = W.n_stripes;
  if (use_tc(W, M)) {
    a.wtc = W.wtc;
    a.M = M;
    a.m0 = 0;
    return launch_gemm_tc(a, epi, tc_ksplit(W, nsm), st, true);
  }
  const int nt = nt_for_tokens(M);
  const int G = groups_for_tokens(M);
  const uint8_t* x = a.x;
  const int* xexp = a.xexp;
  const void* next_w = a.next_w;
  const size_t group_bytes = (size_t)W.KB * 64 * nt * 4;
  const int grid = gemv_grid(W, nsm, nt, bps);
  for (int g = 0; g < G; ++g) {
    a.x = x + g * group_bytes;
    a.xexp = xexp + g * kGroupTokens;
    a.m0 = g * kGroupTokens;
    a.M = std::min(kGroupTokens, M - a.m0);
    a.next_w = (g == G - 1) ? next_w : nullptr;
    cudaError_t e = launch_gemv(a, epi, nt, gemv_wf(W), grid, st, true);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Source matrix staged on the device: int8 [rows][cols] + f32 row scales, or
// q4_0 blocks [rows][cols/32][18] (fmt WF_Q4).
struct SrcI8 {
  int rows = 0, cols = 0;
  int fmt = WF_I8;
  int8_t* q = nullptr;
  float* s = nullptr;
  uint8_t* q4 = nullptr;
  std::vector<void*> tmp;
  ~SrcI8() {
    for (void* p : tmp) cudaFree(p);
  }
};

// f32 rows accepted only when exactly representable as int8 codes times a
// power-of-two row scale (e.g. the reference's integer-valued test fixtures).
static bool f32_row_exact_i8(const float* x, int K, int8_t* q, float* scale) {
  float amax = 0.0f;
  for (int c = 0; c < K; ++c) {
    if (!isfinite(x[c])) return false;
    amax = fmaxf(amax, fabsf(x[c]));
  }
  if (amax == 0.0f) {
    memset(q, 0, K);
    *scale = 1.0f;
    return true;
  }
  int p = -160;
  while (ldexpf(127.0f, p) < amax) ++p;
  const float s = ldexpf(1.0f, p);
  for (int c = 0; c < K; ++c) {
    const float v = ldexpf(x[c], -p);
    if (v != rintf(v) || fabsf(v) > 127.0f) return false;
    q[c] = (int8_t)v;
  }
  *scale = s;
  return true;
}

static mc_status stage_matrix(const mc_tensor_desc* t, SrcI8* out) {
  if (t->ndim != 2) return set_err(MC_E_SHAPE, "%s: expected a matrix", t->name);
  const int rows = (int)t->shape[0], cols = (int)t->shape[1];
  out->rows = rows;
  out->cols = cols;
  const size_t n = (size_t)rows * cols;
  if (t->dtype == MC_DTYPE_Q4_0) {
    // blocks run along each row (dequant.rs:33-44 is flat over elements, so a
    // row that is not a whole number of blocks would share a block)
    if (cols % 32)
      return set_err(MC_E_SHAPE, "%s: q4_0 needs in_features %% 32 == 0 (got %d)", t->name, cols);
    const size_t bytes = n / 32 * kQ4BlockBytes;
    void* q4 = nullptr;
    CK(cudaMalloc(&q4, std::max<size_t>(bytes, 16)));
    out->tmp.push_back(q4);
    out->q4 = (uint8_t*)q4;
    out->fmt = WF_Q4;
    CK(cudaMemcpy(q4, t->data, bytes,
                  t->location == MC_MEM_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice));
    return MC_OK;
  }
  void* q = nullptr;
  void* s = nullptr;
  CK(cudaMalloc(&q, std::max<size_t>(n, 16)));
  out->tmp.push_back(q);
  CK(cudaMalloc(&s, std::max<size_t>((size_t)rows * 4, 16)));
  out->tmp.push_back(s);
  out->q = (int8_t*)q;
  out->s = (float*)s;
  const cudaMemcpyKind kind =
      t->location == MC_MEM_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  switch (t->dtype) {
    case MC_DTYPE_I8_ROW:
      if (!t->scales) return set_err(MC_E_INVALID, "%s: I8_ROW needs scales", t->name);
      CK(cudaMemcpy(q, t->data, n, kind));
      CK(cudaMemcpy(s, t->scales, (size_t)rows * 4, kind));
      break;
    case MC_DTYPE_I8_TENSOR: {
      if (!t->scales) return set_err(MC_E_INVALID, "%s: I8_TENSOR needs a scale", t->name);
      float sc = 0.0f;
      CK(cudaMemcpy(&sc, t->scales, 4, t->location == MC_MEM_DEVICE ? cudaMemcpyDeviceToHost
                                                                    : cudaMemcpyHostToHost));
      std::vector<float> sv(rows, sc);
      CK(cudaMemcpy(q, t->data, n, kind));
      CK(cudaMemcpy(s, sv.data(), (size_t)rows * 4, cudaMemcpyHostToDevice));
      break;
    }
    case MC_DTYPE_F32: {
      std::vector<float> host;
      const float* src = (const float*)t->data;
      if (t->location == MC_MEM_DEVICE) {
        host.resize(n);
        CK(cudaMemcpy(host.data(), t->data, n * 4, cudaMemcpyDeviceToHost));
        src = host.data();
      }
      std::vector<int8_t> hq(n);
      std::vector<float> hs(rows);
      for (int r = 0; r < rows; ++r)
        if (!f32_row_exact_i8(src + (size_t)r * cols, cols, hq.data() + (size_t)r * cols, &hs[r]))
          return set_err(MC_E_DTYPE,
                         "%s: f32 matrix row %d is not exactly representable as int8 "
                         "codes with a power-of-two scale; quantize it (int8 rows) first",
                         t->name, r);
      CK(cudaMemcpy(q, hq.data(), n, cudaMemcpyHostToDevice));
      CK(cudaMemcpy(s, hs.data(), (size_t)rows * 4, cudaMemcpyHostToDevice));
      break;
    }
    default:
      return set_err(MC_E_DTYPE, "%s: dtype %d is not supported by this build", t->name,
                     t->dtype);
  }
  return MC_OK;
}

static mc_status stage_vector(const mc_tensor_desc* t, int n_expect, std::vector<float>* out) {
  const int n = (int)(t->ndim == 1 ? t->shape[0] : t->shape[0] * t->shape[1]);
  if (n != n_expect) return set_err(MC_E_SHAPE, "%s: %d elements, expected %d", t->name, n, n_expect);
  out->resize(n);
  const cudaMemcpyKind kind =
      t->location == MC_MEM_DEVICE ? cudaMemcpyDeviceToHost : cudaMemcpyHostToHost;
  if (t->dtype == MC_DTYPE_F32) {
    CK(cudaMemcpy(out->data(), t->data, (size_t)n * 4, kind));
  } else if (t->dtype == MC_DTYPE_I8_TENSOR || t->dtype == MC_DTYPE_I8_ROW) {
    std::vector<int8_t> q(n);
    float sc = 0.0f;
    CK(cudaMemcpy(q.data(), t->data, n, kind));
    CK(cudaMemcpy(&sc, t->scales, 4, kind));
    for (int i = 0; i < n; ++i) (*out)[i] = (float)q[i] * sc;  // model.rs:182-185
  } else {
    return set_err(MC_E_DTYPE, "%s: unsupported vector dtype", t->name);
  }
  return MC_OK;
}

// Concatenate staged sources row-wise into one device int8 matrix.
static mc_status concat_rows(const std::vector<const SrcI8*>& parts, SrcI8* out) {
  int rows = 0;
  const int cols = parts[0]->cols;
  for (auto* p : parts) {
    if (p->cols != cols) return set_err(MC_E_SHAPE, "fused projections disagree on input width");
    if (p->fmt != parts[0]->fmt)
      return set_err(MC_E_DTYPE, "fused projections (q/k/v or gate/up) must share one dtype");
    rows += p->rows;
  }
  out->rows = rows;
  out->cols = cols;
  if (parts[0]->fmt == WF_Q4) {
    const size_t row_bytes = (size_t)cols / 32 * kQ4BlockBytes;
    void* q4 = nullptr;
    CK(cudaMalloc(&q4, std::max<size_t>((size_t)rows * row_bytes, 16)));
    out->tmp.push_back(q4);
    out->q4 = (uint8_t*)q4;
    out->fmt = WF_Q4;
    size_t r0 = 0;
    for (auto* p : parts) {
      CK(cudaMemcpy(out->q4 + r0 * row_bytes, p->q4, (size_t)p->rows * row_bytes,
                    cudaMemcpyDeviceToDevice));
      r0 += p->rows;
    }
    return MC_OK;
  }
  void* q = nullptr;
  void* s = nullptr;
  CK(cudaMalloc(&q, std::max<size_t>((size_t)rows * cols, 16)));
  out->tmp.push_back(q);
  CK(cudaMalloc(&s, std::max<size_t>((size_t)rows * 4, 16)));
  out->tmp.push_back(s);
  out->q = (int8_t*)q;
  out->s = (float*)s;
  size_t r0 = 0;
  for (auto* p : parts) {
    CK(cudaMemcpy((int8_t*)q + r0 * cols, p->q, (size_t)p->rows * cols, cudaMemcpyDeviceToDevice));
    CK(cudaMemcpy((float*)s + r0, p->s, (size_t)p->rows * 4, cudaMemcpyDeviceToDevice));
    r0 += p->rows;
  }
  return MC_OK;
}

// Pack src through row_map (size n_stripes*16) and col_map (size KB*32).
static mc_status pack_matrix(const SrcI8& src, const std::vector<int>& row_map,
                             const std::vector<int>& col_map, int n_real_rows, int n_real_cols,
                             Allocs& al, PMat* out) {
  out->n_stripes = (int)row_map.size() / 16;
  out->KB = (int)col_map.size() / 32;
  out->N = n_real_rows;
  out->K = n_real_cols;
  out->algo_bytes = (long long)n_real_rows * n_real_cols + 4ll * n_real_rows;
  if (src.fmt == WF_Q4) {
    // q4_0 keeps its blocks: a contiguous, block-aligned column range only
    const int c0 = col_map.empty() ? 0 : col_map[0];
    bool ok = c0 >= 0 && c0 % 32 == 0 && col_map.size() % 32 == 0 &&
              c0 + (long long)col_map.size() <= src.cols;
    for (size_t c = 0; ok && c < col_map.size(); ++c) ok = col_map[c] == c0 + (int)c;
    if (!ok)
      return set_err(MC_E_SHAPE,
                     "q4_0 matrix %dx%d cannot be re-laid-out (head_dim must be a multiple of "
                     "16, and tensor-parallel slices multiples of 32 columns)", src.rows, src.cols);
    out->fmt = WF_Q4;
    out->algo_bytes = (long long)n_real_rows * n_real_cols / 32 * kQ4BlockBytes;
    const size_t units = (size_t)out->n_stripes * out->KB * 32;
    CKS(al.alloc(&out->w, units / 2));  // 8 bytes per unit (int4 = 16 bytes)
    CKS(al.alloc(&out->qscale, (size_t)out->n_stripes * out->KB * 8));
    int* drm = nullptr;
    CK(cudaMalloc(&drm, row_map.size() * 4));
    cudaMemcpy(drm, row_map.data(), row_map.size() * 4, cudaMemcpyHostToDevice);
    cudaError_t e = launch_pack_q4(src.q4, drm, out->n_stripes, out->KB, src.cols / 32, c0 / 32,
                                   reinterpret_cast<uint2*>(out->w), out->qscale, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaFree(drm);
    if (e != cudaSuccess) return set_err(MC_E_CUDA, "q4_0 packing failed: %s", cudaGetErrorString(e));
    return MC_OK;
  }
  CKS(al.alloc(&out->w, (size_t)out->n_stripes * out->KB * 32));
  CKS(al.alloc(&out->scale, (size_t)out->n_stripes * 16));
  int* drm = nullptr;
  int* dcm = nullptr;
  CK(cudaMalloc(&drm, row_map.size() * 4));
  CK(cudaMalloc(&dcm, col_map.size() * 4));
  cudaMemcpy(drm, row_map.data(), row_map.size() * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(dcm, col_map.data(), col_map.size() * 4, cudaMemcpyHostToDevice);
  cudaError_t e = launch_pack_int8(src.q, src.cols, src.s, drm, dcm, out->n_stripes, out->KB,
                                   out->w, out->scale, 0);
  const int n_tiles = (out->n_stripes + 7) / 8;
  mc_status st = MC_OK;
  // swizzled tcgen05 copy: 128 x 128 bytes (1024 int4) per tile and K atom
  if (e == cudaSuccess) st = al.alloc(&out->wtc, (size_t)n_tiles * tc_atoms(out->KB) * 1024);
  if (e == cudaSuccess && st == MC_OK)
    e = launch_pack_tc(src.q, src.cols, drm, dcm, (int)row_map.size(), n_tiles, out->KB, out->wtc, 0);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaFree(drm);
  cudaFree(dcm);
  if (st != MC_OK) return st;
  if (e != cudaSuccess) return set_err(MC_E_CUDA, "packing failed: %s", cudaGetErrorString(e));
  return MC_OK;
}

static std::vector<int> identity_map(int n_real, int n_padded) {
  std::vector<int> m(n_padded, -1);
  for (int i = 0; i < n_real && i < n_padded; ++i) m[i] = i;
  return m;
}

// ------------------------------------------------------------------ weights
struct LayerW {
  bool attn = false, mlp = false;
  float* attn_norm = nullptr;
  float* mlp_norm = nullptr;
  PMat qkv, o, gu, down;
  int sq = 0, sk = 0;
};

struct mc_weights {
  int dev = 0;
  int L = 0, d = 0, H = 0, Hkv = 0, hd = 0, half = 0, half_p = 0, hdp = 0, F = 0, V = 0;
  float theta = 10000.0f, eps = 1e-6f;
  std::vector<LayerW> layers;
  float* final_norm = nullptr;
  PMat head;
  bool has_head = false;
  int8_t* emb_q = nullptr;
  float* emb_scale = nullptr;
  uint8_t* emb_q4 = nullptr;  // q4_0 embedding blocks (emb_q unused then)
  // tensor parallelism: H, Hkv, F above are this rank's shares; the LM head
  // holds vocabulary rows [head_row0, head_row0 + V_loc)
  int tp_rank = 0, tp_world = 1;
  int V_loc = 0, head_row0 = 0;
  Allocs al;
  long long algo_bytes_per_forward = 0;  // streamed weight bytes of one forward
};

static const mc_tensor_desc* find_t(const mc_tensor_desc* ts, size_t n, const std::string& name) {
  for (size_t i = 0; i < n; ++i)
    if (ts[i].name && name == ts[i].name) return &ts[i];
  return nullptr;
}

// Padded head layout: first-half dims at [0, half), second-half dims at
// [half_p, half_p + half); a dim p of the padded head maps to a source
// index inside the real head, or -1.
static int padded_src(int p, int half, int half_p) {
  if (p < half_p) return p < half ? p : -1;
  const int j = p - half_p;
  return j < half ? half + j : -1;
}

static mc_status load_model(const mc_tensor_desc* ts, size_t n, const mc_model_cfg* cfg,
                            mc_weights* W) {
  W->L = cfg->n_layers;
  W->d = cfg->hidden;
  W->F = cfg->ffn;
  W->V = cfg->vocab;
  if (W->L < 0 || W->d <= 0 || W->V <= 0) return set_err(MC_E_INVALID, "bad model config");
  // q_proj rows define the query width (transformer.rs:944-946).
  int q_rows = W->d;
  if (W->L > 0) {
    const mc_tensor_desc* q = find_t(ts, n, "model.layers.0.self_attn.q_proj.weight");
    if (q && q->ndim == 2) q_rows = (int)q->shape[0];
  }
  if (cfg->mode == MC_MODE_REFERENCE) {
    int nh = W->d / 64;
    if (nh < 1) nh = 1;
    W->H = nh;
    W->Hkv = nh;
    W->hd = q_rows / nh;
    W->theta = 10000.0f;
    W->eps = 1e-6f;
  } else {
    W->H = cfg->n_heads;
    W->Hkv = cfg->n_kv_heads;
    W->hd = cfg->head_dim;
    W->theta = cfg->rope_theta;
    W->eps = cfg->eps;
  }
  if (W->H <= 0 || W->Hkv <= 0 || W->hd <= 0 || W->H % W->Hkv)
    return set_err(MC_E_SHAPE, "bad head geometry H=%d Hkv=%d hd=%d", W->H, W->Hkv, W->hd);
  if (W->hd % 2) return set_err(MC_E_SHAPE, "odd head_dim %d is not supported", W->hd);
  if (W->H / W->Hkv > 128)  // query rows of one attention CTA
    return set_err(MC_E_SHAPE, "query group %d too large", W->H / W->Hkv);
  W->half = W->hd / 2;
  W->half_p = round_up(W->half, 8);
  W->hdp = 2 * W->half_p;
  // tensor-parallel shard (global sizes Hg, Hkvg, Fg; local H, Hkv, F)
  const int R = cfg->tp_world > 1 ? cfg->tp_world : 1;
  const int rank = R > 1 ? cfg->tp_rank : 0;
  if (rank < 0 || rank >= R) return set_err(MC_E_INVALID, "tp_rank %d outside [0, %d)", rank, R);
  if (W->H % R || W->Hkv % R || W->F % R || W->V % R)
    return set_err(MC_E_SHAPE, "heads %d/%d, ffn %d and vocab %d must divide by tp_world %d",
                   W->H, W->Hkv, W->F, W->V, R);
  if (R > 1 && (W->F / R) % 32)
    return set_err(MC_E_SHAPE, "ffn / tp_world = %d must be a multiple of 32", W->F / R);
  const int Hg = W->H, Hkvg = W->Hkv, Fg = W->F;
  W->tp_world = R;
  W->tp_rank = rank;
  W->H = Hg / R;
  W->Hkv = Hkvg / R;
  W->F = Fg / R;
  W->V_loc = W->V / R;
  W->head_row0 = rank * W->V_loc;
  const int h0 = rank * W->H, kv0 = rank * W->Hkv, f0 = rank * W->F;
  const int H = W->H, Hkv = W->Hkv, hd = W->hd, half = W->half, half_p = W->half_p,
            hdp = W->hdp, d = W->d, F = W->F;
  Allocs& al = W->al;

  // embedding (row-major int8 for the gather)
  const mc_tensor_desc* te = find_t(ts, n, "model.embed_tokens.weight");
  SrcI8 emb;
  if (te && te->dtype == MC_DTYPE_Q4_0) {
    CKS(stage_matrix(te, &emb));
    if (emb.rows != W->V || emb.cols != d)
      return set_err(MC_E_SHAPE, "embed_tokens is %dx%d, expected %dx%d", emb.rows, emb.cols,
                     W->V, d);
    const size_t bytes = (size_t)W->V * (d / 32) * kQ4BlockBytes;
    CKS(al.alloc(&W->emb_q4, bytes));
    CK(cudaMemcpy(W->emb_q4, emb.q4, bytes, cudaMemcpyDeviceToDevice));
  } else if (te) {
    CKS(stage_matrix(te, &emb));
    if (emb.rows != W->V || emb.cols != d)
      return set_err(MC_E_SHAPE, "embed_tokens is %dx%d, expected %dx%d", emb.rows, emb.cols,
                     W->V, d);
    CKS(al.alloc(&W->emb_q, (size_t)W->V * d));
    CKS(al.alloc(&W->emb_scale, (size_t)W->V));
    CK(cudaMemcpy(W->emb_q, emb.q, (size_t)W->V * d, cudaMemcpyDeviceToDevice));
    CK(cudaMemcpy(W->emb_scale, emb.s, (size_t)W->V * 4, cudaMemcpyDeviceToDevice));
  } else {
    // token_embedding returns zeros without an embedding (generate.rs:858-862)
    CKS(al.alloc(&W->emb_q, (size_t)W->V * d));
    CKS(al.alloc(&W->emb_scale, (size_t)W->V));
    CK(cudaMemset(W->emb_q, 0, (size_t)W->V * d));
    CK(cudaMemset(W->emb_scale, 0, (size_t)W->V * 4));
  }

  auto upload_vec = [&](const char* name, int len, float** dst) -> mc_status {
    const mc_tensor_desc* t = find_t(ts, n, name);
    if (!t) {
      *dst = nullptr;
      return MC_OK;
    }
    std::vector<float> v;
    CKS(stage_vector(t, len, &v));
    CKS(al.alloc(dst, (size_t)len));
    CK(cudaMemcpy(*dst, v.data(), (size_t)len * 4, cudaMemcpyHostToDevice));
    return MC_OK;
  };

  W->layers.resize(W->L);
  long long bytes = 0;
  for (int l = 0; l < W->L; ++l) {
    LayerW& Lw = W->layers[l];
    const std::string p = "model.layers." + std::to_string(l) + ".";
    const mc_tensor_desc* tq = find_t(ts, n, p + "self_attn.q_proj.weight");
    const mc_tensor_desc* tk = find_t(ts, n, p + "self_attn.k_proj.weight");
    const mc_tensor_desc* tv = find_t(ts, n, p + "self_attn.v_proj.weight");
    const mc_tensor_desc* to = find_t(ts, n, p + "self_attn.o_proj.weight");
    Lw.attn = tq && tk && tv && to;  // llama_attention returns None otherwise (:769-772)
    if (Lw.attn) {
      CKS(upload_vec((p + "input_layernorm.weight").c_str(), d, &Lw.attn_norm));
      SrcI8 sq, sk, sv, so;
      CKS(stage_matrix(tq, &sq));
      CKS(stage_matrix(tk, &sk));
      CKS(stage_matrix(tv, &sv));
      CKS(stage_matrix(to, &so));
      if (sq.rows != Hg * hd || sk.rows != Hkvg * hd || sv.rows != Hkvg * hd || sq.cols != d ||
          so.rows != d || so.cols != Hg * hd)
        return set_err(MC_E_SHAPE, "layer %d attention shapes do not match H=%d Hkv=%d hd=%d d=%d",
                       l, Hg, Hkvg, hd, d);
      SrcI8 cat;
      CKS(concat_rows({&sq, &sk, &sv}, &cat));
      const int per_head = half_p / 8;
      Lw.sq = H * per_head;
      Lw.sk = Hkv * per_head;
      const int sv_n = Hkv * per_head;
      std::vector<int> rm((size_t)(Lw.sq + Lw.sk + sv_n) * 16, -1);
      for (int s = 0; s < Lw.sq + Lw.sk; ++s) {
        const bool isq = s < Lw.sq;
        const int s2 = isq ? s : s - Lw.sq;
        const int hh = s2 / per_head, j = s2 % per_head;
        const int base = isq ? (h0 + hh) * hd : Hg * hd + (kv0 + hh) * hd;
        for (int g = 0; g < 8; ++g) {
          const int i = 8 * j + g;
          rm[s * 16 + g] = i < half ? base + i : -1;
          rm[s * 16 + g + 8] = i < half ? base + half + i : -1;
        }
      }
      for (int s = 0; s < sv_n; ++s) {
        const int hh = s / per_head, j = s % per_head;
        for (int r = 0; r < 16; ++r) {
          const int src = padded_src(16 * j + r, half, half_p);
          rm[(Lw.sq + Lw.sk + s) * 16 + r] =
              src < 0 ? -1 : (Hg + Hkvg) * hd + (kv0 + hh) * hd + src;
        }
      }
      CKS(pack_matrix(cat, rm, identity_map(d, round_up(d, 32)), (H + 2 * Hkv) * hd, d, al,
                      &Lw.qkv));
      if (Lw.qkv.fmt == WF_I8)  // padded head rows are not algorithmic bytes
        Lw.qkv.algo_bytes = (long long)(H + 2 * Hkv) * hd * d + 4ll * (H + 2 * Hkv) * hd;
      // O projection: columns follow the padded head layout of the attention output
      std::vector<int> cm(round_up(H * hdp, 32), -1);
      for (int hh = 0; hh < H; ++hh)
        for (int pp = 0; pp < hdp; ++pp) {
          const int src = padded_src(pp, half, half_p);
          cm[hh * hdp + pp] = src < 0 ? -1 : (h0 + hh) * hd + src;
        }
      CKS(pack_matrix(so, identity_map(d, round_up(d, 16)), cm, d, H * hd, al, &Lw.o));
      bytes += Lw.qkv.algo_bytes + Lw.o.algo_bytes;
    }
    const mc_tensor_desc* tg = find_t(ts, n, p + "mlp.gate_proj.weight");
    const mc_tensor_desc* tu = find_t(ts, n, p + "mlp.up_proj.weight");
    const mc_tensor_desc* td = find_t(ts, n, p + "mlp.down_proj.weight");
    Lw.mlp = tg && tu && td;  // llama_mlp returns None otherwise (:801-803)
    if (Lw.mlp) {
      CKS(upload_vec((p + "post_attention_layernorm.weight").c_str(), d, &Lw.mlp_norm));
      SrcI8 sg, su, sdn;
      CKS(stage_matrix(tg, &sg));
      CKS(stage_matrix(tu, &su));
      CKS(stage_matrix(td, &sdn));
      if (sg.rows != Fg || su.rows != Fg || sg.cols != d || su.cols != d || sdn.rows != d ||
          sdn.cols != Fg)
        return set_err(MC_E_SHAPE, "layer %d MLP shapes do not match d=%d ffn=%d", l, d, Fg);
      SrcI8 cat;
      CKS(concat_rows({&sg, &su}, &cat));
      const int ns = (F + 7) / 8;
      std::vector<int> rm((size_t)ns * 16, -1);
      for (int s = 0; s < ns; ++s)
        for (int g = 0; g < 8; ++g) {
          const int i = 8 * s + g;
          rm[s * 16 + g] = i < F ? f0 + i : -1;
          rm[s * 16 + g + 8] = i < F ? Fg + f0 + i : -1;
        }
      CKS(pack_matrix(cat, rm, identity_map(d, round_up(d, 32)), 2 * F, d, al, &Lw.gu));
      std::vector<int> dcm = identity_map(F, round_up(F, 32));
      for (int& c : dcm)
        if (c >= 0) c += f0;
      CKS(pack_matrix(sdn, identity_map(d, round_up(d, 16)), dcm, d, F, al, &Lw.down));
      bytes += Lw.gu.algo_bytes + Lw.down.algo_bytes;
    }
  }
  CKS(upload_vec("model.norm.weight", d, &W->final_norm));
  const mc_tensor_desc* th = find_t(ts, n, "lm_head.weight");
  if (!th) th = te;  // tied head (transformer.rs:94-95)
  if (th) {
    SrcI8 sh;
    CKS(stage_matrix(th, &sh));
    if (sh.rows != W->V || sh.cols != d)
      return set_err(MC_E_SHAPE, "lm_head is %dx%d, expected %dx%d", sh.rows, sh.cols, W->V, d);
    std::vector<int> hrm = identity_map(W->V_loc, round_up(W->V_loc, 16));
    for (int& r : hrm)
      if (r >= 0) r += W->head_row0;
    CKS(pack_matrix(sh, hrm, identity_map(d, round_up(d, 32)), W->V_loc, d, al, &W->head));
    W->has_head = true;
    bytes += W->head.algo_bytes;
  }
  W->algo_bytes_per_forward = bytes;
  return MC_OK;
}

extern "C" mc_status mc_weights_load(const mc_tensor_desc* tensors, size_t n,
                                     const mc_model_cfg* cfg, int32_t device, mc_weights** out) {
  if (!tensors || !cfg || !out) return set_err(MC_E_INVALID, "null argument");
  *out = nullptr;
  CKS(check_device(device));
  mc_weights* W = new mc_weights();
  W->dev = device;
  mc_status st = load_model(tensors, n, cfg, W);
  if (st != MC_OK) {
    W->al.free_all();
    delete W;
    return st;
  }
  *out = W;
  return MC_OK;
}

extern "C" mc_status mc_weights_destroy(mc_weights* w) {
  if (!w) return MC_OK;
  cudaSetDevice(w->dev);
  w->al.free_all();
  delete w;
  return MC_OK;
}

extern "C" int64_t mc_weights_bytes(const mc_weights* w) {
  return w ? (int64_t)w->algo_bytes_per_forward : 0;
}

// ------------------------------------------------------------------ sessions
constexpr int kPage = 64;       // KV positions per page
constexpr int kMaxAttnPages = 64;  // pages one attention launch combines per request
constexpr int kChunk = kMaxTokens;  // prefill tokens per forward launch

struct KVSet {
  float* k = nullptr;
  float* v = nullptr;
  size_t layer_stride = 0;  // floats per layer
  int* page_table = nullptr;  // [requests][n_pages]
  int n_pages = 0;            // pages per request
  float* rope_cos = nullptr;
  float* rope_sin = nullptr;
};

#ifndef MC_DEFAULT_TAILS
#define MC_DEFAULT_TAILS 0
#endif
constexpr int kDefaultTails = MC_DEFAULT_TAILS;  // MODELC_CUDA_ENCODER_TAILS unset

struct mc_session {
  const mc_weights* tw = nullptr;
  const mc_weights* dw = nullptr;
  mc_spec_cfg cfg{};
  int B = 1;           // concurrent requests
  int cap = 0;         // KV capacity per request (tokens)
  int ctx_stride = 0;  // ids between the requests' contexts (and round logs)
  int dev = 0;
  int nsm = 0;
  cudaStream_t stream = nullptr;
  Allocs al;
  // shared scratch
  float* h = nullptr;
  uint8_t* xq = nullptr;
  int* xexp = nullptr;
  float* qb = nullptr;
  float* act = nullptr;
  float* logits = nullptr;
  float* dlogits = nullptr;  // draft logits of a stochastic round [kMaxTokens][V]
  int* ws = nullptr;
  int* cnt = nullptr;
  float* part_o = nullptr;
  float* part_ml = nullptr;
  int* err = nullptr;  // device flag raised by an expired bounded wait
  // activation statistics handed from each producer to the next encoder:
  // two max|x*w| slots used alternately, and per-stripe sums of squares
  unsigned* st_amax = nullptr;  // [2][kMaxTokens]
  float* st_pss = nullptr;      // [kMaxTokens][max stripes]
  int st_np_cap = 0;
  KVSet tkv, dkv;
  // device-resident speculative state, one per request
  SpecState* st = nullptr;      // [B]
  uint32_t* ctx = nullptr;      // [B][ctx_stride]
  int* acc_log = nullptr;       // [B][ctx_stride]
  unsigned long long* fkeys = nullptr;  // argmax keys of plain forwards [kMaxTokens]
  uint32_t* ids = nullptr;
  int* pos = nullptr;  // [2]: target / draft length for the plain forward API
  // host mirrors (request 0 for the plain forward API)
  int lt = 0, ld = 0;
  int prompt_len = 0;
  std::vector<int> prompt_lens;  // per request
  std::vector<uint32_t> draft_tokens;  // tokens in the draft KV (mc_draft)
  uint32_t* h_ids = nullptr;           // pinned staging
  cudaGraphExec_t round_exec = nullptr;
  cudaGraphExec_t verify_exec = nullptr;
  int round_launches = 0;
  int bps[3][6][7] = {};
  int bps_tail[3][2][7] = {};  // encoding-tail variants of RESID / SWIGLU
  // encoding tails (GemvArgs::bar, AttnArgs::bar): the grid barrier's
  // words, and which producers run them -- bit 0 the o / gate-up / down
  // GEMVs, bit 1 the attention -- from MODELC_CUDA_ENCODER_TAILS at session
  // creation (a number; 0 keeps every encoder a launch of its own; the
  // digits are the same either way)
  unsigned* gbar = nullptr;  // [2]
  int tails = kDefaultTails;
  // MIXED target cache: the originals of the tokens verify steps quantize
  // ([B][vm][L][2][Hkv * hdp]); each request's window count after its prime;
  // the window count of the plain forward API's cache
  float* mx_bak = nullptr;
  std::vector<int> mx_hot0;
  int plain_hot = 0;
  // MC_TRACE builds: timeline slots handed to the launches of one capture
  bool trace_on = false;
  int trace_next = 0;
  // tensor parallelism (target weights sharded over tp_world ranks)
  nccl::Comm comm = nullptr;
  float* tp_part = nullptr;  // [kMaxTokens][d] partial sums of o / down
  // P2P reduce region (IPC-exported; see TPArgs), peers' regions once opened
  void* tp_region = nullptr;
  size_t tp_red_bytes = 0;
  unsigned* tp_epoch = nullptr;
  int* tp_cnt_gemv = nullptr;
  int* tp_cnt_red = nullptr;
  bool tp_p2p = false;
  TPArgs tp{};
  std::vector<void*> tp_opened;  // peers' regions mapped here (CUDA IPC)
  size_t tp_keyx_off = 0, tp_kflag_off = 0;  // key slots and key flags in the region
  unsigned* tp_kepoch = nullptr;
  // limit of every bounded device wait, in nanoseconds (device word)
  long long* wait_ns = nullptr;
  bool failed = false;  // an earlier bounded wait expired: the session is unusable
  // drafters without a transformer draft: the MLP drafter (borrowed; the
  // caller keeps it alive), or, with neither, the n-gram drafter
  const mc_mlp_drafter* mlp = nullptr;
  float* mlp_hid = nullptr;  // [B][dh]
  uint32_t* ng = nullptr;    // [B][ng_cap][kNgram + 1] n-gram index entries (key, next)
  int* ng_list = nullptr;    // [B][ng_cap] n-gram scratch
  int ng_cap = 0;            // index entries per request
};

// The drafter a session's rounds run (DraftModel, draft.rs:18-21; without a
// draft model speculative_generate drafts from its trigram index,
// generate.rs:615, :642-646).
enum DraftKind { DRAFT_LLAMA = 0, DRAFT_MLP = 1, DRAFT_NGRAM = 2 };
constexpr int kNgram = 3;  // generate.rs:615: let n = 3usize
static DraftKind draft_kind(const mc_session* s) {
  return s->dw ? DRAFT_LLAMA : (s->mlp ? DRAFT_MLP : DRAFT_NGRAM);
}

static int trace_slot(mc_session* s) { return s->trace_on ? ++s->trace_next : 0; }

static int bps_of(mc_session* s, int epi, int nt, int wf, bool tail = false) {
  int& b = tail ? s->bps_tail[wf][epi == EPI_SWIGLU][nt] : s->bps[wf][epi][nt];
  if (!b) b = std::max(1, gemv_blocks_per_sm(epi, nt, wf, tail));
  return b;
}

// Paged K/V of every request: request z owns pages [z * n_pages, (z + 1) *
// n_pages), listed in row z of the page table.
static mc_status alloc_kv(mc_session* s, const mc_weights* W, KVSet* kv) {
  kv->n_pages = (s->cap + kPage - 1) / kPage;
  const int pages = kv->n_pages * s->B;
  kv->layer_stride = (size_t)pages * W->Hkv * kPage * W->hdp;
  const size_t total = kv->layer_stride * std::max(W->L, 1);
  CKS(s->al.alloc(&kv->k, total));
  CKS(s->al.alloc(&kv->v, total));
  CK(cudaMemset(kv->k, 0, total * 4));
  CK(cudaMemset(kv->v, 0, total * 4));
  CKS(s->al.alloc(&kv->page_table, (size_t)pages));
  std::vector<int> pt(pages);
  for (int i = 0; i < pages; ++i) pt[i] = i;
  CK(cudaMemcpy(kv->page_table, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice));
  // RoPE factors computed on the host with libm exactly as transformer.rs:926-927:
  // theta = pos * base^(-i/half) in f32, then sin/cos.
  const int hp = W->half_p;
  std::vector<float> c((size_t)s->cap * hp), sn((size_t)s->cap * hp);
  for (int p = 0; p < s->cap; ++p)
    for (int i = 0; i < hp; ++i) {
      float cv = 1.0f, sv = 0.0f;
      if (i < W->half) {
        const float expo = -(float)i / (float)W->half;
        const float theta = (float)p * powf(W->theta, expo);
        cv = cosf(theta);
        sv = sinf(theta);
      }
      c[(size_t)p * hp + i] = cv;
      sn[(size_t)p * hp + i] = sv;
    }
  CKS(s->al.alloc(&kv->rope_cos, c.size()));
  CKS(s->al.alloc(&kv->rope_sin, sn.size()));
  CK(cudaMemcpy(kv->rope_cos, c.data(), c.size() * 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(kv->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
  return MC_OK;
}

// Widest activation (input columns), rounded to whole 128-column K atoms of
// the tcgen05 digit layout.
static int max_kp(const mc_weights* W) {
  int m = round_up(W->d, 128);
  m = std::max(m, round_up(W->H * W->hdp, 128));
  m = std::max(m, round_up(W->F, 128));
  return m;
}

static int max_stripes(const mc_weights* W) {
  int m = W->has_head ? W->head.n_stripes : 0;
  for (const LayerW& L : W->layers) {
    m = std::max(m, L.qkv.n_stripes);
    m = std::max(m, L.o.n_stripes);
    m = std::max(m, L.gu.n_stripes);
    m = std::max(m, L.down.n_stripes);
  }
  return m;
}

// Default limit of a bounded device wait (a peer's flag in tensor
// parallelism): far above any healthy wait, short enough that a missing peer
// ends in an error instead of a stalled GPU.
constexpr long long kDefaultWaitNs = 5000000000ll;

// Exchange regions this process exported (mc_session_tp_ipc_handle): a peer
// in the same process (one thread per GPU) opens them directly, since CUDA
// IPC cannot map an allocation into the process that made it.
struct ExportedRegion {
  char handle[64];
  int dev;
  void* ptr;
};
static std::mutex g_export_mu;
static std::vector<ExportedRegion> g_exports;

static mc_status session_alloc(mc_session* s) {
  const mc_weights* ws[2] = {s->tw, s->dw};
  int d = 0, kp = 0, hq = 0, F = 0, V = 0, stripes = 0, hkv = 0;
  size_t po = 0, pml = 0;  // attention partials per page
  for (const mc_weights* W : ws) {
    if (!W) continue;
    d = std::max(d, W->d);
    kp = std::max(kp, max_kp(W));
    hq = std::max(hq, W->H * W->hdp);
    F = std::max(F, W->F);
    V = std::max(V, W->V);
    stripes = std::max(stripes, max_stripes(W));
    // attention partials: query blocks x block capacity < 2 x tokens per
    // forward (blocks of qblk <= seq_len tokens)
    const size_t rows = (size_t)(W->H / W->Hkv) * 2 * kMaxTokens;
    po = std::max(po, (size_t)W->Hkv * rows * W->hdp);
    pml = std::max(pml, (size_t)W->Hkv * rows * 2);
    hkv = std::max(hkv, W->Hkv);
  }
  const int M = kMaxTokens;
  CKS(s->al.alloc(&s->h, (size_t)M * d));
  // digits: 48 bytes per input column per group of 16 tokens
  CKS(s->al.alloc(&s->xq, (size_t)kp * 48 * kMaxGroups));
  CK(cudaMemset(s->xq, 0, (size_t)kp * 48 * kMaxGroups));
  CKS(s->al.alloc(&s->xexp, (size_t)M));
  CKS(s->al.alloc(&s->qb, (size_t)M * hq));
  CKS(s->al.alloc(&s->act, (size_t)M * std::max(F, 1)));
  CKS(s->al.alloc(&s->logits, (size_t)M * V));
  if (s->cfg.temperature > 0.0f) CKS(s->al.alloc(&s->dlogits, (size_t)kGroupTokens * V));
  // split-K workspace: one 16 x 48 int tile and counter per (stripe, group)
  CKS(s->al.alloc(&s->ws, (size_t)stripes * kMaxGroups * 16 * 48));
  CK(cudaMemset(s->ws, 0, (size_t)stripes * kMaxGroups * 16 * 48 * 4));
  CKS(s->al.alloc(&s->cnt, (size_t)stripes * kMaxGroups));
  CK(cudaMemset(s->cnt, 0, (size_t)stripes * kMaxGroups * 4));
  const int n_pages = (s->cap + kPage - 1) / kPage;
  CKS(s->al.alloc(&s->part_o, po * n_pages));
  CKS(s->al.alloc(&s->part_ml, pml * n_pages));
  CKS(s->al.alloc(&s->err, 1));
  CK(cudaMemset(s->err, 0, 4));
  CKS(s->al.alloc(&s->wait_ns, 1));
  const long long wait_default = kDefaultWaitNs;
  CK(cudaMemcpy(s->wait_ns, &wait_default, sizeof(wait_default), cudaMemcpyHostToDevice));
  CKS(s->al.alloc(&s->st_amax, (size_t)2 * kMaxTokens));
  CK(cudaMemset(s->st_amax, 0, (size_t)2 * kMaxTokens * 4));
  CKS(s->al.alloc(&s->gbar, 2));
  CK(cudaMemset(s->gbar, 0, 2 * sizeof(unsigned)));
  if (s->cfg.kv_mode == KV_MIXED) {
    const int vm = s->cfg.gamma + (s->cfg.bonus ? 1 : 0);
    CKS(s->al.alloc(&s->mx_bak, (size_t)s->B * std::max(vm, 1) * std::max(s->tw->L, 1) * 2 *
                                     s->tw->Hkv * s->tw->hdp));
  }
  if (const char* e = getenv("MODELC_CUDA_ENCODER_TAILS")) s->tails = atoi(e) & 3;
  s->st_np_cap = std::max(stripes, 1);
  CKS(s->al.alloc(&s->st_pss, (size_t)kMaxTokens * s->st_np_cap));
  if (s->tw->tp_world > 1) {
    const int R = s->tw->tp_world, dd = s->tw->d;
    CKS(s->al.alloc(&s->tp_part, (size_t)kMaxTokens * dd));
    // exchange region: partial slots, their flags, key slots, key flags; one
    // allocation for one IPC handle
    s->tp_red_bytes = (size_t)2 * R * kMaxTokens * dd * sizeof(float);
    s->tp_keyx_off = (s->tp_red_bytes + 2 * kMaxTP * sizeof(unsigned) + 255) / 256 * 256;
    s->tp_kflag_off = s->tp_keyx_off + (size_t)2 * kMaxTP * kMaxTokens * sizeof(unsigned long long);
    const size_t bytes = s->tp_kflag_off + 2 * kMaxTP * sizeof(unsigned);
    CK(cudaMalloc(&s->tp_region, bytes));
    CK(cudaMemset(s->tp_region, 0, bytes));
    CKS(s->al.alloc(&s->tp_epoch, 1));
    CKS(s->al.alloc(&s->tp_kepoch, 1));
    const unsigned one = 1u;  // epochs start at 1; flags start at 0
    CK(cudaMemcpy(s->tp_epoch, &one, 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(s->tp_kepoch, &one, 4, cudaMemcpyHostToDevice));
    CKS(s->al.alloc(&s->tp_cnt_gemv, 1));
    CKS(s->al.alloc(&s->tp_cnt_red, 1));
    CK(cudaMemset(s->tp_cnt_gemv, 0, 4));
    CK(cudaMemset(s->tp_cnt_red, 0, 4));
  }
  CKS(alloc_kv(s, s->tw, &s->tkv));
  if (s->dw) CKS(alloc_kv(s, s->dw, &s->dkv));
  // kernel limits and occupancy are settled here, never inside a capture
  size_t qsm = 0, asm_ = 0;
  for (const mc_weights* W : ws) {
    if (!W) continue;
    qsm = std::max(qsm, (size_t)max_kp(W) * sizeof(float));
    const int G = W->H / W->Hkv;
    asm_ = std::max(asm_, attention_smem_bytes(G, attention_qblk(G, kMaxTokens), W->hdp, kPage));
  }
  CK(prepare_kernels(qsm, asm_));
  CK(prepare_tc());
  for (int wf : {(int)WF_I8, (int)WF_Q4, (int)WF_I8R})
    for (int epi = 0; epi < 6; ++epi)
      for (int nt : {1, 2, 3, 6}) {
        bps_of(s, epi, nt, wf);
        if (epi == EPI_RESID || epi == EPI_SWIGLU) bps_of(s, epi, nt, wf, true);
      }
  CKS(s->al.alloc(&s->st, (size_t)s->B));
  CK(cudaMemset(s->st, 0, sizeof(SpecState) * s->B));
  s->ctx_stride = s->cap + 8;
  CKS(s->al.alloc(&s->ctx, (size_t)s->B * s->ctx_stride));
  if (!s->dw) {
    // the prompt's windows plus one per round or step; context shifts let a
    // request run past its capacity, so room for three more contexts' rounds
    s->ng_cap = 4 * s->ctx_stride;
    CKS(s->al.alloc(&s->ng, (size_t)s->B * s->ng_cap * (kNgram + 1)));
    CKS(s->al.alloc(&s->ng_list, (size_t)s->B * s->ng_cap));
  }
  if (s->mlp) CKS(s->al.alloc(&s->mlp_hid, (size_t)s->B * mlp_hidden(s->mlp)));
  CKS(s->al.alloc(&s->acc_log, (size_t)s->B * s->ctx_stride));
  CKS(s->al.alloc(&s->fkeys, (size_t)kMaxTokens));
  CKS(s->al.alloc(&s->ids, (size_t)M));
  CKS(s->al.alloc(&s->pos, 2));
  CK(cudaMemset(s->pos, 0, 8));
  CK(cudaMallocHost(&s->h_ids, (size_t)std::max(s->B * s->ctx_stride, M) * 4));
  return MC_OK;
}

static mc_status session_create(const mc_weights* target, const mc_weights* draft,
                                const mc_mlp_drafter* mlp, const mc_spec_cfg* cfg,
                                mc_session** out) {
  if (!target || !cfg || !out) return set_err(MC_E_INVALID, "null argument");
  *out = nullptr;
  if (mlp && mlp_device(mlp) != target->dev)
    return set_err(MC_E_INVALID, "target and MLP drafter live on different devices");
  if (mlp && mlp_vocab(mlp) != target->V)
    return set_err(MC_E_SHAPE, "MLP drafter vocab %d != target vocab %d", mlp_vocab(mlp),
                   target->V);
  if (mlp && cfg->temperature > 0.0f)
    return set_err(MC_E_INVALID, "the MLP drafter drafts greedily: use temperature 0 (the "
                   "reference samples it with an unseeded generator, draft.rs:140)");
  if (draft && draft->dev != target->dev)
    return set_err(MC_E_INVALID, "target and draft live on different devices");
  if (cfg->gamma < 0 || cfg->gamma + 1 > kGroupTokens)
    return set_err(MC_E_INVALID, "gamma %d outside [0, %d]", cfg->gamma, kGroupTokens - 1);
  const int B = std::max(1, (int)cfg->n_requests);
  if (cfg->n_requests < 0 || B * (cfg->gamma + (cfg->bonus ? 1 : 0)) > kMaxTokens)
    return set_err(MC_E_INVALID, "%d requests x %d verify positions exceed %d tokens per forward",
                   B, cfg->gamma + (cfg->bonus ? 1 : 0), kMaxTokens);
  if (B > 1 && cfg->temperature > 0.0f)
    return set_err(MC_E_INVALID, "batched sessions decode greedily (temperature 0)");
  if (cfg->max_context <= 0) return set_err(MC_E_INVALID, "max_context must be positive");
  if (round_up(cfg->max_context + kChunk + 2, kPage) / kPage > kMaxAttnPages)
    return set_err(MC_E_CAPACITY,
                   "max_context %d above this build's limit %d (the attention combines at most "
                   "%d KV pages of %d positions per request)",
                   cfg->max_context, kMaxAttnPages * kPage - kChunk - 2, kMaxAttnPages, kPage);
  if (!(cfg->temperature >= 0.0f) || !isfinite(cfg->temperature))
    return set_err(MC_E_INVALID, "temperature must be finite and >= 0");
  if (cfg->accept_mode != 0 && cfg->accept_mode != 1)
    return set_err(MC_E_INVALID, "accept_mode must be 0 (min(1,p/q)) or 1 (sample == draft)");
  if (cfg->temperature > 0.0f && target->V > kSampleMaxVocab)
    return set_err(MC_E_SHAPE, "vocab %d above the sampler's limit %d", target->V,
                   kSampleMaxVocab);
  if (draft && (draft->V != target->V))
    return set_err(MC_E_SHAPE, "draft vocab %d != target vocab %d", draft->V, target->V);
  if (draft && draft->tp_world > 1)
    return set_err(MC_E_INVALID, "the draft model is replicated: load it with tp_world 1");
  if (target->tp_world > 1 && cfg->temperature > 0.0f)
    return set_err(MC_E_INVALID, "tensor-parallel sessions decode greedily (temperature 0)");
  if (cfg->kv_mode != KV_FP32 && cfg->kv_mode != KV_INT8 && cfg->kv_mode != KV_MIXED)
    return set_err(MC_E_INVALID, "kv_mode %d is not MC_KV_FP32, MC_KV_INT8 or MC_KV_MIXED",
                   cfg->kv_mode);
  if (cfg->kv_mode != KV_FP32 && target->tp_world > 1)
    return set_err(MC_E_INVALID, "int8 and mixed KV caches quantize each token over all KV "
                   "heads: tensor-parallel sessions keep an f32 cache");
  if (cfg->kv_mode == KV_MIXED && cfg->temperature > 0.0f)
    return set_err(MC_E_INVALID, "mixed KV caches run in greedy sessions (temperature 0)");
  if (cfg->shift_context < 0 || cfg->anchor_tokens < 0)
    return set_err(MC_E_INVALID, "shift_context and anchor_tokens must be >= 0");
  if (cfg->shift_context > 0 && cfg->temperature > 0.0f)
    return set_err(MC_E_INVALID, "the context shift runs in greedy sessions (temperature 0)");
  if (cfg->shift_context > 0 && cfg->shift_context + cfg->gamma + 2 > cfg->max_context)
    return set_err(MC_E_INVALID, "shift_context %d + gamma + 2 exceeds max_context %d (a round "
                   "must fit before the shift)", cfg->shift_context, cfg->max_context);
  CK(cudaSetDevice(target->dev));
  mc_session* s = new mc_session();
  s->tw = target;
  s->dw = draft;
  s->mlp = mlp;
  s->cfg = *cfg;
  s->B = B;
  s->dev = target->dev;
  s->cap = round_up(cfg->max_context + kChunk + 2, kPage);
  cudaDeviceGetAttribute(&s->nsm, cudaDevAttrMultiProcessorCount, s->dev);
  mc_status st = MC_OK;
  if (cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking) != cudaSuccess)
    st = set_err(MC_E_CUDA, "stream creation failed");
  if (st == MC_OK) st = session_alloc(s);
  if (st != MC_OK) {
    if (s->h_ids) cudaFreeHost(s->h_ids);
    if (s->stream) cudaStreamDestroy(s->stream);
    s->al.free_all();
    delete s;
    return st;
  }
  *out = s;
  return MC_OK;
}

extern "C" mc_status mc_session_create(const mc_weights* target, const mc_weights* draft,
                                       const mc_spec_cfg* cfg, mc_session** out) {
  return session_create(target, draft, nullptr, cfg, out);
}

extern "C" mc_status mc_session_create_mlp(const mc_weights* target, const mc_mlp_drafter* draft,
                                           const mc_spec_cfg* cfg, mc_session** out) {
  if (!draft) return set_err(MC_E_INVALID, "null MLP drafter");
  return session_create(target, nullptr, draft, cfg, out);
}

extern "C" mc_status mc_session_destroy(mc_session* s) {
  if (!s) return MC_OK;
  cudaSetDevice(s->dev);
  if (s->stream) cudaStreamSynchronize(s->stream);
  if (s->round_exec) cudaGraphExecDestroy(s->round_exec);
  if (s->verify_exec) cudaGraphExecDestroy(s->verify_exec);
  if (s->comm) nccl::g_api.comm_destroy(s->comm);  // after the graphs holding its calls
  for (void* p : s->tp_opened) cudaIpcCloseMemHandle(p);
  if (s->tp_region) {
    std::lock_guard<std::mutex> lock(g_export_mu);
    for (size_t i = 0; i < g_exports.size();)
      if (g_exports[i].ptr == s->tp_region) g_exports.erase(g_exports.begin() + i);
      else ++i;
  }
  if (s->tp_region) cudaFree(s->tp_region);
  if (s->h_ids) cudaFreeHost(s->h_ids);
  if (s->stream) cudaStreamDestroy(s->stream);
  s->al.free_all();
  delete s;
  return MC_OK;
}

// ------------------------------------------------------------------ forward
// A raised device error flag means a bounded wait expired inside a kernel
// (a tensor-parallel peer that never published, or a stalled copy).  The
// session's cross-rank epochs are then out of step, so it stays failed.
static mc_status check_err(mc_session* s) {
  int v = 0;
  CK(cudaMemcpy(&v, s->err, 4, cudaMemcpyDeviceToHost));
  if (v) {
    s->failed = true;
    return set_err(MC_E_TIMEOUT, "a bounded device wait expired (a peer never arrived or the "
                                 "pipeline stalled); destroy this session");
  }
  return MC_OK;
}
static mc_status check_usable(const mc_session* s) {
  if (s->failed)
    return set_err(MC_E_TIMEOUT, "an earlier bounded device wait expired; destroy this session");
  return MC_OK;
}

#ifndef MC_NEXT_PREFETCH_MB
#define MC_NEXT_PREFETCH_MB 24
#endif
// L2 bytes of the next GEMV's weights warmed by the running one
constexpr long long kNextPrefetch = (long long)MC_NEXT_PREFETCH_MB << 20;
// Kernels that leave HBM idle (attention, encoders) warm L2 with the part of
// an upcoming GEMV's weights beyond what the GEMV before it prefetches.
#ifndef MC_IDLE_PREFETCH_MB
#define MC_IDLE_PREFETCH_MB 32
#endif
constexpr long long kIdlePrefetch = (long long)MC_IDLE_PREFETCH_MB << 20;

static long long packed_bytes(const PMat& W) {
  return (long long)W.n_stripes * W.KB * (W.fmt == WF_Q4 ? kFragBytes / 2 : kFragBytes);
}
// [kNextPrefetch, kNextPrefetch + cap) of W's packed codes, clipped
static void idle_prefetch(const PMat* W, long long cap, const void** p, long long* bytes) {
  *p = nullptr;
  *bytes = 0;
  if (!W || !W->w || cap <= 0) return;
  const long long total = packed_bytes(*W);
  if (total <= kNextPrefetch) return;
  *p = reinterpret_cast<const char*>(W->w) + kNextPrefetch;
  *bytes = std::min(total - kNextPrefetch, cap);
}

// Statistics an encoder takes from its producer (see QuantArgs).
struct StatIO {
  const float* pss;
  int np;
  const unsigned* amax;
  unsigned* amax_next;
  const PMat* pf = nullptr;  // upcoming GEMV to warm in L2 (idle_prefetch)
};

static void fill_quant(mc_session* s, QuantArgs& q, const float* h, int ld, int d, int M,
                       const float* w, float eps, int do_norm, const StatIO* io, bool tc,
                       const AttnArgs* att) {
  q = QuantArgs{};
  if (att) {  // combine the attention's page partials while encoding
    q.att_o = att->part_o;
    q.att_ml = att->part_ml;
    q.att_chunks = att->max_chunks;
    q.att_Hkv = att->Hkv;
    q.att_G = att->H / att->Hkv;
    q.att_hdp = att->hdp;
    q.att_qblk = att->qblk;
    q.att_page = att->page;
    q.att_seq = att->seq;
    q.att_pos = att->pos_ptr;
    q.att_pos_add = att->pos_add;
  }
  q.tc_layout = tc ? 1 : 0;
  if (io) {
    q.use_stats = 1;
    q.pss = io->pss;
    q.np = io->np;
    q.np_stride = io->np;
    q.amax = io->amax;
    q.amax_next = io->amax_next;
    idle_prefetch(io->pf, kIdlePrefetch, &q.pf, &q.pf_bytes);
  }
  q.h = h;
  q.ld = ld;
  q.d = d;
  q.M = M;
  q.w = w;
  q.wlen = d;
  q.eps = eps;
  q.do_norm = do_norm;
  q.xq = s->xq;
  q.KB = (d + 31) / 32;
  q.nt = nt_for_tokens(M);
  q.xexp = s->xexp;
}

static mc_status enq_quant(mc_session* s, const float* h, int ld, int d, int M, const float* w,
                           float eps, int do_norm, const StatIO* io = nullptr, bool tc = false,
                           const AttnArgs* att = nullptr) {
  QuantArgs q;
  fill_quant(s, q, h, ld, d, M, w, eps, do_norm, io, tc, att);
  q.trace_slot = trace_slot(s);
  CK(launch_quant(q, s->stream, true));
  return MC_OK;
}




static mc_status enq_gemv(mc_session* s, const PMat& W, int epi, int M, GemvArgs a,
                          const PMat* next = nullptr) {
  if (next && next->w) {
    a.next_w = next->w;
    // packed code bytes of the next matrix (q4_0: 256 per stripe k-block)
    a.next_bytes = (long long)next->n_stripes * next->KB * (next->fmt == WF_Q4 ? kFragBytes / 2
                                                                               : kFragBytes);
    a.next_pf_bytes = std::min(a.next_bytes, kNextPrefetch);
  }
  a.x = s->xq;
  a.xexp = s->xexp;
  a.ws = s->ws;
  a.cnt = s->cnt;
  a.err = s->err;
  a.trace_slot = trace_slot(s);
  const bool tail = a.bar != nullptr;
  CK(run_projection(W, epi, M, a, s->nsm, s->stream,
                    [&](int t) { return bps_of(s, epi, t, gemv_wf(W), tail); }));
  return MC_OK;
}

// One batched forward of M tokens through W (forward_llama_cached,
// transformer.rs:64-96, for M positions at once): sm.seq_len tokens of each
// of M / sm.seq_len sequences, whose positions, KV page-table rows and key
// slots sm maps (one sequence: sm.seq_len = M).
// A MIXED target forward's place in the cache's append sequence (KvMixArgs):
// the window count before it (hot_ptr[z * hot_stride], or hot_const), the
// appends before it (step), and for a verify step the originals' buffer and
// the round's first position.
struct MixStep {
  const int* hot_ptr = nullptr;
  int hot_stride = 0;
  int hot_const = 0;
  int step = 0;
  float* bak = nullptr;
  int bak_steps = 0;
  int* base_out = nullptr;
  int base_stride = 0;
};

static mc_status enq_forward(mc_session* s, const mc_weights* W, const KVSet& kv, int M,
                             SeqMap sm, EmbedArgs ea, const int* pos_ptr, int pos_add,
                             unsigned long long* keys, float* logits_dev, bool kv_pre = false,
                             const MixStep* mix = nullptr) {
  if (M < 1 || M > kMaxTokens || sm.seq_len < 1 || M % sm.seq_len)
    return set_err(MC_E_INVALID, "forward of %d tokens in sequences of %d", M, sm.seq_len);
  if (!W->has_head) return set_err(MC_E_NO_HEAD, "model has no lm_head and no embedding");
  const bool tp = W->tp_world > 1;
  if (tp && !s->comm && !s->tp_p2p)
    return set_err(MC_E_INVALID,
                   "tensor-parallel weights: call mc_session_tp_init or mc_session_tp_open_peers");
  if (tp && logits_dev) return set_err(MC_E_INVALID, "tensor-parallel forwards return argmax only");
  ea.emb_q = W->emb_q;
  ea.emb_scale = W->emb_scale;
  ea.emb_q4 = W->emb_q4;
  ea.d = W->d;
  ea.vocab = W->V;
  ea.M = M;
  ea.h = s->h;
  ea.seq = sm;
  ea.ctx_stride = s->ctx_stride;
  ea.zero_keys = keys;
  ea.n_zero = keys ? M : 0;
  // Encoders in launch order: the rows each reads, the RMSNorm weight it
  // applies (nullptr: no norm) and the projection that reads its digits.
  // Producer j (embedding, attention, or a GEMV epilogue) folds the
  // statistics of its output into slot j % 2 for encoder j, which zeroes the
  // other slot for producer j + 1.
  struct EncSpec {
    const float* h;  // nullptr: the attention's page partials
    int ld;
    const float* w;
    const PMat* cons;
  };
  std::vector<EncSpec> encs;
  for (const LayerW& Lw : W->layers) {
    if (Lw.attn) {
      encs.push_back({s->h, W->d, Lw.attn_norm, &Lw.qkv});
      encs.push_back({nullptr, W->H * W->hdp, nullptr, &Lw.o});
    }
    if (Lw.mlp) {
      encs.push_back({s->h, W->d, Lw.mlp_norm, &Lw.gu});
      encs.push_back({s->act, W->F, nullptr, &Lw.down});
    }
  }
  encs.push_back({s->h, W->d, W->final_norm, &W->head});
  size_t ej = 0;  // next encoder
  size_t tailed = (size_t)-1;  // encoder run as its producer's tail (GemvArgs::bar)
  auto slot = [&](size_t j) { return s->st_amax + (j & 1) * kMaxTokens; };
  auto io_for = [&](size_t j, int np) {
    return StatIO{s->st_pss, np, slot(j), slot(j + 1), nullptr};
  };
  ea.st_pss = s->st_pss;
  ea.st_np = 1;
  ea.st_amax = slot(0);
  ea.st_w = encs[0].w;
  ea.trace_slot = trace_slot(s);
  CK(launch_embed(ea, s->stream, true));
  int prod_np = 1;  // sum-of-squares partials written by the last h producer
  // residual producers fill st_* for the encoder that follows them
  auto resid_stats = [&](GemvArgs& g, const PMat& Wm) {
    g.st_pss = s->st_pss;
    g.st_np = Wm.n_stripes;
    g.st_amax = slot(ej);
    g.st_w = encs[ej].w;
    prod_np = Wm.n_stripes;
  };
  // the next encoder as the tail of the single-launch GEMV that produces its
  // rows (np: that GEMV's sum-of-squares partials; pf: L2 warm-up of upcoming
  // weights, as the encoder's own launch would issue)
  auto attach_tail = [&](GemvArgs& g, const PMat& Wm, int np, const PMat* pf) {
    if (!(s->tails & 1) || M > kGroupTokens || use_tc(Wm, M) || ej >= encs.size() || !encs[ej].h)
      return;
    const EncSpec& e = encs[ej];
    StatIO io = io_for(ej, np);
    io.pf = pf;
    fill_quant(s, g.enc, e.h, e.ld, e.ld, M, e.w, W->eps, e.w ? 1 : 0, &io, use_tc(*e.cons, M),
               nullptr);
    g.bar = s->gbar;
    tailed = ej;
  };
  // o / down: h += W x (+ statistics); row-parallel across ranks: partial
  // sums, one all-reduce, then the residual add and the statistics
  auto residual_gemv = [&](const PMat& Wm, const PMat* next) -> mc_status {
    const int d = W->d;
    GemvArgs g{};
    g.ldo = d;
    g.n_out = d;
    if (!tp) {
      g.out = s->h;
      resid_stats(g, Wm);
      attach_tail(g, Wm, Wm.n_stripes, nullptr);
      return enq_gemv(s, Wm, EPI_RESID, M, g, next);
    }
    ResidArgs r{};
    // fused: the GEMV stores its rows into every rank's buffer (one launch,
    // whose last CTA publishes the epoch: not for the per-group GEMV passes)
    if (s->tp_p2p && (M <= kGroupTokens || use_tc(Wm, M))) {
      g.tp = s->tp;
      CKS(enq_gemv(s, Wm, EPI_TP, M, g, next));
      r.h = s->h;
      r.d = d;
      r.M = M;
      r.pss = s->st_pss;
      r.amax = slot(ej);
      r.w = encs[ej].w;
      r.trace_slot = trace_slot(s);
      CK(launch_tp_reduce(r, s->tp, s->tp_epoch, s->tp_cnt_red, s->stream, true));
      prod_np = (d + kResidBlock - 1) / kResidBlock;
      return MC_OK;
    }
    if (!s->comm)
      return set_err(MC_E_INVALID, "this forward (%d tokens of q4_0 weights) reduces with NCCL: "
                     "call mc_session_tp_init", M);
    g.out = s->tp_part;
    CKS(enq_gemv(s, Wm, EPI_STORE, M, g, next));
    CKS(nccl::check(nccl::g_api.all_reduce(s->tp_part, s->tp_part, (size_t)M * d, nccl::kFloat32,
                                           nccl::kSum, s->comm, s->stream),
                    "all-reduce of row-parallel partial sums"));
    r.h = s->h;
    r.y = s->tp_part;
    r.d = d;
    r.M = M;
    r.pss = s->st_pss;
    r.amax = slot(ej);
    r.w = encs[ej].w;
    r.trace_slot = trace_slot(s);
    CK(launch_resid_stats(r, s->stream, true));
    prod_np = (d + kResidBlock - 1) / kResidBlock;
    return MC_OK;
  };
  const int d = W->d, F = W->F;
  // the GEMVs of this forward in launch order (each warms L2 for the next)
  std::vector<const PMat*> seq;
  for (const LayerW& Lw : W->layers) {
    if (Lw.attn) { seq.push_back(&Lw.qkv); seq.push_back(&Lw.o); }
    if (Lw.mlp) { seq.push_back(&Lw.gu); seq.push_back(&Lw.down); }
  }
  seq.push_back(&W->head);
  size_t gi = 0;
  auto nxt = [&]() -> const PMat* { ++gi; return gi < seq.size() ? seq[gi] : nullptr; };
  for (int l = 0; l < W->L; ++l) {
    const LayerW& Lw = W->layers[l];
    if (Lw.attn) {
      StatIO io = io_for(ej, prod_np);
      if (tailed != ej)
        CKS(enq_quant(s, s->h, d, d, M, Lw.attn_norm, W->eps, Lw.attn_norm ? 1 : 0, &io,
                      use_tc(Lw.qkv, M)));
      ++ej;
      GemvArgs a{};
      a.q_out = s->qb;
      a.kc = kv.k + (size_t)l * kv.layer_stride;
      a.vc = kv.v + (size_t)l * kv.layer_stride;
      a.page_table = kv.page_table;
      a.pos_ptr = pos_ptr;
      a.pos_add = pos_add;
      a.seq = sm;
      a.rope_cos = kv.rope_cos;
      a.rope_sin = kv.rope_sin;
      a.half_p = W->half_p;
      a.hdp = W->hdp;
      a.H = W->H;
      a.Hkv = W->Hkv;
      a.page = kPage;
      a.sq = Lw.sq;
      a.sk = Lw.sk;
      a.kv_prefetch = 1;
      CKS(enq_gemv(s, Lw.qkv, EPI_QKV, M, a, nxt()));
      if (kv.k == s->tkv.k && s->cfg.kv_mode == KV_INT8) {  // KvLayer::append of an INT8 layer
        KvQArgs q{};
        q.kc = a.kc;
        q.vc = a.vc;
        q.page_table = kv.page_table;
        q.pos_ptr = pos_ptr;
        q.pos_add = pos_add;
        q.seq = sm;
        q.M = M;
        q.Hkv = W->Hkv;
        q.hd = W->hdp;  // padding elements are zero: they change neither the scale nor stay nonzero
        q.hdp = W->hdp;
        q.page = kPage;
        CK(launch_kv_qdq(q, s->stream, true));
      }
      if (kv.k == s->tkv.k && s->cfg.kv_mode == KV_MIXED) {  // KvLayer::append of a MIXED layer
        if (!mix || sm.seq_len != 1)
          return set_err(MC_E_INVALID, "mixed KV forwards append one token per request");
        KvMixArgs x{};
        x.kc = a.kc;
        x.vc = a.vc;
        x.page_table = kv.page_table;
        x.pos_ptr = pos_ptr;
        x.pos_add = pos_add;
        x.seq = sm;
        x.B = M;
        x.Hkv = W->Hkv;
        x.hdp = W->hdp;
        x.page = kPage;
        x.window = kMixedWindow;
        x.hot_ptr = mix->hot_ptr;
        x.hot_stride = mix->hot_stride;
        x.hot_const = mix->hot_const;
        x.step = mix->step;
        x.bak = mix->bak;
        x.bak_steps = mix->bak_steps;
        x.layer = l;
        x.layers = W->L;
        x.base_out = mix->base_out;
        x.base_stride = mix->base_stride;
        CK(launch_kv_mixed_age(x, s->stream, true));
      }
      AttnArgs t{};
      t.q = s->qb;
      t.kc = a.kc;
      t.vc = a.vc;
      t.page_table = kv.page_table;
      t.pos_ptr = pos_ptr;
      t.pos_add = pos_add;
      t.seq = sm;
      t.qblk = attention_qblk(W->H / W->Hkv, sm.seq_len);
      t.kv_pre = kv_pre ? 1 : 0;
      t.M = M;
      t.H = W->H;
      t.Hkv = W->Hkv;
      t.hdp = W->hdp;
      t.page = kPage;
      t.inv_scale_den = sqrtf((float)W->hd);
      t.max_chunks = kv.n_pages;
      t.part_o = s->part_o;
      t.part_ml = s->part_ml;
      t.st_amax = slot(ej);
      // the gate/up projection after O: its weights beyond the O GEMV's prefetch
      idle_prefetch(Lw.mlp ? &Lw.gu : nullptr, kIdlePrefetch, &t.pf, &t.pf_bytes);
      io = io_for(ej, 0);
      if (s->tails & 2) {  // the O projection's encoder as the attention's tail
        fill_quant(s, t.enc, nullptr, W->H * W->hdp, W->H * W->hdp, M, nullptr, 0.0f, 0, &io,
                   use_tc(Lw.o, M), &t);
        if (attention_tail_fits(t, s->nsm)) {
          t.bar = s->gbar;
          t.err = s->err;
          tailed = ej;
        }
      }
      t.trace_slot = trace_slot(s);
      CK(launch_attention(t, s->stream, true));
      if (tailed != ej)
        CKS(enq_quant(s, nullptr, W->H * W->hdp, W->H * W->hdp, M, nullptr, 0.0f, 0, &io,
                      use_tc(Lw.o, M), &t));
      ++ej;
      CKS(residual_gemv(Lw.o, nxt()));
    }
    if (Lw.mlp) {
      StatIO io = io_for(ej, prod_np);
      if (tailed != ej)
        CKS(enq_quant(s, s->h, d, d, M, Lw.mlp_norm, W->eps, Lw.mlp_norm ? 1 : 0, &io,
                      use_tc(Lw.gu, M)));
      ++ej;
      GemvArgs g{};
      g.out = s->act;
      g.ldo = F;
      g.n_out = F;
      g.st_amax = slot(ej);
      // the down weights beyond the gate/up GEMV's prefetch go with the encoder
      attach_tail(g, Lw.gu, 0, &Lw.down);
      CKS(enq_gemv(s, Lw.gu, EPI_SWIGLU, M, g, nxt()));
      io = io_for(ej, 0);
      io.pf = &Lw.down;
      if (tailed != ej) CKS(enq_quant(s, s->act, F, F, M, nullptr, 0.0f, 0, &io, use_tc(Lw.down, M)));
      ++ej;
      CKS(residual_gemv(Lw.down, nxt()));
    }
  }
  StatIO io = io_for(ej, prod_np);
  if (tailed != ej)
    CKS(enq_quant(s, s->h, d, d, M, W->final_norm, W->eps, W->final_norm ? 1 : 0, &io,
                  use_tc(W->head, M)));
  GemvArgs hd{};
  hd.out = logits_dev;
  hd.ldo = W->V;
  hd.n_out = W->V_loc;
  hd.keys = keys;
  hd.seq = sm;
  hd.row_offset = W->head_row0;
  CKS(enq_gemv(s, W->head, EPI_LMHEAD, M, hd));
  if (tp && s->tp_p2p) {  // vocab-parallel head over peer memory (bounded waits)
    CK(launch_tp_keys(s->tp, keys, M / sm.seq_len, sm.seq_len, sm.key_stride, s->stream, true));
  } else if (tp) {  // vocab-parallel head: the largest (value, lowest index) key wins
    // the key slots of each sequence are contiguous (seq_len of them)
    const int n_seq = M / sm.seq_len;
    for (int z = 0; z < n_seq; ++z)
      CKS(nccl::check(nccl::g_api.all_reduce(keys + (size_t)z * sm.key_stride,
                                             keys + (size_t)z * sm.key_stride, (size_t)sm.seq_len,
                                             nccl::kUint64, nccl::kMax, s->comm, s->stream),
                      "all-reduce of argmax keys"));
  }
  return MC_OK;
}

// Plain batched forward through the C ABI (target: which=0, draft: which=1).
static mc_status forward_api(mc_session* s, int which, const uint32_t* ids, int n, float* logits) {
  const mc_weights* W = which ? s->dw : s->tw;
  if (!W) return set_err(MC_E_INVALID, "session has no draft model");
  const KVSet& kv = which ? s->dkv : s->tkv;
  int& len = which ? s->ld : s->lt;
  if (n < 0 || (n > 0 && !ids)) return set_err(MC_E_INVALID, "bad ids");
  if (len + n > s->cap - 1) return set_err(MC_E_CAPACITY, "KV capacity %d exceeded", s->cap);
  CKS(check_usable(s));
  CK(cudaSetDevice(s->dev));
  // a MIXED target cache appends token by token (plain_hot: its window count)
  const bool mixed = !which && s->cfg.kv_mode == KV_MIXED;
  const int chunk = mixed ? 1 : kChunk;
  for (int c0 = 0; c0 < n; c0 += chunk) {
    const int M = std::min(chunk, n - c0);
    memcpy(s->h_ids, ids + c0, (size_t)M * 4);
    CK(cudaMemcpyAsync(s->ids, s->h_ids, (size_t)M * 4, cudaMemcpyHostToDevice, s->stream));
    CK(launch_set_int(s->pos + which, len, s->stream));
    EmbedArgs ea{};
    ea.src = SRC_IDS;
    ea.ids = s->ids;
    MixStep mx;
    mx.hot_const = s->plain_hot;
    CKS(enq_forward(s, W, kv, M, SeqMap{M, 0, 0, 0}, ea, s->pos + which, 0, s->fkeys,
                    logits ? s->logits : nullptr, false, mixed ? &mx : nullptr));
    if (mixed) s->plain_hot = std::min(s->plain_hot + 1, kMixedWindow);
    if (logits)
      CK(cudaMemcpyAsync(logits + (size_t)c0 * W->V, s->logits, (size_t)M * W->V * 4,
                         cudaMemcpyDeviceToHost, s->stream));
    CK(cudaStreamSynchronize(s->stream));
    CKS(check_err(s));
    len += M;
  }
  if (which) s->draft_tokens.insert(s->draft_tokens.end(), ids, ids + n);
  return MC_OK;
}

extern "C" mc_status mc_forward(mc_session* s, const uint32_t* ids, int32_t n, float* logits_out) {
  if (!s) return set_err(MC_E_INVALID, "null session");
  return forward_api(s, 0, ids, n, logits_out);
}

extern "C" mc_status mc_draft_forward(mc_session* s, const uint32_t* ids, int32_t n,
                                      float* logits_out) {
  if (!s) return set_err(MC_E_INVALID, "null session");
  return forward_api(s, 1, ids, n, logits_out);
}

extern "C" int32_t mc_kv_len(const mc_session* s) { return s ? s->lt : 0; }

extern "C" mc_status mc_kv_truncate(mc_session* s, int32_t len) {
  if (!s || len < 0) return set_err(MC_E_INVALID, "bad arguments");
  if (len < s->lt) {
    s->plain_hot = std::max(0, s->plain_hot - (s->lt - len));
    s->lt = len;
  }
  return MC_OK;
}

// DraftModel::draft (draft.rs:18-21) for the transformer draft.
extern "C" mc_status mc_draft(mc_session* s, const uint32_t* context, int32_t n, int32_t gamma,
                              uint32_t* out, int32_t* n_out) {
  if (!s || !out || !n_out || n < 0 || gamma < 0) return set_err(MC_E_INVALID, "bad arguments");
  *n_out = 0;
  if (!s->dw) return set_err(MC_E_INVALID, "session has no draft model");
  if (n == 0 || gamma == 0) return MC_OK;
  if (n + gamma > s->cap - 1) return set_err(MC_E_CAPACITY, "KV capacity %d exceeded", s->cap);
  size_t p = 0;
  while (p < s->draft_tokens.size() && p < (size_t)n && s->draft_tokens[p] == context[p]) ++p;
  if (p > (size_t)n - 1) p = n - 1;
  s->draft_tokens.resize(p);
  s->ld = (int)p;
  // forward the uncached context (chunks); keep only the last chunk's argmax
  std::vector<uint32_t> rest(context + p, context + n);
  CKS(forward_api(s, 1, rest.data(), (int)rest.size(), nullptr));
  for (int j = 0; j < gamma; ++j) {
    unsigned long long key = 0;
    const int last = (int)((rest.size() - 1) % kChunk);
    CK(cudaMemcpy(&key, &s->fkeys[last], 8, cudaMemcpyDeviceToHost));
    out[j] = key_index(key);
    if (j + 1 < gamma) {
      rest.assign(1, out[j]);
      CKS(forward_api(s, 1, &out[j], 1, nullptr));
    }
  }
  *n_out = gamma;
  return MC_OK;
}

// ------------------------------------------------------------------ speculative loop

// Verify forward of every request: vm positions each (request z's tokens are
// z * vm .. z * vm + vm - 1), at the request's own target length.
static mc_status enq_verify(mc_session* s, float* logits = nullptr) {
  const int vm = s->cfg.gamma + (s->cfg.bonus ? 1 : 0);
  if (s->cfg.kv_mode == KV_MIXED) {
    // a MIXED cache appends and ages token by token (each step's attention
    // sees the window as the reference's sequential verify leaves it): vm
    // forwards of one token per request -- the context's last token, then
    // the drafts -- their originals kept for the acceptance's roll-back
    const SeqMap sm{1, kStateInts, s->tkv.n_pages, kStateKeys};
    for (int i = 0; i < vm; ++i) {
      EmbedArgs ea{};
      if (i == 0) {
        ea.src = SRC_CTX_AT;
        ea.ctx = s->ctx;
        ea.off = &s->st->ld;
      } else {
        ea.src = SRC_KEYS;
        ea.keys = &s->st->dkeys[i - 1];
      }
      MixStep mx;
      mx.hot_ptr = &s->st->kv_hot;
      mx.hot_stride = kStateInts;
      mx.step = i;
      mx.bak = s->mx_bak;
      mx.bak_steps = vm;
      mx.base_out = &s->st->mx_base;
      mx.base_stride = kStateInts;
      CKS(enq_forward(s, s->tw, s->tkv, s->B, sm, ea, &s->st->lt, i, &s->st->tkeys[i],
                      logits ? logits + (size_t)i * s->tw->V : nullptr, false, &mx));
    }
    return MC_OK;
  }
  EmbedArgs ea{};
  ea.src = SRC_VERIFY;
  ea.ctx = s->ctx;
  ea.off = &s->st->ctx_len;
  ea.keys = s->st->dkeys;
  const SeqMap sm{vm, kStateInts, s->tkv.n_pages, kStateKeys};
  // captured alone in a graph: the target K/V below each request's length
  // (and the length itself) were written by earlier graph launches or
  // stream work, which completes before this graph starts
  return enq_forward(s, s->tw, s->tkv, vm * s->B, sm, ea, &s->st->lt, 0, s->st->tkeys, logits,
                     true);
}

static mc_status capture_verify(mc_session* s) {
  if (s->verify_exec) return MC_OK;
  CK(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
#ifdef MC_TRACE
  s->trace_on = true;
  s->trace_next = 0;
#endif
  mc_status rc = enq_verify(s);
  s->trace_on = false;
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(s->stream, &graph);
  if (rc != MC_OK) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (e != cudaSuccess) return set_err(MC_E_CUDA, "capture failed: %s", cudaGetErrorString(e));
  e = cudaGraphInstantiate(&s->verify_exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) return set_err(MC_E_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
  return MC_OK;
}

// Kernel launches of one round: the drafter's steps, the verify forward,
// the acceptance (and the stochastic draft samples).
// The session's caches for the context shift: the target KV and, with a
// transformer draft, the draft KV.
static KvPlanes kv_planes(const mc_weights* W, const KVSet& kv, int n_pages) {
  KvPlanes p{};
  if (!W) return p;
  p.k = kv.k;
  p.v = kv.v;
  p.layer_stride = kv.layer_stride;
  p.layers = W->L;
  p.Hkv = W->Hkv;
  p.hd = W->hdp;  // padding elements are zero
  p.hdp = W->hdp;
  p.page = kPage;
  p.pt = kv.page_table;
  p.pt_stride = n_pages;
  return p;
}
static ShiftArgs shift_args(mc_session* s) {
  ShiftArgs a{};
  a.st = s->st;
  a.ctx = s->ctx;
  a.ctx_stride = s->ctx_stride;
  a.B = s->B;
  a.shift_context = s->cfg.shift_context;
  a.anchor = s->cfg.anchor_tokens;
  a.requant = s->cfg.kv_mode != KV_FP32 && s->cfg.anchor_tokens > 0;
  a.window = s->cfg.kv_mode == KV_MIXED ? kMixedWindow : 0;
  a.t = kv_planes(s->tw, s->tkv, s->tkv.n_pages);
  a.d = kv_planes(s->dw, s->dkv, s->dkv.n_pages);
  return a;
}

static mc_status capture_round(mc_session* s) {
  if (s->round_exec) return MC_OK;
  const int g = s->cfg.gamma;
  const int bonus = s->cfg.bonus ? 1 : 0;
  const int vm = g + bonus;
  const int dsteps = g + bonus;
  SpecState* st = s->st;
  CK(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
  mc_status rc = MC_OK;
  const bool stochastic = s->cfg.temperature > 0.0f;
  const int V = s->tw->V;
  // draft step j: one token per request (request z's at its draft length + j)
  const SeqMap dsm{1, kStateInts, s->dkv.n_pages, kStateKeys};
  if (draft_kind(s) == DRAFT_MLP) {
    cudaError_t e = mlp_round(s->mlp, st, s->ctx, s->ctx_stride, s->B, g, s->mlp_hid, s->stream);
    if (e != cudaSuccess) rc = set_err(MC_E_CUDA, "MLP draft: %s", cudaGetErrorString(e));
  } else if (draft_kind(s) == DRAFT_NGRAM) {
    cudaError_t e = launch_ngram_round(st, s->ctx, s->ng, s->ng_list, s->ctx_stride, s->ng_cap, s->B,
                                       s->stream);
    if (e != cudaSuccess) rc = set_err(MC_E_CUDA, "n-gram draft: %s", cudaGetErrorString(e));
  }
  for (int j = 0; j < dsteps && rc == MC_OK && s->dw; ++j) {
    EmbedArgs ea{};
    if (j == 0) {
      ea.src = SRC_CTX_AT;
      ea.ctx = s->ctx;
      ea.off = &st->ld;
    } else {
      ea.src = SRC_KEYS;
      ea.keys = &st->dkeys[j - 1];
    }
    float* dl = stochastic && j < g ? s->dlogits + (size_t)j * V : nullptr;
    rc = enq_forward(s, s->dw, s->dkv, s->B, dsm, ea, &st->ld, j, &st->dkeys[j], dl);
    if (rc == MC_OK && dl) {  // x_j ~ softmax(q_j / T) replaces the argmax key
      cudaError_t e = launch_sample_draft(st, dl, V, j, &st->dkeys[j], s->stream, true);
      if (e != cudaSuccess) rc = set_err(MC_E_CUDA, "draft sample: %s", cudaGetErrorString(e));
    }
  }
  if (rc == MC_OK) rc = enq_verify(s, stochastic ? s->logits : nullptr);
  if (rc == MC_OK) {
    cudaError_t e = stochastic
                        ? launch_accept_stochastic(st, s->ctx, s->acc_log, vm, s->logits,
                                                   s->dlogits, V, s->stream, true)
                        : launch_accept_greedy(st, s->ctx, s->acc_log, vm, s->B, s->ctx_stride,
                                               s->ctx_stride, s->stream, true);
    if (e != cudaSuccess) rc = set_err(MC_E_CUDA, "accept launch: %s", cudaGetErrorString(e));
  }
  if (rc == MC_OK && s->cfg.kv_mode == KV_MIXED) {  // roll back dropped steps' window moves
    cudaError_t e = launch_kv_mixed_commit(s->st, kv_planes(s->tw, s->tkv, s->tkv.n_pages),
                                           s->mx_bak, s->B, vm, kMixedWindow, s->stream, true);
    if (e != cudaSuccess) rc = set_err(MC_E_CUDA, "mixed KV commit: %s", cudaGetErrorString(e));
  }
  if (rc == MC_OK && s->cfg.shift_context > 0) {  // generate.rs:738-748: the context shift
    cudaError_t e = launch_context_shift(shift_args(s), s->nsm, s->stream, true);
    if (e != cudaSuccess) rc = set_err(MC_E_CUDA, "context shift: %s", cudaGetErrorString(e));
  }
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(s->stream, &graph);
  if (rc != MC_OK) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (e != cudaSuccess) return set_err(MC_E_CUDA, "capture failed: %s", cudaGetErrorString(e));
  // the round's kernel launches, as captured
  size_t n_nodes = 0;
  int kernels = 0;
  if (cudaGraphGetNodes(graph, nullptr, &n_nodes) == cudaSuccess) {
    std::vector<cudaGraphNode_t> nodes(n_nodes);
    if (cudaGraphGetNodes(graph, nodes.data(), &n_nodes) == cudaSuccess)
      for (size_t i = 0; i < n_nodes; ++i) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(nodes[i], &t) == cudaSuccess && t == cudaGraphNodeTypeKernel)
          ++kernels;
      }
  }
  e = cudaGraphInstantiate(&s->round_exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) return set_err(MC_E_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
  s->round_launches = kernels;
  return MC_OK;
}

// Round state right after priming n_prompt tokens.
static SpecState fresh_state(const mc_session* s, int n_prompt) {
  SpecState h{};
  h.ctx_len = n_prompt;
  h.lt = n_prompt;
  h.ld = n_prompt - 1;
  h.generated = 0;
  h.prompt_len = n_prompt;
  h.gamma = s->cfg.gamma;
  h.bonus = s->cfg.bonus ? 1 : 0;
  h.rounds_cap = s->cap;
  h.accept_mode = s->cfg.accept_mode;
  h.temperature = s->cfg.temperature;
  h.seed_lo = (uint32_t)s->cfg.seed;
  h.seed_hi = (uint32_t)(s->cfg.seed >> 32);
  h.top_p = s->cfg.top_p;
  h.min_p = s->cfg.min_p;
  h.n_draft = s->cfg.gamma;
  h.ngram = kNgram;
  h.ng_len = std::max(0, n_prompt - kNgram);  // build_ngram_index over the prompt
  h.ng_last_len = n_prompt;
  return h;
}
static SpecState fresh_state(const mc_session* s, int z, int n_prompt) {
  SpecState h = fresh_state(s, n_prompt);
  if (s->cfg.kv_mode == KV_MIXED && z < (int)s->mx_hot0.size()) h.kv_hot = s->mx_hot0[z];
  return h;
}

// Prime request z (generate.rs:629-636): its prompt through the target and,
// all but the last token, through the draft, into its own KV pages.
// Target forwards over prompt tokens [t0, n_prompt) (t0 > 0: the K/V of the
// first t0 were restored from a prefix snapshot), draft forwards over all but
// the last.
static mc_status prime_request(mc_session* s, int z, int n_prompt, int t0 = 0, int hot0 = 0) {
  uint32_t* ctx = s->ctx + (size_t)z * s->ctx_stride;
  KVSet tkv = s->tkv, dkv = s->dkv;
  tkv.page_table += (size_t)z * tkv.n_pages;
  dkv.page_table += (size_t)z * dkv.n_pages;
  // a MIXED cache appends token by token (hot0: its window count at t0)
  const bool mixed = s->cfg.kv_mode == KV_MIXED;
  const int chunk = mixed ? 1 : kChunk;
  for (int c0 = t0; c0 < n_prompt; c0 += chunk) {
    const int M = std::min(chunk, n_prompt - c0);
    CK(launch_set_int(s->pos, c0, s->stream));
    EmbedArgs ea{};
    ea.src = SRC_IDS;
    ea.ids = ctx + c0;
    MixStep mx;
    mx.hot_const = hot0;
    mx.step = c0 - t0;
    CKS(enq_forward(s, s->tw, tkv, M, SeqMap{M, 0, 0, 0}, ea, s->pos, 0, s->fkeys, nullptr,
                    false, mixed ? &mx : nullptr));
  }
  if (mixed) s->mx_hot0[z] = std::min(hot0 + n_prompt - t0, kMixedWindow);
  // the draft gets all but the last prompt token (the first round forwards it)
  for (int c0 = 0; c0 < n_prompt - 1 && s->dw; c0 += kChunk) {
    const int M = std::min(kChunk, n_prompt - 1 - c0);
    CK(launch_set_int(s->pos + 1, c0, s->stream));
    EmbedArgs ea{};
    ea.src = SRC_IDS;
    ea.ids = ctx + c0;
    CKS(enq_forward(s, s->dw, dkv, M, SeqMap{M, 0, 0, 0}, ea, s->pos + 1, 0, s->fkeys, nullptr));
  }
  return MC_OK;
}

// A prefix-cache entry (prefix_cache.rs:14-24 CachedPrefix): the context
// tokens of one request and its target K/V -- the pages holding positions
// [0, len), every layer -- as they stood when it was taken.
struct mc_kv_snapshot {
  const mc_weights* W = nullptr;
  int dev = 0, kv_mode = 0, len = 0, pages = 0;
  int hot = 0;             // MIXED: tokens in the f32 window
  size_t page_floats = 0;  // floats of one KV page (Hkv heads x kPage positions x hdp)
  float* k = nullptr;      // [L][pages * page_floats]
  float* v = nullptr;
  std::vector<uint32_t> tokens;
};

static mc_status prime_impl(mc_session* s, const uint32_t* prompts, const int32_t* lens,
                            int32_t n_requests, const mc_kv_snapshot* snap);

extern "C" mc_status mc_spec_prime_batch(mc_session* s, const uint32_t* prompts,
                                         const int32_t* lens, int32_t n_requests) {
  return prime_impl(s, prompts, lens, n_requests, nullptr);
}

static mc_status prime_impl(mc_session* s, const uint32_t* prompts, const int32_t* lens,
                            int32_t n_requests, const mc_kv_snapshot* snap) {
  if (!s || !lens || !prompts) return set_err(MC_E_INVALID, "bad arguments");
  if (n_requests != s->B)
    return set_err(MC_E_INVALID, "%d prompts for a session of %d requests", n_requests, s->B);
  if (!s->dw && s->cfg.temperature > 0.0f)
    return set_err(MC_E_INVALID, "stochastic rounds need a transformer draft model (their "
                   "acceptance reads the draft's distributions)");
  if (s->cfg.gamma < 1) return set_err(MC_E_INVALID, "gamma must be >= 1");
  for (int z = 0; z < n_requests; ++z) {
    if (lens[z] <= 0) return set_err(MC_E_INVALID, "empty prompt (generate.rs:609-611 returns nothing)");
    if (lens[z] + s->cfg.gamma + 2 > s->cap)
      return set_err(MC_E_CAPACITY, "prompt of %d does not fit KV capacity %d", lens[z], s->cap);
  }
  CKS(check_usable(s));
  CK(cudaSetDevice(s->dev));
  s->prompt_len = lens[0];
  s->prompt_lens.assign(lens, lens + n_requests);
  s->draft_tokens.clear();
  size_t off = 0;
  for (int z = 0; z < n_requests; ++z) {
    memcpy(s->h_ids + (size_t)z * s->ctx_stride, prompts + off, (size_t)lens[z] * 4);
    off += (size_t)lens[z];
  }
  CK(cudaMemcpyAsync(s->ctx, s->h_ids, (size_t)n_requests * s->ctx_stride * 4,
                     cudaMemcpyHostToDevice, s->stream));
  if (s->ng) {  // the n-gram index of each prompt: every window, in order
    const size_t row = (size_t)s->ng_cap * (kNgram + 1);
    std::vector<uint32_t> ents((size_t)n_requests * row, 0u);
    off = 0;
    for (int z = 0; z < n_requests; ++z) {
      for (int i = 0; i + kNgram < lens[z]; ++i)
        memcpy(&ents[z * row + (size_t)i * (kNgram + 1)], prompts + off + i, (kNgram + 1) * 4);
      off += (size_t)lens[z];
    }
    CK(cudaMemcpyAsync(s->ng, ents.data(), ents.size() * 4, cudaMemcpyHostToDevice, s->stream));
    CK(cudaStreamSynchronize(s->stream));  // ents is a host temporary
  }
  int t0 = 0, hot0 = 0;
  s->mx_hot0.assign(n_requests, 0);
  if (snap) {  // request 0's first snap->len positions from the snapshot
    const size_t per_layer = (size_t)snap->pages * snap->page_floats;
    for (int l = 0; l < s->tw->L; ++l) {
      CK(cudaMemcpyAsync(s->tkv.k + l * s->tkv.layer_stride, snap->k + l * per_layer,
                         per_layer * sizeof(float), cudaMemcpyDeviceToDevice, s->stream));
      CK(cudaMemcpyAsync(s->tkv.v + l * s->tkv.layer_stride, snap->v + l * per_layer,
                         per_layer * sizeof(float), cudaMemcpyDeviceToDevice, s->stream));
    }
    t0 = snap->len;
    hot0 = snap->hot;
  }
  for (int z = 0; z < n_requests; ++z)
    CKS(prime_request(s, z, lens[z], z == 0 ? t0 : 0, z == 0 ? hot0 : 0));
  std::vector<SpecState> h(n_requests);
  for (int z = 0; z < n_requests; ++z) h[z] = fresh_state(s, z, lens[z]);
  CK(cudaMemcpyAsync(s->st, h.data(), sizeof(SpecState) * n_requests, cudaMemcpyHostToDevice,
                     s->stream));
  CK(cudaStreamSynchronize(s->stream));
  CKS(check_err(s));
  s->lt = lens[0];
  s->ld = lens[0] - 1;
  return MC_OK;
}

extern "C" mc_status mc_spec_prime(mc_session* s, const uint32_t* prompt, int32_t n_prompt) {
  if (!s || (!prompt && n_prompt > 0) || n_prompt < 0) return set_err(MC_E_INVALID, "bad arguments");
  if (s->B != 1) return set_err(MC_E_INVALID, "batched session: use mc_spec_prime_batch");
  return mc_spec_prime_batch(s, prompt, &n_prompt, 1);
}

extern "C" mc_status mc_kv_snapshot_take(mc_session* s, int32_t request, mc_kv_snapshot** out) {
  if (!s || !out) return set_err(MC_E_INVALID, "null argument");
  *out = nullptr;
  if (request < 0 || request >= s->B)
    return set_err(MC_E_INVALID, "request %d outside [0, %d)", request, s->B);
  if (!s->prompt_len) return set_err(MC_E_INVALID, "call mc_spec_prime first");
  if (s->tw->tp_world > 1) return set_err(MC_E_INVALID, "tensor-parallel sessions take no snapshot");
  CKS(check_usable(s));
  CK(cudaSetDevice(s->dev));
  CK(cudaStreamSynchronize(s->stream));
  SpecState h{};
  CK(cudaMemcpy(&h, s->st + request, sizeof(h), cudaMemcpyDeviceToHost));
  mc_kv_snapshot* snap = new mc_kv_snapshot();
  snap->W = s->tw;
  snap->dev = s->dev;
  snap->kv_mode = s->cfg.kv_mode;
  snap->len = h.lt;  // equal to the context length after a prime or a round
  snap->hot = h.kv_hot;
  snap->pages = (h.lt + kPage - 1) / kPage;
  snap->page_floats = (size_t)s->tw->Hkv * kPage * s->tw->hdp;
  snap->tokens.resize((size_t)h.ctx_len);
  mc_status st = MC_OK;
  if (h.ctx_len > 0 &&
      cudaMemcpy(snap->tokens.data(), s->ctx + (size_t)request * s->ctx_stride, (size_t)h.ctx_len * 4,
                 cudaMemcpyDeviceToHost) != cudaSuccess)
    st = set_err(MC_E_CUDA, "snapshot token copy failed");
  const size_t per_layer = (size_t)snap->pages * snap->page_floats;
  const size_t total = std::max<size_t>(per_layer * s->tw->L, 1);
  if (st == MC_OK && (cudaMalloc(&snap->k, total * sizeof(float)) != cudaSuccess ||
                      cudaMalloc(&snap->v, total * sizeof(float)) != cudaSuccess))
    st = set_err(MC_E_OOM, "snapshot of %zu bytes", 2 * total * sizeof(float));
  // request z's pages are [z * n_pages, (z + 1) * n_pages) of every layer
  const size_t first = (size_t)request * s->tkv.n_pages * snap->page_floats;
  for (int l = 0; l < s->tw->L && st == MC_OK; ++l)
    if (cudaMemcpy(snap->k + l * per_layer, s->tkv.k + l * s->tkv.layer_stride + first,
                   per_layer * sizeof(float), cudaMemcpyDeviceToDevice) != cudaSuccess ||
        cudaMemcpy(snap->v + l * per_layer, s->tkv.v + l * s->tkv.layer_stride + first,
                   per_layer * sizeof(float), cudaMemcpyDeviceToDevice) != cudaSuccess)
      st = set_err(MC_E_CUDA, "snapshot copy failed");
  if (st != MC_OK) {
    mc_kv_snapshot_destroy(snap);
    return st;
  }
  *out = snap;
  return MC_OK;
}

extern "C" int32_t mc_kv_snapshot_tokens(const mc_kv_snapshot* snap, uint32_t* out, int32_t cap) {
  if (!snap) return 0;
  const int n = (int)snap->tokens.size();
  if (out && cap > 0) memcpy(out, snap->tokens.data(), (size_t)std::min(n, (int)cap) * 4);
  return n;
}

extern "C" mc_status mc_kv_snapshot_destroy(mc_kv_snapshot* snap) {
  if (!snap) return MC_OK;
  cudaSetDevice(snap->dev);
  if (snap->k) cudaFree(snap->k);
  if (snap->v) cudaFree(snap->v);
  delete snap;
  return MC_OK;
}

extern "C" mc_status mc_spec_prime_cached(mc_session* s, const mc_kv_snapshot* snap,
                                          const uint32_t* prompt, int32_t n_prompt) {
  if (!s || !snap || !prompt || n_prompt <= 0) return set_err(MC_E_INVALID, "bad arguments");
  if (s->B != 1) return set_err(MC_E_INVALID, "batched session: prime requests one by one");
  if (snap->W != s->tw || snap->dev != s->dev)
    return set_err(MC_E_INVALID, "the snapshot was taken from another target model or device");
  if (snap->kv_mode != s->cfg.kv_mode)
    return set_err(MC_E_INVALID, "the snapshot holds another KV variant (%d, session %d)",
                   snap->kv_mode, s->cfg.kv_mode);
  const int n = (int)snap->tokens.size();
  if (n > n_prompt || snap->len != n ||
      memcmp(snap->tokens.data(), prompt, (size_t)n * 4) != 0)
    return set_err(MC_E_INVALID, "the snapshot's %d tokens are not a prefix of the prompt", n);
  if ((size_t)snap->pages * snap->page_floats > s->tkv.layer_stride)
    return set_err(MC_E_CAPACITY, "the snapshot does not fit this session's KV");
  return prime_impl(s, prompt, &n_prompt, 1, snap);
}

// Round loop of every request until each holds >= max_tokens generated ids.
// The reference checks the budget only at round start (generate.rs:638):
// each request's acceptance leaves it unchanged once its budget is spent, and
// launching ceil(max remaining / max_emit) rounds per batch keeps every
// launched round one that the request with the most left would also run.
constexpr int kRoundsPerBatch = 64;
extern "C" mc_status mc_spec_decode(mc_session* s, int32_t max_tokens, int32_t* n_generated) {
  if (!s || max_tokens < 0) return set_err(MC_E_INVALID, "bad arguments");
  if (!s->prompt_len) return set_err(MC_E_INVALID, "call mc_spec_prime first");
  CKS(check_usable(s));
  CK(cudaSetDevice(s->dev));
  CKS(capture_round(s));
  const int B = s->B;
  const int max_emit = s->cfg.gamma + (s->cfg.bonus ? 1 : 0);
  std::vector<SpecState> h(B);
  CK(cudaMemcpy(h.data(), s->st, sizeof(SpecState) * B, cudaMemcpyDeviceToHost));
  for (int z = 0; z < B; ++z)
    CK(cudaMemcpyAsync(&s->st[z].max_tokens, &max_tokens, 4, cudaMemcpyHostToDevice, s->stream));
  // with the context shift the context stays within shift_context + a round
  // (checked at session creation), but the generated count can fall when
  // generated tokens are evicted, as in the reference's loop; a bound on the
  // rounds ends a decode whose budget the shifts never let it reach
  const bool shifting = s->cfg.shift_context > 0;
  long long rounds_left = 8ll * ((long long)max_tokens + s->cap);
  for (;;) {
    if (s->cfg.cancel && *s->cfg.cancel) return set_err(MC_E_CANCELLED, "cancelled");
    int most = 0;
    for (int z = 0; z < B; ++z) most = std::max(most, max_tokens - h[z].generated);
    if (most <= 0) break;
    // at most kRoundsPerBatch rounds between two looks at the cancel flag
    const int R = std::min((most + max_emit - 1) / max_emit, kRoundsPerBatch);
    for (int z = 0; z < B && !shifting; ++z) {
      const int remaining = max_tokens - h[z].generated;
      if (remaining <= 0) continue;
      const int growth = std::min(max_emit * R, remaining + max_emit - 1);
      if (h[z].ctx_len + growth + max_emit + 2 > s->cap)
        return set_err(MC_E_CAPACITY, "generation would exceed KV capacity %d", s->cap);
    }
    if ((rounds_left -= R) < 0)
      return set_err(MC_E_CAPACITY, "the context shift keeps the generated count below %d "
                     "(max_tokens above what a shifted context holds)", max_tokens);
    for (int r = 0; r < R; ++r) CK(cudaGraphLaunch(s->round_exec, s->stream));
    CK(cudaMemcpyAsync(h.data(), s->st, sizeof(SpecState) * B, cudaMemcpyDeviceToHost, s->stream));
    CK(cudaStreamSynchronize(s->stream));
    CKS(check_err(s));
  }
  s->lt = h[0].lt;
  s->ld = h[0].ld;
  if (n_generated) {
    int total = 0;
    for (int z = 0; z < B; ++z) total += h[z].generated;
    *n_generated = total;
  }
  return MC_OK;
}

extern "C" mc_status mc_spec_read_request(mc_session* s, int32_t z, uint32_t* out, int32_t cap,
                                          int32_t* n_out, int32_t* accepted, int32_t accepted_cap,
                                          int32_t* n_rounds) {
  if (!s) return set_err(MC_E_INVALID, "null session");
  if (z < 0 || z >= s->B) return set_err(MC_E_INVALID, "request %d outside [0, %d)", z, s->B);
  CK(cudaSetDevice(s->dev));
  SpecState h{};
  CK(cudaMemcpy(&h, s->st + z, sizeof(h), cudaMemcpyDeviceToHost));
  const uint32_t* ctx = s->ctx + (size_t)z * s->ctx_stride;
  const int gen = h.ctx_len - h.prompt_len;
  const int nc = std::max(0, std::min(gen, (int)cap));
  if (out && nc) CK(cudaMemcpy(out, ctx + h.prompt_len, (size_t)nc * 4, cudaMemcpyDeviceToHost));
  if (n_out) *n_out = nc;
  if (accepted && accepted_cap > 0) {
    const int na = std::min(h.n_rounds, (int)accepted_cap);
    if (na)
      CK(cudaMemcpy(accepted, s->acc_log + (size_t)z * s->ctx_stride, (size_t)na * 4,
                    cudaMemcpyDeviceToHost));
  }
  if (n_rounds) *n_rounds = h.n_rounds;
  return MC_OK;
}

extern "C" mc_status mc_spec_read(mc_session* s, uint32_t* out, int32_t cap, int32_t* n_out,
                                  int32_t* accepted, int32_t accepted_cap, int32_t* n_rounds) {
  return mc_spec_read_request(s, 0, out, cap, n_out, accepted, accepted_cap, n_rounds);
}

extern "C" mc_status mc_spec_rewind(mc_session* s) {
  if (!s || !s->prompt_len) return set_err(MC_E_INVALID, "call mc_spec_prime first");
  CK(cudaSetDevice(s->dev));
  std::vector<SpecState> h(s->B);
  if (s->cfg.shift_context > 0) {  // a shifted context no longer holds the prompt
    CK(cudaMemcpy(h.data(), s->st, sizeof(SpecState) * s->B, cudaMemcpyDeviceToHost));
    for (int z = 0; z < s->B; ++z)
      if (h[z].n_shifts > 0)
        return set_err(MC_E_INVALID, "request %d's context was shifted: prime it again", z);
  }
  for (int z = 0; z < s->B; ++z) h[z] = fresh_state(s, z, s->prompt_lens[z]);
  CK(cudaMemcpyAsync(s->st, h.data(), sizeof(SpecState) * s->B, cudaMemcpyHostToDevice, s->stream));
  CK(cudaStreamSynchronize(s->stream));
  s->lt = h[0].lt;
  s->ld = h[0].ld;
  return MC_OK;
}

extern "C" mc_status mc_tp_unique_id(char id_out[128]) {
  if (!id_out) return set_err(MC_E_INVALID, "null argument");
  CKS(nccl::load());
  nccl::UniqueId id;
  CKS(nccl::check(nccl::g_api.get_unique_id(&id), "ncclGetUniqueId"));
  memcpy(id_out, id.internal, sizeof(id.internal));
  return MC_OK;
}

extern "C" mc_status mc_session_tp_init(mc_session* s, const char id[128], int32_t rank,
                                        int32_t world) {
  if (!s || !id) return set_err(MC_E_INVALID, "null argument");
  if (s->comm) return set_err(MC_E_INVALID, "tensor parallelism already initialised");
  if (world != s->tw->tp_world || rank != s->tw->tp_rank)
    return set_err(MC_E_INVALID, "rank %d of %d does not match the weights' shard %d of %d", rank,
                   world, s->tw->tp_rank, s->tw->tp_world);
  if (world < 2) return set_err(MC_E_INVALID, "tp_world must be at least 2");
  CKS(nccl::load());
  CK(cudaSetDevice(s->dev));
  nccl::UniqueId uid;
  memcpy(uid.internal, id, sizeof(uid.internal));
  nccl::Comm comm = nullptr;
  CKS(nccl::check(nccl::g_api.comm_init_rank(&comm, world, uid, rank), "ncclCommInitRank"));
  s->comm = comm;
  return MC_OK;
}

extern "C" mc_status mc_session_tp_ipc_handle(mc_session* s, char handle_out[64]) {
  if (!s || !handle_out) return set_err(MC_E_INVALID, "null argument");
  if (!s->tp_region) return set_err(MC_E_INVALID, "session has no tensor-parallel target");
  CK(cudaSetDevice(s->dev));
  cudaIpcMemHandle_t h;
  CK(cudaIpcGetMemHandle(&h, s->tp_region));
  static_assert(sizeof(h) == 64, "IPC handle size");
  memcpy(handle_out, &h, 64);
  std::lock_guard<std::mutex> lock(g_export_mu);
  bool known = false;
  for (const ExportedRegion& x : g_exports) known |= x.ptr == s->tp_region;
  if (!known) {
    ExportedRegion x{};
    memcpy(x.handle, &h, 64);
    x.dev = s->dev;
    x.ptr = s->tp_region;
    g_exports.push_back(x);
  }
  return MC_OK;
}

extern "C" mc_status mc_session_tp_open_peers(mc_session* s, const char* handles) {
  if (!s || !handles) return set_err(MC_E_INVALID, "null argument");
  if (!s->tp_region) return set_err(MC_E_INVALID, "session has no tensor-parallel target");
  if (s->tp_p2p) return set_err(MC_E_INVALID, "peers already open");
  if (s->round_exec || s->verify_exec)
    return set_err(MC_E_INVALID, "open the peers before the first decode");
  const int R = s->tw->tp_world, rank = s->tw->tp_rank;
  if (R > kMaxTP) return set_err(MC_E_INVALID, "tp_world %d above %d for peer reduction", R, kMaxTP);
  CK(cudaSetDevice(s->dev));
  TPArgs t{};
  t.rank = rank;
  t.world = R;
  t.d = s->tw->d;
  t.epoch = s->tp_epoch;
  t.kepoch = s->tp_kepoch;
  t.cnt = s->tp_cnt_gemv;
  t.err = s->err;
  t.wait_ns = s->wait_ns;
  for (int r = 0; r < R; ++r) {
    char* base = nullptr;
    ExportedRegion local{};
    bool in_process = false;
    if (r != rank) {
      std::lock_guard<std::mutex> lock(g_export_mu);
      for (const ExportedRegion& x : g_exports)
        if (!memcmp(x.handle, handles + 64 * r, 64)) {
          local = x;
          in_process = true;
        }
    }
    if (r == rank) {
      base = (char*)s->tp_region;
    } else if (in_process) {  // a peer session of this process: its pointer as is
      if (local.dev != s->dev) {
        int can = 0;
        CK(cudaDeviceCanAccessPeer(&can, s->dev, local.dev));
        if (!can) return set_err(MC_E_CUDA, "device %d cannot access device %d", s->dev, local.dev);
        cudaError_t e = cudaDeviceEnablePeerAccess(local.dev, 0);
        if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
        else CK(e);
      }
      base = (char*)local.ptr;
    } else {
      cudaIpcMemHandle_t h;
      memcpy(&h, handles + 64 * r, 64);
      void* p = nullptr;
      cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) {
        for (void* q : s->tp_opened) cudaIpcCloseMemHandle(q);
        s->tp_opened.clear();
        return set_err(MC_E_CUDA, "opening rank %d's reduce buffer: %s", r, cudaGetErrorString(e));
      }
      s->tp_opened.push_back(p);
      base = (char*)p;
    }
    t.red[r] = (float*)base;
    t.flag[r] = (unsigned*)(base + s->tp_red_bytes);
    t.keyx[r] = (unsigned long long*)(base + s->tp_keyx_off);
    t.kflag[r] = (unsigned*)(base + s->tp_kflag_off);
  }
  s->tp = t;
  s->tp_p2p = true;
  return MC_OK;
}

extern "C" mc_status mc_spec_set_seed(mc_session* s, uint64_t seed) {
  if (!s) return set_err(MC_E_INVALID, "null session");
  s->cfg.seed = seed;
  if (!s->prompt_len) return MC_OK;  // taken at the next mc_spec_prime
  CK(cudaSetDevice(s->dev));
  const uint32_t v[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  CK(cudaMemcpyAsync(&s->st->seed_lo, v, sizeof(v), cudaMemcpyHostToDevice, s->stream));
  CK(cudaStreamSynchronize(s->stream));
  return MC_OK;
}

extern "C" mc_status mc_spec_verify_launch(mc_session* s, int32_t n) {
  if (!s || n < 0) return set_err(MC_E_INVALID, "bad arguments");
  if (!s->prompt_len) return set_err(MC_E_INVALID, "call mc_spec_prime first");
  CK(cudaSetDevice(s->dev));
  CKS(capture_verify(s));
  for (int i = 0; i < n; ++i) CK(cudaGraphLaunch(s->verify_exec, s->stream));
  return MC_OK;
}

extern "C" void* mc_session_stream(mc_session* s) { return s ? (void*)s->stream : nullptr; }

extern "C" mc_status mc_session_set_wait_timeout(mc_session* s, int32_t ms) {
  if (!s || ms < 1) return set_err(MC_E_INVALID, "bad arguments");
  CK(cudaSetDevice(s->dev));
  const long long ns = (long long)ms * 1000000ll;
  CK(cudaMemcpyAsync(s->wait_ns, &ns, sizeof(ns), cudaMemcpyHostToDevice, s->stream));
  CK(cudaStreamSynchronize(s->stream));
  return MC_OK;
}

extern "C" int32_t mc_session_round_launches(const mc_session* s) {
  return s ? s->round_launches : 0;
}

extern "C" mc_status mc_speculative_generate(mc_session* s, const uint32_t* prompt,
                                             int32_t n_prompt, int32_t max_tokens, uint32_t* out,
                                             int32_t cap, int32_t* n_out, int32_t* accepted,
                                             int32_t accepted_cap, int32_t* n_rounds) {
  if (n_out) *n_out = 0;
  if (n_rounds) *n_rounds = 0;
  if (s && n_prompt == 0) return MC_OK;  // generate.rs:609-611
  CKS(mc_spec_prime(s, prompt, n_prompt));
  CKS(mc_spec_decode(s, max_tokens, nullptr));
  return mc_spec_read(s, out, cap, n_out, accepted, accepted_cap, n_rounds);
}

extern "C" mc_status mc_speculative_generate_batch(mc_session* s, const uint32_t* prompts,
                                                   const int32_t* lens, int32_t n_requests,
                                                   int32_t max_tokens, uint32_t* out,
                                                   int32_t out_stride, int32_t* n_out,
                                                   int32_t* accepted, int32_t accepted_stride,
                                                   int32_t* n_rounds) {
  if (!s || !n_out || out_stride < 0 || (accepted && accepted_stride < 0))
    return set_err(MC_E_INVALID, "bad arguments");
  CKS(mc_spec_prime_batch(s, prompts, lens, n_requests));
  CKS(mc_spec_decode(s, max_tokens, nullptr));
  for (int z = 0; z < n_requests; ++z)
    CKS(mc_spec_read_request(s, z, out ? out + (size_t)z * out_stride : nullptr, out_stride,
                             &n_out[z], accepted ? accepted + (size_t)z * accepted_stride : nullptr,
                             accepted ? accepted_stride : 0, n_rounds ? &n_rounds[z] : nullptr));
  return MC_OK;
}

// ------------------------------------------------------------------ standalone linear
struct mc_linear {
  int dev = 0;
  PMat m;
  Allocs al;
  uint8_t* xq = nullptr;
  int* xexp = nullptr;
  unsigned* amax = nullptr;  // per-token max |x| for the encoder
  int* ws = nullptr;
  int* cnt = nullptr;
  int* err = nullptr;
  int nsm = 0;
  int bps[3][7] = {};
};

static int linear_grid(mc_linear* l, int nt) {
  return gemv_grid(l->m, l->nsm, nt, [&](int t) {
    int& b = l->bps[gemv_wf(l->m)][t];
    if (!b) b = std::max(1, gemv_blocks_per_sm(EPI_STORE, t, gemv_wf(l->m)));
    return b;
  });
}

extern "C" mc_status mc_linear_create(const mc_tensor_desc* w, int32_t device, mc_linear** out) {
  if (!w || !out) return set_err(MC_E_INVALID, "null argument");
  *out = nullptr;
  CKS(check_device(device));
  mc_linear* L = new mc_linear();
  L->dev = device;
  SrcI8 src;
  mc_status st = stage_matrix(w, &src);
  if (st == MC_OK)
    st = pack_matrix(src, identity_map(src.rows, round_up(src.rows, 16)),
                     identity_map(src.cols, round_up(src.cols, 32)), src.rows, src.cols, L->al,
                     &L->m);
  const int kp = round_up(src.cols, 128);  // whole K atoms of the tcgen05 digit layout
  if (st == MC_OK && (prepare_kernels(0, 0) != cudaSuccess || prepare_tc() != cudaSuccess))
    st = set_err(MC_E_CUDA, "kernel preparation failed");
  if (st == MC_OK) st = L->al.alloc(&L->xq, (size_t)kp * 48 * kMaxGroups);
  if (st == MC_OK) st = L->al.alloc(&L->xexp, (size_t)kMaxTokens);
  if (st == MC_OK) st = L->al.alloc(&L->amax, (size_t)kMaxTokens);
  if (st == MC_OK) st = L->al.alloc(&L->ws, (size_t)L->m.n_stripes * kMaxGroups * 16 * 48);
  if (st == MC_OK) st = L->al.alloc(&L->cnt, (size_t)L->m.n_stripes * kMaxGroups);
  if (st == MC_OK) st = L->al.alloc(&L->err, 1);
  if (st == MC_OK && cudaMemset(L->err, 0, 4) != cudaSuccess) st = set_err(MC_E_CUDA, "memset");
  if (st == MC_OK &&
      (cudaMemset(L->xq, 0, (size_t)kp * 48 * kMaxGroups) != cudaSuccess ||
       cudaMemset(L->ws, 0, (size_t)L->m.n_stripes * kMaxGroups * 16 * 48 * 4) != cudaSuccess ||
       cudaMemset(L->cnt, 0, (size_t)L->m.n_stripes * kMaxGroups * 4) != cudaSuccess))
    st = set_err(MC_E_CUDA, "memset failed");
  cudaDeviceGetAttribute(&L->nsm, cudaDevAttrMultiProcessorCount, device);
  if (st == MC_OK)
    for (int nt : {1, 2, 3, 6})
      L->bps[gemv_wf(L->m)][nt] = std::max(1, gemv_blocks_per_sm(EPI_STORE, nt, gemv_wf(L->m)));
  if (st != MC_OK) {
    L->al.free_all();
    delete L;
    return st;
  }
  *out = L;
  return MC_OK;
}

extern "C" mc_status mc_linear_destroy(mc_linear* l) {
  if (!l) return MC_OK;
  cudaSetDevice(l->dev);
  l->al.free_all();
  delete l;
  return MC_OK;
}

extern "C" int64_t mc_linear_weight_bytes(const mc_linear* l) { return l ? l->m.algo_bytes : 0; }

extern "C" mc_status mc_linear_run(mc_linear* l, const float* x_dev, int32_t m, float* y_dev,
                                   void* stream) {
  if (!l || (!x_dev && m > 0) || (!y_dev && m > 0) || m < 0)
    return set_err(MC_E_INVALID, "bad arguments");
  CK(cudaSetDevice(l->dev));
  cudaStream_t s = (cudaStream_t)stream;
  for (int r0 = 0; r0 < m; r0 += kMaxTokens) {
    const int M = std::min(kMaxTokens, m - r0);
    CK(launch_act_amax(x_dev + (size_t)r0 * l->m.K, l->m.K, l->m.K, M, l->amax, s, true));
    QuantArgs q{};
    q.h = x_dev + (size_t)r0 * l->m.K;
    q.ld = l->m.K;
    q.d = l->m.K;
    q.M = M;
    q.xq = l->xq;
    q.KB = l->m.KB;
    q.nt = nt_for_tokens(M);
    q.xexp = l->xexp;
    q.tc_layout = use_tc(l->m, M) ? 1 : 0;
    q.use_stats = 1;  // max |x| per token from k_act_amax; no norm, no partial sums
    q.amax = l->amax;
    CK(launch_quant(q, s, true));
    GemvArgs a{};
    a.x = l->xq;
    a.xexp = l->xexp;
    a.ws = l->ws;
    a.cnt = l->cnt;
    a.err = l->err;
    a.out = y_dev + (size_t)r0 * l->m.N;
    a.ldo = l->m.N;
    a.n_out = l->m.N;
    CK(run_projection(l->m, EPI_STORE, M, a, l->nsm, s, [&](int t) {
      int& b = l->bps[gemv_wf(l->m)][t];
      if (!b) b = std::max(1, gemv_blocks_per_sm(EPI_STORE, t, gemv_wf(l->m)));
      return b;
    }));
  }
  return MC_OK;
}

// ------------------------------------------------ allocation-free projection
// mc_linear_run_static: the encoder + GEMV pair of mc_linear_run with its
// activation scratch in one module-scope device array instead of buffers the
// handle owns.  Layout: packed digit words (48 bytes per input column: up to
// 6 n8 tiles x 8 columns, one byte each) then kMaxTokens int exponents.
constexpr int kStaticMaxK = 16384;
constexpr size_t kStaticXqBytes = (size_t)kStaticMaxK * 48;  // 768 KiB
constexpr size_t kStaticBytes = kStaticXqBytes + 256;        // + exponents
static_assert(kMaxTokens * sizeof(int) <= 256, "exponent slot too small");
static __device__ __align__(256) unsigned char g_static_scratch[kStaticBytes];

constexpr int kStaticMaxDevices = 64;
static std::mutex g_static_mu;
static unsigned char* g_static_ptr[kStaticMaxDevices];

// Set-up, once per device, with that device current: the array's device
// address.  Nothing in the array has to be zero at the start of a call, so
// there is no clear (a clear on another stream than the caller's would not be
// ordered before the first encoder): every call's encoder rewrites all digit
// words the GEMV reads, the zero digits of columns past in_features and the
// padding columns of the last n8 tile included, and the exponents of its
// tokens.  The address is cached for the life of the process, so
// cudaDeviceReset on a device is not supported while this library is in use
// there: the module is reloaded and the array may move.
static mc_status static_scratch(int dev, unsigned char** out) {
  if (dev < 0 || dev >= kStaticMaxDevices)
    return set_err(MC_E_INVALID, "device %d outside [0, %d)", dev, kStaticMaxDevices);
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_ptr[dev]) {
    unsigned char* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress((void**)&ptr, g_static_scratch);
    if (e != cudaSuccess || !ptr)
      return set_err(MC_E_CUDA, "static scratch address on device %d: %s", dev,
                     cudaGetErrorString(e));
    g_static_ptr[dev] = ptr;
  }
  *out = g_static_ptr[dev];
  return MC_OK;
}

extern "C" mc_status mc_linear_run_static(mc_linear* l, const float* x_dev, int32_t m,
                                          float* y_dev, void* stream) {
  if (!l || (!x_dev && m > 0) || (!y_dev && m > 0) || m < 0)
    return set_err(MC_E_INVALID, "bad arguments");
  if (l->m.K > kStaticMaxK)
    return set_err(MC_E_CAPACITY,
                   "mc_linear_run_static: in_features %d exceeds the static scratch limit %d "
                   "(use mc_linear_run)", l->m.K, kStaticMaxK);
  CK(cudaSetDevice(l->dev));
  unsigned char* scratch = nullptr;
  CKS(static_scratch(l->dev, &scratch));
  uint8_t* xq = scratch;
  int* xexp = reinterpret_cast<int*>(scratch + kStaticXqBytes);
  cudaStream_t s = (cudaStream_t)stream;
  for (int r0 = 0; r0 < m; r0 += kGroupTokens) {  // the scratch holds one token group
    const int M = std::min(kGroupTokens, m - r0);
    const int nt = nt_for_tokens(M);
    QuantArgs q{};
    q.h = x_dev + (size_t)r0 * l->m.K;
    q.ld = l->m.K;
    q.d = l->m.K;
    q.M = M;
    q.xq = xq;
    q.KB = l->m.KB;
    q.nt = nt;
    q.xexp = xexp;
    CK(launch_quant(q, s, true));
    GemvArgs a{};
    a.w = l->m.w;
    a.scale = l->m.scale;
    a.qscale = l->m.qscale;
    a.x = xq;
    a.xexp = xexp;
    a.KB = l->m.KB;
    a.n_stripes = l->m.n_stripes;
    a.M = M;
    a.out = y_dev + (size_t)r0 * l->m.N;
    a.ldo = l->m.N;
    a.n_out = l->m.N;
    CK(launch_gemv(a, EPI_STORE, nt, gemv_wf(l->m), linear_grid(l, nt), s, true));
  }
  return MC_OK;
}

#ifdef MC_TRACE
// Timeline of the verify graph's launches (trace builds only; not part of
// the public header).
extern "C" MC_API int32_t mc_trace_reset(void) { return trace_reset() == cudaSuccess ? MC_OK : MC_E_CUDA; }
extern "C" MC_API int32_t mc_trace_read(unsigned long long* out, int32_t n) {
  return trace_read(out, n) == cudaSuccess ? MC_OK : MC_E_CUDA;
}
#endif

// generate.rs:948-969 sample, one token per row of device logits.
extern "C" mc_status mc_sample_rows(const float* logits_dev, int32_t n_rows, int32_t vocab,
                                    float temperature, float top_p, float min_p, uint64_t seed,
                                    uint32_t round, uint32_t* tokens_dev, void* stream) {
  if (n_rows < 0 || (n_rows > 0 && (!logits_dev || !tokens_dev)))
    return set_err(MC_E_INVALID, "bad arguments");
  if (vocab <= 0 || vocab > kSampleMaxVocab)
    return set_err(MC_E_SHAPE, "vocab %d outside [1, %d]", vocab, kSampleMaxVocab);
  if (!isfinite(temperature)) return set_err(MC_E_INVALID, "temperature must be finite");
  if (n_rows == 0) return MC_OK;
  cudaPointerAttributes pa{};
  CK(cudaPointerGetAttributes(&pa, logits_dev));
  if (pa.type != cudaMemoryTypeDevice && pa.type != cudaMemoryTypeManaged)
    return set_err(MC_E_INVALID, "logits must be device memory");
  CK(cudaSetDevice(pa.device));
  CK(launch_sample_rows(logits_dev, n_rows, vocab, temperature, top_p, min_p, seed, round,
                        tokens_dev, (cudaStream_t)stream));
  return MC_OK;
}
