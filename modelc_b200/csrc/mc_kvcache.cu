// mc_kvcache.cu -- the reference's KV cache variants and context shift on the
// paged device KV.
//
//  INT8 layer (KvLayer::Int8, transformer.rs:167-420): every appended token's
//  K and V are quantized with one scale per token (max |x| / 127 over all KV
//  heads); the cache then holds code * scale, the values k_all()/v_all()
//  return, in its f32 pages.
//
//  Context shift (generate.rs:26-63, KvCache::shift / shift_anchored,
//  transformer.rs:424-583): after a round whose context exceeds max_context,
//  overflow = len - max_ctx + max_ctx / 4 tokens leave the token list and
//  every layer's K/V -- the oldest ones, or (anchored) the ones right after
//  the first anchor_tokens -- and the kept positions move down.  Keys keep the
//  rotation of their old positions, as in the reference.  An anchored shift
//  re-appends the kept tokens, so an INT8 layer re-quantizes them.
#include <cuda_runtime.h>
#include <math.h>

#include "mc_internal.cuh"

namespace mc {

namespace {

constexpr int kKvqThreads = 256;

// The code and value of x at `scale` (quantize, transformer.rs:201-206, then
// q as f32 * scale): round half away from zero, clamp to +-127, NaN -> 0
// (Rust's saturating cast).
__device__ __forceinline__ float qdq_value(float x, float scale) {
  const float r = roundf(__fdiv_rn(x, scale));
  const float q = isnan(r) ? 0.0f : fminf(fmaxf(r, -127.0f), 127.0f);
  return __fmul_rn(q, scale);
}

// quantize_scale (transformer.rs:196-199) of the n = Hkv * hd values at
// base + (i / hd) * head_stride + i % hd, then every value through
// qdq_value: one warp.  f32::max skips NaN, as fmaxf does.
__device__ __forceinline__ void qdq_token_warp(float* base, int n, int hd, size_t head_stride,
                                               int lane) {
  float mx = 0.0f;
  for (int i = lane; i < n; i += 32) {
    const int h = i / hd;
    mx = fmaxf(mx, fabsf(base[(size_t)h * head_stride + (i - h * hd)]));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float scale = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
  for (int i = lane; i < n; i += 32) {
    const int h = i / hd;
    float* p = base + (size_t)h * head_stride + (i - h * hd);
    *p = qdq_value(*p, scale);
  }
}

// KvLayer::append of an INT8 layer (transformer.rs:375-388) for the tokens
// a forward just wrote: one warp per (token, K or V).
__global__ void __launch_bounds__(kKvqThreads) k_kv_qdq(KvQArgs a) {
  grid_launch_dependents();
  grid_wait();
  const int warp = (int)(blockIdx.x * (kKvqThreads / 32) + (threadIdx.x >> 5));
  const int lane = threadIdx.x & 31;
  if (warp >= 2 * a.M) return;
  const int m = warp >> 1;
  const int z = seq_of(a.seq, m);
  const int pos = a.pos_ptr[z * a.seq.pos_stride] + a.pos_add + seq_off(a.seq, m);
  const int pg = a.page_table[z * a.seq.pt_stride + pos / a.page];
  float* base = ((warp & 1) ? a.vc : a.kc) +
                ((size_t)pg * a.Hkv * a.page + (size_t)(pos % a.page)) * a.hdp;
  qdq_token_warp(base, a.Hkv * a.hd, a.hd, (size_t)a.page * a.hdp, lane);
}

// KvLayer::append of a MIXED layer (transformer.rs:389-419): one warp per
// (request, K or V).  The hot part holds the last min(hot + step, window)
// tokens before this append; when that is the window, the append pushes the
// oldest hot token -- `window` positions back -- into the cold part.
__global__ void __launch_bounds__(kKvqThreads) k_kv_mixed_age(KvMixArgs a) {
  grid_launch_dependents();
  grid_wait();
  const int warp = (int)(blockIdx.x * (kKvqThreads / 32) + (threadIdx.x >> 5));
  const int lane = threadIdx.x & 31;
  if (warp >= 2 * a.B) return;
  const int z = warp >> 1, sel = warp & 1;
  const int pos = a.pos_ptr[z * a.seq.pos_stride] + a.pos_add;
  if (a.base_out && a.step == 0 && a.layer == 0 && sel == 0 && lane == 0)
    a.base_out[z * a.base_stride] = pos;
  const int hot = a.hot_ptr ? a.hot_ptr[z * a.hot_stride] : a.hot_const;
  if (min(hot + a.step, a.window) < a.window) return;  // warp-uniform
  const int c = pos - a.window;
  const int pg = a.page_table[z * a.seq.pt_stride + c / a.page];
  float* base = (sel ? a.vc : a.kc) + ((size_t)pg * a.Hkv * a.page + (size_t)(c % a.page)) * a.hdp;
  const int n = a.Hkv * a.hdp;
  const size_t head_stride = (size_t)a.page * a.hdp;
  if (a.bak) {
    float* b = a.bak + ((((size_t)z * a.bak_steps + a.step) * a.layers + a.layer) * 2 + sel) * n;
    for (int i = lane; i < n; i += 32) b[i] = base[(size_t)(i / a.hdp) * head_stride + i % a.hdp];
    __syncwarp();
  }
  qdq_token_warp(base, n, a.hdp, head_stride, lane);
}

// Position p of head h in one layer of request z's KV (K or V base).
__device__ __forceinline__ float* kv_at(const KvPlanes& P, float* layer_base, int z, int h,
                                        int p) {
  const int pg = P.pt[(size_t)z * P.pt_stride + p / P.page];
  return layer_base + (((size_t)pg * P.Hkv + h) * P.page + (size_t)(p % P.page)) * P.hdp;
}

// The plan of every request's shift (one CTA each; thread 0 decides, the
// block moves the tokens).  generate.rs:32-63: overflow = len - max_ctx +
// max_ctx / 4; the anchored form when anchor > 0 and len > anchor + overflow
// (then the prompt length loses the removed prompt tokens past the anchor),
// else the oldest tokens (the prompt length saturating at 0).  The target KV
// holds len positions, the draft KV ld of them; both lose the removed range
// as far as they reach.  The n-gram index holds token content, so it is
// unchanged.
__global__ void __launch_bounds__(kKvqThreads) k_shift_plan(ShiftArgs a) {
  grid_launch_dependents();
  grid_wait();
  __shared__ int s_n, s_at, s_len;
  SpecState* st = a.st + blockIdx.x;
  uint32_t* ctx = a.ctx + (size_t)blockIdx.x * a.ctx_stride;
  if (threadIdx.x == 0) {
    const int L = st->ctx_len, mc_ = a.shift_context;
    int n = 0, at = 0, anch = 0;
    if (mc_ > 0 && L > mc_) {
      n = L - mc_ + mc_ / 4;
      anch = a.anchor > 0 && n > 0 && L > a.anchor + n;
      at = anch ? a.anchor : 0;
    }
    st->sh_n = n;
    st->sh_at = at;
    st->sh_anch = anch;
    st->sh_lt = st->lt;
    st->sh_ld = st->ld;
    if (n > 0) {
      if (anch) {
        if (st->prompt_len > at) {
          const int non_anchor = st->prompt_len - at;
          st->prompt_len = at + non_anchor - min(n, non_anchor);
        }
      } else {
        st->prompt_len = max(st->prompt_len - n, 0);
      }
      if (a.window > 0) {  // MIXED: shift drops cold tokens first; shift_anchored re-appends
        if (anch) {
          st->kv_hot = min(L - n, a.window);
        } else {
          const int cold = st->lt - st->kv_hot;
          if (n > cold) st->kv_hot -= n - cold;
        }
      }
      st->ctx_len = L - n;
      st->lt = st->lt - min(n, max(st->lt - at, 0));
      st->ld = st->ld - min(n, max(st->ld - at, 0));
      st->generated = st->ctx_len - st->prompt_len;
      // the index update of this round runs at the next round's start, on
      // the window ending at the last token (which the shift keeps): it
      // stays pending
      st->ng_last_len = max(st->ng_last_len - n, 0);
      st->n_shifts += 1;
    }
    s_n = n;
    s_at = at;
    s_len = L;
  }
  __syncthreads();
  const int n = s_n, at = s_at, L = s_len;
  if (n <= 0) return;
  // tokens [at + n, L) -> [at, L - n), chunks of at most n positions so a
  // chunk's reads and writes never overlap; the barrier orders the chunks
  for (int p0 = at; p0 < L - n; p0 += n) {
    const int c = min(n, L - n - p0);
    for (int i = threadIdx.x; i < c; i += blockDim.x) ctx[p0 + i] = ctx[p0 + n + i];
    __syncthreads();
  }
}

// The K/V moves: one (request, cache, layer, head, K or V) plane per
// iteration of a CTA, positions [at + rm, len) -> [at, len - rm) with rm the
// removed positions the cache holds, in chunks of at most rm positions (a
// chunk's reads and writes never overlap; the barrier orders the chunks).
__global__ void __launch_bounds__(kKvqThreads) k_shift_kv(ShiftArgs a) {
  grid_launch_dependents();
  grid_wait();
  const int per_t = a.t.layers * a.t.Hkv * 2, per_d = a.d.layers * a.d.Hkv * 2;
  const int per_z = per_t + per_d;
  for (int task = blockIdx.x; task < a.B * per_z; task += gridDim.x) {
    const int z = task / per_z;
    int r = task - z * per_z;
    const SpecState* st = a.st + z;
    const int n = st->sh_n, at = st->sh_at;
    if (n <= 0) continue;  // block-uniform
    const bool tgt = r < per_t;
    if (!tgt) r -= per_t;
    const KvPlanes& P = tgt ? a.t : a.d;
    const int len = tgt ? st->sh_lt : st->sh_ld;
    const int rm = min(n, max(len - at, 0));
    if (rm <= 0) continue;
    const int layer = r / (P.Hkv * 2), h = (r >> 1) % P.Hkv;
    float* base = ((r & 1) ? P.v : P.k) + (size_t)layer * P.layer_stride;
    const int hd4 = P.hdp / 4;
    for (int p0 = at; p0 < len - rm; p0 += rm) {
      const int c = min(rm, len - rm - p0);
      for (int i = threadIdx.x; i < c * hd4; i += blockDim.x) {
        const int t = i / hd4, q = i - t * hd4;
        const float4 v = reinterpret_cast<const float4*>(kv_at(P, base, z, h, p0 + rm + t))[q];
        reinterpret_cast<float4*>(kv_at(P, base, z, h, p0 + t))[q] = v;
      }
      __syncthreads();
    }
  }
}

// After an anchored shift of an INT8 or MIXED target: the kept tokens
// re-appended (transformer.rs:577-582), each one that reaches the int8 part
// re-quantized from its current values; one warp per (request, layer,
// position, K or V).
__global__ void __launch_bounds__(kKvqThreads) k_shift_requant(ShiftArgs a) {
  grid_launch_dependents();
  grid_wait();
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (kKvqThreads / 32);
  const long long per_z = (long long)a.t.layers * a.ctx_stride * 2;
  for (long long w = (long long)blockIdx.x * (kKvqThreads / 32) + (threadIdx.x >> 5);
       w < (long long)a.B * per_z; w += warps) {
    const int z = (int)(w / per_z);
    const SpecState* st = a.st + z;
    if (st->sh_n <= 0 || !st->sh_anch) continue;  // warp-uniform
    long long r = w - z * per_z;
    const int layer = (int)(r / ((long long)a.ctx_stride * 2));
    r -= (long long)layer * a.ctx_stride * 2;
    const int p = (int)(r >> 1);
    // re-appended tokens land in the cold part: all of them in an INT8
    // layer, all but the last `window` in a MIXED one
    if (p >= st->lt - a.window) continue;
    float* lb = ((r & 1) ? a.t.v : a.t.k) + (size_t)layer * a.t.layer_stride;
    qdq_token_warp(kv_at(a.t, lb, z, 0, p), a.t.Hkv * a.t.hd, a.t.hd,
                   (size_t)a.t.page * a.t.hdp, lane);
  }
}

// The verify steps a MIXED round's acceptance dropped: each one that moved a
// token to the cold part gets it back from bak.  One warp per (request,
// step, layer, K or V).
__global__ void __launch_bounds__(kKvqThreads) k_kv_mixed_restore(SpecState* st, KvPlanes t,
                                                                  const float* bak, int B,
                                                                  int steps, int window) {
  grid_launch_dependents();
  grid_wait();
  const int lane = threadIdx.x & 31;
  const long long w = (long long)blockIdx.x * (kKvqThreads / 32) + (threadIdx.x >> 5);
  if (w >= (long long)B * steps * t.layers * 2) return;
  const int sel = (int)(w & 1);
  long long r = w >> 1;
  const int layer = (int)(r % t.layers);
  r /= t.layers;
  const int i = (int)(r % steps), z = (int)(r / steps);
  const SpecState* q = st + z;
  const int kept = q->lt - q->mx_base;
  if (i < kept || min(q->kv_hot + i, window) < window) return;
  const int c = q->mx_base + i - window;
  const int n = t.Hkv * t.hdp;
  const float* b = bak + ((((size_t)z * steps + i) * t.layers + layer) * 2 + sel) * n;
  float* lb = (sel ? t.v : t.k) + (size_t)layer * t.layer_stride;
  for (int e = lane; e < n; e += 32) {
    const int h = e / t.hdp;
    kv_at(t, lb, z, h, c)[e - h * t.hdp] = b[e];
  }
}

__global__ void k_kv_mixed_hot(SpecState* st, int B, int window) {
  grid_launch_dependents();
  grid_wait();
  const int z = blockIdx.x * blockDim.x + threadIdx.x;
  if (z >= B) return;
  SpecState* q = st + z;
  q->kv_hot = min(q->kv_hot + (q->lt - q->mx_base), window);
}

cudaError_t launch_pdl(const void* f, dim3 grid, dim3 block, void** args, cudaStream_t s,
                       bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, f, args);
}

}  // namespace

cudaError_t launch_kv_qdq(const KvQArgs& a, cudaStream_t s, bool pdl) {
  if (a.M < 1 || a.Hkv < 1 || a.hd < 1 || a.hd > a.hdp || a.page < 1) return cudaErrorInvalidValue;
  KvQArgs x = a;
  void* args[] = {&x};
  const int warps = 2 * a.M, per = kKvqThreads / 32;
  return launch_pdl((const void*)k_kv_qdq, dim3((warps + per - 1) / per), dim3(kKvqThreads), args,
                    s, pdl);
}

cudaError_t launch_kv_mixed_age(const KvMixArgs& a, cudaStream_t s, bool pdl) {
  if (a.B < 1 || a.Hkv < 1 || a.hdp < 1 || a.page < 1 || a.window < 1 || a.step < 0 ||
      (a.bak && (a.step >= a.bak_steps || a.layer >= a.layers)))
    return cudaErrorInvalidValue;
  KvMixArgs x = a;
  void* args[] = {&x};
  const int warps = 2 * a.B, per = kKvqThreads / 32;
  return launch_pdl((const void*)k_kv_mixed_age, dim3((warps + per - 1) / per), dim3(kKvqThreads),
                    args, s, pdl);
}

cudaError_t launch_kv_mixed_commit(SpecState* st, const KvPlanes& t, const float* bak, int B,
                                   int steps, int window, cudaStream_t s, bool pdl) {
  if (B < 1 || steps < 1 || window < 1 || t.layers < 1) return cudaErrorInvalidValue;
  SpecState* st_ = st;
  KvPlanes t_ = t;
  const float* bak_ = bak;
  int B_ = B, steps_ = steps, window_ = window;
  void* args[] = {&st_, &t_, &bak_, &B_, &steps_, &window_};
  const long long warps = (long long)B * steps * t.layers * 2;
  const int per = kKvqThreads / 32;
  cudaError_t e = launch_pdl((const void*)k_kv_mixed_restore, dim3((unsigned)((warps + per - 1) / per)),
                             dim3(kKvqThreads), args, s, pdl);
  if (e != cudaSuccess) return e;
  void* args2[] = {&st_, &B_, &window_};
  return launch_pdl((const void*)k_kv_mixed_hot, dim3((B + 127) / 128), dim3(128), args2, s, pdl);
}

cudaError_t launch_context_shift(const ShiftArgs& a, int nsm, cudaStream_t s, bool pdl) {
  if (a.B < 1 || a.shift_context < 1 || a.t.layers < 0 || (a.t.hdp & 3) || (a.d.hdp & 3))
    return cudaErrorInvalidValue;
  ShiftArgs x = a;
  void* args[] = {&x};
  cudaError_t e = launch_pdl((const void*)k_shift_plan, dim3(a.B), dim3(kKvqThreads), args, s, pdl);
  if (e == cudaSuccess)
    e = launch_pdl((const void*)k_shift_kv, dim3(nsm > 0 ? 2 * nsm : 296), dim3(kKvqThreads), args,
                   s, pdl);
  if (e == cudaSuccess && a.requant)
    e = launch_pdl((const void*)k_shift_requant, dim3(nsm > 0 ? 2 * nsm : 296),
                   dim3(kKvqThreads), args, s, pdl);
  return e;
}

}  // namespace mc
