// mc_kernels.cu -- sm_100a kernels of the speculative-decoding step.
//
//  k_gemv      quantized int8 x fixed-point-digit GEMV/skinny GEMM on the
//              tensor cores (mma.m16n8k32.s8, exact int32 accumulation),
//              stream-K split over all warps of one persistent wave, fused
//              epilogues (RoPE + paged-KV append, SwiGLU, residual, argmax).
//  k_quant     RMSNorm (transformer.rs:888-896) + per-token fixed-point
//              digit packing of the next GEMV's activations.
//  k_attention paged KV verify attention, causal over the new positions,
//              split over KV pages with a last-arriver combine
//              (attention_kv, transformer.rs:944-982).
//  k_embed     token_embedding (generate.rs:843-863) from int8 rows.
//  k_accept    greedy acceptance (generate.rs:695-726).
#include <math.h>

#include "mc_internal.cuh"

namespace mc {

// ------------------------------------------------------------ PTX helpers
__device__ __forceinline__ int4 ldg_stream(const int4* p) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ldg_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ldg_u2(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p));
  return v;
}
__device__ __forceinline__ void grid_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void red_add(int* p, int v) {
  asm volatile("red.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_cg(const int* p) {
  int v;
  asm volatile("ld.global.cg.s32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float ld_cg_f(const float* p) {
  float v;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
// D += A(16x32 s8, row) * B(32x8 s8, col), int32 accumulate.
__device__ __forceinline__ void imma(int* c, const int4& a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

template <int NT>
__device__ __forceinline__ void load_x(uint32_t* xv, const uint8_t* p) {
  if constexpr (NT == 1) {
    uint2 v = ldg_u2(p);
    xv[0] = v.x; xv[1] = v.y;
  } else if constexpr (NT == 2) {
    uint4 v = ldg_u4(p);
    xv[0] = v.x; xv[1] = v.y; xv[2] = v.z; xv[3] = v.w;
  } else if constexpr (NT == 3) {
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      uint2 v = ldg_u2(p + 8 * i);
      xv[2 * i] = v.x; xv[2 * i + 1] = v.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < NT / 2; ++i) {
      uint4 v = ldg_u4(p + 16 * i);
      xv[4 * i] = v.x; xv[4 * i + 1] = v.y; xv[4 * i + 2] = v.z; xv[4 * i + 3] = v.w;
    }
  }
}

// y = scale * (d0*2^14 + d1*2^7 + d2) * 2^-e: the int32 digit sums are exact,
// so the only rounding is the final double product and its narrowing.
__device__ __forceinline__ float combine_digits(const int* row, int m, float scale, int e) {
  if (e == kExpNonFinite) return __int_as_float(0x7fc00000);
  long long X = ((long long)row[3 * m] << 14) + ((long long)row[3 * m + 1] << 7) +
                (long long)row[3 * m + 2];
  double v = (double)X * (double)scale;
  v *= __longlong_as_double((long long)(1023 - e) << 52);
  return __double2float_rn(v);
}

__device__ __forceinline__ float silu_mul(float g, float u) {
  // transformer.rs:907-909 silu (v / (1 + e^-v)), then the SwiGLU product
  // of transformer.rs:812.
  float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
  return __fmul_rn(s, u);
}

// ------------------------------------------------------------ GEMV
template <int NT>
struct GemvCfg {
  static constexpr int U = (NT <= 2) ? 8 : 4;  // k-blocks per load batch
  static constexpr int COLS = 8 * NT;
};

constexpr int kGemvWarps = 8;

template <int NT, int EPI>
__device__ __forceinline__ void gemv_epilogue(const GemvArgs& a, int stripe,
                                              int (*sm)[8 * NT + 1], const int (&acc)[NT][4],
                                              int lane, unsigned long long* kmax) {
  const int g = lane >> 2, tq = lane & 3;
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    sm[g][t * 8 + 2 * tq] = acc[t][0];
    sm[g][t * 8 + 2 * tq + 1] = acc[t][1];
    sm[g + 8][t * 8 + 2 * tq] = acc[t][2];
    sm[g + 8][t * 8 + 2 * tq + 1] = acc[t][3];
  }
  __syncwarp();
  const int M = a.M;
  for (int it = 0; it * 32 < 8 * M; ++it) {
    const int idx = it * 32 + lane;
    if (idx < 8 * M) {
      const int r = idx & 7, m = idx >> 3;
      const int e = a.xexp[m];
      const int prow = stripe * 16 + r;
      const float y0 = combine_digits(sm[r], m, a.scale[prow], e);
      const float y1 = combine_digits(sm[r + 8], m, a.scale[prow + 8], e);
      if constexpr (EPI == EPI_STORE || EPI == EPI_RESID || EPI == EPI_LMHEAD) {
        float* o = a.out ? a.out + (size_t)m * a.ldo : nullptr;
        if (prow < a.n_out) {
          if constexpr (EPI == EPI_RESID) o[prow] = __fadd_rn(o[prow], y0);
          else if (o) o[prow] = y0;
          if constexpr (EPI == EPI_LMHEAD) {
            if (!isnan(y0)) {
              unsigned long long k = argmax_key(y0, (uint32_t)prow);
              kmax[it] = k > kmax[it] ? k : kmax[it];
            }
          }
        }
        if (prow + 8 < a.n_out) {
          if constexpr (EPI == EPI_RESID) o[prow + 8] = __fadd_rn(o[prow + 8], y1);
          else if (o) o[prow + 8] = y1;
          if constexpr (EPI == EPI_LMHEAD) {
            if (!isnan(y1)) {
              unsigned long long k = argmax_key(y1, (uint32_t)(prow + 8));
              kmax[it] = k > kmax[it] ? k : kmax[it];
            }
          }
        }
      } else if constexpr (EPI == EPI_SWIGLU) {
        const int i = stripe * 8 + r;  // row r = gate_i, row r+8 = up_i
        if (i < a.n_out) a.out[(size_t)m * a.ldo + i] = silu_mul(y0, y1);
      } else if constexpr (EPI == EPI_QKV) {
        const int pos = *a.pos_ptr + a.pos_add + m;
        const int per_head = a.half_p >> 3;  // stripes per head (Q/K) = hdp/16
        const int slot = pos % a.page;
        const int pg = a.page_table[pos / a.page];
        if (stripe < a.sq + a.sk) {
          // rows r and r+8 are the RoPE pair (i, i + half) (transformer.rs:921-938)
          const bool isq = stripe < a.sq;
          const int s2 = isq ? stripe : stripe - a.sq;
          const int hh = s2 / per_head;
          const int i = (s2 - hh * per_head) * 8 + r;
          const float c = a.rope_cos[(size_t)pos * a.half_p + i];
          const float sn = a.rope_sin[(size_t)pos * a.half_p + i];
          const float o0 = __fsub_rn(__fmul_rn(y0, c), __fmul_rn(y1, sn));
          const float o1 = __fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, c));
          if (isq) {
            float* q = a.q_out + ((size_t)m * a.H + hh) * a.hdp;
            q[i] = o0;
            q[a.half_p + i] = o1;
          } else {
            float* k = a.kc + (((size_t)pg * a.Hkv + hh) * a.page + slot) * a.hdp;
            k[i] = o0;
            k[a.half_p + i] = o1;
          }
        } else {
          const int s2 = stripe - a.sq - a.sk;
          const int hh = s2 / per_head;
          const int j = (s2 - hh * per_head) * 16 + r;
          float* v = a.vc + (((size_t)pg * a.Hkv + hh) * a.page + slot) * a.hdp;
          v[j] = y0;
          v[j + 8] = y1;
        }
      }
    }
  }
  __syncwarp();
}

template <int NT, int EPI>
__global__ void __launch_bounds__(kGemvWarps * 32, 2) k_gemv(GemvArgs a) {
  constexpr int U = GemvCfg<NT>::U;
  constexpr int COLS = GemvCfg<NT>::COLS;
  __shared__ int sm_epi[kGemvWarps][16][COLS + 1];
  __shared__ unsigned long long sm_keys[kMaxTokens];

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const long long gw = (long long)blockIdx.x * kGemvWarps + warp;
  const long long nw = (long long)gridDim.x * kGemvWarps;
  const long long T = (long long)a.n_stripes * a.KB;
  const long long r0 = T * gw / nw, r1 = T * (gw + 1) / nw;

  if (EPI == EPI_LMHEAD && threadIdx.x < kMaxTokens) sm_keys[threadIdx.x] = 0ull;

  // Weights never depend on the producer grid: start streaming them (and
  // warm L2 with the next part of this warp's range) before the wait.
  int4 wv[U];
  if (r0 < r1) {
    const int s0 = (int)(r0 / a.KB);
    const long long e0 = min(r1, (long long)(s0 + 1) * a.KB);
    const int nb0 = (int)min((long long)U, e0 - r0);
#pragma unroll
    for (int j = 0; j < U; ++j)
      if (j < nb0) wv[j] = ldg_stream(a.w + (r0 + j) * 32 + lane);
    if (lane == 0 && r1 - r0 > U) {
      const long long pf = min(r1 - r0 - U, 64ll);
      prefetch_l2_bulk(a.w + (r0 + U) * 32, (uint32_t)(pf * kFragBytes));
    }
  }
  grid_wait();
  if (EPI == EPI_LMHEAD) __syncthreads();

  unsigned long long kmax[(8 * kMaxTokens + 31) / 32];
#pragma unroll
  for (int i = 0; i < (8 * kMaxTokens + 31) / 32; ++i) kmax[i] = 0ull;

  bool pre = true;
  long long seg = r0;
  while (seg < r1) {
    const int stripe = (int)(seg / a.KB);
    const int kb0 = (int)(seg - (long long)stripe * a.KB);
    const int n = (int)(min(r1, (long long)(stripe + 1) * a.KB) - seg);
    int acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0;
    const int4* wp = a.w + seg * 32 + lane;
    const uint8_t* xp = a.x + ((size_t)kb0 * 32 + lane) * COLS;
    for (int i = 0; i < n; i += U) {
      const int nb = min(U, n - i);
      if (!pre) {
#pragma unroll
        for (int j = 0; j < U; ++j)
          if (j < nb) wv[j] = ldg_stream(wp + (size_t)(i + j) * 32);
      }
      pre = false;
      uint32_t xv[U][2 * NT];
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (j < nb) load_x<NT>(xv[j], xp + (size_t)(i + j) * 32 * COLS);
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (j < nb) {
#pragma unroll
          for (int t = 0; t < NT; ++t) imma(acc[t], wv[j], xv[j][2 * t], xv[j][2 * t + 1]);
        }
    }
    // flush this stripe segment
    if (kb0 == 0 && n == a.KB) {
      gemv_epilogue<NT, EPI>(a, stripe, sm_epi[warp], acc, lane, kmax);
    } else {
      int* wsp = a.ws + ((size_t)stripe * 32 + lane) * (4 * NT);
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int q = 0; q < 4; ++q) red_add(wsp + t * 4 + q, acc[t][q]);
      __threadfence();
      int last = 0;
      if (lane == 0) last = (atomicAdd(a.cnt + stripe, n) + n == a.KB);
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last) {
        __threadfence();
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            acc[t][q] = ld_cg(wsp + t * 4 + q);
            wsp[t * 4 + q] = 0;
          }
        if (lane == 0) atomicExch(a.cnt + stripe, 0);
        gemv_epilogue<NT, EPI>(a, stripe, sm_epi[warp], acc, lane, kmax);
      }
    }
    seg += n;
  }
  grid_launch_dependents();

  if constexpr (EPI == EPI_LMHEAD) {
#pragma unroll
    for (int it = 0; it < (8 * kMaxTokens + 31) / 32; ++it) {
      unsigned long long k = kmax[it];
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        unsigned long long k2 = __shfl_xor_sync(0xffffffffu, k, o);
        k = k2 > k ? k2 : k;
      }
      const int m = (it * 32 + lane) >> 3;
      if ((lane & 7) == 0 && m < a.M && k) atomicMax(&sm_keys[m], k);
    }
    __syncthreads();
    if (threadIdx.x < a.M && sm_keys[threadIdx.x])
      atomicMax(a.keys + threadIdx.x, sm_keys[threadIdx.x]);
  }
}

template <int NT, int EPI>
static cudaError_t launch_gemv_t(const GemvArgs& a, int grid, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemvWarps * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_gemv<NT, EPI>, a);
}

template <int NT>
static cudaError_t launch_gemv_nt(const GemvArgs& a, int epi, int grid, cudaStream_t s, bool pdl) {
  switch (epi) {
    case EPI_STORE: return launch_gemv_t<NT, EPI_STORE>(a, grid, s, pdl);
    case EPI_RESID: return launch_gemv_t<NT, EPI_RESID>(a, grid, s, pdl);
    case EPI_SWIGLU: return launch_gemv_t<NT, EPI_SWIGLU>(a, grid, s, pdl);
    case EPI_QKV: return launch_gemv_t<NT, EPI_QKV>(a, grid, s, pdl);
    case EPI_LMHEAD: return launch_gemv_t<NT, EPI_LMHEAD>(a, grid, s, pdl);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_gemv(const GemvArgs& a, int epi, int nt, int grid, cudaStream_t s, bool pdl) {
  switch (nt) {
    case 1: return launch_gemv_nt<1>(a, epi, grid, s, pdl);
    case 2: return launch_gemv_nt<2>(a, epi, grid, s, pdl);
    case 3: return launch_gemv_nt<3>(a, epi, grid, s, pdl);
    case 6: return launch_gemv_nt<6>(a, epi, grid, s, pdl);
  }
  return cudaErrorInvalidValue;
}

template <int NT>
static int bps_nt(int epi) {
  int n = 0;
  switch (epi) {
    case EPI_STORE: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_gemv<NT, EPI_STORE>, kGemvWarps * 32, 0); break;
    case EPI_RESID: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_gemv<NT, EPI_RESID>, kGemvWarps * 32, 0); break;
    case EPI_SWIGLU: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_gemv<NT, EPI_SWIGLU>, kGemvWarps * 32, 0); break;
    case EPI_QKV: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_gemv<NT, EPI_QKV>, kGemvWarps * 32, 0); break;
    case EPI_LMHEAD: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_gemv<NT, EPI_LMHEAD>, kGemvWarps * 32, 0); break;
  }
  return n;
}

int gemv_blocks_per_sm(int epi, int nt) {
  switch (nt) {
    case 1: return bps_nt<1>(epi);
    case 2: return bps_nt<2>(epi);
    case 3: return bps_nt<3>(epi);
    case 6: return bps_nt<6>(epi);
  }
  return 0;
}

// ------------------------------------------------------------ quantize
// One block per token.  Optional RMSNorm (transformer.rs:888-896:
// ms = sum(v*v)/n, rms = sqrt(ms + eps), out = v / rms * w), then the
// fixed-point digit encoding of the GEMV's B operand.
constexpr int kQuantThreads = 1024;
static int g_quant_smem = 48 * 1024;  // current dynamic smem limits (per process;
static int g_attn_smem = 48 * 1024;   // single-device use assumed per limit)

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.0f;
  if (threadIdx.x < 32) {
    t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

__device__ __forceinline__ uint32_t block_max_u(uint32_t v, uint32_t* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    uint32_t t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0u;
#pragma unroll
    for (int o = 16; o; o >>= 1) t = max(t, __shfl_xor_sync(0xffffffffu, t, o));
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

__global__ void __launch_bounds__(kQuantThreads) k_quant(QuantArgs a) {
  extern __shared__ float sx[];
  __shared__ float redf[32];
  __shared__ uint32_t redu[32];
  grid_launch_dependents();
  grid_wait();
  const int m = blockIdx.x;
  const float* h = a.h + (size_t)m * a.ld;
  const int d = a.d;
  float rms = 1.0f;
  if (a.do_norm) {
    float ss = 0.0f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
      float v = h[i];
      ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
    ss = block_sum(ss, redf);
    float nf = (float)(d > 1 ? d : 1);
    rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, nf), a.eps));
  }
  uint32_t amax = 0u, bad = 0u;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    float v = h[i];
    if (a.do_norm) {
      float wi = (a.w && i < a.wlen) ? a.w[i] : 1.0f;
      v = __fmul_rn(__fdiv_rn(v, rms), wi);
    }
    sx[i] = v;
    uint32_t b = __float_as_uint(fabsf(v));
    if (!isfinite(v)) bad = 1u;
    amax = max(amax, b);
  }
  amax = block_max_u(amax, redu);
  bad = block_max_u(bad, redu);
  int e = 0;
  if (bad) {
    e = kExpNonFinite;
  } else if (amax != 0u) {
    int E;
    frexpf(__uint_as_float(amax), &E);
    e = 20 - E;  // |x| * 2^e < 2^20
  }
  if (threadIdx.x == 0) a.xexp[m] = e;
  const int nt = a.nt;
  const int cols = 8 * nt;
  uint32_t* xq = reinterpret_cast<uint32_t*>(a.xq);
  const int ngroups = a.KB * 8;
  for (int gi = threadIdx.x; gi < ngroups; gi += blockDim.x) {
    const int k0 = gi * 4;
    const int kb = k0 >> 5, kk = k0 & 31;
    const int reg = kk >> 4, t = (kk & 15) >> 2;
    uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = k0 + j;
      int X = 0;
      if (k < d && e != kExpNonFinite) X = __float2int_rn(ldexpf(sx[k], e));
      const int d2 = ((X + 64) & 127) - 64;
      const int X1 = (X - d2) >> 7;
      const int d1 = ((X1 + 64) & 127) - 64;
      const int d0 = (X1 - d1) >> 7;
      w0 |= (uint32_t)(d0 & 0xff) << (8 * j);
      w1 |= (uint32_t)(d1 & 0xff) << (8 * j);
      w2 |= (uint32_t)(d2 & 0xff) << (8 * j);
    }
    const uint32_t wd[3] = {w0, w1, w2};
#pragma unroll
    for (int s = 0; s < 3; ++s) {
      const int c = 3 * m + s;
      const int tile = c >> 3, n = c & 7, ln = n * 4 + t;
      xq[(((size_t)kb * 32 + ln) * cols + tile * 8 + reg * 4) >> 2] = wd[s];
    }
    if (m == a.M - 1) {
      for (int c = 3 * a.M; c < cols; ++c) {
        const int tile = c >> 3, n = c & 7, ln = n * 4 + t;
        xq[(((size_t)kb * 32 + ln) * cols + tile * 8 + reg * 4) >> 2] = 0u;
      }
    }
  }
}

cudaError_t launch_quant(const QuantArgs& a, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.M);
  cfg.blockDim = dim3(kQuantThreads);
  cfg.dynamicSmemBytes = (size_t)a.KB * 32 * sizeof(float);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cfg.dynamicSmemBytes > (size_t)g_quant_smem) return cudaErrorInvalidConfiguration;
  return cudaLaunchKernelEx(&cfg, k_quant, a);
}

// ------------------------------------------------------------ attention
// One CTA per (KV head, KV page).  Query rows are the G query heads sharing
// the KV head times the M new tokens; token m sees positions <= pos0 + m.
// Scores: dot / sqrt(head_dim) (transformer.rs:959-966); softmax with the
// max subtracted (transformer.rs:985-1000), combined across pages by the
// last-arriving CTA of the head.
constexpr int kAttnThreads = 256;

__global__ void __launch_bounds__(kAttnThreads) k_attention(AttnArgs a) {
  extern __shared__ float smem[];
  grid_launch_dependents();
  grid_wait();
  const int kvh = blockIdx.x, chunk = blockIdx.y;
  const int G = a.H / a.Hkv;
  const int R = G * a.M;
  const int hdp = a.hdp, P = a.page;
  const int pos0 = *a.pos_ptr + a.pos_add;
  const int L = pos0 + a.M;
  const int n_chunks = (L + P - 1) / P;
  if (chunk >= n_chunks) return;
  const int t0 = chunk * P;
  const int nt = min(P, L - t0);
  const int ks = hdp + 1;  // padded K row stride (bank-conflict free)
  float* sq = smem;                    // [R][hdp]
  float* sk = sq + (size_t)R * hdp;    // [P][hdp+1]
  float* sv = sk + (size_t)P * ks;     // [P][hdp]
  float* ss = sv + (size_t)P * hdp;    // [R][P]
  __shared__ float s_m[128], s_l[128];

  const int pg = a.page_table[chunk];
  const float* kbase = a.kc + ((size_t)pg * a.Hkv + kvh) * P * hdp;
  const float* vbase = a.vc + ((size_t)pg * a.Hkv + kvh) * P * hdp;
  for (int i = threadIdx.x; i < R * hdp; i += blockDim.x) {
    const int row = i / hdp, c = i - row * hdp;
    const int m = row / G, gi = row - m * G;
    sq[i] = a.q[((size_t)m * a.H + kvh * G + gi) * hdp + c];
  }
  for (int i = threadIdx.x; i < nt * hdp; i += blockDim.x) {
    const int t = i / hdp, c = i - t * hdp;
    sk[t * ks + c] = kbase[i];
    sv[i] = vbase[i];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < R * nt; i += blockDim.x) {
    const int row = i / nt, t = i - row * nt;
    const int m = row / G;
    float s = -INFINITY;
    if (t0 + t <= pos0 + m) {
      const float* qr = sq + (size_t)row * hdp;
      const float* kr = sk + (size_t)t * ks;
      float dot = 0.0f;
      for (int c = 0; c < hdp; ++c) dot = __fmaf_rn(qr[c], kr[c], dot);
      s = __fdiv_rn(dot, a.inv_scale_den);
    }
    ss[row * P + t] = s;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int row = warp; row < R; row += blockDim.x >> 5) {
    float mx = -INFINITY;
    for (int t = lane; t < nt; t += 32) mx = fmaxf(mx, ss[row * P + t]);
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    for (int t = lane; t < nt; t += 32) {
      const float s = ss[row * P + t];
      const float p = (mx == -INFINITY) ? 0.0f : expf(s - mx);
      ss[row * P + t] = p;
      sum += p;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) { s_m[row] = mx; s_l[row] = sum; }
  }
  __syncthreads();
  const size_t pbase = ((size_t)kvh * a.max_chunks + chunk) * R;
  for (int i = threadIdx.x; i < R * hdp; i += blockDim.x) {
    const int row = i / hdp, c = i - row * hdp;
    float o = 0.0f;
    for (int t = 0; t < nt; ++t) o = __fmaf_rn(ss[row * P + t], sv[t * hdp + c], o);
    a.part_o[(pbase + row) * hdp + c] = o;
  }
  for (int row = threadIdx.x; row < R; row += blockDim.x) {
    a.part_ml[(pbase + row) * 2] = s_m[row];
    a.part_ml[(pbase + row) * 2 + 1] = s_l[row];
  }
  __threadfence();
  __syncthreads();
  __shared__ int s_last;
  if (threadIdx.x == 0) s_last = (atomicAdd(a.cnt + kvh, 1) == n_chunks - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // combine the pages of this KV head
  for (int row = threadIdx.x; row < R; row += blockDim.x) {
    float M_ = -INFINITY;
    for (int c = 0; c < n_chunks; ++c)
      M_ = fmaxf(M_, ld_cg_f(a.part_ml + (((size_t)kvh * a.max_chunks + c) * R + row) * 2));
    float l = 0.0f;
    for (int c = 0; c < n_chunks; ++c) {
      const size_t b = (((size_t)kvh * a.max_chunks + c) * R + row) * 2;
      const float mc = ld_cg_f(a.part_ml + b);
      if (mc != -INFINITY) l += ld_cg_f(a.part_ml + b + 1) * expf(mc - M_);
    }
    s_m[row] = M_;
    s_l[row] = l;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < R * hdp; i += blockDim.x) {
    const int row = i / hdp, c = i - row * hdp;
    float o = 0.0f;
    for (int ch = 0; ch < n_chunks; ++ch) {
      const size_t b = ((size_t)kvh * a.max_chunks + ch) * R + row;
      const float mc = ld_cg_f(a.part_ml + b * 2);
      if (mc != -INFINITY) o += ld_cg_f(a.part_o + b * hdp + c) * expf(mc - s_m[row]);
    }
    const int m = row / G, gi = row - m * G;
    a.out[((size_t)m * a.H + kvh * G + gi) * hdp + c] = __fdiv_rn(o, s_l[row]);
  }
  if (threadIdx.x == 0) atomicExch(a.cnt + kvh, 0);
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl) {
  const int G = a.H / a.Hkv;
  const int R = G * a.M;
  size_t smem = ((size_t)R * a.hdp + (size_t)a.page * (a.hdp + 1) + (size_t)a.page * a.hdp +
                 (size_t)R * a.page) * sizeof(float);
  if (R > 128) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.Hkv, a.max_chunks);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (smem > (size_t)g_attn_smem) return cudaErrorInvalidConfiguration;
  return cudaLaunchKernelEx(&cfg, k_attention, a);
}

size_t attention_smem_bytes(int G, int M, int hdp, int page) {
  const size_t R = (size_t)G * M;
  return (R * hdp + (size_t)page * (hdp + 1) + (size_t)page * hdp + R * page) * sizeof(float);
}

// Raise the dynamic shared-memory limits once, outside any stream capture.
cudaError_t prepare_kernels(size_t quant_smem, size_t attn_smem) {
  if (quant_smem > (size_t)g_quant_smem) {
    cudaError_t e = cudaFuncSetAttribute(k_quant, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)quant_smem);
    if (e != cudaSuccess) return e;
    g_quant_smem = (int)quant_smem;
  }
  if (attn_smem > (size_t)g_attn_smem) {
    cudaError_t e = cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)attn_smem);
    if (e != cudaSuccess) return e;
    g_attn_smem = (int)attn_smem;
  }
  return cudaSuccess;
}

// ------------------------------------------------------------ embedding
__global__ void __launch_bounds__(256) k_embed(EmbedArgs a) {
  grid_launch_dependents();
  grid_wait();
  const int m = blockIdx.x;
  uint32_t id;
  switch (a.src) {
    case SRC_IDS: id = a.ids[m]; break;
    case SRC_CTX_AT: id = a.ctx[*a.off + m]; break;
    case SRC_KEYS: id = key_index(a.keys[m]); break;
    default: id = (m == 0) ? a.ctx[*a.off - 1] : key_index(a.keys[m - 1]); break;
  }
  if (a.ids_out && threadIdx.x == 0) a.ids_out[m] = id;
  float* h = a.h + (size_t)m * a.d;
  if (id < (uint32_t)a.vocab) {
    const int8_t* q = a.emb_q + (size_t)id * a.d;
    const float sc = a.emb_scale[id];
    for (int i = threadIdx.x; i < a.d; i += blockDim.x) h[i] = __fmul_rn((float)q[i], sc);
  } else {
    for (int i = threadIdx.x; i < a.d; i += blockDim.x) h[i] = 0.0f;
  }
  if (m == 0)
    for (int i = threadIdx.x; i < a.n_zero; i += blockDim.x) a.zero_keys[i] = 0ull;
}

cudaError_t launch_embed(const EmbedArgs& a, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.M);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_embed, a);
}

// ------------------------------------------------------------ acceptance
// Greedy acceptance of one speculative round (generate.rs:695-726): the
// verify forward saw [last, d1 .. d_vm-1]; key[j] is the target's argmax
// after position j.  Drafts are accepted while they equal the target's
// token; the first mismatch pushes the target's token.  Without the bonus
// (the reference, vm == gamma) a fully accepted round pushes d_gamma unverified
// by a further forward; with the bonus (vm == gamma+1) the target's token after
// d_gamma is pushed as well.  KV lengths are rolled back to what a
// sequential verify would have forwarded.
__global__ void k_accept_greedy(SpecState* st, uint32_t* ctx, int* acc_log, int vm) {
  grid_launch_dependents();
  grid_wait();
  if (threadIdx.x != 0) return;
  const int g = st->gamma;
  int a = 0;
  while (a < g && key_index(st->tkeys[a]) == key_index(st->dkeys[a])) ++a;
  int len = st->ctx_len;
  for (int j = 0; j < a; ++j) ctx[len + j] = key_index(st->dkeys[j]);
  int emitted = a;
  if (a < vm) {
    ctx[len + a] = key_index(st->tkeys[a]);
    emitted = a + 1;
  }
  st->ctx_len = len + emitted;
  st->lt += (a + 1 < vm) ? a + 1 : vm;
  st->ld = st->ctx_len - 1;
  st->generated += emitted;
  if (acc_log && st->n_rounds < st->rounds_cap) acc_log[st->n_rounds] = a;
  st->n_rounds += 1;
}

cudaError_t launch_accept_greedy(SpecState* st, uint32_t* ctx, int* acc_log, int vm,
                                 cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_accept_greedy, st, ctx, acc_log, vm);
}

__global__ void k_set_int(int* p, int v) { *p = v; }
cudaError_t launch_set_int(int* p, int v, cudaStream_t s) {
  k_set_int<<<1, 1, 0, s>>>(p, v);
  return cudaGetLastError();
}

// ------------------------------------------------------------ packing
// One thread per lane-fragment (16 bytes).  row_map / col_map give, for each
// packed row / column, the source row / column or -1 for zero padding.
__global__ void k_pack_int8(const int8_t* __restrict__ src, long long src_ld,
                            const int* __restrict__ row_map, const int* __restrict__ col_map,
                            int n_stripes, int KB, int4* __restrict__ dst) {
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = (long long)n_stripes * KB * 32;
  if (gid >= total) return;
  const int lane = (int)(gid & 31);
  const long long sk = gid >> 5;
  const int kb = (int)(sk % KB);
  const int stripe = (int)(sk / KB);
  const int g = lane >> 2, t = lane & 3;
  const int ra = row_map[stripe * 16 + g];
  const int rb = row_map[stripe * 16 + g + 8];
  uint32_t regs[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int row = (r & 1) ? rb : ra;
    const int cbase = kb * 32 + (r >> 1) * 16 + 4 * t;
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = col_map[cbase + j];
      uint8_t b = 0;
      if (row >= 0 && c >= 0) b = (uint8_t)src[(long long)row * src_ld + c];
      word |= (uint32_t)b << (8 * j);
    }
    regs[r] = word;
  }
  dst[gid] = make_int4((int)regs[0], (int)regs[1], (int)regs[2], (int)regs[3]);
}

__global__ void k_pack_scale(const float* src_scale, const int* row_map, int n, float* dst) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = row_map[i] >= 0 ? src_scale[row_map[i]] : 0.0f;
}

cudaError_t launch_pack_int8(const int8_t* src, long long src_ld, const float* src_scale,
                             const int* row_map, const int* col_map, int n_stripes, int KB,
                             int4* dst, float* dst_scale, cudaStream_t s) {
  const long long total = (long long)n_stripes * KB * 32;
  const int bs = 256;
  k_pack_int8<<<(unsigned)((total + bs - 1) / bs), bs, 0, s>>>(src, src_ld, row_map, col_map,
                                                                 n_stripes, KB, dst);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int n = n_stripes * 16;
  k_pack_scale<<<(n + 255) / 256, 256, 0, s>>>(src_scale, row_map, n, dst_scale);
  return cudaGetLastError();
}

}  // namespace mc
