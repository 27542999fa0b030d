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
#include <cuda_fp16.h>
#include <math.h>

#include <algorithm>
#include <climits>
#include <type_traits>

#include "mc_internal.cuh"

namespace mc {

// ------------------------------------------------------------ tracing
#ifdef MC_TRACE
struct TraceRec {
  unsigned long long start, waited, end;
};
__device__ TraceRec g_trace[kTraceSlots];
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#define MC_TRACE_T0                          \
  const unsigned long long mc_t0 = gtimer(); \
  unsigned long long mc_tp = mc_t0;          \
  (void)mc_tp;
// per-phase time summed over CTAs (divide by the CTAs that reached it)
__device__ unsigned long long g_phase[kTraceSlots][8];
__device__ unsigned int g_phase_n[kTraceSlots][8];
#define MC_TRACE_PHASE(ts, k, tprev)                                   \
  do {                                                                 \
    if ((ts) > 0 && threadIdx.x == 0) {                                \
      const unsigned long long tn = gtimer();                          \
      atomicAdd(&g_phase[(ts) - 1][k], tn - (tprev));                  \
      atomicAdd(&g_phase_n[(ts) - 1][k], 1u);                          \
      (tprev) = tn;                                                    \
    }                                                                  \
  } while (0)
#define MC_TRACE_WAITED(ts)                                 \
  do {                                                      \
    if ((ts) > 0 && threadIdx.x == 0) {                     \
      atomicMin(&g_trace[(ts) - 1].start, mc_t0);           \
      atomicMin(&g_trace[(ts) - 1].waited, gtimer());       \
    }                                                       \
  } while (0)
// called by every thread of the CTA at a common exit point
#define MC_TRACE_END(ts)                                                    \
  do {                                                                      \
    __syncthreads();                                                        \
    if ((ts) > 0 && threadIdx.x == 0) atomicMax(&g_trace[(ts) - 1].end, gtimer()); \
  } while (0)
#else
#define MC_TRACE_T0
#define MC_TRACE_WAITED(ts) \
  do {                      \
  } while (0)
#define MC_TRACE_END(ts) \
  do {                   \
  } while (0)
#define MC_TRACE_PHASE(ts, k, tprev) \
  do {                               \
  } while (0)
#endif

cudaError_t trace_reset() {
#ifdef MC_TRACE
  static TraceRec h[kTraceSlots];
  static unsigned long long z[kTraceSlots][8];
  static unsigned int zn[kTraceSlots][8];
  for (auto& r : h) r = TraceRec{~0ull, ~0ull, 0ull};
  cudaError_t e = cudaMemcpyToSymbol(g_phase, z, sizeof(z));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_phase_n, zn, sizeof(zn));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_trace, h, sizeof(h));
#else
  return cudaErrorNotSupported;
#endif
}

cudaError_t trace_read(unsigned long long* out, int n) {
#ifdef MC_TRACE
  if (n > kTraceSlots) n = kTraceSlots;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_trace, (size_t)n * sizeof(TraceRec));
  if (e != cudaSuccess) return e;
  // then per slot 8 phase sums and 8 counts
  static unsigned long long ph[kTraceSlots][8];
  static unsigned int pn[kTraceSlots][8];
  e = cudaMemcpyFromSymbol(ph, g_phase, sizeof(ph));
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(pn, g_phase_n, sizeof(pn));
  for (int i = 0; i < n && e == cudaSuccess; ++i)
    for (int k = 0; k < 8; ++k) {
      out[3 * n + 16 * i + k] = ph[i][k];
      out[3 * n + 16 * i + 8 + k] = pn[i][k];
    }
  return e;
#else
  (void)out;
  (void)n;
  return cudaErrorNotSupported;
#endif
}

// ------------------------------------------------------------ PTX helpers
// Weight stream: read once per forward, so it bypasses L1 and is marked
// evict-first in L2 (it must not evict the next GEMV's prefetched lines).
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ int4 ldg_stream(const int4* p, uint64_t pol) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.s32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}
__device__ __forceinline__ uint2 ldg_stream2(const uint2* p, uint64_t pol) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.u32 {%0,%1}, [%2], %3;"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p), "l"(pol));
  return v;
}
__device__ __forceinline__ uint32_t ldg_stream1(const uint32_t* p, uint64_t pol) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.u32 %0, [%1], %2;"
               : "=r"(v)
               : "l"(p), "l"(pol));
  return v;
}
// Activation digits are rewritten by the previous kernel while this grid may
// already be resident (programmatic dependent launch), so they are read
// through L2 (.cg), never through the non-coherent path.
__device__ __forceinline__ uint4 ldg_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ldg_u2(const void* p) {
  uint2 v;
  asm volatile("ld.global.cg.v2.u32 {%0,%1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p));
  return v;
}
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes)
               : "memory");
}
// This CTA's share of an L2 prefetch of `bytes` at p (16-byte multiples,
// 32 KB per instruction), issued by one thread.
__device__ __forceinline__ void prefetch_share(const void* p, long long bytes, int cta, int n_ctas) {
  const long long share = (bytes / n_ctas) & ~15ll;
  if (share < 16) return;
  const char* q = reinterpret_cast<const char*>(p) + share * cta;
  for (long long left = share; left >= 16;) {
    const uint32_t b = (uint32_t)min(left, 32768ll) & ~15u;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(q), "r"(b) : "memory");
    q += b;
    left -= b;
  }
}
// mbarriers and bulk copies (cp.async.bulk, completion counted in bytes on
// an mbarrier): shared by the GEMV's weight ring and the tcgen05 GEMM.
constexpr long long kMbarSpin = 1ll << 22;  // try_wait rounds before giving up
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(b)),
               "r"(bytes)
               : "memory");
}
// Bounded wait for the completion of the phase with this parity.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity) {
  uint32_t done = 0;
  for (long long i = 0; i < kMbarSpin && !done; ++i)
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(b)), "r"(parity)
        : "memory");
  return done != 0;
}
// the same with an L2 cache policy (createpolicy) for the source lines
__device__ __forceinline__ void bulk_load_hint(void* dst, const void* src, uint32_t bytes,
                                               uint64_t* b, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(b)), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* b) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(b))
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

// This lane's B fragments of one k-block (base: the k-block's 256 * NT
// bytes; layout as digit_word): one 16-byte load per pair of tiles and an
// 8-byte one for an odd last tile, each contiguous across the warp.
template <int NT>
__device__ __forceinline__ void load_x(uint32_t* xv, const uint8_t* base, int lane) {
#pragma unroll
  for (int i = 0; i < NT / 2; ++i) {
    uint4 v = ldg_u4(base + i * 512 + lane * 16);
    xv[4 * i] = v.x; xv[4 * i + 1] = v.y; xv[4 * i + 2] = v.z; xv[4 * i + 3] = v.w;
  }
  if constexpr (NT & 1) {
    uint2 w = ldg_u2(base + (NT / 2) * 512 + lane * 8);
    xv[NT * 2 - 2] = w.x; xv[NT * 2 - 1] = w.y;
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

// q4_0 tiles hold per-digit sums already scaled by the block scales (f32).
__device__ __forceinline__ float combine_digits(const float* row, int m, float, int e) {
  if (e == kExpNonFinite) return __int_as_float(0x7fc00000);
  double v = (double)row[3 * m] * 16384.0 + (double)row[3 * m + 1] * 128.0 +
             (double)row[3 * m + 2];
  v *= __longlong_as_double((long long)(1023 - e) << 52);
  return __double2float_rn(v);
}

// Four unsigned 4-bit codes (one per byte, 0..15) -> signed bytes code - 8.
// Bytes stay below 0x80 after the add, so no carry crosses a byte.
__device__ __forceinline__ uint32_t q4_signed(uint32_t u) {
  return (u + 0x78787878u) ^ 0x80808080u;
}
__device__ __forceinline__ int4 q4_fragment(uint2 w) {
  return make_int4((int)q4_signed(w.x & 0x0F0F0F0Fu), (int)q4_signed((w.x >> 4) & 0x0F0F0F0Fu),
                   (int)q4_signed(w.y & 0x0F0F0F0Fu), (int)q4_signed((w.y >> 4) & 0x0F0F0F0Fu));
}
// Exact int -> float for |c| < 2^22 on the full-rate integer and FP32 pipes:
// c + 0x4B400000 is the bit pattern of 1.5 * 2^23 + c.
__device__ __forceinline__ float small_int_to_float(int c) {
  return __fsub_rn(__int_as_float(c + 0x4B400000), 12582912.0f);
}

__device__ __forceinline__ float silu_mul(float g, float u) {
  // transformer.rs:907-909 silu (v / (1 + e^-v)), then the SwiGLU product
  // of transformer.rs:812.
  float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
  return __fmul_rn(s, u);
}

// ------------------------------------------------------------ activation encoding
// Per-token statistics of an activation row block, reduced with one fixed
// tree of kStatLanes virtual lanes (partials per lane, xor-shuffles within a
// virtual warp, then the 16 virtual warps summed in order), so every kernel
// that encodes activations -- whatever its block size -- gets bit-identical
// exponents and multipliers.  RMSNorm follows transformer.rs:888-896
// (ms = sum(v*v)/n, rms = sqrt(ms + eps), x = v / rms * w).  The exponent
// makes |x| * 2^e < 2^20 with a one-ulp margin (digits tolerate |X| < 2^21).
constexpr int kStatLanes = 512;
constexpr int kStatWarps = kStatLanes / 32;

struct StatArgs {
  const float* h;
  int ld, d, M;
  const float* w;
  int wlen;
  float eps;
  int do_norm;
};

// Slice capture: if cap != nullptr, elements [lo, hi) of every token are also
// stored to cap[m * (hi - lo) + (i - lo)].  Tokens are reduced in groups of
// kStatTokens (one register partial per token of the group; the grouping
// does not change any token's reduction order).
constexpr int kStatTokens = 8;
__device__ __forceinline__ void token_stats(const StatArgs& a, float (*red_ss)[kMaxTokens],
                                            float (*red_hw)[kMaxTokens], uint32_t* s_bad,
                                            float* s_mul, int* s_e, float* cap, int lo, int hi) {
  const int M = a.M, d = a.d;
  const bool vec = ((a.ld & 3) == 0) && ((d & 3) == 0) &&
                   ((reinterpret_cast<uintptr_t>(a.h) & 15) == 0);
  const int span = hi - lo;
  if (threadIdx.x < kMaxTokens / kStatTokens) s_bad[threadIdx.x] = 0u;
  __syncthreads();
  for (int g0 = 0; g0 < M; g0 += kStatTokens) {
    const int MG = min(kStatTokens, M - g0);
    uint32_t bad = 0u;
    for (int v = threadIdx.x; v < kStatLanes; v += blockDim.x) {
      float ss[kStatTokens], hw[kStatTokens];
#pragma unroll
      for (int m = 0; m < kStatTokens; ++m) { ss[m] = 0.0f; hw[m] = 0.0f; }
      if (vec) {
#pragma unroll 4
        for (int i = v * 4; i < d; i += kStatLanes * 4) {
          float4 wv = make_float4(1.0f, 1.0f, 1.0f, 1.0f);
          if (a.do_norm && a.w) {
            wv.x = i < a.wlen ? a.w[i] : 1.0f;
            wv.y = i + 1 < a.wlen ? a.w[i + 1] : 1.0f;
            wv.z = i + 2 < a.wlen ? a.w[i + 2] : 1.0f;
            wv.w = i + 3 < a.wlen ? a.w[i + 3] : 1.0f;
          }
#pragma unroll
          for (int m = 0; m < kStatTokens; ++m)
            if (m < MG) {
              const int mt = g0 + m;
              const float4 x = __ldcg(reinterpret_cast<const float4*>(a.h + (size_t)mt * a.ld + i));
              if (cap && i >= lo && i < hi) *reinterpret_cast<float4*>(cap + mt * span + (i - lo)) = x;
              ss[m] = __fadd_rn(ss[m], __fmul_rn(x.x, x.x));
              ss[m] = __fadd_rn(ss[m], __fmul_rn(x.y, x.y));
              ss[m] = __fadd_rn(ss[m], __fmul_rn(x.z, x.z));
              ss[m] = __fadd_rn(ss[m], __fmul_rn(x.w, x.w));
              hw[m] = fmaxf(hw[m], fmaxf(fmaxf(fabsf(__fmul_rn(x.x, wv.x)), fabsf(__fmul_rn(x.y, wv.y))),
                                         fmaxf(fabsf(__fmul_rn(x.z, wv.z)), fabsf(__fmul_rn(x.w, wv.w)))));
              if (!(isfinite(x.x) && isfinite(x.y) && isfinite(x.z) && isfinite(x.w))) bad |= 1u << m;
            }
        }
      } else {
        for (int i = v; i < d; i += kStatLanes) {
          const float wi = (a.do_norm && a.w && i < a.wlen) ? a.w[i] : 1.0f;
#pragma unroll
          for (int m = 0; m < kStatTokens; ++m)
            if (m < MG) {
              const int mt = g0 + m;
              const float x = __ldcg(a.h + (size_t)mt * a.ld + i);
              if (cap && i >= lo && i < hi) cap[mt * span + (i - lo)] = x;
              ss[m] = __fadd_rn(ss[m], __fmul_rn(x, x));
              hw[m] = fmaxf(hw[m], fabsf(__fmul_rn(x, wi)));
              if (!isfinite(x)) bad |= 1u << m;
            }
        }
      }
      const int vw = v >> 5;
#pragma unroll
      for (int m = 0; m < kStatTokens; ++m) {
        if (m < MG) {
          float x = ss[m], y = hw[m];
#pragma unroll
          for (int o = 16; o; o >>= 1) {
            x += __shfl_xor_sync(0xffffffffu, x, o);
            y = fmaxf(y, __shfl_xor_sync(0xffffffffu, y, o));
          }
          if ((v & 31) == 0) { red_ss[vw][g0 + m] = x; red_hw[vw][g0 + m] = y; }
        }
      }
    }
    bad = __reduce_or_sync(0xffffffffu, bad);
    if ((threadIdx.x & 31) == 0 && bad) atomicOr(s_bad + g0 / kStatTokens, bad);
  }
  __syncthreads();
  if (threadIdx.x < M) {
    const int m = threadIdx.x;
    float x = 0.0f, y = 0.0f;
    for (int w = 0; w < kStatWarps; ++w) { x += red_ss[w][m]; y = fmaxf(y, red_hw[w][m]); }
    float rms = 1.0f;
    if (a.do_norm) rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(x, (float)(d > 1 ? d : 1)), a.eps));
    const float amax = a.do_norm ? y / rms : y;
    int e = 0;
    if (((s_bad[m / kStatTokens] >> (m % kStatTokens)) & 1u) || !isfinite(amax)) {
      e = kExpNonFinite;
    } else if (amax > 0.0f) {
      int E;
      frexpf(amax * 1.0000002f, &E);
      e = 20 - E;
    }
    // x * 2^e = (h * w) * (2^e / rms): the power-of-two factor is exact; one
    // reciprocal per token replaces the per-element division (<= 1 ulp).
    float mul = 0.0f;
    if (e != kExpNonFinite) mul = ldexpf(a.do_norm ? 1.0f / rms : 1.0f, e);
    s_mul[m] = mul;
    s_e[m] = e;
  }
  __syncthreads();
}

// Encodes k-blocks [kb0, kb1) of the digit operand: one task per (token,
// 4 consecutive k) computes the 4 fixed-point values once and writes its
// three digit words; leftover columns of the last n8 tile get zero words.
// Tasks run in batches of kEncBatch per thread with all their loads issued
// first.  src4(m, k) returns the raw activations k..k+3 (k % 4 == 0, zeros
// past d); dst(word, value) stores a word.
constexpr int kEncBatch = 8;

// Word index of the 4 digit bytes of column c, k-block kb, k = kk..kk+3
// (kk % 4 == 0).  mma.sync layout: [kb][lane][tile][reg], lane = (c%8)*4 +
// (kk%16)/4, the B fragment of m16n8k32, in planes of two tiles:
// [kb][tile/2][lane][tile%2][reg], an odd last tile as its own plane
// [lane][reg].  Each of the GEMV's loads then reads a contiguous span across
// the warp (a 24- or 48-byte lane stride costs three times the L1
// wavefronts).  tcgen05 layout (tc): K-major with
// the 128-byte swizzle, [kb/4][column][128 bytes] with the row's 16-byte
// chunk q = (kb%4)*2 + kk/16 stored at q ^ (column % 8).
__device__ __forceinline__ size_t digit_word(int kb, int c, int kk, int nt, bool tc) {
  if (tc) {
    const int q = ((kb & 3) << 1) | (kk >> 4);
    return ((size_t)(kb >> 2) * (8 * nt) + c) * 32 + (size_t)(((q ^ (c & 7)) << 2) + ((kk & 15) >> 2));
  }
  const int lane = (c & 7) * 4 + ((kk & 15) >> 2), t = c >> 3, r = kk >> 4;
  const size_t plane = (size_t)kb * 64 * nt + (t >> 1) * 128;
  return plane + ((nt & 1) && t == nt - 1 ? lane * 2 + r : lane * 4 + (t & 1) * 2 + r);
}
// Word index of column c of a forward of `groups` token groups: the tcgen05
// layout spans all groups (nt * groups tiles); the mma.sync layout keeps each
// group's 8 * nt columns in its own block of KB * 64 * nt words, the operand
// of one GEMV launch.
__device__ __forceinline__ size_t digit_index(int kb, int c, int kk, int nt, int groups, int KB,
                                              bool tc) {
  if (tc) return digit_word(kb, c, kk, nt * groups, true);
  const int g = c / (8 * nt);
  return (size_t)g * KB * 64 * nt + digit_word(kb, c - g * 8 * nt, kk, nt, false);
}

template <int BATCH = kEncBatch, class Src4, class Dst>
__device__ __forceinline__ void encode_digits(const StatArgs& a, int nt, int KB, int kb0, int kb1,
                                              const float* s_mul, const int* s_e, Src4 src4,
                                              Dst dst, bool tc = false) {
  const int M = a.M, d = a.d;
  const int groups = groups_for_tokens(M);
  const int pad_cols = 8 * nt * groups - 3 * M;
  const int ngroups = (kb1 - kb0) * 8;
  const int tasks = ngroups * (M + pad_cols);
  for (int t0 = threadIdx.x; t0 < tasks; t0 += blockDim.x * BATCH) {
    float4 v[BATCH];
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int task = t0 + u * blockDim.x;
      v[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (task < tasks) {
        const int grp = task % ngroups, q = task / ngroups;
        if (q < M && s_e[q] != kExpNonFinite)
          v[u] = src4(q, (kb0 + (grp >> 3)) * 32 + (grp & 7) * 4);
      }
    }
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int task = t0 + u * blockDim.x;
      if (task >= tasks) continue;
      const int grp = task % ngroups;
      const int q = task / ngroups;  // token (q < M) or padding column (q >= M)
      const int kb = kb0 + (grp >> 3);
      const int kk = (grp & 7) * 4;
      if (q >= M) {
        dst(digit_index(kb, 3 * M + (q - M), kk, nt, groups, KB, tc), 0u);
        continue;
      }
      const int m = q;
      uint32_t w0 = 0, w1 = 0, w2 = 0;
      if (s_e[m] != kExpNonFinite) {
        const float mul = s_mul[m];
        const float vv[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int k = kb * 32 + kk + j;
          int X = 0;
          if (k < d) {
            float x = vv[j];
            if (a.do_norm) x = __fmul_rn(x, (a.w && k < a.wlen) ? a.w[k] : 1.0f);
            X = __float2int_rn(__fmul_rn(x, mul));
          }
          const int d2 = ((X + 64) & 127) - 64;
          const int X1 = (X - d2) >> 7;
          const int d1 = ((X1 + 64) & 127) - 64;
          const int d0 = (X1 - d1) >> 7;
          w0 |= (uint32_t)(d0 & 0xff) << (8 * j);
          w1 |= (uint32_t)(d1 & 0xff) << (8 * j);
          w2 |= (uint32_t)(d2 & 0xff) << (8 * j);
        }
      }
      const uint32_t wd[3] = {w0, w1, w2};
#pragma unroll
      for (int dg = 0; dg < 3; ++dg) dst(digit_index(kb, 3 * m + dg, kk, nt, groups, KB, tc), wd[dg]);
    }
  }
}

// encode_digits for an encoder whose statistics come from the producer:
// the first batch's activations and RMSNorm weights do not depend on those
// statistics, so they are loaded before ready() (which computes s_mul / s_e
// and ends with a block barrier) and their round trip overlaps it.  The
// digits are those of encode_digits, bit for bit.
template <int BATCH = kEncBatch, class Src4, class Dst, class Ready>
__device__ __forceinline__ void encode_digits_early(const StatArgs& a, int nt, int KB, int kb0,
                                                    int kb1, const float* s_mul, const int* s_e,
                                                    Src4 src4, Dst dst, bool tc, Ready ready) {
  const int M = a.M, d = a.d;
  const int groups = groups_for_tokens(M);
  const int pad_cols = 8 * nt * groups - 3 * M;
  const int ngroups = (kb1 - kb0) * 8;
  const int tasks = ngroups * (M + pad_cols);
  const bool use_w = a.do_norm && a.w;
  float4 v[BATCH], wv[BATCH];
  auto load = [&](int t0) {
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int task = t0 + u * blockDim.x;
      v[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      wv[u] = make_float4(1.0f, 1.0f, 1.0f, 1.0f);
      if (task < tasks) {
        const int grp = task % ngroups, q = task / ngroups;
        if (q < M) {
          const int k = (kb0 + (grp >> 3)) * 32 + (grp & 7) * 4;
          v[u] = src4(q, k);
          if (use_w) {
            const float* wp = a.w + k;
            if (k + 3 < a.wlen && ((reinterpret_cast<uintptr_t>(wp) & 15) == 0)) {
              wv[u] = __ldg(reinterpret_cast<const float4*>(wp));
            } else {
              wv[u].x = k < a.wlen ? __ldg(wp) : 1.0f;
              wv[u].y = k + 1 < a.wlen ? __ldg(wp + 1) : 1.0f;
              wv[u].z = k + 2 < a.wlen ? __ldg(wp + 2) : 1.0f;
              wv[u].w = k + 3 < a.wlen ? __ldg(wp + 3) : 1.0f;
            }
          }
        }
      }
    }
  };
  load(threadIdx.x);
  ready();
  for (int t0 = threadIdx.x; t0 < tasks; t0 += blockDim.x * BATCH) {
    if (t0 != (int)threadIdx.x) load(t0);
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int task = t0 + u * blockDim.x;
      if (task >= tasks) continue;
      const int grp = task % ngroups;
      const int q = task / ngroups;  // token (q < M) or padding column (q >= M)
      const int kb = kb0 + (grp >> 3);
      const int kk = (grp & 7) * 4;
      if (q >= M) {
        dst(digit_index(kb, 3 * M + (q - M), kk, nt, groups, KB, tc), 0u);
        continue;
      }
      const int m = q;
      uint32_t w0 = 0, w1 = 0, w2 = 0;
      if (s_e[m] != kExpNonFinite) {
        const float mul = s_mul[m];
        const float vv[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        const float ww[4] = {wv[u].x, wv[u].y, wv[u].z, wv[u].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int k = kb * 32 + kk + j;
          int X = 0;
          if (k < d) {
            float x = vv[j];
            if (a.do_norm) x = __fmul_rn(x, ww[j]);
            X = __float2int_rn(__fmul_rn(x, mul));
          }
          const int d2 = ((X + 64) & 127) - 64;
          const int X1 = (X - d2) >> 7;
          const int d1 = ((X1 + 64) & 127) - 64;
          const int d0 = (X1 - d1) >> 7;
          w0 |= (uint32_t)(d0 & 0xff) << (8 * j);
          w1 |= (uint32_t)(d1 & 0xff) << (8 * j);
          w2 |= (uint32_t)(d2 & 0xff) << (8 * j);
        }
      }
      const uint32_t wd[3] = {w0, w1, w2};
#pragma unroll
      for (int dg = 0; dg < 3; ++dg) dst(digit_index(kb, 3 * m + dg, kk, nt, groups, KB, tc), wd[dg]);
    }
  }
}

// Four consecutive activations of token m starting at k (k % 4 == 0), zero
// past d; vectorised when the row is float4-aligned.  Read through L2: the
// producing kernel may have finished after this grid was scheduled.
__device__ __forceinline__ float4 load_act4(const float* h, int ld, int d, int m, int k) {
  const float* p = h + (size_t)m * ld + k;
  if (k + 3 < d && ((reinterpret_cast<uintptr_t>(p) & 15) == 0))
    return __ldcg(reinterpret_cast<const float4*>(p));
  float4 r;
  r.x = k < d ? __ldcg(p) : 0.0f;
  r.y = k + 1 < d ? __ldcg(p + 1) : 0.0f;
  r.z = k + 2 < d ? __ldcg(p + 2) : 0.0f;
  r.w = k + 3 < d ? __ldcg(p + 3) : 0.0f;
  return r;
}

// The O projection's input straight from the attention's page partials
// (QuantArgs::att_o): the CTA's slice [lo, hi) of every token is combined
// into shared memory, then encoded.  Output (token m, head h, columns c..c+3)
// = sum_p e^(m_p - M) o_p / sum_p e^(m_p - M) l_p over the pages p of its
// query block, M = max_p m_p.  kCombLanes adjacent lanes share an output:
// lane j of the group takes pages j, j + kCombLanes, ..., adding them in
// order (B of them in flight, which leaves the arithmetic unchanged), and the
// group's sums meet in an xor-shuffle tree, whose sums are bitwise the same
// on every lane -- the same result for every B.  The exponent comes from the
// attention's bound (amax), read meanwhile.  `lead`: this CTA writes the
// exponents and zeroes the next producer's max slot.  EB: encode_digits'
// batch.
constexpr int kCombLanes = 16;
template <int B, int EB>
__device__ __forceinline__ void attn_combine_encode(const QuantArgs& a, int lo, int hi, int kb0,
                                                    int kb1, bool lead, uint32_t* s_bound,
                                                    float* s_mul, int* s_e, float* s_slice,
                                                    uint32_t* xq) {
  constexpr int LN = kCombLanes;
  if (threadIdx.x < a.M) s_bound[threadIdx.x] = __ldcg(a.amax + threadIdx.x);
  const int hd = a.att_hdp, G = a.att_G, Rs = G * a.att_qblk;
  const int n_qb = (a.att_seq.seq_len + a.att_qblk - 1) / a.att_qblk;
  const int span = hi - lo, q4 = span / 4, n_out = a.M * q4;
  const size_t cs4 = (size_t)Rs * hd / 4;  // float4s between pages
  const int sub = (int)threadIdx.x & (LN - 1);
  for (int base = 0; base < LN * n_out; base += blockDim.x) {  // block-uniform trip count
    const int t = base + (int)threadIdx.x, o = t / LN;
    const bool live = o < n_out;
    const int m = live ? o / q4 : 0;
    const int k = lo + 4 * (live ? o - m * q4 : 0);
    const bool in = live && k < a.d;
    int nch = 0;
    const float2* ml = nullptr;
    const float4* src = nullptr;
    if (in) {
      const int hh = k / hd;
      const int z = seq_of(a.att_seq, m), i = seq_off(a.att_seq, m);
      const int qb = i / a.att_qblk, i0 = qb * a.att_qblk;
      const int Mq = min(a.att_qblk, a.att_seq.seq_len - i0);
      const int L = a.att_pos[z * a.att_seq.pos_stride] + a.att_pos_add + i0 + Mq;
      nch = min((L + a.att_page - 1) / a.att_page, a.att_chunks);
      const size_t cslot = (size_t)(z * n_qb + qb) * a.att_Hkv + hh / G;
      const size_t row = cslot * a.att_chunks * Rs + (size_t)((i - i0) * G + hh % G);
      ml = reinterpret_cast<const float2*>(a.att_ml) + row;
      src = reinterpret_cast<const float4*>(a.att_o + row * hd + (k - hh * hd));
    }
    // M over every page of the row (all lanes' pages): a pre-pass only when
    // the pages do not fit one batch
    float M_ = -INFINITY;
    if (nch > LN * B)
      for (int p = sub; p < nch; p += LN) M_ = fmaxf(M_, __ldcg(&ml[(size_t)p * Rs].x));
    float l = 0.0f;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    // every lane runs the warp's longest page loop (the shuffles below need
    // all of them; lanes past their own pages load nothing)
    for (int p0 = 0; __any_sync(0xffffffffu, p0 < nch); p0 += LN * B) {
      float2 mv[B];
      float4 v[B];
#pragma unroll
      for (int u = 0; u < B; ++u) {
        const int p = p0 + LN * u + sub;
        mv[u] = p < nch ? __ldcg(ml + (size_t)p * Rs) : make_float2(-INFINITY, 0.0f);
        v[u] = p < nch ? __ldcg(src + (size_t)p * cs4) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
      if (p0 == 0) {
        if (nch <= LN * B) {
#pragma unroll
          for (int u = 0; u < B; ++u) M_ = fmaxf(M_, mv[u].x);
        }
#pragma unroll
        for (int off = LN / 2; off; off >>= 1) M_ = fmaxf(M_, __shfl_xor_sync(0xffffffffu, M_, off));
      }
#pragma unroll
      for (int u = 0; u < B; ++u) {
        const float w = (mv[u].x == -INFINITY) ? 0.0f : expf(mv[u].x - M_);
        l = __fadd_rn(l, __fmul_rn(w, mv[u].y));
        acc.x = __fmaf_rn(v[u].x, w, acc.x);
        acc.y = __fmaf_rn(v[u].y, w, acc.y);
        acc.z = __fmaf_rn(v[u].z, w, acc.z);
        acc.w = __fmaf_rn(v[u].w, w, acc.w);
      }
    }
#pragma unroll
    for (int off = LN / 2; off; off >>= 1) {
      l = __fadd_rn(l, __shfl_xor_sync(0xffffffffu, l, off));
      acc.x = __fadd_rn(acc.x, __shfl_xor_sync(0xffffffffu, acc.x, off));
      acc.y = __fadd_rn(acc.y, __shfl_xor_sync(0xffffffffu, acc.y, off));
      acc.z = __fadd_rn(acc.z, __shfl_xor_sync(0xffffffffu, acc.z, off));
      acc.w = __fadd_rn(acc.w, __shfl_xor_sync(0xffffffffu, acc.w, off));
    }
    if (live && sub == 0) {
      float4 r = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (in) {
        r.x = __fdiv_rn(acc.x, l);
        r.y = __fdiv_rn(acc.y, l);
        r.z = __fdiv_rn(acc.z, l);
        r.w = __fdiv_rn(acc.w, l);
      }
      *reinterpret_cast<float4*>(s_slice + (size_t)m * span + (k - lo)) = r;
    }
  }
  __syncthreads();
  // exponents from the bound (no norm), as the encoder's statistics path
  if (threadIdx.x < a.M) {
    const int m = threadIdx.x;
    const float amax = __uint_as_float(s_bound[m]);
    int e = 0;
    if (!isfinite(amax)) {
      e = kExpNonFinite;
    } else if (amax > 0.0f) {
      int E;
      frexpf(amax * 1.0000002f, &E);
      e = 20 - E;
    }
    s_mul[m] = (e != kExpNonFinite) ? ldexpf(1.0f, e) : 0.0f;
    s_e[m] = e;
    if (lead) a.xexp[m] = e;
  }
  if (lead && a.amax_next && threadIdx.x < kMaxTokens) a.amax_next[threadIdx.x] = 0u;
  __syncthreads();
  const StatArgs sa{nullptr, 0, a.d, a.M, nullptr, 0, 0.0f, 0};
  encode_digits<EB>(sa, a.nt, a.KB, kb0, kb1, s_mul, s_e,
                [&](int m, int k) {
                  const float* p = s_slice + (size_t)m * span + (k - lo);
                  return make_float4(k < a.d ? p[0] : 0.0f, k + 1 < a.d ? p[1] : 0.0f,
                                     k + 2 < a.d ? p[2] : 0.0f, k + 3 < a.d ? p[3] : 0.0f);
                },
                [&](size_t wi, uint32_t v) { xq[wi] = v; }, a.tc_layout != 0);
}

// The encoder's statistics path over k-blocks [kb0, kb1) of a.xq: the
// exponents come from the producer's statistics, then the slice is encoded;
// block 0 also writes the exponents and zeroes the next producer's max slot.
// s_mul / s_e: kMaxTokens each (shared).  phase(k) marks trace phases 1-3.
template <int BATCH = kEncBatch, class Phase>
__device__ __forceinline__ void encode_slice_stats_t(const QuantArgs& a, int kb0, int kb1,
                                                     float* s_mul, int* s_e, Phase phase) {
  uint32_t* xq = reinterpret_cast<uint32_t*>(a.xq);
  const StatArgs sa{a.h, a.ld, a.d, a.M, a.w, a.wlen, a.eps, a.do_norm};
  auto src4 = [&](int m, int k) { return load_act4(a.h, a.ld, a.d, m, k); };
  auto ready = [&]() {
    // statistics from the producing kernel: one warp per token sums the
    // partials in a fixed order (lane-strided, then an xor-shuffle tree)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int m = warp; m < a.M; m += blockDim.x >> 5) {
      const unsigned mxb = lane == 0 ? __ldcg(a.amax + m) : 0u;  // issued with the partials
      float ss = 0.0f;
      if (a.do_norm) {
        // the lane's partials j = lane, lane + 32, ... in batches of 8 whose
        // loads are all in flight before the (in-order) adds
        const float* pr = a.pss + (size_t)m * a.np_stride;
        for (int j0 = lane; j0 < a.np; j0 += 32 * 8) {
          float v[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) v[u] = j0 + 32 * u < a.np ? __ldcg(pr + j0 + 32 * u) : 0.0f;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            if (j0 + 32 * u < a.np) ss = __fadd_rn(ss, v[u]);
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      if (lane == 0) {
        const float mx = __uint_as_float(mxb);
        float rms = 1.0f;
        if (a.do_norm) rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)(a.d > 1 ? a.d : 1)), a.eps));
        const float amax = a.do_norm ? mx / rms : mx;
        int e = 0;
        if (!isfinite(amax)) {  // a NaN/inf element makes the bit-max non-finite
          e = kExpNonFinite;
        } else if (amax > 0.0f) {
          int E;
          frexpf(amax * 1.0000002f, &E);
          e = 20 - E;
        }
        s_mul[m] = (e != kExpNonFinite) ? ldexpf(a.do_norm ? 1.0f / rms : 1.0f, e) : 0.0f;
        s_e[m] = e;
      }
    }
    if (blockIdx.x == 0 && a.amax_next && threadIdx.x < kMaxTokens) a.amax_next[threadIdx.x] = 0u;
    phase(1);
    __syncthreads();
    phase(2);
    if (blockIdx.x == 0 && threadIdx.x < a.M) a.xexp[threadIdx.x] = s_e[threadIdx.x];
  };
  encode_digits_early<BATCH>(sa, a.nt, a.KB, kb0, kb1, s_mul, s_e, src4,
                      [&](size_t wi, uint32_t v) { xq[wi] = v; }, a.tc_layout != 0, ready);
  phase(3);
}

// All CTAs of the grid (every dimension; at most one wave, so all resident)
// meet here.  Thread 0 of each CTA arrives with an acquire-release add (the
// CTA's writes before the block barrier are released with it); the last to
// arrive resets the count and publishes the next generation (release); the
// others poll it (acquire), at most 2 s of %globaltimer, after which the
// error word is raised and they go on.  wait = false: arrive only (a CTA that
// reads nothing the others wrote).
__device__ __forceinline__ void grid_barrier(unsigned* bar, int* err, bool wait = true) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned n_cta = gridDim.x * gridDim.y * gridDim.z;
    unsigned gen, old;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(gen) : "l"(bar + 1) : "memory");
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(bar) : "memory");
    if (old == n_cta - 1) {
      // every CTA has arrived: nobody reads the count until the next use
      asm volatile("st.relaxed.gpu.global.u32 [%0], 0;" ::"l"(bar) : "memory");
      asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(bar + 1), "r"(gen + 1u) : "memory");
    } else if (wait) {
      unsigned long long t0;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
      for (long long i = 0;; ++i) {
        unsigned g;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(g) : "l"(bar + 1) : "memory");
        if (g != gen) break;
        if ((i & 63) == 63) {
          unsigned long long t1;
          asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
          if (t1 - t0 > 2000000000ull || i > (1ll << 26)) {
            if (err) atomicExch(err, 1);
            break;
          }
        }
      }
    }
  }
  __syncthreads();
}

// ------------------------------------------------------------ GEMV
// Work split: each CTA owns a contiguous range of the linear (stripe,
// k-block) index (stream-K, balanced to one k-block); its 8 warps own
// contiguous eighths of it.  A warp streams its weights with 16-byte loads
// (U k-blocks in flight), the first batch issued before griddepcontrol.wait.
// A stripe finished inside one warp goes straight to the epilogue.  Stripes
// shared by warps of one CTA are summed with shared-memory atomics and the
// last contributing warp finishes them; only a CTA's first and last stripe
// can be shared with other CTAs, and those go through the global split-K
// workspace (int32 sums, so the reduction order never changes the result).
template <int NT>
struct GemvCfg {
  // k-blocks per load batch: its weight fragments and activation words stay
  // in registers, 8 up to three tiles (24 columns, 8 tokens), 4 beyond
  static constexpr int U = (NT <= 3) ? 8 : 4;
  static constexpr int COLS = 8 * NT;
};

constexpr int kGemvWarps = 8;

// Epilogue of a finished stripe from a row-major [16][ld] int tile holding
// MG <= 16 tokens (forward-wide tokens m0 .. m0 + MG - 1), run by one warp.
// Lane (it, lane) handles rows r and r+8 of tile token m, with
// idx = it*32 + lane, r = idx & 7, m = idx >> 3; the 8 lanes of a token form
// one shuffle group for the encoding statistics.  xexp holds the tile's
// token exponents; tok (or nullptr) its tokens' (position, KV page), resolved
// ahead for the QKV epilogue.  A lane's rows are the same in every
// iteration, so all its global loads (row scales, next-norm weights, then per
// iteration the residual rows or the RoPE factors) are issued before the
// arithmetic -- or read from `pre`, the same values staged in shared memory
// while the tile's main loop ran.
struct EpiPre {
  int row0;            // first row of the staged tile
  const float* scale;  // [128] row scales
  const float* w;      // [128] next RMSNorm weights (RESID)
  const float* h;      // [tokens][128] residual rows (RESID), token index from m0 of the launch
  const float* cs;     // [tokens][64] RoPE cos of (stripe, pair row) (QKV)
  const float* sn;
};

template <int NT, int EPI, typename T>
__device__ __forceinline__ void gemv_epilogue(const GemvArgs& a, int stripe, const T* tile,
                                              int ld, int lane, unsigned long long* kmax,
                                              const float* scale, const int* xexp, int m0,
                                              int MG, const int2* tok = nullptr,
                                              const EpiPre* pre = nullptr) {
  constexpr int NIT = (8 * kGroupTokens) / 32;
  const int r = lane & 7;
  const int prow = stripe * 16 + r;
  const int lrow = pre ? prow - pre->row0 : 0;  // row within the staged tile
  // q4_0 tiles carry their block scales already; int8 tiles take the row scale
  float sc0 = 1.0f, sc1 = 1.0f;
  if (pre) {
    sc0 = pre->scale[lrow];
    sc1 = pre->scale[lrow + 8];
  } else if (scale) {
    sc0 = scale[prow];
    sc1 = scale[prow + 8];
  }
  float w0 = 1.0f, w1 = 1.0f;  // next RMSNorm weight of the rows (RESID statistics)
  if constexpr (EPI == EPI_RESID) {
    if (pre) {
      w0 = pre->w[lrow];
      w1 = pre->w[lrow + 8];
    } else if (a.st_w) {
      if (prow < a.n_out) w0 = a.st_w[prow];
      if (prow + 8 < a.n_out) w1 = a.st_w[prow + 8];
    }
  }
  // per iteration: RESID the current h rows; QKV position, page, cos, sin
  float p0[NIT], p1[NIT];
  int ppos[NIT], ppg[NIT];
  // QKV geometry of this stripe and lane (rows r and r+8 are the RoPE pair
  // (i, i + half), transformer.rs:921-938; V stripes hold 16 plain rows)
  const int per_head = a.half_p >> 3;  // stripes per head (Q/K) = hdp/16
  const bool rope = stripe < a.sq + a.sk;
  const bool isq = stripe < a.sq;
  const int s2 = rope ? (isq ? stripe : stripe - a.sq) : stripe - a.sq - a.sk;
  const int hh = per_head > 0 ? s2 / per_head : 0;
  const int ri = (s2 - hh * per_head) * (rope ? 8 : 16) + r;  // i (RoPE) or j (V)
#pragma unroll
  for (int it = 0; it < NIT; ++it) {
    const int m = it * 4 + (lane >> 3);
    p0[it] = p1[it] = 0.0f;
    ppos[it] = ppg[it] = 0;
    if (it * 32 >= 8 * MG || m >= MG) continue;
    const int mt = m0 + m;
    if constexpr (EPI == EPI_RESID) {
      if (pre) {
        const float* hr = pre->h + (size_t)(mt - a.m0) * kTcTileRows;
        p0[it] = hr[lrow];
        p1[it] = hr[lrow + 8];
      } else {
        const float* o = a.out + (size_t)mt * a.ldo;
        if (prow < a.n_out) p0[it] = o[prow];
        if (prow + 8 < a.n_out) p1[it] = o[prow + 8];
      }
    } else if constexpr (EPI == EPI_QKV) {
      int pos, pg;
      if (tok) {
        pos = tok[m].x;
        pg = tok[m].y;
      } else {
        const int z = seq_of(a.seq, mt);
        pos = a.pos_ptr[z * a.seq.pos_stride] + a.pos_add + seq_off(a.seq, mt);
        pg = a.page_table[z * a.seq.pt_stride + pos / a.page];
      }
      ppos[it] = pos;
      ppg[it] = pg;
      if (rope) {
        if (pre) {
          const int q = (stripe * 8 + r) - pre->row0 / 2;  // (stripe, pair row) in the tile
          p0[it] = pre->cs[(size_t)(mt - a.m0) * 64 + q];
          p1[it] = pre->sn[(size_t)(mt - a.m0) * 64 + q];
        } else {
          p0[it] = a.rope_cos[(size_t)pos * a.half_p + ri];
          p1[it] = a.rope_sin[(size_t)pos * a.half_p + ri];
        }
      }
    }
  }
#pragma unroll
  for (int it = 0; it < NIT; ++it) {
    if (it * 32 >= 8 * MG) break;  // warp-uniform
    const int idx = it * 32 + lane;
    const bool valid = idx < 8 * MG;
    const int m = valid ? (idx >> 3) : 0;
    const int mt = m0 + m;  // forward-wide token
    // statistics contribution of this lane: sum(h*h) and max|h*w| kept as
    // float bits, whose unsigned order matches |x| and lets NaN/inf win
    float st_sq = 0.0f;
    uint32_t st_mx = 0u;
    if (valid) {
      const int e = xexp[m];
      const float y0 = combine_digits(tile + r * ld, m, sc0, e);
      const float y1 = combine_digits(tile + (r + 8) * ld, m, sc1, e);
      if constexpr (EPI == EPI_TP) {
        // this rank's partial rows into slot `rank` of every rank's buffer
        const TPArgs& t = a.tp;
        const size_t off = (((size_t)(__ldcg(t.epoch) & 1u) * t.world + t.rank) * kMaxTokens + mt) * t.d;
        for (int q = 0; q < t.world; ++q) {
          float* o = t.red[q] + off;
          if (prow < a.n_out) o[prow] = y0;
          if (prow + 8 < a.n_out) o[prow + 8] = y1;
        }
      } else if constexpr (EPI == EPI_STORE || EPI == EPI_RESID || EPI == EPI_LMHEAD) {
        float* o = a.out ? a.out + (size_t)mt * a.ldo : nullptr;
        if (prow < a.n_out) {
          if constexpr (EPI == EPI_RESID) {
            const float h0 = __fadd_rn(p0[it], y0);
            o[prow] = h0;
            st_sq = __fmul_rn(h0, h0);
            st_mx = __float_as_uint(fabsf(__fmul_rn(h0, w0)));
          } else if (o) {
            o[prow] = y0;
          }
          if constexpr (EPI == EPI_LMHEAD) {
            if (y0 > -INFINITY) {  // NaN and -inf never win (generate.rs:1088-1098)
              unsigned long long k =
                  argmax_key(__fadd_rn(y0, 0.0f), (uint32_t)(prow + a.row_offset));
              kmax[it] = k > kmax[it] ? k : kmax[it];
            }
          }
        }
        if (prow + 8 < a.n_out) {
          if constexpr (EPI == EPI_RESID) {
            const float h1 = __fadd_rn(p1[it], y1);
            o[prow + 8] = h1;
            st_sq = __fadd_rn(st_sq, __fmul_rn(h1, h1));
            st_mx = max(st_mx, __float_as_uint(fabsf(__fmul_rn(h1, w1))));
          } else if (o) {
            o[prow + 8] = y1;
          }
          if constexpr (EPI == EPI_LMHEAD) {
            if (y1 > -INFINITY) {
              unsigned long long k =
                  argmax_key(__fadd_rn(y1, 0.0f), (uint32_t)(prow + 8 + a.row_offset));
              kmax[it] = k > kmax[it] ? k : kmax[it];
            }
          }
        }
      } else if constexpr (EPI == EPI_SWIGLU) {
        const int i = stripe * 8 + r;  // row r = gate_i, row r+8 = up_i
        if (i < a.n_out) {
          const float act = silu_mul(y0, y1);
          a.out[(size_t)mt * a.ldo + i] = act;
          st_mx = __float_as_uint(fabsf(act));
        }
      } else if constexpr (EPI == EPI_QKV) {
        const int pos = ppos[it], pg = ppg[it];
        const int slot = pos % a.page;
        if (rope) {
          const float c = p0[it], sn = p1[it];
          const float o0 = __fsub_rn(__fmul_rn(y0, c), __fmul_rn(y1, sn));
          const float o1 = __fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, c));
          if (isq) {
            float* q = a.q_out + ((size_t)mt * a.H + hh) * a.hdp;
            q[ri] = o0;
            q[a.half_p + ri] = o1;
          } else {
            float* k = a.kc + (((size_t)pg * a.Hkv + hh) * a.page + slot) * a.hdp;
            k[ri] = o0;
            k[a.half_p + ri] = o1;
          }
        } else {
          float* v = a.vc + (((size_t)pg * a.Hkv + hh) * a.page + slot) * a.hdp;
          v[ri] = y0;
          v[ri + 8] = y1;
        }
      }
    }
    if constexpr (EPI == EPI_RESID || EPI == EPI_SWIGLU) {
      if (a.st_amax) {  // warp-uniform; every lane takes part in the shuffles
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) {
          if constexpr (EPI == EPI_RESID)
            st_sq = __fadd_rn(st_sq, __shfl_xor_sync(0xffffffffu, st_sq, off, 8));
          st_mx = max(st_mx, __shfl_xor_sync(0xffffffffu, st_mx, off, 8));
        }
        if (valid && r == 0) {
          if constexpr (EPI == EPI_RESID) a.st_pss[(size_t)mt * a.st_np + stripe] = st_sq;
          atomicMax(a.st_amax + mt, st_mx);
        }
      }
    }
  }
}

// Work split (whole stripes, no cross-CTA reduction): CTA c owns stripes
// [c*S/G, (c+1)*S/G).  With s stripes per CTA each stripe is cut into
// F = ceil(8/s) k-ranges so that all 8 warps have units; unit u (stripe
// u/F, k-range u%F) belongs to warp u%8.  A stripe cut into F > 1 units is
// summed with shared-memory atomics and finished by its last warp.
// Per-SM streaming capacity exceeds each SM's share of HBM bandwidth, so the
// mild imbalance of whole-stripe ownership costs nothing.
constexpr int kTileSlots = 8;      // stripes in flight per CTA when F > 1
constexpr int kMaxCtaStripes = 64; // scales staged per CTA (before the wait)

// Shared memory of a k-split: int8 sums arrive by integer atomics (exact, so
// order-free) in one tile per stripe; q4_0 sums are f32, so every unit keeps
// its own partial tile and the last warp adds them in k order (results do
// not depend on arrival order).
// End of a row-parallel GEMV: the block barrier orders the CTA's peer stores
// before thread 0's system-scope fence (release is cumulative over them),
// then the grid's last CTA publishes the epoch in every rank's flags.
__device__ __forceinline__ void tp_publish(const TPArgs& t) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const int n = gridDim.x * gridDim.y;
    if (atomicAdd(t.cnt, 1) == n - 1) {
      __threadfence_system();
      const unsigned e = __ldcg(t.epoch);
      for (int r = 0; r < t.world; ++r)
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(t.flag[r] + (e & 1u) * kMaxTP + t.rank),
                     "r"(e)
                     : "memory");
      atomicExch(t.cnt, 0);
    }
  }
}

constexpr int kMaxSplitUnits = 16;  // units per CTA when F > 1 (ns * F <= 14)

// Weight ring of one warp: NB chunk buffers of up to U k-blocks, filled by
// cp.async.bulk copies (lane 0) that complete on one mbarrier per buffer.
// WF_I8 k-block: 512 bytes (each lane's 16-byte A fragment); WF_Q4: 256
// bytes of nibbles, then (after the chunk's U nibble blocks) 32 bytes of
// block scales.  The buffers hold what the warp streams next, so the first
// NB chunks -- the whole slice of a small projection -- load before
// griddepcontrol.wait, while the producer of its activations still runs.
// Used by the WF_I8R variant only (large int8 matrices, where the deeper
// stream pays; the register path is faster for small ones).
// Ring chunks issued before the dependency wait: one (more competes with the
// producer -- an encoder on the critical path -- for memory bandwidth, and
// measured slower).
#ifndef MC_RING_PREWAIT
#define MC_RING_PREWAIT 1
#endif
constexpr int kRingPreWait = MC_RING_PREWAIT;

template <int NT, int WF>
struct GemvRing {
  static constexpr bool On = WF == WF_I8R;
  static constexpr int U = GemvCfg<NT>::U;
  static constexpr int KBW = 512;
  static constexpr int KBS = 0;
  static constexpr int ChunkBytes = U * (KBW + KBS);
  static constexpr int NB = NT <= 3 ? 2 : 3;  // two 4 KB chunks, or three 2 KB ones
  static constexpr int PreWait = kRingPreWait < NB ? kRingPreWait : NB;
  static constexpr int WarpBytes = On ? NB * ChunkBytes : 0;
  static constexpr size_t Base = ((((size_t)kGemvWarps * 16 * (8 * NT + 1) +
                                    (size_t)(WF == WF_Q4 ? kMaxSplitUnits : kTileSlots) * 16 *
                                        8 * NT) * 4) + 127) / 128 * 128;
  static constexpr int kMaxNB = 3;
};

template <int NT, int WF>
static constexpr size_t gemv_dyn_smem() {
  return GemvRing<NT, WF>::Base + (size_t)kGemvWarps * GemvRing<NT, WF>::WarpBytes;
}

// TAIL (RESID and SWIGLU, one launch per projection): after its epilogues
// the grid meets at a bounded barrier (the grid is at most one wave, so every
// CTA is resident), then encodes the next projection's input -- the rows it
// just wrote, with the statistics its epilogues folded -- exactly as k_quant
// would (a.enc, k-blocks split over the grid), saving that launch.
template <int NT, int EPI, int WF, bool TAIL>
__global__ void __launch_bounds__(kGemvWarps * 32, 2) k_gemv(GemvArgs a) {
  constexpr int U = GemvCfg<NT>::U;
  constexpr int COLS = GemvCfg<NT>::COLS;
  constexpr bool Q4 = WF == WF_Q4;
  constexpr bool RING = WF == WF_I8R;
  using Acc = typename std::conditional<Q4, float, int>::type;
  extern __shared__ __align__(16) int gemv_smem[];
  // per-warp fragment staging [warp][16][COLS+1], then the k-split area
  Acc (*sm_epi)[16][COLS + 1] = reinterpret_cast<Acc (*)[16][COLS + 1]>(gemv_smem);
  Acc (*sm_tile)[16 * COLS] =
      reinterpret_cast<Acc (*)[16 * COLS]>(gemv_smem + kGemvWarps * 16 * (COLS + 1));
  __shared__ int sm_cnt[kTileSlots];
  __shared__ float sm_scale[kMaxCtaStripes * 16];
  __shared__ int sm_exp[kGemvWarps][kGroupTokens];  // per warp: filled at its first epilogue
  __shared__ unsigned long long sm_keys[kGroupTokens];
  __shared__ __align__(8) uint64_t sm_mbar[kGemvWarps][GemvRing<NT, WF>::kMaxNB];
  using R = GemvRing<NT, WF>;
  uint8_t* ring = reinterpret_cast<uint8_t*>(gemv_smem) + R::Base;

  MC_TRACE_T0
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int s0 = (int)((long long)a.n_stripes * blockIdx.x / gridDim.x);
  const int s1 = (int)((long long)a.n_stripes * (blockIdx.x + 1) / gridDim.x);
  const int ns = s1 - s0;
  const int F = ns >= kGemvWarps ? 1 : (kGemvWarps + max(ns, 1) - 1) / max(ns, 1);
  const int n_units = ns * F;

  if (threadIdx.x < kTileSlots) sm_cnt[threadIdx.x] = 0;
  if (threadIdx.x < kGroupTokens) sm_keys[threadIdx.x] = 0ull;
  if (!Q4 && F > 1)
    for (int i = threadIdx.x; i < kTileSlots * 16 * COLS; i += blockDim.x) (&sm_tile[0][0])[i] = 0;
  const bool scale_smem = !Q4 && ns <= kMaxCtaStripes;
  if (scale_smem)
    for (int i = threadIdx.x; i < ns * 16; i += blockDim.x) sm_scale[i] = a.scale[s0 * 16 + i];

  auto unit_range = [&](int u, int& stripe, int& kb0, int& kb1) {
    stripe = s0 + u / F;
    const int part = u - (u / F) * F;
    kb0 = a.KB * part / F;  // KB * F < 2^31
    kb1 = a.KB * (part + 1) / F;
  };
  // Weights never depend on the producer grid: start streaming them before
  // the wait.  Register path: the first batch of this warp's first unit.
  // Ring path (WF_I8R): lane 0 streams this warp's k-blocks (its units u =
  // warp, warp + 8, ... in order, U per chunk) into the ring, chunk c into
  // buffer c % NB; the consumer below walks the same order.
  const uint64_t pol = policy_evict_first();
  int4 wv[Q4 || RING ? 1 : U];
  uint2 wq[Q4 ? U : 1];
  uint32_t wsc[Q4 ? U : 1];
  auto load_batch = [&](int stripe, int kb, int nb) {
    if constexpr (Q4) {
      const uint2* wp = reinterpret_cast<const uint2*>(a.w) + ((size_t)stripe * a.KB + kb) * 32 + lane;
      const uint32_t* sp = a.qscale + ((size_t)stripe * a.KB + kb) * 8 + (lane >> 2);
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (j < nb) {
          wq[j] = ldg_stream2(wp + (size_t)j * 32, pol);
          wsc[j] = ldg_stream1(sp + (size_t)j * 8, pol);
        }
    } else if constexpr (!RING) {
      const int4* wp = a.w + ((size_t)stripe * a.KB + kb) * 32 + lane;
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (j < nb) wv[j] = ldg_stream(wp + (size_t)j * 32, pol);
    }
  };
  uint8_t* wring = ring + (size_t)warp * R::WarpBytes;
  uint64_t* mbar = sm_mbar[warp];
  int pu = warp, pk = 0, pk1 = -1, pstripe = 0;  // producer: unit, next k-block, its end
  auto issue = [&](int b) {  // lane 0: the next chunk of this warp into buffer b
    while (pu < n_units && pk >= pk1) {
      if (pk1 >= 0) pu += kGemvWarps;
      if (pu >= n_units) break;
      unit_range(pu, pstripe, pk, pk1);
    }
    if (pu >= n_units) return;
    const int nb = min(U, pk1 - pk);
    uint8_t* dst = wring + (size_t)b * R::ChunkBytes;
    const size_t blk = (size_t)pstripe * a.KB + pk;
    mbar_expect_tx(&mbar[b], (uint32_t)(nb * R::KBW));
    bulk_load_hint(dst, reinterpret_cast<const uint8_t*>(a.w) + blk * R::KBW,
                   (uint32_t)(nb * R::KBW), &mbar[b], pol);
    pk += nb;
  };
  if constexpr (RING) {
    // the first kRingPreWait chunks go out before the wait
    if (lane == 0) {
      for (int b = 0; b < R::NB; ++b) mbar_init(&mbar[b], 1);
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      for (int b = 0; b < R::PreWait; ++b) issue(b);
    }
    __syncwarp();
  } else if (warp < n_units) {
    int st, k0, k1;
    unit_range(warp, st, k0, k1);
    load_batch(st, k0, min(U, k1 - k0));
  }
  // Warm L2 with the next GEMV's weights (split like this grid) so HBM keeps
  // streaming through this grid's tail and the small kernels in between.
  if (a.next_w && lane == 1 && a.next_bytes > 0) {
    const long long nw = (long long)gridDim.x * kGemvWarps;
    const long long gw = (long long)blockIdx.x * kGemvWarps + warp;
    const long long chunk = (a.next_bytes / nw) & ~15ll;
    if (chunk >= 16) {
      const char* p = reinterpret_cast<const char*>(a.next_w) + chunk * gw;
      long long left = min(chunk, a.next_pf_bytes / nw);
      while (left >= 16) {
        const uint32_t b = (uint32_t)min(left, 32768ll) & ~15u;
        prefetch_l2_bulk(p, b);
        p += b;
        left -= b;
      }
    }
  }
  // Warm L2 with the K/V pages the attention after this QKV projection reads
  // (positions below the ones this grid appends were written by earlier
  // launches; the position counter is final two launches back).
  if constexpr (EPI == EPI_QKV) {
    if (a.kv_prefetch && lane == 2) {
      const long long blk = (long long)a.page * a.hdp;  // floats of one (page, kv head)
      const long long nw = (long long)gridDim.x * kGemvWarps;
      const int z0 = seq_of(a.seq, a.m0), z1 = seq_of(a.seq, a.m0 + a.M - 1);
      for (int z = z0; z <= z1; ++z) {  // the sequences of this launch's tokens
        const int L = a.pos_ptr[z * a.seq.pos_stride] + a.pos_add + a.seq.seq_len;
        const int np = (L + a.page - 1) / a.page;
        const int* pt = a.page_table + z * a.seq.pt_stride;
        const long long items = (long long)np * 2 * a.Hkv;
        for (long long i = (long long)blockIdx.x * kGemvWarps + warp; i < items; i += nw) {
          const int pg = (int)(i / (2 * a.Hkv));
          const int rem = (int)(i - (long long)pg * 2 * a.Hkv);
          const float* base = (rem & 1) ? a.vc : a.kc;
          const float* p = base + ((long long)pt[pg] * a.Hkv + (rem >> 1)) * blk;
          prefetch_l2_bulk(p, (uint32_t)(blk * 4));
        }
      }
    }
  }
  __syncthreads();  // shared tiles, counters and scales are initialised
  grid_wait();
  MC_TRACE_WAITED(a.trace_slot);
  if (RING && lane == 0)
    for (int b = R::PreWait; b < R::NB; ++b) issue(b);
  // The token exponents are only needed by the epilogue: issue the load now,
  // consume it there, so its L2 round trip overlaps the first batches.
  const int xe = lane < a.M ? __ldcg(a.xexp + lane) : 0;
  bool xe_staged = false;
  auto stage_exp = [&]() {
    if (!xe_staged) {
      if (lane < kGroupTokens) sm_exp[warp][lane] = xe;
      __syncwarp();
      xe_staged = true;
    }
  };

  unsigned long long kmax[(8 * kGroupTokens) / 32];
#pragma unroll
  for (int i = 0; i < (8 * kGroupTokens) / 32; ++i) kmax[i] = 0ull;
  const float* scl = Q4 ? nullptr : (scale_smem ? sm_scale - s0 * 16 : a.scale);

  int c = 0;        // chunks consumed by this warp (ring path)
  bool ring_ok = true;
  bool pre = true;  // the register path's first batch is in flight
  for (int u = warp; u < n_units; u += kGemvWarps) {
    int stripe, k0, k1;
    unit_range(u, stripe, k0, k1);
    const int n = k1 - k0;

    if (n <= 0) {  // empty k-range (K shorter than the split): contributes nothing
      pre = false;
      continue;
    }
    Acc acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0;
    const uint8_t* xp = a.x + (size_t)k0 * 32 * COLS;
    for (int i = 0; i < n; i += U, ++c) {
      const int nb = min(U, n - i);
      if (!RING && !pre) load_batch(stripe, k0 + i, nb);
      pre = false;
      uint32_t xv[U][2 * NT];
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (j < nb) load_x<NT>(xv[j], xp + (size_t)(i + j) * 32 * COLS, lane);
      const int b = RING ? c % R::NB : 0;
      if constexpr (RING) ring_ok &= mbar_wait(&mbar[b], (uint32_t)((c / R::NB) & 1));
      const uint8_t* cb = wring + (size_t)b * R::ChunkBytes;
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (j < nb) {
          if constexpr (Q4) {
            // one k-block per MMA: exact int32 sums, then its block scales
            const int4 af = q4_fragment(wq[j]);
            const float d0 = __half2float(__ushort_as_half((unsigned short)(wsc[j] & 0xffffu)));
            const float d1 = __half2float(__ushort_as_half((unsigned short)(wsc[j] >> 16)));
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              int c[4] = {0, 0, 0, 0};
              imma(c, af, xv[j][2 * t], xv[j][2 * t + 1]);
              acc[t][0] = __fmaf_rn(small_int_to_float(c[0]), d0, acc[t][0]);
              acc[t][1] = __fmaf_rn(small_int_to_float(c[1]), d0, acc[t][1]);
              acc[t][2] = __fmaf_rn(small_int_to_float(c[2]), d1, acc[t][2]);
              acc[t][3] = __fmaf_rn(small_int_to_float(c[3]), d1, acc[t][3]);
            }
          } else {
            const int4 w = RING ? *reinterpret_cast<const int4*>(cb + j * R::KBW + lane * 16)
                                : wv[RING ? 0 : j];
#pragma unroll
            for (int t = 0; t < NT; ++t) imma(acc[t], w, xv[j][2 * t], xv[j][2 * t + 1]);
          }
        }
      if constexpr (RING) {
        // the MMAs above consumed every lane's fragments: the buffer is free
        __syncwarp();
        if (lane == 0) issue(b);
      }
    }
    const int g = lane >> 2, tq = lane & 3;
    if (F == 1) {
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        sm_epi[warp][g][t * 8 + 2 * tq] = acc[t][0];
        sm_epi[warp][g][t * 8 + 2 * tq + 1] = acc[t][1];
        sm_epi[warp][g + 8][t * 8 + 2 * tq] = acc[t][2];
        sm_epi[warp][g + 8][t * 8 + 2 * tq + 1] = acc[t][3];
      }
      __syncwarp();
      stage_exp();
      gemv_epilogue<NT, EPI>(a, stripe, &sm_epi[warp][0][0], COLS + 1, lane, kmax, scl,
                             sm_exp[warp], a.m0, a.M);
      __syncwarp();
    } else {
      // F <= 8 and ns < 8, so a stripe's slot is its index in the CTA
      const int slot = stripe - s0;
      if constexpr (Q4) {
        Acc* part = sm_tile[u];
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          part[g * COLS + t * 8 + 2 * tq] = acc[t][0];
          part[g * COLS + t * 8 + 2 * tq + 1] = acc[t][1];
          part[(g + 8) * COLS + t * 8 + 2 * tq] = acc[t][2];
          part[(g + 8) * COLS + t * 8 + 2 * tq + 1] = acc[t][3];
        }
      } else {
        Acc* tile = sm_tile[slot];
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          atomicAdd(tile + g * COLS + t * 8 + 2 * tq, acc[t][0]);
          atomicAdd(tile + g * COLS + t * 8 + 2 * tq + 1, acc[t][1]);
          atomicAdd(tile + (g + 8) * COLS + t * 8 + 2 * tq, acc[t][2]);
          atomicAdd(tile + (g + 8) * COLS + t * 8 + 2 * tq + 1, acc[t][3]);
        }
      }
      __syncwarp();
      int last = 0;
      if (lane == 0) {
        __threadfence_block();
        last = (atomicAdd(&sm_cnt[slot], n) + n == a.KB);
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last) {
        __threadfence_block();
        if constexpr (Q4) {
          // add the stripe's non-empty partial tiles in k order into this
          // warp's staging (empty k-ranges wrote no tile); which parts are
          // non-empty is settled once, not per element
          unsigned live = 0;
          for (int p = 0; p < F; ++p)
            if (a.KB * (p + 1) / F > a.KB * p / F) live |= 1u << p;
          const Acc* parts = sm_tile[slot * F];
          for (int i = lane; i < 16 * COLS; i += 32) {
            float v = 0.0f;
            for (int p = 0; p < F; ++p)
              if ((live >> p) & 1u) v = __fadd_rn(v, parts[p * 16 * COLS + i]);
            sm_epi[warp][i / COLS][i % COLS] = v;
          }
          __syncwarp();
          stage_exp();
          gemv_epilogue<NT, EPI>(a, stripe, &sm_epi[warp][0][0], COLS + 1, lane, kmax, scl,
                                 sm_exp[warp], a.m0, a.M);
        } else {
          stage_exp();
          gemv_epilogue<NT, EPI>(a, stripe, sm_tile[slot], COLS, lane, kmax, scl, sm_exp[warp],
                                 a.m0, a.M);
        }
      }
      __syncwarp();
    }
  }
  grid_launch_dependents();
  if (!ring_ok && lane == 0 && a.err) atomicExch(a.err, 1);

  if constexpr (EPI == EPI_LMHEAD) {
#pragma unroll
    for (int it = 0; it < (8 * kGroupTokens) / 32; ++it) {
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
      atomicMax(a.keys + key_slot(a.seq, a.m0 + threadIdx.x), sm_keys[threadIdx.x]);
  }
  if constexpr (EPI == EPI_TP) tp_publish(a.tp);
  if constexpr (TAIL) {
    // HBM is idle while the grid meets: warm L2 with upcoming weights
    if (a.enc.pf && threadIdx.x == 0)
      prefetch_share(a.enc.pf, a.enc.pf_bytes, blockIdx.x, gridDim.x);
    __shared__ float t_mul[kMaxTokens];
    __shared__ int t_e[kMaxTokens];
    const int kbs = (a.enc.KB + gridDim.x - 1) / gridDim.x;
    const int kb0 = blockIdx.x * kbs, kb1 = min(a.enc.KB, kb0 + kbs);
    // every epilogue's rows and statistics are out; a CTA without k-blocks to
    // encode only arrives, and leaves its SM to the next kernel
    grid_barrier(a.bar, a.err, kb0 < kb1);
    if (kb0 < kb1) encode_slice_stats_t<1>(a.enc, kb0, kb1, t_mul, t_e, [](int) {});
  }
  MC_TRACE_END(a.trace_slot);
}

template <int NT, int EPI, int WF, bool TAIL = false>
static cudaError_t launch_gemv_t(const GemvArgs& a, int grid, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemvWarps * 32);
  cfg.dynamicSmemBytes = gemv_dyn_smem<NT, WF>();
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_gemv<NT, EPI, WF, TAIL>, a);
}

template <int NT, int WF>
static cudaError_t launch_gemv_nt(const GemvArgs& a, int epi, int grid, cudaStream_t s, bool pdl) {
  switch (epi) {
    case EPI_STORE: return launch_gemv_t<NT, EPI_STORE, WF>(a, grid, s, pdl);
    case EPI_RESID:
      return a.bar ? launch_gemv_t<NT, EPI_RESID, WF, true>(a, grid, s, pdl)
                   : launch_gemv_t<NT, EPI_RESID, WF>(a, grid, s, pdl);
    case EPI_SWIGLU:
      return a.bar ? launch_gemv_t<NT, EPI_SWIGLU, WF, true>(a, grid, s, pdl)
                   : launch_gemv_t<NT, EPI_SWIGLU, WF>(a, grid, s, pdl);
    case EPI_QKV: return launch_gemv_t<NT, EPI_QKV, WF>(a, grid, s, pdl);
    case EPI_LMHEAD: return launch_gemv_t<NT, EPI_LMHEAD, WF>(a, grid, s, pdl);
    case EPI_TP: return launch_gemv_t<NT, EPI_TP, WF>(a, grid, s, pdl);
  }
  return cudaErrorInvalidValue;
}

template <int WF>
static cudaError_t launch_gemv_wf(const GemvArgs& a, int epi, int nt, int grid, cudaStream_t s,
                                  bool pdl) {
  switch (nt) {
    case 1: return launch_gemv_nt<1, WF>(a, epi, grid, s, pdl);
    case 2: return launch_gemv_nt<2, WF>(a, epi, grid, s, pdl);
    case 3: return launch_gemv_nt<3, WF>(a, epi, grid, s, pdl);
    case 6: return launch_gemv_nt<6, WF>(a, epi, grid, s, pdl);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_gemv(const GemvArgs& a, int epi, int nt, int wf, int grid, cudaStream_t s,
                        bool pdl) {
  // one token group per launch: its tiles, exponents and keys are 16 wide
  if (a.M < 1 || a.M > kGroupTokens || 8 * nt < kDigits * a.M || a.m0 < 0 ||
      a.m0 + a.M > kMaxTokens)
    return cudaErrorInvalidValue;
  // the encoding tail: RESID / SWIGLU only, a grid the caller sized to one
  // wave of the tail variant (gemv_blocks_per_sm(..., true)), one group
  if (a.bar && ((epi != EPI_RESID && epi != EPI_SWIGLU) || a.m0 != 0 || a.enc.M != a.M ||
                a.enc.KB < 1 || !a.enc.use_stats || a.enc.att_o))
    return cudaErrorInvalidValue;
  if (wf == WF_Q4) {
    if (!a.qscale) return cudaErrorInvalidValue;
    return launch_gemv_wf<WF_Q4>(a, epi, nt, grid, s, pdl);
  }
  if (wf == WF_I8R) return launch_gemv_wf<WF_I8R>(a, epi, nt, grid, s, pdl);
  return launch_gemv_wf<WF_I8>(a, epi, nt, grid, s, pdl);
}

template <int NT, int EPI, int WF, bool TAIL = false>
static int bps_t() {
  const size_t sm = gemv_dyn_smem<NT, WF>();
  if (sm > 48 * 1024)
    cudaFuncSetAttribute(k_gemv<NT, EPI, WF, TAIL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)sm);
  int n = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_gemv<NT, EPI, WF, TAIL>, kGemvWarps * 32,
                                                sm);
  return n;
}

// Occupancy of a GEMV variant; also raises its dynamic shared-memory limit,
// so it is called once per variant outside any stream capture.
template <int NT, int WF>
static int bps_nt(int epi, bool tail) {
  switch (epi) {
    case EPI_STORE: return bps_t<NT, EPI_STORE, WF>();
    case EPI_RESID: return tail ? bps_t<NT, EPI_RESID, WF, true>() : bps_t<NT, EPI_RESID, WF>();
    case EPI_SWIGLU:
      return tail ? bps_t<NT, EPI_SWIGLU, WF, true>() : bps_t<NT, EPI_SWIGLU, WF>();
    case EPI_QKV: return bps_t<NT, EPI_QKV, WF>();
    case EPI_LMHEAD: return bps_t<NT, EPI_LMHEAD, WF>();
    case EPI_TP: return bps_t<NT, EPI_TP, WF>();
  }
  return 0;
}

template <int WF>
static int bps_wf(int epi, int nt, bool tail) {
  switch (nt) {
    case 1: return bps_nt<1, WF>(epi, tail);
    case 2: return bps_nt<2, WF>(epi, tail);
    case 3: return bps_nt<3, WF>(epi, tail);
    case 6: return bps_nt<6, WF>(epi, tail);
  }
  return 0;
}

int gemv_blocks_per_sm(int epi, int nt, int wf, bool tail) {
  return wf == WF_Q4 ? bps_wf<WF_Q4>(epi, nt, tail)
                     : (wf == WF_I8R ? bps_wf<WF_I8R>(epi, nt, tail)
                                     : bps_wf<WF_I8>(epi, nt, tail));
}

size_t gemv_ws_ints_per_stripe(int nt) { return (size_t)16 * 8 * nt; }


// ------------------------------------------------------------ quantize
// Encodes the next GEMV's B operand.  Every CTA first recomputes, for all M
// tokens, sum(h*h) and max|h*w| over the whole vector (vectorised L2 reads;
// cheap next to a grid-wide reduction), then writes its own slice of the
// packed digit words, one coalesced 4-byte word per thread.  RMSNorm follows
// transformer.rs:888-896 (ms = sum(v*v)/n, rms = sqrt(ms + eps),
// x = v / rms * w).  The exponent makes |x| * 2^e < 2^20 with a one-ulp
// margin (digits tolerate |X| < 2^21).
constexpr int kQuantThreads = 512;
constexpr int kQuantMaxCtas = 64;
// Function attributes (the dynamic shared-memory limits) belong to one
// device's context, so what has been set is kept per device.
constexpr int kMaxDevices = 64;
static int cur_device() {
  int d = 0;
  cudaGetDevice(&d);
  return (d >= 0 && d < kMaxDevices) ? d : 0;
}
static int g_attn_smem[kMaxDevices];  // attention dynamic smem limit set beyond 48 KB, per device
static int attn_smem_limit() { return std::max(g_attn_smem[cur_device()], 48 * 1024); }

// STATS: the producer supplied the statistics (use_stats); otherwise the
// kernel reduces them itself (two instances keep the forward's one lean).
template <bool STATS>
__global__ void __launch_bounds__(kQuantThreads) k_quant(QuantArgs a) {
  __shared__ float red_ss[kStatWarps][kMaxTokens];
  __shared__ float red_hw[kStatWarps][kMaxTokens];
  __shared__ float s_mul[kMaxTokens];
  __shared__ int s_e[kMaxTokens];
  __shared__ uint32_t s_bad[kMaxTokens / kStatTokens];
  extern __shared__ float s_x[];
  MC_TRACE_T0
  if (a.pf && threadIdx.x == 0) prefetch_share(a.pf, a.pf_bytes, blockIdx.x, gridDim.x);
  grid_launch_dependents();
  grid_wait();
  MC_TRACE_WAITED(a.trace_slot);
  MC_TRACE_PHASE(a.trace_slot, 0, mc_tp);
  const StatArgs sa{a.h, a.ld, a.d, a.M, a.w, a.wlen, a.eps, a.do_norm};
  // this CTA's k-blocks
  const int kbs = (a.KB + gridDim.x - 1) / gridDim.x;
  const int kb0 = blockIdx.x * kbs, kb1 = min(a.KB, kb0 + kbs);
  const int lo = kb0 * 32, hi = kb0 * 32 + max(kb1 - kb0, 0) * 32;
  uint32_t* xq = reinterpret_cast<uint32_t*>(a.xq);
  if constexpr (STATS) {
    encode_slice_stats_t(a, kb0, kb1, s_mul, s_e,
                         [&](int k) { MC_TRACE_PHASE(a.trace_slot, k, mc_tp); });
    MC_TRACE_END(a.trace_slot);
    return;
  } else {
  // no producer statistics: reduce over the whole vector here, capturing
  // this CTA's slice in shared memory
  token_stats(sa, red_ss, red_hw, s_bad, s_mul, s_e, s_x, lo, hi);
  if (blockIdx.x == 0 && threadIdx.x < a.M) a.xexp[threadIdx.x] = s_e[threadIdx.x];
  const int span = hi - lo;
  encode_digits(sa, a.nt, a.KB, kb0, kb1, s_mul, s_e,
                [&](int m, int k) {
                  const float* p = s_x + m * span + (k - lo);
                  float4 r;
                  r.x = k < a.d ? p[0] : 0.0f;
                  r.y = k + 1 < a.d ? p[1] : 0.0f;
                  r.z = k + 2 < a.d ? p[2] : 0.0f;
                  r.w = k + 3 < a.d ? p[3] : 0.0f;
                  return r;
                },
                [&](size_t wi, uint32_t v) { xq[wi] = v; }, a.tc_layout != 0);
  MC_TRACE_END(a.trace_slot);
  }
}

// Per-token max |x| (float bits; NaN and inf order above every finite value)
// of un-normalised activations, one CTA per token: the statistics the
// encoder takes from a producer, for standalone projections.
__global__ void __launch_bounds__(256) k_act_amax(const float* __restrict__ x, int ld, int d,
                                                  unsigned* __restrict__ amax) {
  grid_launch_dependents();
  grid_wait();
  const float* row = x + (size_t)blockIdx.x * ld;
  uint32_t mx = 0u;
  const bool vec = ((ld & 3) == 0) && ((d & 3) == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  if (vec) {
    for (int i = threadIdx.x * 4; i < d; i += blockDim.x * 4) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(row + i));
      mx = max(max(mx, __float_as_uint(fabsf(v.x))), __float_as_uint(fabsf(v.y)));
      mx = max(max(mx, __float_as_uint(fabsf(v.z))), __float_as_uint(fabsf(v.w)));
    }
  } else {
    for (int i = threadIdx.x; i < d; i += blockDim.x) mx = max(mx, __float_as_uint(fabsf(__ldcg(row + i))));
  }
  mx = __reduce_max_sync(0xffffffffu, mx);
  __shared__ uint32_t red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t m = 0u;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = max(m, red[w]);
    amax[blockIdx.x] = m;
  }
}

// The O projection's encoder reading the attention's page partials
// (QuantArgs::att_o): attn_combine_encode on this CTA's k-blocks.
__global__ void __launch_bounds__(kQuantThreads) k_quant_att(QuantArgs a) {
  __shared__ float s_mul[kMaxTokens];
  __shared__ int s_e[kMaxTokens];
  __shared__ uint32_t s_bound[kMaxTokens];
  extern __shared__ float s_x[];
  MC_TRACE_T0
  if (a.pf && threadIdx.x == 0) prefetch_share(a.pf, a.pf_bytes, blockIdx.x, gridDim.x);
  grid_launch_dependents();
  grid_wait();
  MC_TRACE_WAITED(a.trace_slot);
  const int kbs = (a.KB + gridDim.x - 1) / gridDim.x;
  const int kb0 = blockIdx.x * kbs, kb1 = min(a.KB, kb0 + kbs);
  const int lo = kb0 * 32, hi = kb0 * 32 + max(kb1 - kb0, 0) * 32;
  attn_combine_encode<2, kEncBatch>(a, lo, hi, kb0, kb1, blockIdx.x == 0, s_bound, s_mul, s_e,
                                    s_x, reinterpret_cast<uint32_t*>(a.xq));
  MC_TRACE_END(a.trace_slot);
}

cudaError_t launch_act_amax(const float* x, int ld, int d, int M, unsigned* amax, cudaStream_t s,
                            bool pdl) {
  if (M < 1 || M > kMaxTokens) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_act_amax, x, ld, d, amax);
}

cudaError_t launch_quant(const QuantArgs& a, cudaStream_t s, bool pdl) {
  if (a.M < 1 || a.M > kMaxTokens) return cudaErrorInvalidValue;
  if (a.nt != nt_for_tokens(a.M)) return cudaErrorInvalidValue;
  const int words = a.KB * 32 * 2 * a.nt * groups_for_tokens(a.M);
  int ctas = (words + kQuantThreads - 1) / kQuantThreads;
  ctas = ctas < 1 ? 1 : (ctas > kQuantMaxCtas ? kQuantMaxCtas : ctas);
  // staged slice <= 32 KB: with the 8.8 KB of static statistics arrays it
  // stays under the 48 KB default shared-memory limit
  const int kbs_fit = (32 * 1024) / (a.M * 32 * (int)sizeof(float));
  if (kbs_fit < 1) return cudaErrorInvalidConfiguration;
  const int need = (a.KB + kbs_fit - 1) / kbs_fit;
  ctas = ctas < need ? need : ctas;
  if (a.att_o) {
    // the page combine: kCombLanes lanes per 4 outputs of a token, the CTA's
    // threads covering its k-blocks in one pass where the grid allows
    const int lanes_per_kb = kCombLanes * 8 * a.M;
    const int kb_per_cta = std::max(1, kQuantThreads / lanes_per_kb);
    ctas = std::max(ctas, std::min((a.KB + kb_per_cta - 1) / kb_per_cta, 4 * kQuantMaxCtas));
  }
  ctas = ctas > a.KB ? a.KB : ctas;
  const int kbs = (a.KB + ctas - 1) / ctas;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(kQuantThreads);
  cfg.dynamicSmemBytes =
      (a.use_stats && !a.att_o) ? 0 : (size_t)a.M * kbs * 32 * sizeof(float);
  if (a.att_o && (!a.use_stats || a.att_hdp < 4 || (a.att_hdp & 3) || a.att_chunks > 64 ||
                  a.att_G < 1 || a.att_qblk < 1))
    return cudaErrorInvalidValue;
  if (cfg.dynamicSmemBytes > 40 * 1024) return cudaErrorInvalidConfiguration;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (a.att_o) return cudaLaunchKernelEx(&cfg, k_quant_att, a);
  return a.use_stats ? cudaLaunchKernelEx(&cfg, k_quant<true>, a)
                     : cudaLaunchKernelEx(&cfg, k_quant<false>, a);
}

// ------------------------------------------------------------ attention
// One CTA per (KV head, KV page of 64 positions, query block).  A query
// block is up to qblk consecutive new tokens of one sequence (sequence z =
// block / blocks per sequence); its query rows are the G query heads sharing
// the KV head times those tokens, and token i of the sequence sees positions
// <= pos_z + i.  Scores are dot / sqrt(head_dim) (transformer.rs:959-966);
// the softmax subtracts the row max (transformer.rs:985-1000).  Each CTA
// writes its page's partials (flash-decoding split); the O projection's
// encoder combines them (k_quant_att, or the tensor-core kernel's tail).
constexpr int kAttnThreads = 512;

// The page partials are combined by the O projection's encoder (k_quant
// reading AttnArgs' partials), which needs each token's max |output| for its
// exponent before it has the output.  The output of a (token, head) is a
// convex combination of the pages' normalised partials o_p / l_p (weights
// e^(m_p - M) l_p / sum), so max over pages and heads of |o_p| / l_p bounds
// it; a CTA folds its page's share of that bound into st_amax[token].
// page_bound: this thread's |o_p| value of query row `row`, into s_mx.
__device__ __forceinline__ void page_bound(uint32_t* s_mx, const float* s_l, int row, int G,
                                           float abs_o) {
  const float l = s_l[row];
  if (!(l > 0.0f)) return;  // no visible position on this page: no share
  // as float bits (|x| only, so their unsigned order is |x|'s; NaN wins)
  atomicMax(s_mx + row / G, __float_as_uint(fabsf(__fdiv_rn(abs_o, l))));
}
// s_mx (zeroed before the partials) complete: fold it into st_amax.
__device__ __forceinline__ void publish_bound(const AttnArgs& a, const uint32_t* s_mx, int mt0,
                                              int Mq) {
  if (a.st_amax)
    for (int i = threadIdx.x; i < Mq; i += blockDim.x)
      if (s_mx[i]) atomicMax(a.st_amax + mt0 + i, s_mx[i]);
}

// 16-byte global -> shared copy that holds no registers (L2 only, as __ldcg).
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(smem_dst)),
               "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// Wait until at most N of this thread's committed copy groups are pending.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// RB: query rows per thread (all of them valid: R is a multiple of the
// number of row groups in both passes, checked by the launcher).  MINB: CTAs
// per SM the registers are sized for -- 2 for grids of several waves with
// few rows per CTA (the verify of a batch of requests), else 1.
template <int RB, int MINB>
__global__ void __launch_bounds__(kAttnThreads, MINB) k_attention(AttnArgs a) {
  MC_TRACE_T0
  extern __shared__ float smem[];
  __shared__ float s_m[128], s_l[128];
  __shared__ uint32_t s_mx[64];  // page share of each token's output bound (float bits)
  if (threadIdx.x < 64) s_mx[threadIdx.x] = 0u;
  if (a.pf && threadIdx.x == 0)
    prefetch_share(a.pf, a.pf_bytes, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
  grid_launch_dependents();
  grid_wait();
  MC_TRACE_WAITED(a.trace_slot);
  MC_TRACE_PHASE(a.trace_slot, 0, mc_tp);
  const int kvh = blockIdx.x, chunk = blockIdx.y, zb = blockIdx.z;
  const int G = a.H / a.Hkv;
  const int n_qb = (a.seq.seq_len + a.qblk - 1) / a.qblk;
  const int z = zb / n_qb, i0 = (zb - z * n_qb) * a.qblk;
  const int Mq = min(a.qblk, a.seq.seq_len - i0);  // tokens of this block
  const int mt0 = z * a.seq.seq_len + i0;           // forward-wide first token
  const int R = G * Mq;
  const int Rs = G * a.qblk;                        // row stride of the partials
  const int hdp = a.hdp, P = a.page;
  // rows padded with zero queries to a multiple of both passes' row groups
  // (from the block capacity, as the launcher chose RB)
  const int rgmax = max(kAttnThreads / P, kAttnThreads / hdp);
  const int Rp = (Rs + rgmax - 1) / rgmax * rgmax;
  const int pos0 = a.pos_ptr[z * a.seq.pos_stride] + a.pos_add + i0;
  const int L = pos0 + Mq;
  const int n_chunks = (L + P - 1) / P;
  const int cslot = zb * a.Hkv + kvh;  // (query block, KV head)
  if (chunk >= n_chunks) {
    MC_TRACE_END(a.trace_slot);
    return;
  }
  const int t0 = chunk * P;
  const int nt = min(P, L - t0);
  const int ks = hdp + 4;  // K row stride: float4-aligned, conflict-free float4 reads
  float* sq = smem;                    // [Rp][hdp]
  float* sk = sq + (size_t)Rp * hdp;   // [P][hdp+4]
  float* sv = sk + (size_t)P * ks;     // [P][hdp]
  float* ss = sv + (size_t)P * hdp;    // [Rp][P]

  const int pg = a.page_table[z * a.seq.pt_stride + chunk];
  const float4* kbase = reinterpret_cast<const float4*>(a.kc + ((size_t)pg * a.Hkv + kvh) * P * hdp);
  const float4* vbase = reinterpret_cast<const float4*>(a.vc + ((size_t)pg * a.Hkv + kvh) * P * hdp);
  const int h4 = hdp >> 2;
  // K/V copies go straight to shared memory (cp.async, no registers held);
  // the q loads follow while they are in flight
  {
    const int n4 = nt * h4;
    for (int i = threadIdx.x; i < n4; i += kAttnThreads) {
      const int t = i / h4, c4 = i - t * h4;
      cp_async16(sk + (size_t)t * ks + 4 * c4, kbase + i);
      cp_async16(reinterpret_cast<float4*>(sv) + i, vbase + i);
    }
    // q: four loads in flight per batch (the K/V loads above are already out)
    for (int i0 = threadIdx.x; i0 < Rp * h4; i0 += 4 * kAttnThreads) {
      float4 qr[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * kAttnThreads;
        qr[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (i < R * h4) {
          const int row = i / h4, c4 = i - row * h4;
          const int m = row / G, gi = row - m * G;
          qr[u] = __ldcg(reinterpret_cast<const float4*>(a.q + ((size_t)(mt0 + m) * a.H + kvh * G + gi) * hdp) + c4);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * kAttnThreads;
        if (i < Rp * h4) reinterpret_cast<float4*>(sq)[i] = qr[u];
      }
    }
    // the P.V pass steps 4 positions at a time: zero V rows past the last
    // position (their probabilities are 0, and 0 * stale data could be NaN)
    const int ntr = (nt + 3) & ~3;
    for (int i = nt * h4 + threadIdx.x; i < ntr * h4; i += blockDim.x)
      reinterpret_cast<float4*>(sv)[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    cp_async_wait_all();
  }
  __syncthreads();
  MC_TRACE_PHASE(a.trace_slot, 1, mc_tp);
  // scores: thread -> position t and rows rq, rq+RG, ... (RB of them)
  {
    const int t = threadIdx.x % P;
    const int RG = kAttnThreads / P;  // row groups
    for (int rq = threadIdx.x / P; rq < Rp; rq += RG * RB) {
      float acc[RB];
#pragma unroll
      for (int j = 0; j < RB; ++j) acc[j] = 0.0f;
      if (t < nt) {
        const float* kr = sk + (size_t)t * ks;
        for (int c = 0; c < hdp; c += 4) {
          const float4 kv = *reinterpret_cast<const float4*>(kr + c);
#pragma unroll
          for (int j = 0; j < RB; ++j) {
            const float4 qv = *reinterpret_cast<const float4*>(sq + (rq + j * RG) * hdp + c);
            acc[j] = __fmaf_rn(qv.x, kv.x, acc[j]);
            acc[j] = __fmaf_rn(qv.y, kv.y, acc[j]);
            acc[j] = __fmaf_rn(qv.z, kv.z, acc[j]);
            acc[j] = __fmaf_rn(qv.w, kv.w, acc[j]);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < RB; ++j) {
        const int row = rq + j * RG;
        const int m = min(row, R - 1) / G;
        ss[row * P + t] = (t < nt && t0 + t <= pos0 + m) ? __fdiv_rn(acc[j], a.inv_scale_den)
                                                          : -INFINITY;
      }
    }
  }
  __syncthreads();
  MC_TRACE_PHASE(a.trace_slot, 2, mc_tp);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int row = warp; row < Rp; row += blockDim.x >> 5) {
    float mx = -INFINITY;
    for (int t = lane; t < P; t += 32) mx = fmaxf(mx, ss[row * P + t]);
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    for (int t = lane; t < P; t += 32) {
      const float sc = ss[row * P + t];
      const float p = (sc == -INFINITY) ? 0.0f : expf(sc - mx);
      ss[row * P + t] = p;
      sum += p;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) { s_m[row] = mx; s_l[row] = sum; }
  }
  __syncthreads();
  MC_TRACE_PHASE(a.trace_slot, 3, mc_tp);
  // P.V: thread -> column c and rows rq, rq+RG, ... ; four positions per step
  const size_t pbase = ((size_t)cslot * a.max_chunks + chunk) * Rs;
  {
    const int c = threadIdx.x % hdp;
    const int RG = kAttnThreads / hdp;
    for (int rq = threadIdx.x / hdp; rq < Rp; rq += RG * RB) {
      float acc[RB];
#pragma unroll
      for (int j = 0; j < RB; ++j) acc[j] = 0.0f;
      for (int t = 0; t < nt; t += 4) {  // nt < P only on the last page: p == 0 there
        const float v0 = sv[(t + 0) * hdp + c], v1 = sv[(t + 1) * hdp + c];
        const float v2 = sv[(t + 2) * hdp + c], v3 = sv[(t + 3) * hdp + c];
#pragma unroll
        for (int j = 0; j < RB; ++j) {
          const float4 p = *reinterpret_cast<const float4*>(ss + (rq + j * RG) * P + t);
          acc[j] = __fmaf_rn(p.x, v0, acc[j]);
          acc[j] = __fmaf_rn(p.y, v1, acc[j]);
          acc[j] = __fmaf_rn(p.z, v2, acc[j]);
          acc[j] = __fmaf_rn(p.w, v3, acc[j]);
        }
      }
#pragma unroll
      for (int j = 0; j < RB; ++j)
        if (rq + j * RG < R) {
          a.part_o[(pbase + rq + j * RG) * hdp + c] = acc[j];
          page_bound(s_mx, s_l, rq + j * RG, G, fabsf(acc[j]));
        }
    }
  }
  for (int row = threadIdx.x; row < R; row += blockDim.x) {
    a.part_ml[(pbase + row) * 2] = s_m[row];
    a.part_ml[(pbase + row) * 2 + 1] = s_l[row];
  }
  __syncthreads();
  publish_bound(a, s_mx, mt0, Mq);
  MC_TRACE_PHASE(a.trace_slot, 4, mc_tp);
  MC_TRACE_END(a.trace_slot);
}

// ------------------------------------------------------------ attention on the tensor cores
// The same split as k_attention (one CTA per (KV head, page, query block)),
// for up to 64 query rows and head dims of 32, 64 or 128: q.K^T and P.V on
// mma.sync m16n8k8 TF32 with each f32 operand split into a TF32 high part
// and a TF32 remainder (hi*hi + hi*lo + lo*hi: f32-level products).  Eight
// warps run the MMAs -- one 8-position n-tile of scores each, then the head
// dimension for P.V -- and all 16 warps stage K/V/q and run the combine; the
// softmax reduces rows over quads (shuffles) and warps (shared).  Partials
// (m, l, o) and the last-arriver combine are those of k_attention.
constexpr int kAttnTcThreads = 512;
constexpr int kAttnTcMmaWarps = 8;

__device__ __forceinline__ void tf32_split(float x, uint32_t& hi, uint32_t& lo) {
  uint32_t h, l;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
  const float r = x - __uint_as_float(h);
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(l) : "f"(r));
  hi = h;
  lo = l;
}
__device__ __forceinline__ void mma_tf32(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
// d += a * b with a = ah + al, b = bh + bl (the al*bl term dropped)
__device__ __forceinline__ void mma_3xtf32(float* d, const uint32_t* ah, const uint32_t* al,
                                           const uint32_t* bh, const uint32_t* bl) {
  mma_tf32(d, al, bh);
  mma_tf32(d, ah, bl);
  mma_tf32(d, ah, bh);
}

// The attention's encoding tail (AttnArgs::bar): the grid meets once every
// CTA's partials and bound are out, then each CTA combines and encodes its
// slice of the O projection's k-blocks (k-blocks split over the linear
// block index) in `smem`, as k_quant_att does.
__device__ __forceinline__ void attn_tail(const AttnArgs& a, float* smem) {
  __shared__ uint32_t t_bound[kMaxTokens];
  __shared__ float t_mul[kMaxTokens];
  __shared__ int t_e[kMaxTokens];
  grid_barrier(a.bar, a.err);
  const int nb = gridDim.x * gridDim.y * gridDim.z;
  const int b = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
  const int kbs = (a.enc.KB + nb - 1) / nb;
  const int kb0 = b * kbs, kb1 = min(a.enc.KB, kb0 + kbs);
  if (kb0 < kb1)
    attn_combine_encode<2, 2>(a.enc, kb0 * 32, kb1 * 32, kb0, kb1, b == 0, t_bound, t_mul, t_e,
                              smem, reinterpret_cast<uint32_t*>(a.enc.xq));
}

// MT: 16-row m-tiles (query rows <= 16 MT); HD: head dim (hdp); TAIL: the
// encoding tail (MT == 1 only)
template <int MT, int HD, bool TAIL = false>
__global__ void __launch_bounds__(kAttnTcThreads, MT == 1 ? 2 : 1) k_attention_tc(AttnArgs a) {
  constexpr int P = 64;
  constexpr int KS = HD + 4;   // K / q row stride: conflict-free fragment loads
  constexpr int VS = HD + 8;   // V row stride (B fragments walk positions)
  constexpr int PS = P + 4;    // P row stride
  constexpr int RM = 16 * MT;  // padded query rows
  constexpr int NW = kAttnTcMmaWarps;
  constexpr int PV_WARPS = HD / 8 < NW ? HD / 8 : NW;  // warps with P.V columns
  constexpr int NT_PV = HD / (8 * PV_WARPS);           // 8-column n-tiles each
  MC_TRACE_T0
  extern __shared__ __align__(16) float asmem[];
  float* sK = asmem;               // [64][KS]
  float* sV = sK + P * KS;         // [64][VS]
  float* sQ = sV + P * VS;         // [RM][KS] q, then its TF32 high parts
  float* sQl = sQ + RM * KS;       // [RM][KS] TF32 remainders of q
  float* sP = sQl + RM * KS;       // [RM][PS]
  __shared__ float s_red[NW][RM];
  __shared__ float s_m[RM], s_l[RM];
  __shared__ uint32_t s_mx[64];  // page share of each token's output bound (float bits)
  if (threadIdx.x < 64) s_mx[threadIdx.x] = 0u;
  if (a.pf && threadIdx.x == 0)
    prefetch_share(a.pf, a.pf_bytes, (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x,
                   gridDim.x * gridDim.y * gridDim.z);
  const int kvh = blockIdx.x, chunk = blockIdx.y, zb = blockIdx.z;
  const int G = a.H / a.Hkv;
  const int n_qb = (a.seq.seq_len + a.qblk - 1) / a.qblk;
  const int z = zb / n_qb, i0 = (zb - z * n_qb) * a.qblk;
  // A page wholly below the sequence's first new position holds final K/V
  // when kv_pre is set: its copies start before the wait and overlap the
  // producer's tail (the two copy groups, K then V, as below).
  bool early = false;
  if (a.kv_pre) {
    const int base = a.pos_ptr[z * a.seq.pos_stride] + a.pos_add;
    if ((chunk + 1) * P <= base) {
      const int pg = a.page_table[z * a.seq.pt_stride + chunk];
      const float4* kb4 = reinterpret_cast<const float4*>(a.kc + ((size_t)pg * a.Hkv + kvh) * P * HD);
      const float4* vb4 = reinterpret_cast<const float4*>(a.vc + ((size_t)pg * a.Hkv + kvh) * P * HD);
      constexpr int H4 = HD / 4;
      for (int i = threadIdx.x; i < P * H4; i += kAttnTcThreads) {
        const int t = i / H4, c4 = i - t * H4;
        cp_async16(sK + t * KS + 4 * c4, kb4 + i);
      }
      cp_async_commit();
      for (int i = threadIdx.x; i < P * H4; i += kAttnTcThreads) {
        const int t = i / H4, c4 = i - t * H4;
        cp_async16(sV + t * VS + 4 * c4, vb4 + i);
      }
      cp_async_commit();
      early = true;
    }
  }
  grid_launch_dependents();
  grid_wait();
  MC_TRACE_WAITED(a.trace_slot);
  MC_TRACE_PHASE(a.trace_slot, 0, mc_tp);
  const int Mq = min(a.qblk, a.seq.seq_len - i0);
  const int mt0 = z * a.seq.seq_len + i0;
  const int R = G * Mq;
  const int Rs = G * a.qblk;
  const int pos0 = a.pos_ptr[z * a.seq.pos_stride] + a.pos_add + i0;
  const int L = pos0 + Mq;
  const int n_chunks = (L + P - 1) / P;
  const int cslot = zb * a.Hkv + kvh;
  if (chunk >= n_chunks) {
    if constexpr (TAIL) attn_tail(a, asmem);
    MC_TRACE_END(a.trace_slot);
    return;
  }
  const int t0 = chunk * P;
  const int nt = min(P, L - t0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  {
    constexpr int H4 = HD / 4;
    if (!early) {
      const int pg = a.page_table[z * a.seq.pt_stride + chunk];
      const float4* kbase = reinterpret_cast<const float4*>(a.kc + ((size_t)pg * a.Hkv + kvh) * P * HD);
      const float4* vbase = reinterpret_cast<const float4*>(a.vc + ((size_t)pg * a.Hkv + kvh) * P * HD);
      // two copy groups: K (needed by the scores) then V (needed after the
      // softmax), so the V copies land while the scores are computed
      for (int i = threadIdx.x; i < nt * H4; i += kAttnTcThreads) {
        const int t = i / H4, c4 = i - t * H4;
        cp_async16(sK + t * KS + 4 * c4, kbase + i);
      }
      cp_async_commit();
      for (int i = threadIdx.x; i < nt * H4; i += kAttnTcThreads) {
        const int t = i / H4, c4 = i - t * H4;
        cp_async16(sV + t * VS + 4 * c4, vbase + i);
      }
      cp_async_commit();
    }
    // rows past the page's last position: zero K and V (probability 0 times
    // stale data could be NaN); their scores are masked
    for (int i = nt * H4 + threadIdx.x; i < P * H4; i += kAttnTcThreads) {
      const int t = i / H4, c4 = i - t * H4;
      *reinterpret_cast<float4*>(sV + t * VS + 4 * c4) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      *reinterpret_cast<float4*>(sK + t * KS + 4 * c4) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    for (int i = threadIdx.x; i < RM * H4; i += kAttnTcThreads) {
      const int row = i / H4, c4 = i - row * H4;
      float4 q = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (row < R) {
        const int m = row / G, gi = row - m * G;
        q = __ldcg(reinterpret_cast<const float4*>(a.q + ((size_t)(mt0 + m) * a.H + kvh * G + gi) * HD) + c4);
      }
      *reinterpret_cast<float4*>(sQ + row * KS + 4 * c4) = q;
    }
  }
  __syncthreads();  // q in shared memory (its own loads; cp.async still in flight)
  // q split once for all MMA warps: TF32 high part in place, remainder aside
  for (int i = threadIdx.x; i < RM * HD; i += kAttnTcThreads) {
    const int row = i / HD, c = i - row * HD;
    uint32_t h, l;
    tf32_split(sQ[row * KS + c], h, l);
    sQ[row * KS + c] = __uint_as_float(h);
    sQl[row * KS + c] = __uint_as_float(l);
  }
  cp_async_wait_group<1>();  // K landed (V may still be in flight)
  __syncthreads();
  MC_TRACE_PHASE(a.trace_slot, 1, mc_tp);
  // scores: MMA warp w -> positions 8 w .. 8 w + 7 (one n-tile) of every row;
  // the three products (lo*hi, hi*lo, hi*hi) accumulate separately (shorter
  // dependent MMA chains) and are added small terms first
  const bool mma_warp = warp < NW;
  float sc[MT][4];
#pragma unroll
  for (int mi = 0; mi < MT; ++mi)
#pragma unroll
    for (int e = 0; e < 4; ++e) sc[mi][e] = 0.0f;
  if (mma_warp) {
    float s_lh[MT][4], s_hl[MT][4];
#pragma unroll
    for (int mi = 0; mi < MT; ++mi)
#pragma unroll
      for (int e = 0; e < 4; ++e) s_lh[mi][e] = s_hl[mi][e] = 0.0f;
#pragma unroll 4
    for (int kk = 0; kk < HD / 8; ++kk) {
      uint32_t bh[2], bl[2];
      const float* kr = sK + (8 * warp + g) * KS + 8 * kk;
      tf32_split(kr[tq], bh[0], bl[0]);
      tf32_split(kr[tq + 4], bh[1], bl[1]);
#pragma unroll
      for (int mi = 0; mi < MT; ++mi) {
        const int o0 = (16 * mi + g) * KS + 8 * kk, o1 = o0 + 8 * KS;
        const uint32_t ah[4] = {__float_as_uint(sQ[o0 + tq]), __float_as_uint(sQ[o1 + tq]),
                                __float_as_uint(sQ[o0 + tq + 4]), __float_as_uint(sQ[o1 + tq + 4])};
        const uint32_t al[4] = {__float_as_uint(sQl[o0 + tq]), __float_as_uint(sQl[o1 + tq]),
                                __float_as_uint(sQl[o0 + tq + 4]), __float_as_uint(sQl[o1 + tq + 4])};
        mma_tf32(s_lh[mi], al, bh);
        mma_tf32(s_hl[mi], ah, bl);
        mma_tf32(sc[mi], ah, bh);
      }
    }
#pragma unroll
    for (int mi = 0; mi < MT; ++mi)
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[mi][e] = (s_lh[mi][e] + s_hl[mi][e]) + sc[mi][e];
    // scale (a division, transformer.rs:966), mask, and the row maxima
#pragma unroll
    for (int mi = 0; mi < MT; ++mi)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = 16 * mi + g + 8 * h;
        const int m = min(row, max(R - 1, 0)) / G;
        float mx = -INFINITY;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int t = 8 * warp + 2 * tq + e;
          float v = __fdiv_rn(sc[mi][2 * h + e], a.inv_scale_den);
          if (row >= R || t >= nt || t0 + t > pos0 + m) v = -INFINITY;
          sc[mi][2 * h + e] = v;
          mx = fmaxf(mx, v);
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        if (tq == 0) s_red[warp][row] = mx;
      }
  }
  __syncthreads();
  if (threadIdx.x < RM) {
    float mx = s_red[0][threadIdx.x];
#pragma unroll
    for (int w = 1; w < NW; ++w) mx = fmaxf(mx, s_red[w][threadIdx.x]);
    s_m[threadIdx.x] = mx;
  }
  __syncthreads();
  // probabilities e^(s - max) into sP, and the row sums
  if (mma_warp) {
#pragma unroll
    for (int mi = 0; mi < MT; ++mi)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = 16 * mi + g + 8 * h;
        const float M_ = s_m[row];
        float sum = 0.0f;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float v = sc[mi][2 * h + e];
          const float p = (v == -INFINITY) ? 0.0f : expf(v - M_);
          sP[row * PS + 8 * warp + 2 * tq + e] = p;
          sum += p;
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if (tq == 0) s_red[warp][row] = sum;
      }
  }
  cp_async_wait_group<0>();  // V landed; the barrier publishes it with sP
  __syncthreads();
  if (threadIdx.x < RM) {
    float l = s_red[0][threadIdx.x];
#pragma unroll
    for (int w = 1; w < NW; ++w) l += s_red[w][threadIdx.x];
    s_l[threadIdx.x] = l;
  }
  MC_TRACE_PHASE(a.trace_slot, 2, mc_tp);
  // P.V: warp w < PV_WARPS -> head-dim columns 8 NT_PV w .. 8 NT_PV (w + 1)
  float acc[MT][NT_PV][4];
#pragma unroll
  for (int mi = 0; mi < MT; ++mi)
#pragma unroll
    for (int nj = 0; nj < NT_PV; ++nj)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[mi][nj][e] = 0.0f;
  const int c0 = warp * 8 * NT_PV;
  if (warp < PV_WARPS) {
#pragma unroll 2
    for (int kk = 0; kk < P / 8; ++kk) {
      uint32_t bh[NT_PV][2], bl[NT_PV][2];
#pragma unroll
      for (int nj = 0; nj < NT_PV; ++nj) {
        const float* v0 = sV + (8 * kk + tq) * VS + c0 + 8 * nj + g;
        tf32_split(v0[0], bh[nj][0], bl[nj][0]);
        tf32_split(v0[4 * VS], bh[nj][1], bl[nj][1]);
      }
#pragma unroll
      for (int mi = 0; mi < MT; ++mi) {
        uint32_t ah[4], al[4];
        const float* p0 = sP + (16 * mi + g) * PS + 8 * kk;
        const float* p1 = p0 + 8 * PS;
        tf32_split(p0[tq], ah[0], al[0]);
        tf32_split(p1[tq], ah[1], al[1]);
        tf32_split(p0[tq + 4], ah[2], al[2]);
        tf32_split(p1[tq + 4], ah[3], al[3]);
#pragma unroll
        for (int nj = 0; nj < NT_PV; ++nj) mma_3xtf32(acc[mi][nj], ah, al, bh[nj], bl[nj]);
      }
    }
  }
  MC_TRACE_PHASE(a.trace_slot, 3, mc_tp);
  const size_t pbase = ((size_t)cslot * a.max_chunks + chunk) * Rs;
  __syncthreads();  // s_l complete
  if (warp < PV_WARPS)
#pragma unroll
    for (int mi = 0; mi < MT; ++mi)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = 16 * mi + g + 8 * h;
        if (row < R) {
          uint32_t mx = 0u;  // max |o| as float bits: NaN and inf win
#pragma unroll
          for (int nj = 0; nj < NT_PV; ++nj) {
            *reinterpret_cast<float2*>(a.part_o + (pbase + row) * HD + c0 + 8 * nj + 2 * tq) =
                make_float2(acc[mi][nj][2 * h], acc[mi][nj][2 * h + 1]);
            mx = max(mx, max(__float_as_uint(fabsf(acc[mi][nj][2 * h])),
                             __float_as_uint(fabsf(acc[mi][nj][2 * h + 1]))));
          }
          page_bound(s_mx, s_l, row, G, __uint_as_float(mx));
        }
      }
  for (int row = threadIdx.x; row < R; row += kAttnTcThreads) {
    a.part_ml[(pbase + row) * 2] = s_m[row];
    a.part_ml[(pbase + row) * 2 + 1] = s_l[row];
  }
  __syncthreads();
  publish_bound(a, s_mx, mt0, Mq);
  MC_TRACE_PHASE(a.trace_slot, 4, mc_tp);
  if constexpr (TAIL) attn_tail(a, asmem);
  MC_TRACE_END(a.trace_slot);
}

size_t attention_tc_smem_bytes(int mt, int hd) {
  return ((size_t)64 * (hd + 4) + (size_t)64 * (hd + 8) + (size_t)2 * 16 * mt * (hd + 4) +
          (size_t)16 * mt * 68) * sizeof(float);
}

size_t attention_smem_bytes(int G, int qblk, int hdp, int page) {
  const int rgmax = std::max(kAttnThreads / page, kAttnThreads / hdp);
  const size_t R = (size_t)((G * qblk + rgmax - 1) / rgmax * rgmax);
  return (R * hdp + (size_t)page * (hdp + 4) + (size_t)page * hdp + R * page) * sizeof(float);
}

// Rows per thread for both passes: the score pass has threads/P row groups
// and the P.V pass threads/hdp; RB must divide R / groups in both.
static int attention_rb(int R, int hdp, int page) {
  const int g1 = kAttnThreads / page, g2 = kAttnThreads / hdp;
  for (int rb : {8, 4, 2, 1})
    if (R % (g1 * rb) == 0 && R % (g2 * rb) == 0) return rb;
  return 0;
}

// Tokens of one sequence per attention CTA: query rows G * qblk <= 64 (the
// tensor-core kernel's limit, for every forward of a model alike).
int attention_qblk(int G, int seq_len) {
  const int cap = std::max(1, 64 / std::max(G, 1));
  return std::max(1, std::min(seq_len, cap));
}

// tensor-core attention dynamic smem limit set beyond 48 KB, per device
static int g_attn_tc_smem[kMaxDevices];
static int attn_tc_smem_limit() { return std::max(g_attn_tc_smem[cur_device()], 48 * 1024); }

template <int MT, int HD, bool TAIL = false>
static cudaError_t launch_attention_tc(const AttnArgs& a, dim3 grid, cudaStream_t s, bool pdl) {
  const size_t smem = attention_tc_smem_bytes(MT, HD);
  if (smem > (size_t)attn_tc_smem_limit()) return cudaErrorInvalidConfiguration;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kAttnTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_attention_tc<MT, HD, TAIL>, a);
}

template <int HD>
static cudaError_t launch_attention_tc_hd(const AttnArgs& a, int R, dim3 grid, cudaStream_t s,
                                          bool pdl) {
  if (a.bar) {  // the caller checked attention_tail_fits
    if (R > 16) return cudaErrorInvalidValue;
    return launch_attention_tc<1, HD, true>(a, grid, s, pdl);
  }
  if (R <= 16) return launch_attention_tc<1, HD>(a, grid, s, pdl);
  if (R <= 32) return launch_attention_tc<2, HD>(a, grid, s, pdl);
  return launch_attention_tc<4, HD>(a, grid, s, pdl);
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl) {
  const int G = a.H / a.Hkv;
  if (a.seq.seq_len < 1 || a.qblk < 1 || a.qblk > a.seq.seq_len || a.M % a.seq.seq_len)
    return cudaErrorInvalidValue;
  const int n_seq = a.M / a.seq.seq_len;
  const int n_qb = (a.seq.seq_len + a.qblk - 1) / a.qblk;
  if (a.bar && !attention_tail_fits(a, 0)) return cudaErrorInvalidValue;
  // tensor-core kernel: up to 64 query rows per block, head dims 32 / 64 / 128
  // (the block size depends only on the model, so every forward of a model
  // takes the same kernel)
  if (a.page == 64 && a.max_chunks <= 64 && G * a.qblk <= 64 &&
      (a.hdp == 32 || a.hdp == 64 || a.hdp == 128)) {
    const dim3 grid(a.Hkv, a.max_chunks, n_seq * n_qb);
    switch (a.hdp) {
      case 32: return launch_attention_tc_hd<32>(a, G * a.qblk, grid, s, pdl);
      case 64: return launch_attention_tc_hd<64>(a, G * a.qblk, grid, s, pdl);
      default: return launch_attention_tc_hd<128>(a, G * a.qblk, grid, s, pdl);
    }
  }
  const int R = G * a.qblk;
  // the combine's page weights [R][n_chunks] reuse the score tile [Rp][page]
  if (a.page != 64 || a.max_chunks > a.page || a.hdp > 128 || (a.hdp & 3) ||
      (kAttnThreads % a.hdp))
    return cudaErrorInvalidValue;
  const int rgmax = std::max(kAttnThreads / a.page, kAttnThreads / a.hdp);
  const int Rp = (R + rgmax - 1) / rgmax * rgmax;
  if (Rp > 128) return cudaErrorInvalidValue;
  const int rb = attention_rb(Rp, a.hdp, a.page);
  if (rb == 0) return cudaErrorInvalidValue;
  const size_t smem = attention_smem_bytes(G, a.qblk, a.hdp, a.page);
  if (smem > (size_t)attn_smem_limit()) return cudaErrorInvalidConfiguration;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.Hkv, a.max_chunks, n_seq * n_qb);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static int nsm = 0;
  if (!nsm) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    nsm = nsm > 0 ? nsm : 148;
  }
  const bool two = rb <= 2 && (long long)a.Hkv * a.max_chunks * n_seq * n_qb > 2LL * nsm;
  switch (rb) {
    case 8: return cudaLaunchKernelEx(&cfg, k_attention<8, 1>, a);
    case 4: return cudaLaunchKernelEx(&cfg, k_attention<4, 1>, a);
    case 2: return two ? cudaLaunchKernelEx(&cfg, k_attention<2, 2>, a)
                       : cudaLaunchKernelEx(&cfg, k_attention<2, 1>, a);
    default: return two ? cudaLaunchKernelEx(&cfg, k_attention<1, 2>, a)
                        : cudaLaunchKernelEx(&cfg, k_attention<1, 1>, a);
  }
}

// Raise the dynamic shared-memory limit once, outside any stream capture.
// CTAs of the tail variant k_attention_tc<1, HD, true> resident per SM
// (index 0/1/2: HD 32/64/128) on each device, settled by prepare_kernels.
static int g_attn_tail_bps[kMaxDevices][3];

template <int HD>
static cudaError_t prepare_attention_tc_hd() {
  for (auto f : {k_attention_tc<1, HD>, k_attention_tc<2, HD>, k_attention_tc<4, HD>,
                 k_attention_tc<1, HD, true>}) {
    cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)attention_tc_smem_bytes(4, 128));
    if (e != cudaSuccess) return e;
  }
  int n = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
      &n, k_attention_tc<1, HD, true>, kAttnTcThreads, attention_tc_smem_bytes(1, HD));
  if (e != cudaSuccess) return e;
  g_attn_tail_bps[cur_device()][HD == 32 ? 0 : (HD == 64 ? 1 : 2)] = n;
  return cudaSuccess;
}

bool attention_tail_fits(const AttnArgs& a, int nsm) {
  static int n_sm = 0;
  if (!n_sm) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
  }
  if (nsm <= 0) nsm = n_sm;
  const int G = a.H / std::max(a.Hkv, 1);
  if (a.page != 64 || a.max_chunks > 64 || G * a.qblk > 16 || a.seq.seq_len < 1 ||
      a.M % a.seq.seq_len || a.qblk < 1 || !a.enc.att_o || a.enc.KB < 1 || a.enc.M != a.M)
    return false;
  if (a.hdp != 32 && a.hdp != 64 && a.hdp != 128) return false;
  const int bps = g_attn_tail_bps[cur_device()][a.hdp == 32 ? 0 : (a.hdp == 64 ? 1 : 2)];
  const long long n_qb = (a.seq.seq_len + a.qblk - 1) / a.qblk;
  const long long grid = (long long)a.Hkv * a.max_chunks * (a.M / a.seq.seq_len) * n_qb;
  if (bps < 1 || grid > (long long)nsm * bps) return false;
  const long long kbs = (a.enc.KB + grid - 1) / grid;
  return (long long)a.M * kbs * 32 * (long long)sizeof(float) <=
         (long long)attention_tc_smem_bytes(1, a.hdp);
}

cudaError_t prepare_kernels(size_t quant_smem, size_t attn_smem) {
  (void)quant_smem;
  const int dev = cur_device();
  if (g_attn_tc_smem[dev] < (int)attention_tc_smem_bytes(4, 128)) {
    cudaError_t e = prepare_attention_tc_hd<32>();
    if (e == cudaSuccess) e = prepare_attention_tc_hd<64>();
    if (e == cudaSuccess) e = prepare_attention_tc_hd<128>();
    if (e != cudaSuccess) return e;
    g_attn_tc_smem[dev] = (int)attention_tc_smem_bytes(4, 128);
  }

  if (attn_smem > (size_t)attn_smem_limit()) {
    for (auto f : {k_attention<8, 1>, k_attention<4, 1>, k_attention<2, 1>, k_attention<1, 1>,
                   k_attention<2, 2>, k_attention<1, 2>}) {
      cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)attn_smem);
      if (e != cudaSuccess) return e;
    }
    g_attn_smem[dev] = (int)attn_smem;
  }
  return cudaSuccess;
}

// ------------------------------------------------------------ embedding
__global__ void __launch_bounds__(256) k_embed(EmbedArgs a) {
  MC_TRACE_T0
  grid_launch_dependents();
  grid_wait();
  MC_TRACE_WAITED(a.trace_slot);
  const int m = blockIdx.x;
  const int z = seq_of(a.seq, m), si = seq_off(a.seq, m);
  const uint32_t* ctx = a.ctx + (size_t)z * a.ctx_stride;
  const unsigned long long* keys = a.keys + (size_t)z * a.seq.key_stride;
  uint32_t id;
  switch (a.src) {
    case SRC_IDS: id = a.ids[m]; break;
    case SRC_CTX_AT: id = ctx[a.off[z * a.seq.pos_stride] + si]; break;
    case SRC_KEYS: id = key_index(keys[si]); break;
    default: id = (si == 0) ? ctx[a.off[z * a.seq.pos_stride] - 1] : key_index(keys[si - 1]); break;
  }
  if (a.ids_out && threadIdx.x == 0) a.ids_out[m] = id;
  float* h = a.h + (size_t)m * a.d;
  float ss = 0.0f;
  uint32_t mx = 0u;  // max|h*w| as float bits (NaN/inf win)
  const bool in = id < (uint32_t)a.vocab;
  const bool q4 = a.emb_q4 != nullptr;
  const int8_t* q = (in && !q4) ? a.emb_q + (size_t)id * a.d : nullptr;
  const uint8_t* q4row = (in && q4) ? a.emb_q4 + (size_t)id * (a.d / 32) * kQ4BlockBytes : nullptr;
  const float sc = (in && !q4) ? a.emb_scale[id] : 0.0f;
  // the row is read from HBM: a batch of kEmbBatch elements per thread has
  // all its loads in flight before the first use; the sums keep the
  // element order i = tid, tid + 256, ...
  constexpr int kEmbBatch = 16;
  for (int i0 = threadIdx.x; i0 < a.d; i0 += blockDim.x * kEmbBatch) {
    float v[kEmbBatch], wv[kEmbBatch];
#pragma unroll
    for (int u = 0; u < kEmbBatch; ++u) {
      const int i = i0 + u * blockDim.x;
      v[u] = 0.0f;
      wv[u] = 1.0f;
      if (i < a.d) {
        if (q4row) {
          // dequantize_q4_0 (dequant.rs:33-44): (code - 8) as f32 * d
          const uint8_t* blk = q4row + (i >> 5) * kQ4BlockBytes;
          const int j = i & 31;
          const uint32_t byte = blk[2 + (j & 15)];
          const int code = (int)(j < 16 ? (byte & 0x0Fu) : (byte >> 4)) - 8;
          const float dq =
              __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
          v[u] = __fmul_rn((float)code, dq);
        } else if (q) {
          v[u] = __fmul_rn((float)q[i], sc);
        }
        if (a.st_w) wv[u] = a.st_w[i];
      }
    }
#pragma unroll
    for (int u = 0; u < kEmbBatch; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i < a.d) {
        h[i] = v[u];
        ss = __fadd_rn(ss, __fmul_rn(v[u], v[u]));
        mx = max(mx, __float_as_uint(fabsf(__fmul_rn(v[u], wv[u]))));
      }
    }
  }
  if (m == 0)
    for (int j = threadIdx.x; j < a.n_zero; j += blockDim.x) a.zero_keys[key_slot(a.seq, j)] = 0ull;
  if (m == 0)
    for (int i = threadIdx.x; i < a.n_st_zero; i += blockDim.x) a.st_zero[i] = 0u;
  if (a.st_amax) {
    __shared__ float rs[8];
    __shared__ uint32_t rm[8];
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if ((threadIdx.x & 31) == 0) { rs[threadIdx.x >> 5] = ss; rm[threadIdx.x >> 5] = mx; }
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.0f;
      uint32_t u = 0u;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) { t = __fadd_rn(t, rs[w]); u = max(u, rm[w]); }
      a.st_pss[(size_t)m * a.st_np] = t;
      a.st_amax[m] = u;
    }
  }
  MC_TRACE_END(a.trace_slot);
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
__global__ void k_accept_greedy(SpecState* st_all, uint32_t* ctx_all, int* acc_log_all, int vm,
                                int ctx_stride, int log_stride) {
  grid_launch_dependents();
  grid_wait();
  if (threadIdx.x != 0) return;
  const int z = blockIdx.x;
  SpecState* st = st_all + z;
  uint32_t* ctx = ctx_all + (size_t)z * ctx_stride;
  int* acc_log = acc_log_all ? acc_log_all + (size_t)z * log_stride : nullptr;
  // a request whose budget is spent takes no more rounds (generate.rs:638)
  if (st->max_tokens > 0 && st->generated >= st->max_tokens) return;
  const int g = st->gamma;
  const int nd = min(max(st->n_draft, 0), g);  // draft tokens this round
  const int len = st->ctx_len;
  if (nd == 0) {
    // no draft (the n-gram index had no match): one standard generation
    // step, generate.rs:647-693 -- the target's token after the context's
    // last token, which the verify's first position computed.  Not a round:
    // no accepted count is logged.
    ctx[len] = key_index(st->tkeys[0]);
    st->ctx_len = len + 1;
    st->lt += 1;
    st->ld = len;
    st->generated += 1;
    return;
  }
  int a = 0;
  while (a < nd && key_index(st->tkeys[a]) == key_index(st->dkeys[a])) ++a;
  for (int j = 0; j < a; ++j) ctx[len + j] = key_index(st->dkeys[j]);
  int emitted = a, forwarded = a + 1;
  if (a < nd) {  // the first mismatch pushes the target's token
    ctx[len + a] = key_index(st->tkeys[a]);
    emitted = a + 1;
  } else if (vm > g) {  // every draft accepted: the bonus token (vm == gamma + 1)
    ctx[len + nd] = key_index(st->tkeys[nd]);
    emitted = nd + 1;
  } else {  // the reference: d_nd pushed unverified (quirk Q2)
    forwarded = nd;
  }
  st->ctx_len = len + emitted;
  st->lt += forwarded;
  st->ld = st->ctx_len - 1;
  st->generated += emitted;
  if (acc_log && st->n_rounds < st->rounds_cap) acc_log[st->n_rounds] = a;
  st->n_rounds += 1;
}

cudaError_t launch_accept_greedy(SpecState* st, uint32_t* ctx, int* acc_log, int vm, int n_seq,
                                 int ctx_stride, int log_stride, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_seq);
  cfg.blockDim = dim3(32);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_accept_greedy, st, ctx, acc_log, vm, ctx_stride, log_stride);
}

// ------------------------------------------------------------ sampling
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC 2011): ten rounds of
// (hi0, lo0) = M0 * c0, (hi1, lo1) = M1 * c2, c = (hi1^c1^k0, lo1, hi0^c3^k1,
// lo0), key advanced by the Weyl constants between rounds.  Counter
// (slot, round, 0, 0), key = seed; uniform = top 24 bits * 2^-24.  Slots per
// round: draft sample j -> j, acceptance test j -> 32 + j, residual / target
// / bonus sample j -> 64 + j.
__device__ __forceinline__ float philox_uniform(uint32_t seed_lo, uint32_t seed_hi,
                                                uint32_t round, uint32_t slot) {
  uint32_t c0 = slot, c1 = round, c2 = 0u, c3 = 0u, k0 = seed_lo, k1 = seed_hi;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r > 0) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    const uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
    const uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
  }
  return (float)(c0 >> 8) * (1.0f / 16777216.0f);
}

constexpr int kSampThreads = 1024;  // 32 warps; tile t = elements [1024 t, 1024 t + 1024)
constexpr int kSampTiles = kSampleMaxVocab / 1024;

constexpr int kCutBins = 4096;  // radix digits of 12 bits (the last pass 8)

struct SampSmem {
  float red[32];
  int ired[32];
  float tile[kSampTiles];
  int tile_last[kSampTiles];
  float bcast[4];
  int ibcast[4];  // [0] tile of the target, [1] fallback index, [2] index found, [3] bin
  unsigned long long hist[kCutBins];  // top-p: integer mass per radix digit
  unsigned long long wsum[32];
  unsigned long long ubcast[2];
};

__device__ float block_max(const float* row, int V, SampSmem& sm) {
  float m = -INFINITY;
  for (int v = threadIdx.x; v < V; v += kSampThreads) m = fmaxf(m, row[v]);
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sm.red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float x = sm.red[threadIdx.x];
#pragma unroll
    for (int o = 16; o; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
    if (threadIdx.x == 0) sm.bcast[0] = x;
  }
  __syncthreads();
  return sm.bcast[0];
}

// Sums of the weights w(v) >= 0 per tile (warp w takes tiles w, w+32, ...;
// lane l adds elements 32 i + l of its tile in i order, then an xor tree),
// the last positive index of each tile, and their total in tile order.
template <class W>
__device__ float tile_sums(W w, int V, SampSmem& sm) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = (V + 1023) >> 10;
  for (int t = warp; t < nt; t += 32) {
    float s = 0.0f;
    int last = -1;
    for (int i = 0; i < 32; ++i) {
      const int v = (t << 10) + i * 32 + lane;
      if (v < V) {
        const float x = w(v);
        s = __fadd_rn(s, x);
        if (x > 0.0f) last = v;
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
      last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
    }
    if (lane == 0) {
      sm.tile[t] = s;
      sm.tile_last[t] = last;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.0f;
    for (int t = 0; t < nt; ++t) tot = __fadd_rn(tot, sm.tile[t]);
    sm.bcast[1] = tot;
  }
  __syncthreads();
  return sm.bcast[1];
}

// Inverse CDF in index order over w (tile sums already in sm.tile, total
// `tot`): the first v whose running sum exceeds u * tot; if rounding leaves
// none, the last positive weight.  Returns v to every thread.
template <class W>
__device__ int inv_cdf(W w, int V, float tot, float u, SampSmem& sm) {
  const int nt = (V + 1023) >> 10;
  if (threadIdx.x == 0) {
    const float tau = __fmul_rn(u, tot);
    float c = 0.0f;
    int kt = -1, fallback = -1;
    for (int t = 0; t < nt; ++t) {
      if (sm.tile_last[t] >= 0) fallback = sm.tile_last[t];
      if (kt < 0 && __fadd_rn(c, sm.tile[t]) > tau) {
        kt = t;
      } else if (kt < 0) {
        c = __fadd_rn(c, sm.tile[t]);
      }
    }
    sm.ibcast[0] = kt;
    sm.ibcast[1] = fallback < 0 ? 0 : fallback;
    sm.bcast[2] = __fsub_rn(tau, c);  // remaining mass inside tile kt
  }
  __syncthreads();
  const int kt = sm.ibcast[0];
  int res = sm.ibcast[1];
  if (kt >= 0 && threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const float rem = sm.bcast[2];
    float c = 0.0f;
    int found = -1;
    for (int i = 0; i < 32 && found < 0; ++i) {
      const int v = (kt << 10) + i * 32 + lane;
      const float x = v < V ? w(v) : 0.0f;
      float sc = x;  // inclusive scan over lanes (index order within the row)
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, sc, o);
        if (lane >= o) sc = __fadd_rn(sc, y);
      }
      const float run = __fadd_rn(c, sc);
      const unsigned hit = __ballot_sync(0xffffffffu, run > rem && x > 0.0f);
      if (hit) found = (kt << 10) + i * 32 + (__ffs(hit) - 1);
      c = __fadd_rn(c, __shfl_sync(0xffffffffu, sc, 31));
    }
    if (lane == 0) sm.ibcast[2] = found >= 0 ? found : -2;
  }
  __syncthreads();
  if (kt >= 0) {
    const int f = sm.ibcast[2];
    res = f >= 0 ? f : (sm.tile_last[kt] >= 0 ? sm.tile_last[kt] : res);
  }
  __syncthreads();
  return res;
}

// ---- top-p and min-p (generate.rs:1034-1063 apply_top_p, :1071-1086
// apply_min_p), restated on e_v = exp((l_v - max) / T), whose maximum is 1,
// so that every decision is exact and order-independent:
//   top-p (0 < top_p < 1): order v by (e_v descending, v ascending), as the
//     reference's stable descending sort does; each v has the integer mass
//     m_v = floor(e_v * 2^32); keep the shortest prefix whose mass reaches
//     T = ceil(top_p * sum m_v) (one double rounding).  A three-pass radix
//     select over the bits of e_v (12 + 12 + 8 bits; integer mass histograms
//     in shared memory) finds the e at which the prefix ends, and one more
//     pass the last index kept when the prefix ends inside a run of equal e.
//   min-p (0 < min_p < 1): drop e_v < min_p, i.e. p_v < min_p * max p.
// The sampler draws from the kept e_v unnormalised, so the reference's
// renormalisations need no pass of their own.
struct Cut {
  uint32_t key;  // keep v iff bits(e_v) > key, or == key and v <= last ...
  int last;
  float min_e;   // ... and e_v >= min_e
};

__device__ __forceinline__ unsigned long long cut_mass(float e) {
  return __float2ull_rz(__fmul_rn(e, 4294967296.0f));
}

__device__ __forceinline__ float cut_weight(const Cut& c, float e, int v) {
  const uint32_t k = __float_as_uint(e);
  return (e >= c.min_e && (k > c.key || (k == c.key && v <= c.last))) ? e : 0.0f;
}

// Exclusive prefix sum over the block in thread order; *total gets the sum.
__device__ unsigned long long block_excl_scan(unsigned long long x, SampSmem& sm,
                                              unsigned long long* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) sm.wsum[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const unsigned long long w = sm.wsum[lane];
    unsigned long long wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    sm.wsum[lane] = wi - w;
    if (lane == 31) sm.ubcast[0] = wi;
  }
  __syncthreads();
  const unsigned long long r = sm.wsum[warp] + inc - x;
  *total = sm.ubcast[0];
  __syncthreads();
  return r;
}

// Index of the k-th (1-based, ascending) v with pred(v); INT_MAX if none.
template <class P>
__device__ int kth_index(P pred, int V, int k, SampSmem& sm) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = (V + 1023) >> 10;
  for (int t = warp; t < nt; t += 32) {
    int c = 0;
    for (int i = 0; i < 32; ++i) {
      const int v = (t << 10) + i * 32 + lane;
      c += __popc(__ballot_sync(0xffffffffu, v < V && pred(v)));
    }
    if (lane == 0) sm.tile_last[t] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int r = k, kt = -1;
    for (int t = 0; t < nt; ++t) {
      if (r <= sm.tile_last[t]) {
        kt = t;
        break;
      }
      r -= sm.tile_last[t];
    }
    sm.ibcast[0] = kt;
    sm.ibcast[1] = r;
    sm.ibcast[2] = INT_MAX;
  }
  __syncthreads();
  const int kt = sm.ibcast[0];
  if (kt >= 0 && threadIdx.x < 32) {
    int r = sm.ibcast[1];
    for (int i = 0; i < 32; ++i) {
      const int v = (kt << 10) + i * 32 + lane;
      const unsigned m = __ballot_sync(0xffffffffu, v < V && pred(v));
      const int c = __popc(m);
      if (r <= c) {
        if (((m >> lane) & 1u) && __popc(m & ((1u << lane) - 1u)) == r - 1) sm.ibcast[2] = v;
        break;
      }
      r -= c;
    }
  }
  __syncthreads();
  const int res = sm.ibcast[2];
  __syncthreads();
  return res;
}

template <class E>
__device__ Cut make_cut(E e, int V, float top_p, float min_p, SampSmem& sm) {
  Cut c{0u, INT_MAX, (min_p > 0.0f && min_p < 1.0f) ? min_p : 0.0f};
  if (!(top_p > 0.0f && top_p < 1.0f)) return c;
  uint32_t pfx = 0u, pmask = 0u;
  unsigned long long need = 0ull;
  int bin = 0;
#pragma unroll 1
  for (int pass = 0; pass < 3; ++pass) {
    const int shift = pass == 0 ? 20 : (pass == 1 ? 8 : 0);
    const int nb = pass == 2 ? 256 : kCutBins;
    for (int i = threadIdx.x; i < nb; i += kSampThreads) sm.hist[i] = 0ull;
    __syncthreads();
    for (int v = threadIdx.x; v < V; v += kSampThreads) {
      const float x = e(v);
      const uint32_t k = __float_as_uint(x);
      if ((k & pmask) == pfx) atomicAdd(&sm.hist[(k >> shift) & (uint32_t)(nb - 1)], cut_mass(x));
    }
    __syncthreads();
    // thread t holds digits nb-1-4t .. nb-4-4t: thread order = descending e
    const int hi = nb - 1 - 4 * (int)threadIdx.x;
    unsigned long long loc = 0ull;
    if (hi >= 0)
      for (int b = 0; b < 4; ++b) loc += sm.hist[hi - b];
    unsigned long long tot;
    unsigned long long ex = block_excl_scan(loc, sm, &tot);
    if (pass == 0) need = (unsigned long long)ceil(__dmul_rn((double)top_p, (double)tot));
    if (hi >= 0 && ex < need && need <= ex + loc) {  // exactly one thread
      for (int b = 0; b < 4; ++b) {
        const unsigned long long h = sm.hist[hi - b];
        if (ex + h >= need) {
          sm.ubcast[1] = need - ex;
          sm.ibcast[3] = hi - b;
          break;
        }
        ex += h;
      }
    }
    __syncthreads();
    need = sm.ubcast[1];  // mass still to take inside the chosen digit
    bin = sm.ibcast[3];
    pfx |= (uint32_t)bin << shift;
    pmask |= (uint32_t)(nb - 1) << shift;
  }
  // every v in the last digit has e = pfx and the same mass
  const unsigned long long m1 = cut_mass(__uint_as_float(pfx));
  const unsigned long long cnt = m1 ? sm.hist[bin] / m1 : 0ull;
  const unsigned long long k = m1 ? (need + m1 - 1) / m1 : 0ull;
  __syncthreads();
  c.key = pfx;
  if (k < cnt)
    c.last = kth_index([&](int v) { return __float_as_uint(e(v)) == pfx; }, V, (int)k, sm);
  return c;
}

__global__ void __launch_bounds__(kSampThreads) k_sample_draft(SpecState* st, const float* row,
                                                               int V, int j,
                                                               unsigned long long* key_out) {
  __shared__ SampSmem sm;
  grid_launch_dependents();
  grid_wait();
  const float t = st->temperature;
  const float mx = block_max(row, V, sm);
  auto e = [&](int v) { return expf(__fdiv_rn(__fsub_rn(__ldcg(row + v), mx), t)); };
  const Cut c = make_cut(e, V, st->top_p, st->min_p, sm);
  auto w = [&](int v) { return cut_weight(c, e(v), v); };
  const float tot = tile_sums(w, V, sm);
  const float u = philox_uniform(st->seed_lo, st->seed_hi, (uint32_t)st->n_rounds, (uint32_t)j);
  const int x = inv_cdf(w, V, tot, u, sm);
  if (threadIdx.x == 0) *key_out = argmax_key(0.0f, (uint32_t)x);
}

__global__ void __launch_bounds__(kSampThreads) k_accept_stochastic(
    SpecState* st, uint32_t* ctx, int* acc_log, int vm, const float* tlog, const float* dlog,
    int V) {
  __shared__ SampSmem sm;
  grid_launch_dependents();
  grid_wait();
  const int g = st->gamma;
  const float t = st->temperature, top_p = st->top_p, min_p = st->min_p;
  const uint32_t rnd = (uint32_t)st->n_rounds, s0 = st->seed_lo, s1 = st->seed_hi;
  int a = 0, y = -1;
  for (int j = 0; j < g; ++j) {
    const float* p = tlog + (size_t)j * V;
    const float* q = dlog + (size_t)j * V;
    const uint32_t x = min(key_index(st->dkeys[j]), (uint32_t)(V - 1));
    const float u_res = philox_uniform(s0, s1, rnd, 64u + (uint32_t)j);
    const float mp = block_max(p, V, sm);
    auto ep = [&](int v) { return expf(__fdiv_rn(__fsub_rn(__ldcg(p + v), mp), t)); };
    const Cut cp = make_cut(ep, V, top_p, min_p, sm);
    auto wp = [&](int v) { return cut_weight(cp, ep(v), v); };
    const float sp = tile_sums(wp, V, sm);
    if (st->accept_mode == 1) {
      // the reference's rule (generate.rs:695-726): the target's own sample
      const int z = inv_cdf(wp, V, sp, u_res, sm);
      if ((uint32_t)z == x) {
        ++a;
        continue;
      }
      y = z;
      break;
    }
    const float mq = block_max(q, V, sm);
    auto eq_ = [&](int v) { return expf(__fdiv_rn(__fsub_rn(__ldcg(q + v), mq), t)); };
    const Cut cq = make_cut(eq_, V, top_p, min_p, sm);
    auto wq = [&](int v) { return cut_weight(cq, eq_(v), v); };
    const float sq = tile_sums(wq, V, sm);
    const float px = wp((int)x), qx = wq((int)x);
    const float u = philox_uniform(s0, s1, rnd, 32u + (uint32_t)j);
    if (__fmul_rn(__fmul_rn(u, qx), sp) < __fmul_rn(px, sq)) {  // u < p(x) / q(x)
      ++a;
      continue;
    }
    auto wr = [&](int v) {
      return fmaxf(__fsub_rn(__fdiv_rn(wp(v), sp), __fdiv_rn(wq(v), sq)), 0.0f);
    };
    const float rs = tile_sums(wr, V, sm);
    if (rs > 0.0f) {
      y = inv_cdf(wr, V, rs, u_res, sm);
    } else {
      tile_sums(wp, V, sm);
      y = inv_cdf(wp, V, sp, u_res, sm);
    }
    break;
  }
  if (y < 0 && a == g && vm > g) {  // bonus token from the last verify position
    const float* p = tlog + (size_t)g * V;
    const float mp = block_max(p, V, sm);
    auto ep = [&](int v) { return expf(__fdiv_rn(__fsub_rn(__ldcg(p + v), mp), t)); };
    const Cut cp = make_cut(ep, V, top_p, min_p, sm);
    auto wp = [&](int v) { return cut_weight(cp, ep(v), v); };
    const float sp = tile_sums(wp, V, sm);
    y = inv_cdf(wp, V, sp, philox_uniform(s0, s1, rnd, 64u + (uint32_t)g), sm);
  }
  if (threadIdx.x != 0) return;
  const int len = st->ctx_len;
  for (int j = 0; j < a; ++j) ctx[len + j] = key_index(st->dkeys[j]);
  int emitted = a;
  if (y >= 0) {
    ctx[len + a] = (uint32_t)y;
    emitted = a + 1;
  }
  st->ctx_len = len + emitted;
  st->lt += (a + 1 < vm) ? a + 1 : vm;
  st->ld = st->ctx_len - 1;
  st->generated += emitted;
  if (acc_log && st->n_rounds < st->rounds_cap) acc_log[st->n_rounds] = a;
  st->n_rounds += 1;
}

template <class K, class... Args>
static cudaError_t launch_one_block(K kernel, int threads, cudaStream_t s, bool pdl,
                                    Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(threads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

cudaError_t launch_sample_draft(SpecState* st, const float* logits, int V, int j,
                                unsigned long long* key_out, cudaStream_t s, bool pdl) {
  if (V <= 0 || V > kSampleMaxVocab) return cudaErrorInvalidValue;
  return launch_one_block(k_sample_draft, kSampThreads, s, pdl, st, logits, V, j, key_out);
}

cudaError_t launch_accept_stochastic(SpecState* st, uint32_t* ctx, int* acc_log, int vm,
                                     const float* tlog, const float* dlog, int V,
                                     cudaStream_t s, bool pdl) {
  if (V <= 0 || V > kSampleMaxVocab) return cudaErrorInvalidValue;
  return launch_one_block(k_accept_stochastic, kSampThreads, s, pdl, st, ctx, acc_log, vm, tlog,
                          dlog, V);
}

// One CTA per row of logits (generate.rs:948-969 sample): temperature <= 0
// is the reference's argmax (first strict maximum; NaN and -inf never win;
// 0 when nothing does), otherwise softmax(l / T) after top-p and min-p,
// drawn by inverse CDF with the Philox uniform of (seed, round, slot = row).
__global__ void __launch_bounds__(kSampThreads) k_sample_rows(const float* logits, int V,
                                                              float t, float top_p, float min_p,
                                                              uint32_t s0, uint32_t s1,
                                                              uint32_t rnd, uint32_t* out) {
  __shared__ SampSmem sm;
  const float* row = logits + (size_t)blockIdx.x * V;
  if (!(t > 0.0f)) {
    unsigned long long best = 0ull;
    for (int v = threadIdx.x; v < V; v += kSampThreads) {
      const float x = row[v];
      if (x > -INFINITY) best = max(best, argmax_key(__fadd_rn(x, 0.0f), (uint32_t)v));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    if ((threadIdx.x & 31) == 0) sm.wsum[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x < 32) {
      unsigned long long b = sm.wsum[threadIdx.x];
#pragma unroll
      for (int o = 16; o; o >>= 1) b = max(b, __shfl_xor_sync(0xffffffffu, b, o));
      if (threadIdx.x == 0) out[blockIdx.x] = key_index(b);
    }
    return;
  }
  const float mx = block_max(row, V, sm);
  auto e = [&](int v) { return expf(__fdiv_rn(__fsub_rn(__ldcg(row + v), mx), t)); };
  const Cut c = make_cut(e, V, top_p, min_p, sm);
  auto w = [&](int v) { return cut_weight(c, e(v), v); };
  const float tot = tile_sums(w, V, sm);
  const int y = inv_cdf(w, V, tot, philox_uniform(s0, s1, rnd, blockIdx.x), sm);
  if (threadIdx.x == 0) out[blockIdx.x] = (uint32_t)y;
}

cudaError_t launch_sample_rows(const float* logits, int rows, int V, float t, float top_p,
                               float min_p, uint64_t seed, uint32_t rnd, uint32_t* out,
                               cudaStream_t s) {
  if (V <= 0 || V > kSampleMaxVocab || rows <= 0) return cudaErrorInvalidValue;
  k_sample_rows<<<rows, kSampThreads, 0, s>>>(logits, V, t, top_p, min_p, (uint32_t)seed,
                                             (uint32_t)(seed >> 32), rnd, out);
  return cudaGetLastError();
}

// grid (ceil(d / 1024), M), 256 threads: h += y on one 1024-element block of
// one token, its sum of squares (fixed order: 4 strided elements per thread,
// then warp and block trees) and max |h * w|.
__global__ void __launch_bounds__(256) k_resid_stats(ResidArgs a) {
  MC_TRACE_T0
  grid_launch_dependents();
  grid_wait();
  MC_TRACE_WAITED(a.trace_slot);
  const int m = blockIdx.y, blk = blockIdx.x;
  float ss = 0.0f;
  uint32_t mx = 0u;
  for (int j = 0; j < kResidBlock / 256; ++j) {
    const int i = blk * kResidBlock + j * 256 + threadIdx.x;
    if (i < a.d) {
      float* hp = a.h + (size_t)m * a.d + i;
      const float v = __fadd_rn(*hp, __ldcg(a.y + (size_t)m * a.d + i));
      *hp = v;
      ss = __fadd_rn(ss, __fmul_rn(v, v));
      mx = max(mx, __float_as_uint(fabsf(__fmul_rn(v, a.w ? a.w[i] : 1.0f))));
    }
  }
  __shared__ float rs[8];
  __shared__ uint32_t rm[8];
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if ((threadIdx.x & 31) == 0) {
    rs[threadIdx.x >> 5] = ss;
    rm[threadIdx.x >> 5] = mx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    uint32_t u = 0u;
    for (int w = 0; w < 8; ++w) {
      t = __fadd_rn(t, rs[w]);
      u = max(u, rm[w]);
    }
    a.pss[(size_t)m * gridDim.x + blk] = t;
    atomicMax(a.amax + m, u);
  }
  MC_TRACE_END(a.trace_slot);
}

cudaError_t launch_resid_stats(const ResidArgs& a, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.d + kResidBlock - 1) / kResidBlock, a.M);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_resid_stats, a);
}

// Waits until *p == e (acquire at system scope, so the peer's stores that
// precede its release are visible) for at most limit_ns nanoseconds of
// %globaltimer; a fixed poll count bounds it as well, should the timer not
// advance.  Returns false when the wait expired.
__device__ __forceinline__ bool bounded_wait_eq(const unsigned* p, unsigned e, long long limit_ns) {
  unsigned long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (long long i = 0; i < (1ll << 24); ++i) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    if (v == e) return true;
    if ((i & 31) == 31) {
      unsigned long long t1;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
      if ((long long)(t1 - t0) > limit_ns) return false;
    }
  }
  return false;
}

// One thread: waits (bounded) until flags[r] == e for every rank r; gives up
// at once when the error word is already raised (an earlier wait expired),
// and raises it when a wait expires.
__device__ __forceinline__ int tp_wait_all(const TPArgs& t, const unsigned* flags, unsigned e) {
  int ok = !(t.err && *(volatile int*)t.err);
  const long long limit = t.wait_ns ? *(const volatile long long*)t.wait_ns : 5000000000ll;
  for (int r = 0; r < t.world && ok; ++r) ok = bounded_wait_eq(flags + r, e, limit);
  if (!ok && t.err) atomicExch(t.err, 1);
  return ok;
}

// grid (ceil(d / 1024), M), 256 threads: wait (bounded) for the R partials of
// this epoch, h += their sum in rank order, statistics as k_resid_stats; the
// last CTA advances the epoch.
__global__ void __launch_bounds__(256) k_tp_reduce(ResidArgs a, TPArgs t, unsigned* epoch,
                                                   int* cnt) {
  MC_TRACE_T0
  grid_launch_dependents();
  grid_wait();
  MC_TRACE_WAITED(a.trace_slot);
  __shared__ int s_ok;
  const unsigned e = __ldcg(epoch);
  const unsigned* fl = t.flag[t.rank] + (e & 1u) * kMaxTP;
  if (threadIdx.x == 0) s_ok = tp_wait_all(t, fl, e);
  __syncthreads();
  const int m = blockIdx.y, blk = blockIdx.x;
  const float* red = t.red[t.rank] + (size_t)(e & 1u) * t.world * kMaxTokens * a.d;
  float ss = 0.0f;
  uint32_t mx = 0u;
  for (int j = 0; j < kResidBlock / 256; ++j) {
    const int i = blk * kResidBlock + j * 256 + threadIdx.x;
    if (i < a.d) {
      float sum = 0.0f;
      for (int r = 0; r < t.world; ++r)
        sum = __fadd_rn(sum, __ldcg(red + ((size_t)r * kMaxTokens + m) * a.d + i));
      float* hp = a.h + (size_t)m * a.d + i;
      const float v = __fadd_rn(*hp, s_ok ? sum : __int_as_float(0x7fc00000));
      *hp = v;
      ss = __fadd_rn(ss, __fmul_rn(v, v));
      mx = max(mx, __float_as_uint(fabsf(__fmul_rn(v, a.w ? a.w[i] : 1.0f))));
    }
  }
  __shared__ float rs[8];
  __shared__ uint32_t rm[8];
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if ((threadIdx.x & 31) == 0) {
    rs[threadIdx.x >> 5] = ss;
    rm[threadIdx.x >> 5] = mx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float tt = 0.0f;
    uint32_t u = 0u;
    for (int w = 0; w < 8; ++w) {
      tt = __fadd_rn(tt, rs[w]);
      u = max(u, rm[w]);
    }
    a.pss[(size_t)m * gridDim.x + blk] = tt;
    atomicMax(a.amax + m, u);
    __threadfence();
    if (atomicAdd(cnt, 1) == (int)(gridDim.x * gridDim.y) - 1) {  // every CTA has read e
      atomicExch(epoch, e + 1u);
      atomicExch(cnt, 0);
    }
  }
  MC_TRACE_END(a.trace_slot);
}

cudaError_t launch_tp_reduce(const ResidArgs& a, const TPArgs& t, unsigned* epoch, int* cnt,
                             cudaStream_t s, bool pdl) {
  if (t.world < 2 || t.world > kMaxTP) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.d + kResidBlock - 1) / kResidBlock, a.M);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_tp_reduce, a, t, epoch, cnt);
}

// One CTA of 64 threads, one per token (n_seq * seq_len <= kMaxTokens): this
// rank's argmax keys go into slot `rank` of key set e % 2 in every rank's
// buffer, then its flag e; after a bounded wait for every rank's flag each
// key becomes the largest over the ranks (the largest logit, ties to the
// lowest global index).  On an expired wait the keys stay this rank's own
// and the error word is raised.
__global__ void __launch_bounds__(kMaxTokens) k_tp_keys(TPArgs t, unsigned long long* keys,
                                                        int n_seq, int seq_len, int key_stride) {
  grid_launch_dependents();
  grid_wait();
  __shared__ int s_ok;
  const unsigned e = *(volatile unsigned*)t.kepoch;
  const int set = (int)(e & 1u);
  const int n = n_seq * seq_len;
  const int i = threadIdx.x;
  const size_t kidx = i < n ? (size_t)(i / seq_len) * key_stride + i % seq_len : 0;
  if (i < n) {
    const unsigned long long k = __ldcg(keys + kidx);
    for (int r = 0; r < t.world; ++r)
      t.keyx[r][((size_t)set * kMaxTP + t.rank) * kMaxTokens + i] = k;
  }
  __syncthreads();
  if (i == 0) {
    __threadfence_system();
    for (int r = 0; r < t.world; ++r)
      asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(t.kflag[r] + set * kMaxTP + t.rank),
                   "r"(e)
                   : "memory");
    s_ok = tp_wait_all(t, t.kflag[t.rank] + set * kMaxTP, e);
  }
  __syncthreads();
  if (i < n && s_ok) {
    const unsigned long long* in = t.keyx[t.rank] + (size_t)set * kMaxTP * kMaxTokens + i;
    unsigned long long m = 0ull;
    for (int r = 0; r < t.world; ++r) {
      const unsigned long long k = __ldcg(in + (size_t)r * kMaxTokens);
      m = k > m ? k : m;
    }
    keys[kidx] = m;
  }
  __syncthreads();
  if (i == 0) *(volatile unsigned*)t.kepoch = e + 1u;
}

cudaError_t launch_tp_keys(const TPArgs& t, unsigned long long* keys, int n_seq, int seq_len,
                           int key_stride, cudaStream_t s, bool pdl) {
  if (t.world < 2 || t.world > kMaxTP || n_seq * seq_len > kMaxTokens || n_seq * seq_len < 1)
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kMaxTokens);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_tp_keys, t, keys, n_seq, seq_len, key_stride);
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

// One thread per (stripe, k-block, lane): gathers the nibbles of A registers
// a0..a3 (rows g, g+8; columns 4t..4t+3 and 16+4t..16+4t+3 of the block) from
// the q4_0 source.  In a source block, element j < 16 is the low nibble of
// qs[j] and element 16 + j its high nibble (dequant.rs:33-44).
__global__ void k_pack_q4(const uint8_t* __restrict__ src, const int* __restrict__ row_map,
                          int n_stripes, int KB, int src_KB, int kb_off, uint2* __restrict__ dst,
                          uint32_t* __restrict__ dst_scale) {
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
  const uint8_t* ba = ra >= 0 ? src + ((long long)ra * src_KB + kb_off + kb) * kQ4BlockBytes : nullptr;
  const uint8_t* bb = rb >= 0 ? src + ((long long)rb * src_KB + kb_off + kb) * kQ4BlockBytes : nullptr;
  uint32_t w0 = 0, w1 = 0;
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const uint32_t qa = ba ? ba[2 + 4 * t + b] : 0x88u;  // padding rows: codes 8 (value 0)
    const uint32_t qb = bb ? bb[2 + 4 * t + b] : 0x88u;
    w0 |= ((qa & 0x0Fu) | ((qb & 0x0Fu) << 4)) << (8 * b);
    w1 |= ((qa >> 4) | (qb & 0xF0u)) << (8 * b);
  }
  dst[gid] = make_uint2(w0, w1);
  if (t == 0) {
    const uint32_t da = ba ? (uint32_t)ba[0] | ((uint32_t)ba[1] << 8) : 0u;
    const uint32_t db = bb ? (uint32_t)bb[0] | ((uint32_t)bb[1] << 8) : 0u;
    dst_scale[sk * 8 + g] = da | (db << 16);
  }
}

cudaError_t launch_pack_q4(const uint8_t* src, const int* row_map, int n_stripes, int KB,
                           int src_KB, int kb_off, uint2* dst, uint32_t* dst_scale,
                           cudaStream_t s) {
  const long long total = (long long)n_stripes * KB * 32;
  const int bs = 256;
  k_pack_q4<<<(unsigned)((total + bs - 1) / bs), bs, 0, s>>>(src, row_map, n_stripes, KB, src_KB,
                                                             kb_off, dst, dst_scale);
  return cudaGetLastError();
}

// ------------------------------------------------------------ tcgen05 GEMM
// Projections of 9..64 tokens (48 digit columns per group of 16 tokens, G
// groups) on the 5th-generation tensor cores: D[128 rows][48 G] +=
// A[128][32 k] * B[48 G][32 k] per tcgen05.mma.kind::i8 (exact int32 in
// tensor memory).  One CTA per 128-row tile (and k-split):
// thread 0 streams A (the weight copy in the canonical layout, below) and B
// (the digits, encoded in the same layout) into a 4-stage shared-memory ring
// with cp.async.bulk + mbarrier transaction counts; thread 32 issues the MMAs
// and releases each stage with tcgen05.commit.  Afterwards the 4 warps read
// their 32 tensor-memory lanes (tcgen05.ld 32x32b), one token group at a
// time, and run the same stripe epilogue as the GEMV, so results are
// identical to it bit for bit.
//
// Operands are K-major with the 128-byte swizzle (atoms of 8 rows x 128
// bytes of K = 4 k-steps, 8-row groups 1024 bytes apart = SBO; the MMA of
// k-step j of an atom starts 32 j bytes into it), so the tensor cores read
// shared memory without bank conflicts.
constexpr int kTcRows = 128;
constexpr int kTcMaxStages = 8;
constexpr int kTcRingBudget = 180 * 1024;  // bytes of ring per CTA (one CTA per SM)
constexpr int kTcAStep = kTcRows * 32;  // bytes of A per k-step
constexpr int kTcGroupCols = 48;        // digit columns of one token group
template <int G>
struct TcCfg {
  static constexpr int N = kTcGroupCols * G;  // MMA N (multiple of 16, <= 256)
  static constexpr int BStep = N * 32;        // bytes of B per k-step
  static constexpr int AtomA = kTcRows * 128;  // bytes of one A atom (4 k-steps)
  static constexpr int AtomB = N * 128;
  static constexpr int Chunk = G == 1 ? 8 : 4;  // k-steps per stage (whole atoms)
  static constexpr int StageBytes = Chunk * (kTcAStep + BStep);
  static constexpr int StagesFit = kTcRingBudget / StageBytes;
  static constexpr int Stages = StagesFit > kTcMaxStages ? kTcMaxStages : StagesFit;
  // independent accumulators, k-step j into accumulator j % NAcc: MMAs into
  // one accumulator serialize, so consecutive k-steps go to different ones
  // (summed exactly in the epilogue)
  static constexpr int NAcc = G <= 2 ? 4 : (G == 3 ? 3 : 2);
  static constexpr uint32_t TmemCols = G == 1 ? 256 : 512;  // power of 2 >= NAcc * N
  static constexpr size_t Ring = (size_t)Stages * StageBytes;
  // after the main loop the ring receives, from every CTA of the cluster,
  // the partial rows of the stripes this CTA finishes: [source][owned rows]
  // [N + 4] ints, at most 7 sources x 2 stripes x 16 rows
  static constexpr int LDP = N + 4;  // int row stride: 16-byte rows, conflict-free v4 stores
  static constexpr size_t RecvBytes = (size_t)224 * LDP * sizeof(int);
  // + 1 KB to align the ring to the 1024-byte swizzle atoms
  static constexpr size_t Smem = (Ring > RecvBytes ? Ring : RecvBytes) + 1024;
  static_assert(Smem <= 227 * 1024 - 2048, "tcgen05 GEMM shared memory");
  static_assert(Stages >= 2 && (Chunk & 3) == 0, "tcgen05 GEMM ring");
  // kind::i8 instruction descriptor: s32 accumulator, signed A and B, both
  // K-major, N, M = 128.
  static constexpr uint32_t Idesc = (2u << 4) | (1u << 7) | (1u << 10) |
                                    ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
};

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  // start address, LBO 1 (unused by swizzled K-major), SBO 1024 B (16-byte
  // units), descriptor version 1, layout 128-byte swizzle
  return (uint64_t)((saddr >> 4) & 0x3FFF) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}
__device__ __forceinline__ void umma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* b) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(b))
               : "memory");
}
// Thread-block cluster helpers: rank in the cluster, a full cluster barrier
// (release / acquire), and 16-byte loads from a peer CTA's shared memory.
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}
__device__ __forceinline__ uint32_t peer_addr(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_peer_v4(uint32_t addr, int4 v) {
  asm volatile("st.shared::cluster.v4.s32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ int4 ld_peer_v4(uint32_t addr) {
  int4 v;
  asm volatile("ld.shared::cluster.v4.s32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

template <int EPI, int G>
__global__ void __launch_bounds__(128, 1) k_gemm_tc(GemvArgs a) {
  using C = TcCfg<G>;
  constexpr int GC = kTcGroupCols;
  constexpr int N = C::N, LDP = C::LDP;
  extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
  // the swizzle atoms need 1024-byte alignment (the allocation has 1 KB slack)
  uint8_t* tc_smem = tc_smem_raw + ((1024u - (smem_addr(tc_smem_raw) & 1023u)) & 1023u);
  uint8_t* smA = tc_smem;
  uint8_t* smB = tc_smem + (size_t)C::Stages * C::Chunk * kTcAStep;
  // reused after the main loop: the receive buffer of the partial rows
  int* recv = reinterpret_cast<int*>(tc_smem);
  __shared__ __align__(8) uint64_t full[kTcMaxStages], empty[kTcMaxStages], done;
  __shared__ uint32_t tmem_base;
  __shared__ int sm_exp[kMaxTokens], s_issued, s_consumed, s_fail;
  __shared__ unsigned long long sm_keys[kMaxTokens];
  __shared__ int2 sm_tok[EPI == EPI_QKV ? kMaxTokens : 1];  // (position, KV page) per token
  // epilogue inputs staged during the main loop (EpiPre)
  __shared__ float sm_scl[kTcRows];
  __shared__ float sm_w[EPI == EPI_RESID ? kTcRows : 1];
  __shared__ __align__(16) float sm_h[EPI == EPI_RESID ? kMaxTokens * kTcRows : 1];
  __shared__ float sm_cs[EPI == EPI_QKV ? kMaxTokens * 64 : 1];
  __shared__ float sm_sn[EPI == EPI_QKV ? kMaxTokens * 64 : 1];
  MC_TRACE_T0
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the k-split CTAs of a tile form one cluster (grid y = cluster y)
  const int tile = blockIdx.x, nsplit = gridDim.y, split = blockIdx.y;
  const int KA = tc_atoms(a.KB);  // K atoms (4 k-steps each; padding is zero weights)
  const int a0 = (int)((long long)KA * split / nsplit), a1 = (int)((long long)KA * (split + 1) / nsplit);
  const int nk = 4 * (a1 - a0);  // k-steps of this split
  const int n_chunks = (nk + C::Chunk - 1) / C::Chunk;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(&tmem_base)),
                 "r"(C::TmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_issued = s_consumed = s_fail = 0;
  }
  if (threadIdx.x < kMaxTokens) sm_keys[threadIdx.x] = 0ull;
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  const uint8_t* wsrc = reinterpret_cast<const uint8_t*>(a.wtc) + ((size_t)tile * KA + a0) * C::AtomA;
  const uint8_t* xsrc = a.x + (size_t)a0 * C::AtomB;
  // The weights never depend on the producer grid: the first ring stages'
  // weight copies go out before the dependency wait (their activation
  // copies, after it, complete the same transaction counts).
  const int pre = min(n_chunks, C::Stages);
  if (threadIdx.x == 0)
    for (int i = 0; i < pre; ++i) {
      const int steps = min(C::Chunk, nk - i * C::Chunk);
      mbar_expect_tx(&full[i], (uint32_t)steps * (kTcAStep + C::BStep));
      bulk_load(smA + (size_t)i * C::Chunk * kTcAStep, wsrc + (size_t)i * C::Chunk * kTcAStep,
                (uint32_t)steps * kTcAStep, &full[i]);
    }
  grid_wait();
  MC_TRACE_WAITED(a.trace_slot);
  MC_TRACE_PHASE(a.trace_slot, 0, mc_tp);
  if (threadIdx.x < a.M) sm_exp[threadIdx.x] = __ldcg(a.xexp + threadIdx.x);
  // warps 2-3 stage everything the epilogue reads while the pipeline runs:
  // row scales, next-norm weights and residual rows of the tile (RESID), the
  // tokens' positions, pages and RoPE factors (QKV)
  const int row0 = tile * kTcRows;
  if (threadIdx.x >= 64) {
    const int t = (int)threadIdx.x - 64;
    if constexpr (EPI == EPI_QKV) {
      if (t < a.M) {
        const int mt = a.m0 + t, z = seq_of(a.seq, mt);
        const int pos = a.pos_ptr[z * a.seq.pos_stride] + a.pos_add + seq_off(a.seq, mt);
        sm_tok[t] = make_int2(pos, a.page_table[z * a.seq.pt_stride + pos / a.page]);
      }
      asm volatile("bar.sync 1, 64;" ::: "memory");  // warps 2-3: token table ready
      const int per_head = a.half_p >> 3;
      for (int i = t; i < a.M * 64; i += 64) {
        const int m = i >> 6, q = i & 63;
        const int gs = tile * 8 + (q >> 3), rr = q & 7;
        float c = 1.0f, sn = 0.0f;
        if (gs < a.n_stripes && gs < a.sq + a.sk && per_head > 0) {
          const int s2 = gs < a.sq ? gs : gs - a.sq;
          const int hh = s2 / per_head;
          const int ri = (s2 - hh * per_head) * 8 + rr;
          const size_t at = (size_t)sm_tok[m].x * a.half_p + ri;
          c = a.rope_cos[at];
          sn = a.rope_sin[at];
        }
        sm_cs[i] = c;
        sm_sn[i] = sn;
      }
    }
    for (int r = t; r < kTcRows; r += 64) {
      const int gr = row0 + r;
      sm_scl[r] = gr < a.n_stripes * 16 ? a.scale[gr] : 0.0f;
      if constexpr (EPI == EPI_RESID) sm_w[r] = (a.st_w && gr < a.n_out) ? a.st_w[gr] : 1.0f;
    }
    if constexpr (EPI == EPI_RESID) {
      // residual rows: 16-byte loads where the token's row segment allows
      const bool vec = ((a.ldo & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.out) & 15) == 0) &&
                       row0 + kTcRows <= a.n_out;
      if (vec) {
        for (int i = t; i < a.M * (kTcRows / 4); i += 64) {
          const int m = i / (kTcRows / 4), c4 = i - m * (kTcRows / 4);
          reinterpret_cast<float4*>(sm_h)[i] = *reinterpret_cast<const float4*>(
              a.out + (size_t)(a.m0 + m) * a.ldo + row0 + 4 * c4);
        }
      } else {
        for (int i = t; i < a.M * kTcRows; i += 64) {
          const int m = i / kTcRows, gr = row0 + (i - m * kTcRows);
          sm_h[i] = gr < a.n_out ? a.out[(size_t)(a.m0 + m) * a.ldo + gr] : 0.0f;
        }
      }
    }
  }

  if (threadIdx.x == 0) {  // producer
    int i = 0;
    for (; i < n_chunks; ++i) {
      const int s = i % C::Stages;
      const int steps = min(C::Chunk, nk - i * C::Chunk);
      if (i >= pre) {
        if (!mbar_wait(&empty[s], ((i / C::Stages) - 1) & 1)) {
          s_fail = 1;
          break;
        }
        mbar_expect_tx(&full[s], (uint32_t)steps * (kTcAStep + C::BStep));
        bulk_load(smA + (size_t)s * C::Chunk * kTcAStep, wsrc + (size_t)i * C::Chunk * kTcAStep,
                  (uint32_t)steps * kTcAStep, &full[s]);
      }
      bulk_load(smB + (size_t)s * C::Chunk * C::BStep, xsrc + (size_t)i * C::Chunk * C::BStep,
                (uint32_t)steps * C::BStep, &full[s]);
    }
    s_issued = i;
    MC_TRACE_PHASE(a.trace_slot, 1, mc_tp);
  } else if (threadIdx.x == 32) {  // MMA issuer
    int i = 0;
    for (; i < n_chunks; ++i) {
      const int s = i % C::Stages;
      if (!mbar_wait(&full[s], (i / C::Stages) & 1)) {
        s_fail = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int steps = min(C::Chunk, nk - i * C::Chunk);
      const uint32_t sa = smem_addr(smA + (size_t)s * C::Chunk * kTcAStep);
      const uint32_t sb = smem_addr(smB + (size_t)s * C::Chunk * C::BStep);
      // k-step j: atom j / 4, 32 (j % 4) bytes into its 128-byte rows
      for (int j = 0; j < steps; ++j) {
        const int kidx = i * C::Chunk + j;
        umma_i8(tmem + (uint32_t)((kidx % C::NAcc) * N), umma_desc(sa + (j >> 2) * C::AtomA + (j & 3) * 32),
                umma_desc(sb + (j >> 2) * C::AtomB + (j & 3) * 32), C::Idesc,
                kidx >= C::NAcc ? 1u : 0u);
      }
      umma_commit(&empty[s]);
    }
    s_consumed = i;
    umma_commit(&done);  // tracks completion of every MMA issued above
  }
  __syncthreads();
  // one thread waits for the MMAs (and, after a failed wait, drains copies
  // issued but never consumed); the verdict is block-uniform, as the
  // .aligned tensor-memory loads below require
  if (threadIdx.x == 0) {
    for (int i = s_consumed; i < s_issued; ++i) mbar_wait(&full[i % C::Stages], (i / C::Stages) & 1);
    if (!mbar_wait(&done, 0)) s_fail = 1;
    MC_TRACE_PHASE(a.trace_slot, 2, mc_tp);
  }
  __syncthreads();
  const bool ok = !s_fail;
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (!ok && threadIdx.x == 0 && a.err) atomicExch(a.err, 1);
  // 1) every CTA of the cluster is past its main loop: the rings are idle
  if (nsplit > 1) cluster_sync_all(); else __syncthreads();
  MC_TRACE_PHASE(a.trace_slot, 3, mc_tp);
  // 2) push: thread (warp, lane) holds accumulator row R = 32 * warp + lane of
  //    stripe R / 16, which CTA (R / 16) % nsplit finishes; the row goes to
  //    slot `rank` of that CTA's receive buffer (remote stores do not stall;
  //    an empty k-range contributes 0)
  const int rank = nsplit > 1 ? (int)cluster_rank() : 0;
  {
    const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
    const int R = warp * 32 + lane, s = R >> 4;
    const int owner = s % nsplit, li = s / nsplit;
    const int owned = (8 - owner + nsplit - 1) / nsplit;  // stripes the owner finishes
    const int drow = (rank * owned + li) * 16 + (R & 15);
    const uint32_t dst = smem_addr(recv + (size_t)drow * LDP);
    const bool have = ok && nk > 0;  // block-uniform
#pragma unroll 1
    for (int c = 0; c < N; c += GC) {  // one token group per wait, summed over accumulators
      uint32_t v[GC];
      if (have) {
#pragma unroll
        for (int j = 0; j < GC; j += 16) tmem_ld16(taddr + c + j, v + j);
#pragma unroll 1
        for (int q = 1; q < C::NAcc; ++q) {  // nk >= 4 >= NAcc: every accumulator written
          uint32_t u[GC];
#pragma unroll
          for (int j = 0; j < GC; j += 16) tmem_ld16(taddr + (uint32_t)(q * N) + c + j, u + j);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
          for (int j = 0; j < GC; ++j) v[j] += u[j];
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      } else {
#pragma unroll
        for (int j = 0; j < GC; ++j) v[j] = 0u;
      }
      if (nsplit > 1) {
#pragma unroll
        for (int j = 0; j < GC; j += 4)
          st_peer_v4(peer_addr(dst + (uint32_t)(c + j) * 4u, (uint32_t)owner),
                     make_int4((int)v[j], (int)v[j + 1], (int)v[j + 2], (int)v[j + 3]));
      } else {
#pragma unroll
        for (int j = 0; j < GC; j += 4)
          *reinterpret_cast<int4*>(recv + (size_t)drow * LDP + c + j) =
              make_int4((int)v[j], (int)v[j + 1], (int)v[j + 2], (int)v[j + 3]);
      }
    }
  }
  MC_TRACE_PHASE(a.trace_slot, 4, mc_tp);
  // 3) every push has landed
  if (nsplit > 1) cluster_sync_all(); else __syncthreads();
  MC_TRACE_PHASE(a.trace_slot, 5, mc_tp);
  // 4) this CTA finishes stripes rank, rank + nsplit, ...: the exact int32
  //    sum of the sources' rows (local shared memory) into slot 0, then the
  //    stripe epilogue of each token group
  unsigned long long kmax[(8 * kGroupTokens) / 32];
  const int owned = (8 - rank + nsplit - 1) / nsplit;
  constexpr int V4 = N / 4;  // 16-byte units per row
  for (int j = warp; j < owned; j += 4) {
    const int st_local = rank + j * nsplit;  // stripe within the tile
    const int stripe = tile * 8 + st_local;
    if (stripe >= a.n_stripes) break;  // warp-uniform
    int* rows0 = recv + (size_t)(j * 16) * LDP;  // slot 0 rows of this stripe
    if (nsplit > 1)
      for (int i = lane; i < 16 * V4; i += 32) {
        const int r = i / V4, c4 = i - r * V4;
        const size_t off = (size_t)r * LDP + c4 * 4;
        int4 acc = *reinterpret_cast<const int4*>(rows0 + off);
        for (int q = 1; q < nsplit; ++q) {
          const int4 v = *reinterpret_cast<const int4*>(recv + (size_t)((q * owned + j) * 16) * LDP + off);
          acc.x += v.x;
          acc.y += v.y;
          acc.z += v.z;
          acc.w += v.w;
        }
        *reinterpret_cast<int4*>(rows0 + off) = acc;
      }
    int* wsum = rows0;
    __syncwarp();
    if (ok) {
      for (int g = 0; g < G; ++g) {
        const int gm0 = g * kGroupTokens;
        if (gm0 >= a.M) break;  // warp-uniform
        const int MG = min(kGroupTokens, a.M - gm0);
#pragma unroll
        for (int i = 0; i < (8 * kGroupTokens) / 32; ++i) kmax[i] = 0ull;
        const EpiPre pre{row0, sm_scl, sm_w, sm_h, sm_cs, sm_sn};
        gemv_epilogue<6, EPI>(a, stripe, wsum + g * GC, LDP, lane, kmax, a.scale, sm_exp + gm0,
                              a.m0 + gm0, MG, EPI == EPI_QKV ? sm_tok + gm0 : nullptr, &pre);
        if constexpr (EPI == EPI_LMHEAD) {
#pragma unroll
          for (int it = 0; it < (8 * kGroupTokens) / 32; ++it) {
            unsigned long long k = kmax[it];
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
              unsigned long long k2 = __shfl_xor_sync(0xffffffffu, k, o);
              k = k2 > k ? k2 : k;
            }
            const int m = (it * 32 + lane) >> 3;
            if ((lane & 7) == 0 && m < MG && k) atomicMax(&sm_keys[gm0 + m], k);
          }
        }
      }
    }
    __syncwarp();
  }
  MC_TRACE_PHASE(a.trace_slot, 6, mc_tp);
  grid_launch_dependents();
  __syncthreads();
  MC_TRACE_PHASE(a.trace_slot, 7, mc_tp);
  if constexpr (EPI == EPI_LMHEAD) {
    if (threadIdx.x < a.M && sm_keys[threadIdx.x])
      atomicMax(a.keys + key_slot(a.seq, a.m0 + threadIdx.x), sm_keys[threadIdx.x]);
  }
  if constexpr (EPI == EPI_TP) tp_publish(a.tp);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(C::TmemCols)
                 : "memory");
  MC_TRACE_END(a.trace_slot);
}

// One 16-byte chunk per thread of the swizzled weight copy: (tile, atom,
// row r, stored chunk p) holds K bytes 16 (p ^ (r % 8)) .. + 16 of the atom;
// columns past the map (K padding) and padding rows are zero.
__global__ void k_pack_tc(const int8_t* __restrict__ src, long long src_ld,
                          const int* __restrict__ row_map, const int* __restrict__ col_map,
                          int n_cols, int n_rows, int n_tiles, int KA, int4* __restrict__ dst) {
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = (long long)n_tiles * KA * (kTcRows * 8);
  if (gid >= total) return;
  const int seg = (int)(gid % (kTcRows * 8));
  const long long ta = gid / (kTcRows * 8);
  const int atom = (int)(ta % KA), t = (int)(ta / KA);
  const int r = seg >> 3, lc = (seg & 7) ^ (r & 7);
  const int prow = t * kTcRows + r;
  const int row = prow < n_rows ? row_map[prow] : -1;
  uint32_t w[4] = {0, 0, 0, 0};
  if (row >= 0)
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int k = atom * 128 + lc * 16 + j;
      const int c = k < n_cols ? col_map[k] : -1;
      const uint32_t b = c >= 0 ? (uint8_t)src[(long long)row * src_ld + c] : 0u;
      w[j >> 2] |= b << (8 * (j & 3));
    }
  dst[gid] = make_int4((int)w[0], (int)w[1], (int)w[2], (int)w[3]);
}

cudaError_t launch_pack_tc(const int8_t* src, long long src_ld, const int* row_map,
                           const int* col_map, int n_rows, int n_tiles, int KB, int4* dst,
                           cudaStream_t s) {
  const int KA = tc_atoms(KB);
  const long long total = (long long)n_tiles * KA * (kTcRows * 8);
  k_pack_tc<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(src, src_ld, row_map, col_map, KB * 32,
                                                             n_rows, n_tiles, KA, dst);
  return cudaGetLastError();
}

template <int EPI, int G>
static cudaError_t launch_tc_t(const GemvArgs& a, int ksplit, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.n_stripes + 7) / 8, ksplit);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = TcCfg<G>::Smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;  // the k-splits of a tile
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = (unsigned)ksplit;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, k_gemm_tc<EPI, G>, a);
}

template <int G>
static cudaError_t launch_tc_g(const GemvArgs& a, int epi, int ksplit, cudaStream_t s, bool pdl) {
  switch (epi) {
    case EPI_STORE: return launch_tc_t<EPI_STORE, G>(a, ksplit, s, pdl);
    case EPI_RESID: return launch_tc_t<EPI_RESID, G>(a, ksplit, s, pdl);
    case EPI_SWIGLU: return launch_tc_t<EPI_SWIGLU, G>(a, ksplit, s, pdl);
    case EPI_QKV: return launch_tc_t<EPI_QKV, G>(a, ksplit, s, pdl);
    case EPI_LMHEAD: return launch_tc_t<EPI_LMHEAD, G>(a, ksplit, s, pdl);
    case EPI_TP: return launch_tc_t<EPI_TP, G>(a, ksplit, s, pdl);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_gemm_tc(const GemvArgs& a, int epi, int ksplit, cudaStream_t s, bool pdl) {
  if (!a.wtc || a.M > kMaxTokens || a.M < 1 || ksplit < 1 || ksplit > kTcMaxSplit)
    return cudaErrorInvalidValue;
  switch (groups_for_tokens(a.M)) {
    case 1: return launch_tc_g<1>(a, epi, ksplit, s, pdl);
    case 2: return launch_tc_g<2>(a, epi, ksplit, s, pdl);
    case 3: return launch_tc_g<3>(a, epi, ksplit, s, pdl);
    case 4: return launch_tc_g<4>(a, epi, ksplit, s, pdl);
  }
  return cudaErrorInvalidValue;
}

template <int G>
static cudaError_t prepare_tc_g() {
  for (auto f : {k_gemm_tc<EPI_STORE, G>, k_gemm_tc<EPI_RESID, G>, k_gemm_tc<EPI_SWIGLU, G>,
                 k_gemm_tc<EPI_QKV, G>, k_gemm_tc<EPI_LMHEAD, G>, k_gemm_tc<EPI_TP, G>}) {
    cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)TcCfg<G>::Smem);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t prepare_tc() {
  cudaError_t e = prepare_tc_g<1>();
  if (e == cudaSuccess) e = prepare_tc_g<2>();
  if (e == cudaSuccess) e = prepare_tc_g<3>();
  if (e == cudaSuccess) e = prepare_tc_g<4>();
  return e;
}

}  // namespace mc
