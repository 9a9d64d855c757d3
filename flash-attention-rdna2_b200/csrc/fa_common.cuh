// fa_common.cuh — shared device helpers of the sm_100a attention engine: element conversions,
// the Philox4x32-10 dropout generator, per-sequence geometry (dense / varlen) and the
// host-side launch bookkeeping used by every kernel file.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <math.h>
#include "fable_attn.h"

#include <utility>

// ---------------------------------------------------------------- programmatic dependent launch
// A kernel launched with fa::launch_pdl may start while the kernel before it on the stream is
// still finishing: pdl_wait() returns once that kernel has completed and its writes are visible
// (a no-op after a plain launch), and pdl_trigger() lets the next kernel start early (it still
// waits in its own pdl_wait() before reading anything this kernel writes).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

#define FA_LOG2E 1.4426950408889634f
#define FA_LN2 0.6931471805599453f

// ---------------------------------------------------------------- element conversions
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

// ---------------------------------------------------------------- Philox4x32-10 dropout
// Counter-based generator keyed by the 64-bit seed, counter = (idx lo, idx hi, 0, 0); round
// multipliers 0xD2511F53 / 0xCD9E8D57, key increments 0x9E3779B9 / 0xBB67AE85 (the published
// Philox4x32 constants, Salmon et al. 2011).  Only the first output word decides the keep bit,
// exactly as kernels/fa_common.hpp:71-88 of the reference:  u = (r0 >> 8) / 2^24,
// keep iff u >= p.
__host__ __device__ __forceinline__ uint32_t fa_philox_r0(uint64_t seed, uint64_t idx) {
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
  uint32_t c0 = (uint32_t)idx, c1 = (uint32_t)(idx >> 32), c2 = 0u, c3 = 0u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    // each 32 x 32 -> 64-bit product as one wide multiply (hi and lo halves from one instruction)
    const uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
    const uint32_t hi0 = (uint32_t)(p0 >> 32), hi1 = (uint32_t)(p1 >> 32);
    const uint32_t lo0 = (uint32_t)p0, lo1 = (uint32_t)p1;
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
    k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
  }
  return c0;
}
// multiplier applied to a kept probability: inv_keep if kept, 0 if dropped
__host__ __device__ __forceinline__ float fa_dropout_mul(uint64_t seed, uint64_t idx, float p,
                                                         float inv_keep) {
  const float u = (float)(fa_philox_r0(seed, idx) >> 8) * (1.0f / 16777216.0f);
  return (u >= p) ? inv_keep : 0.0f;
}

// Integer form of the keep test: u = (r0 >> 8) / 2^24 >= p  <=>  (r0 >> 8) >= ceil(p * 2^24).
// Both sides of the float test are exact (r0 >> 8 < 2^24 and scaling by 2^-24 is exact), and
// p * 2^24 is exact in fp32, so the two tests decide identically.  Result in 1 .. 2^24.
__host__ __device__ __forceinline__ uint32_t fa_drop_thresh(float p) {
  return (uint32_t)ceilf(p * 16777216.0f);
}

// Keep bits of the Philox counters base + b*stride, b = 0..31 (bit b set iff that score is
// kept); bits b >= nvalid are 0.  Not inlined: the attention kernels call it once per 32
// scores, and a single copy keeps their unrolled element loops small.  The 32 evaluations are
// independent and are issued 8 at a time to keep the integer pipes busy.
static __device__ __noinline__ uint32_t fa_keep_word(uint64_t seed, uint64_t base, uint64_t stride, uint32_t thresh,
                                              int nvalid) {
  uint32_t word = 0;
#pragma unroll 1
  for (int b0 = 0; b0 < 32; b0 += 8) {
    uint32_t r[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) r[u] = fa_philox_r0(seed, base + (uint64_t)(b0 + u) * stride);
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if ((r[u] >> 8) >= thresh && b0 + u < nvalid) word |= 1u << (b0 + u);
  }
  return word;
}

// index of the keep-mask word holding keys [32*kw, 32*kw + 31] of query row q of head h: the
// fa_dropout_mask_launch layout [NH][ceil(SK/32)][SQ], query row fastest
__host__ __device__ __forceinline__ long long fa_mask_word(int h, int SQ, int SK, int q, int kw) {
  return ((long long)h * ((SK + 31) / 32) + kw) * SQ + q;
}

// keep multiplier of score (q, k) of query head h: from the precomputed bit mask when given,
// else Philox evaluated here; both give the same decision
__device__ __forceinline__ float fa_keep_mul(const unsigned int* bits, uint64_t seed, int h, int SQ, int SK, int q,
                                             int k, float p, float inv_keep) {
  if (bits) return ((bits[fa_mask_word(h, SQ, SK, q, k / 32)] >> (k % 32)) & 1u) ? inv_keep : 0.0f;
  return fa_dropout_mul(seed, ((uint64_t)h * SQ + q) * SK + k, p, inv_keep);
}

// ---------------------------------------------------------------- sequence geometry
// Resolves, for batch index / sequence z, the lengths and the element offsets of row 0 of the
// q / k / o tensors.  Dense: offsets from the batch stride.  Varlen: token offsets from
// cu_seqlens (the batch stride is ignored) and lengths clipped by seqused.
struct SeqGeom {
  int SQ, SK;
  long long q0, k0, v0, o0;   // element offsets of row 0 (head 0)
  long long tok_q;            // first token index of this sequence in the packed q (varlen), else 0
};

__device__ __forceinline__ SeqGeom fa_seq_geom(int z, int SQd, int SKd, const int* cu_q, const int* cu_k,
                                               const int* su_q, const int* su_k, const FaStrides& sq,
                                               const FaStrides& sk, const FaStrides& sv,
                                               const FaStrides& so) {
  SeqGeom g;
  if (cu_q) {
    const int qs = cu_q[z], ks = cu_k[z];
    g.SQ = cu_q[z + 1] - qs;
    g.SK = cu_k[z + 1] - ks;
    if (su_q) { const int u = su_q[z]; if (u < g.SQ) g.SQ = u; }
    if (su_k) { const int u = su_k[z]; if (u < g.SK) g.SK = u; }
    if (g.SQ < 0) g.SQ = 0;
    if (g.SK < 0) g.SK = 0;
    g.q0 = (long long)qs * sq.s; g.k0 = (long long)ks * sk.s; g.v0 = (long long)ks * sv.s;
    g.o0 = (long long)qs * so.s; g.tok_q = qs;
  } else {
    g.SQ = SQd; g.SK = SKd;
    g.q0 = (long long)z * sq.b; g.k0 = (long long)z * sk.b; g.v0 = (long long)z * sv.b;
    g.o0 = (long long)z * so.b; g.tok_q = 0;
  }
  return g;
}

// Cache row of key position k of sequence z in a paged K/V (FaFwdParams block_table): page
// block_table[z][k / page], slot k % page.  Positions past the table's row and invalid entries
// give row k % page of page 0; `bad` is set for an invalid entry of a real key (k < SK).
__device__ __forceinline__ long long fa_paged_row(const FaFwdParams& p, int z, int k, int SK, bool& bad) {
  const int pi = k / p.page;
  long long blk = 0;
  bad = false;
  if (pi < p.max_blocks) {
    blk = p.block_table[(long long)z * p.max_blocks + pi];
    if (blk < 0 || blk >= p.num_blocks) {
      bad = k < SK;
      blk = 0;
    }
  }
  return blk * p.page + k % p.page;
}

// LSE / dsum row address: dense [batch, NH, SQ]; varlen [NH, total_q]
__device__ __forceinline__ long long fa_lse_index(bool varlen, int z, int h, int NH, int SQd,
                                                  long long tok_q, long long total_q, int q) {
  return varlen ? (long long)h * total_q + tok_q + q : ((long long)z * NH + h) * SQd + q;
}

// Key range [lo, hi] that query row q may see (bottom-right aligned masks).  Returns lo > hi
// when the row sees nothing.  Chunk handling follows kernels/fa_forward.hip:227-234.
__host__ __device__ __forceinline__ void fa_key_range(int q, int SQ, int SK, int causal, int wl,
                                                      int wr, int chunk, int& lo, int& hi) {
  const int diag = q + SK - SQ;
  lo = 0; hi = SK - 1;
  if (causal && diag < hi) hi = diag;
  if (wl >= 0 && diag - wl > lo) lo = diag - wl;
  if (wr >= 0 && diag + wr < hi) hi = diag + wr;
  if (chunk > 0) {
    int pp = diag < 0 ? 0 : diag;
    const int cs = (pp / chunk) * chunk;
    if (cs > lo) lo = cs;
    if (cs + chunk - 1 < hi) hi = cs + chunk - 1;
  }
}

// Query rows [qlo, qhi] that see key k under (causal, wl, wr), without attention chunks: the
// inverse of fa_key_range.  Row q's diagonal is key q + SK - SQ, so with off = SQ - SK
//   causal: k <= q - off    <=>  q >= k + off
//   wl>=0:  k >= diag - wl  <=>  q <= k + wl + off
//   wr>=0:  k <= diag + wr  <=>  q >= k - wr + off
// Empty when qlo > qhi.  Computed in 64 bits and clamped to [0, SQ] / [-1, SQ-1].
__host__ __device__ __forceinline__ void fa_query_range(int k, int SQ, int SK, int causal, int wl, int wr,
                                                        int& qlo, int& qhi) {
  const long long off = (long long)SQ - SK;
  long long lo = 0, hi = SQ - 1;
  if (causal && k + off > lo) lo = k + off;
  if (wr >= 0 && k - wr + off > lo) lo = k - wr + off;
  if (wl >= 0 && k + wl + off < hi) hi = k + wl + off;
  qlo = (int)(lo > SQ ? SQ : lo);
  qhi = (int)(hi < -1 ? -1 : hi);
}

// tanh from the identity tanh x = 1 - 2 / (e^(2x) + 1), with e^(2x) = 2^(2x log2 e) on the SFU.
// The exponent is clamped so the power stays finite (tanh is 1 in fp32 long before); below, the
// power flushes to 0 and the result is -1.  Absolute error is a few ulp of 1, which is what the
// softcapped logit cap * tanh(.) needs: its error is then a few ulp of cap.
__device__ __forceinline__ float fa_tanh(float x) {
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(fminf(2.f * FA_LOG2E * x, 64.f)));
  return 1.f - __fdividef(2.f, e + 1.f);
}

// Softcap tanh of the tensor-core kernels: bf16 requests use the SFU's tanh (tanh.approx.f32, one
// SFU operation, relative error below 2^-10.9): with the logit capped at c the error is at most
// c * |tanh| * 2^-10.9, a few 1e-4 of a probability, inside bf16's 2.5e-3 rel_rms budget and
// half the SFU work of fa_tanh (exponential + reciprocal).  fp16 requests (a 3e-4 budget) keep
// fa_tanh.  Forward and backward use the same one, so the backward's recomputed probabilities
// match the forward's LSE.
template <bool BF16>
__device__ __forceinline__ float fa_tanh_tc(float x) {
  if constexpr (BF16) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
  } else {
    return fa_tanh(x);
  }
}

// ---------------------------------------------------------------- host bookkeeping
namespace fa {
void set_error(const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);
void count_launch(unsigned n = 1);
int num_sms();
}  // namespace fa

#define FA_CHECK_ARG(cond, ...)             \
  do {                                      \
    if (!(cond)) {                          \
      fa::set_error(__VA_ARGS__);           \
      return FA_ERR_INVALID;                \
    }                                       \
  } while (0)

namespace fa {
bool pdl_enabled();
// cudaLaunchKernelEx with programmatic stream serialization (a plain launch when disabled)
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
}  // namespace fa
