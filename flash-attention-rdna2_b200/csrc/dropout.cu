// dropout.cu — the dropout keep mask as bits (see fa_dropout_mask_launch in fable_attn.h).
//
// One thread per 32-bit word = 32 consecutive keys of one (head, query row); consecutive threads
// take consecutive query rows, so stores are coalesced in the [NH][ceil(SK/32)][SQ] layout.  The
// 32 Philox evaluations of a word are independent and are issued 4 at a time.  The keep decision
// is the reference's (kernels/fa_common.hpp:71-88), u = (r0 >> 8) / 2^24, keep iff u >= p,
// evaluated as the equivalent integer test r0 >= fa_drop_thresh(p) * 2^8.  Words that hold no key
// the row can see (causal / window) are skipped: no consumer reads them.
//
// The kernel is bound by the integer multiply pipe: a Philox4x32-10 draw is ~17 32 x 32 -> 64-bit
// products (two integer-multiply instructions each) plus the XORs, and with every product on the
// integer multiplier that pipe ran 91 % busy while issue ran at 64 %.  So the high halves of the
// M0 products of rounds 1-9 come from the otherwise idle fp64 pipe instead (philox_r0_split); the
// draw is the same function, bit for bit, as fa_philox_r0.
#include "fa_common.cuh"
#include "fa_launch.h"

#include <cstdlib>

namespace {

constexpr uint32_t kPhiloxM0 = 0xD2511F53u, kPhiloxM1 = 0xCD9E8D57u;

// High 32 bits of M * x for the 32-bit x: with the double 2^52 + x (its bit pattern is x below the
// exponent of 2^52), fma_rd(M * 2^-32, 2^52 + x, 2^52 - M * 2^20) = 2^52 + M * x / 2^32 rounded
// down.  The fused product and sum are exact, and the exact result lies in [2^52, 2^53), where
// doubles are the integers, so rounding down gives 2^52 + floor(M * x / 2^32) exactly; its low
// 32 bits are the high half of the product.
__device__ __forceinline__ uint32_t mulhi_fp64(double m_scaled, double bias, uint32_t x) {
  return (uint32_t)__double2loint(__fma_rd(m_scaled, __hiloint2double(0x43300000, (int)x), bias));
}

// fa_philox_r0(seed, (c1 << 32) | c0): Philox4x32-10, first output word, with the M0 products'
// high halves of rounds 1-9 by mulhi_fp64 and their low halves by a 32-bit multiply (the M1
// products stay 64-bit integer products).  Moving more products measured slower: the kernel
// becomes issue bound.
__device__ __forceinline__ uint32_t philox_r0_split(uint64_t seed, uint32_t c0, uint32_t c1) {
  const double m0s = (double)kPhiloxM0 * 0x1p-32, bias0 = 0x1p52 - (double)kPhiloxM0 * 0x1p20;
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32), c2 = 0u, c3 = 0u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = mulhi_fp64(m0s, bias0, c0), lo0 = c0 * kPhiloxM0;
    const uint64_t p1 = (uint64_t)kPhiloxM1 * c2;
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0; c1 = (uint32_t)p1; c2 = n2; c3 = lo0;
    k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
  }
  return c0;
}

// Draws in flight per thread: 4 measured 0.675 ms on config 3's mask against 0.700 for 8 (the
// integer form was flat from 2 to 32); 16 and 32 were slower (0.82, 0.87 ms).
constexpr int MASK_DRAWS = 4;

// Keep bits of counters base .. base + 31 (bit b set iff draw base + b is kept), bits b >= nvalid
// cleared.  WIDE: counters may exceed 2^32 (64-bit counter per draw); otherwise the high counter
// word is 0 for every draw of the launch.
template <bool WIDE>
__device__ __forceinline__ uint32_t keep_word_split(uint64_t seed, uint64_t base, uint32_t thr8, int nvalid) {
  uint32_t word = 0;
#pragma unroll 1
  for (int b0 = 0; b0 < 32; b0 += MASK_DRAWS) {
    uint32_t r[MASK_DRAWS];
#pragma unroll
    for (int u = 0; u < MASK_DRAWS; ++u) {
      const uint64_t idx = base + (uint64_t)(b0 + u);
      r[u] = philox_r0_split(seed, (uint32_t)idx, WIDE ? (uint32_t)(idx >> 32) : 0u);
    }
#pragma unroll
    for (int u = 0; u < MASK_DRAWS; ++u)
      if (r[u] >= thr8) word |= 1u << (b0 + u);
  }
  return nvalid >= 32 ? word : word & ((1u << nvalid) - 1u);
}

// thr8 = fa_drop_thresh(p) << 8 (fits: p < 1 gives a threshold below 2^24)
template <bool WIDE>
__global__ void __launch_bounds__(256) dropout_mask_kernel(unsigned long long seed, unsigned int thr8, int NH,
                                                           int SQ, int SK, int causal, int wl, int wr,
                                                           unsigned int* bits) {
  const int W = (SK + 31) / 32;
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = (long long)NH * SQ * W;
  if (gid >= total) return;
  const int q = (int)(gid % SQ);
  const long long hw = gid / SQ;            // h*W + kw
  const int kw = (int)(hw % W), h = (int)(hw / W);
  int lo, hi;
  fa_key_range(q, SQ, SK, causal, wl, wr, 0, lo, hi);
  const int k0 = kw * 32;
  if (hi < k0 || lo > k0 + 31 || lo > hi) return;
  bits[gid] = keep_word_split<WIDE>(seed, ((uint64_t)h * SQ + q) * SK + k0, thr8, SK - k0);
}

// One warp per 32 x 32 block (32 query rows x 32 keys): lane l reads the row-major word of row
// 32 qw + l, a 32 x 32 bit transpose across the warp turns rows-of-keys into keys-of-rows, lane b
// writes the word of key 32 kw + b.  The transpose swaps, for each bit j of the index (16, 8, 4, 2,
// 1), the off-diagonal j x j sub-blocks between lanes l and l ^ j: the lane without bit j keeps its
// bits whose index lacks bit j and takes its partner's such bits shifted up by j; the lane with bit
// j keeps its bits whose index has bit j and takes its partner's shifted down by j (five shuffles
// instead of 32 ballots).
// Each warp takes T_BLOCKS consecutive query blocks of one key word and issues their loads before
// the first shuffle (one 128-byte line per lane and block in flight left HBM at 1.6 TB/s).  Warps
// run query blocks fastest, so reads and writes are 128-byte lines.  Blocks whose 32 rows see
// none of the word's keys (causal / window) are neither read nor written: the mask kernel did not
// write them and the dK/dV kernel masks those scores to zero probability whatever their bits.
// IDX: the integer type of the warp index (32-bit whenever the count fits, so that the per-warp
// index split is not a 64-bit division)
constexpr int T_BLOCKS = 4;

template <typename IDX>
__global__ void __launch_bounds__(256) dropout_mask_t_kernel(const unsigned int* __restrict__ bits,
                                                             unsigned int* __restrict__ bits_t, int NH, int SQ,
                                                             int SK, int causal, int wl, int wr) {
  const IDX W = (SK + 31) / 32, QW = (SQ + 31) / 32, QG = (QW + T_BLOCKS - 1) / T_BLOCKS;
  const IDX wid = ((IDX)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= (IDX)NH * W * QG) return;   // whole warps
  const int qg = (int)(wid % QG);
  const IDX hk = wid / QG;
  const int kw = (int)(hk % W), h = (int)(hk / W);
  const int k0 = kw * 32;
  unsigned int t[T_BLOCKS], live = 0;
#pragma unroll
  for (int i = 0; i < T_BLOCKS; ++i) {
    const int q = (qg * T_BLOCKS + i) * 32 + lane;
    bool sees = false;
    if (q < SQ) {
      int lo, hi;
      fa_key_range(q, SQ, SK, causal, wl, wr, 0, lo, hi);
      sees = !(hi < k0 || lo > k0 + 31 || lo > hi);
    }
    if (__ballot_sync(0xffffffffu, sees)) live |= 1u << i;
    t[i] = (q < SQ && ((live >> i) & 1u)) ? bits[((long long)h * W + kw) * SQ + q] : 0u;
  }
  // bits whose index lacks bit j: 0x0000FFFF, 0x00FF00FF, 0x0F0F0F0F, 0x33333333, 0x55555555
  const unsigned int lo_mask[5] = {0x0000FFFFu, 0x00FF00FFu, 0x0F0F0F0Fu, 0x33333333u, 0x55555555u};
  const int k = k0 + lane;
#pragma unroll
  for (int i = 0; i < T_BLOCKS; ++i) {
    if (!((live >> i) & 1u)) continue;   // warp-uniform
    unsigned int v = t[i];
#pragma unroll
    for (int s = 0, j = 16; s < 5; ++s, j >>= 1) {
      const unsigned int m = lo_mask[s], o = __shfl_xor_sync(0xffffffffu, v, j);
      v = (lane & j) ? ((v & ~m) | ((o & ~m) >> j)) : ((v & m) | ((o & m) << j));
    }
    if (k < SK) bits_t[((long long)h * QW + qg * T_BLOCKS + i) * SK + k] = v;
  }
}

}  // namespace

namespace fa {

int dropout_mask_transpose(const unsigned int* bits, unsigned int* bits_t, int NH, int SQ, int SK, int causal,
                           int wl, int wr, cudaStream_t st) {
  const long long qg = ((SQ + 31) / 32 + T_BLOCKS - 1) / T_BLOCKS;
  const long long warps = (long long)NH * ((SK + 31) / 32) * qg;
  if (warps == 0) return FA_OK;
  const long long blocks = (warps + 7) / 8;
  if (blocks >= (1ll << 31)) {
    set_error("dropout mask transpose: %lld blocks is too large", blocks);
    return FA_ERR_SIZE;
  }
  if (blocks * 256 < (1ll << 32))
    dropout_mask_t_kernel<unsigned int><<<(unsigned)blocks, 256, 0, st>>>(bits, bits_t, NH, SQ, SK, causal, wl, wr);
  else
    dropout_mask_t_kernel<unsigned long long><<<(unsigned)blocks, 256, 0, st>>>(bits, bits_t, NH, SQ, SK, causal, wl,
                                                                               wr);
  count_launch();
  return cuda_status(cudaGetLastError(), "dropout mask transpose launch");
}

}  // namespace fa

extern "C" FA_API long long fa_dropout_mask_words(int NH, int SQ, int SK) {
  if (NH <= 0 || SQ <= 0 || SK <= 0) return 0;
  return (long long)NH * SQ * ((SK + 31) / 32);
}

extern "C" FA_API int fa_dropout_mask_launch(unsigned long long seed, float p, int NH, int SQ, int SK, int causal,
                                             int win_left, int win_right, unsigned int* bits, void* stream) {
  if (!bits) {
    fa::set_error("dropout mask: null output");
    return FA_ERR_INVALID;
  }
  if (!(p > 0.f && p < 1.f) || NH <= 0 || SQ < 0 || SK < 0) {
    fa::set_error("dropout mask: p=%f NH=%d SQ=%d SK=%d", p, NH, SQ, SK);
    return FA_ERR_INVALID;
  }
  const long long total = fa_dropout_mask_words(NH, SQ, SK);
  if (total == 0) return FA_OK;
  const long long blocks = (total + 255) / 256;
  if (blocks >= (1ll << 31)) {
    fa::set_error("dropout mask: %lld words is too large", total);
    return FA_ERR_SIZE;
  }
  const unsigned int thr8 = fa_drop_thresh(p) << 8;
  // 32-bit counters when every counter drawn, at most (NH*SQ - 1)*SK + ceil(SK/32)*32 - 1, is
  // below 2^32; FABLE_ATTN_MASK_WIDE forces the 64-bit form (a test hook: both give the same bits)
  const bool wide = (unsigned long long)NH * SQ * ((SK + 31) / 32 * 32) > (1ull << 32) ||
                    getenv("FABLE_ATTN_MASK_WIDE") != nullptr;
  if (wide)
    dropout_mask_kernel<true><<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(seed, thr8, NH, SQ, SK, causal,
                                                                               win_left, win_right, bits);
  else
    dropout_mask_kernel<false><<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(seed, thr8, NH, SQ, SK, causal,
                                                                                win_left, win_right, bits);
  fa::count_launch();
  return fa::cuda_status(cudaGetLastError(), "dropout mask launch");
}
