// bwd_sm100.cu — exact attention backward on the Blackwell tensor cores (tcgen05 + TMEM + TMA),
// deterministic: no atomics, every output element is produced by exactly one CTA in a fixed
// order (the decomposition of the reference, kernels/backward.hip:86-387).
//
//   dq kernel   : one CTA per 128-row query tile; loops over 64-key tiles
//                 S = Q K^T, dP = dO V^T (SS MMAs into TMEM, double-buffered);
//                 softmax warps (thread = query row) form dS = P (Z dP - dsum) (1 - tanh^2);
//                 dQ += dS K (TS MMA, dS read from TMEM).
//   dkdv kernel : one CTA per 128-key tile of one kv head; loops over every query head of the
//                 group and every 64-row query tile that can see the keys
//                 S^T = K Q^T, dP^T = V dO^T (SS), thread = key row forms P~^T = Z P^T and dS^T;
//                 dV += P~^T dO, dK += dS^T Q (TS).
// dS feeds its MMAs as a pair of 16-bit numbers hi + lo (lo = dS - hi), two MMAs each, so the
// 16-bit rounding of dS does not reach dQ/dK; P~ goes in as one 16-bit number.  The preprocess
// dsum = rowsum(O*dO) is the CUDA-core kernel of bwd_simt.cu.  Every mbarrier wait is bounded.
// Warp roles (320 threads): warps 0-7 elementwise, two per TMEM lane quadrant (w and w + 4 share
// the quadrant's 32 rows; w / 4 takes half of each 64-wide tile and D/2 output columns, and
// writes its packed P~ / dS into its own TMEM columns), warp 8 TMA, warp 9 MMA.
#include <cudaTypedefs.h>
#include <type_traits>
#include "fa_common.cuh"
#include "fa_launch.h"
#include "sm100_ptx.cuh"

namespace {

using namespace sm100;

constexpr int NTHREADS = 320;        // warps 0-7 elementwise (two per TMEM quadrant), 8 TMA, 9 MMA
constexpr int WARP_TMA = 8, WARP_MMA = 9, NELEM = 256;
__device__ int g_bwd_error = 0;
__device__ __forceinline__ void record_error(int code) { atomicOr(&g_bwd_error, code); }

// named barrier 1 over the 256 elementwise threads, AND-reducing a predicate (uniform break)
__device__ __forceinline__ bool bar_and_elem(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.and.pred po, 1, 256, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v)
      : "memory");
  return r != 0;
}

// 16-bit pair packing
template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (BF16) {
    const __nv_bfloat162 t = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&t);
  } else {
    const __half2 t = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&t);
  }
}
// the two floats a packed 16-bit pair holds (exact)
template <bool BF16>
__device__ __forceinline__ void unpack2(uint32_t w, float& a, float& b) {
  if constexpr (BF16) {
    a = __uint_as_float(w << 16);
    b = __uint_as_float(w & 0xffff0000u);
  } else {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
    a = f.x;
    b = f.y;
  }
}
// dS as hi + lo 16-bit pairs: hi = dS rounded, lo = the rounding remainder rounded (one packing
// conversion per pair for each; hi is read back from its packed bits)
template <bool BF16>
__device__ __forceinline__ void split2(float d0, float d1, uint32_t& hi, uint32_t& lo) {
  hi = pack2<BF16>(d0, d1);
  float h0, h1;
  unpack2<BF16>(hi, h0, h1);
  lo = pack2<BF16>(d0 - h0, d1 - h1);
}

// the same split for a pair held as float2: the remainder dS - hi (exact in fp32) by one FFMA2
template <bool BF16>
__device__ __forceinline__ void split2p(float2 d, uint32_t& hi, uint32_t& lo) {
  hi = pack2<BF16>(d.x, d.y);
  float h0, h1;
  unpack2<BF16>(hi, h0, h1);
  const float2 r = __ffma2_rn(make_float2(h0, h1), make_float2(-1.f, -1.f), d);
  lo = pack2<BF16>(r.x, r.y);
}

// Per-sequence geometry: dense uses the batch index z; varlen reads the token offsets and lengths
// of sequence z from cu_seqlens (clipped by seqused) and addresses the packed (total, H, D) rows.
struct BwdGeom {
  int SQ, SK;        // this sequence's lengths
  int qtok0, ktok0;  // first token of the sequence in the packed q / k (varlen), else 0
  int bcoord;        // batch coordinate of the 4-D TMA maps (0 for varlen)
};
__device__ __forceinline__ BwdGeom bwd_geom(const FaBwdParams& p, int z) {
  BwdGeom g{p.SQ, p.SK, 0, 0, z};
  if (p.cu_q) {
    g.qtok0 = p.cu_q[z];
    g.ktok0 = p.cu_k[z];
    g.SQ = p.cu_q[z + 1] - g.qtok0;
    g.SK = p.cu_k[z + 1] - g.ktok0;
    if (p.seqused_q && p.seqused_q[z] < g.SQ) g.SQ = p.seqused_q[z];
    if (p.seqused_k && p.seqused_k[z] < g.SK) g.SK = p.seqused_k[z];
    g.SQ = max(g.SQ, 0);
    g.SK = max(g.SK, 0);
    g.bcoord = 0;
  }
  return g;
}

// Varlen tiles can hold rows of the next sequence (or unused rows past seqused): the warp zeroes
// tile rows [r0, rows) of a [rows][D] tile (D/64 chunks of rows x 128 B) so that a probability or
// dS of 0 never meets a non-finite value in an MMA.  Generic-proxy stores, then the fence that
// makes them visible to the tensor core.
template <int D>
__device__ __forceinline__ void zero_tile_rows(uint8_t* tile, int rows, int r0, int lane) {
  constexpr int NCH = D / 64;
  for (int c = 0; c < NCH; ++c)   // rows [r0, rows) of every 64-column chunk, 16 bytes per lane
    for (int e = r0 * 8 + lane; e < rows * 8; e += 32)
      *reinterpret_cast<uint4*>(tile + c * rows * 128 + (e / 8) * 128 + (e % 8) * 16) = make_uint4(0, 0, 0, 0);
}

// K-major / MN-major descriptors of a [rows][D] tile stored as D/64 chunks of rows x 128 B
// (TMA SWIZZLE_128B boxes).  kstep = 16-element step along the contracted dimension.  The MMA
// issuers build the step-0 descriptor once and add each step's byte offset / 16 to it (the start
// address field holds address / 16 in 14 bits, and every shared-memory address stays below 2^18):
// the single issuing thread spends fewer instructions per MMA, which the short N = 64 MMAs need.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t tile, int rows, int kstep) {
  const int c = kstep / 4, off = (kstep % 4) * 32;
  return sdesc_sw128(tile + c * rows * 128 + off, 16, 1024);
}
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t tile, int rows, int kstep) {
  // contracted dim = rows: 16 rows per step; the D (N) dim spans chunks rows*128 bytes apart
  return sdesc_sw128(tile + kstep * 16 * 128, rows * 128, 1024);
}

// =====================================================================================
// dQ kernel
// =====================================================================================
template <int D>
struct DqCfg {
  static constexpr int BM = 128, BN = 64, NS = 4, NCH = D / 64;
  static constexpr int Q_BYTES = BM * D * 2, KV_BYTES = BN * D * 2;
  static constexpr int OFF_Q = 0, OFF_DO = Q_BYTES, OFF_K = 2 * Q_BYTES, OFF_V = OFF_K + NS * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + NS * KV_BYTES;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  // TMEM columns: S[2] at 0/64, dP[2] at 128/192, dQ at 256
  static constexpr uint32_t S_COL = 0, DP_COL = 128, DQ_COL = 256;
};
struct DqBars {
  static constexpr int Q_FULL = 0, K_FULL = 8, K_EMPTY = 40, V_FULL = 72, V_EMPTY = 104, SP_FULL = 136,
                       DS_FULL = 152, DQ_DONE = 168, DRAIN = 176, TMEM_ADDR = 184;
};

template <int D, bool BF16, bool FEAT>
__global__ void __launch_bounds__(NTHREADS, 1)
    bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                     const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                     const FaBwdParams p) {
  using C = DqCfg<D>;
  using Bz = DqBars;
  constexpr int BM = C::BM, BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  const uint32_t sQ = sbase + C::OFF_Q, sDO = sbase + C::OFF_DO, sK = sbase + C::OFF_K, sV = sbase + C::OFF_V;
  const uint32_t bar = sbase + C::OFF_BAR;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + C::OFF_BAR + Bz::TMEM_ADDR);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int z = blockIdx.z, h = blockIdx.y, kvh = h / p.gqa;
  const bool varlen = p.cu_q != nullptr;
  const BwdGeom g = bwd_geom(p, z);
  const int SQ = g.SQ, SK = g.SK;
  const int qb = (gridDim.x - 1 - blockIdx.x) * BM;
  if (qb >= SQ) return;

  int klo, khi, dmy;
  fa_key_range(qb, SQ, SK, p.causal, p.win_left, p.win_right, 0, klo, dmy);
  fa_key_range(min(qb + BM, SQ) - 1, SQ, SK, p.causal, p.win_left, p.win_right, 0, dmy, khi);
  klo = max(klo, 0);
  khi = min(khi, SK - 1);
  const int t0 = klo / BN;
  const int ntiles = (khi >= klo) ? (khi / BN - t0 + 1) : 0;

  if (tid == 0) {
    mbar_init(bar + Bz::Q_FULL, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(bar + Bz::K_FULL + 8 * s, 1);
      mbar_init(bar + Bz::K_EMPTY + 8 * s, 1);
      mbar_init(bar + Bz::V_FULL + 8 * s, 1);
      mbar_init(bar + Bz::V_EMPTY + 8 * s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar + Bz::SP_FULL + 8 * s, 1);
      mbar_init(bar + Bz::DS_FULL + 8 * s, NELEM);
    }
    mbar_init(bar + Bz::DQ_DONE, 1);
    mbar_init(bar + Bz::DRAIN, 1);
    fence_barrier_init();
  }
  if (warp == WARP_MMA) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == WARP_TMA) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && ntiles > 0) {
      mbar_expect_tx(bar + Bz::Q_FULL, 2 * C::Q_BYTES);
      for (int c = 0; c < C::NCH; ++c) {
        tma_load_4d(sQ + c * BM * 128, &tmQ, c * 64, g.qtok0 + qb, h, g.bcoord, bar + Bz::Q_FULL);
        tma_load_4d(sDO + c * BM * 128, &tmDO, c * 64, g.qtok0 + qb, h, g.bcoord, bar + Bz::Q_FULL);
      }
      for (int j = 0; j < ntiles; ++j) {
        const int s = j % C::NS, krow = g.ktok0 + (t0 + j) * BN;
        if (j >= C::NS && !mbar_wait(bar + Bz::K_EMPTY + 8 * s, ((j / C::NS) - 1) & 1)) { record_error(1); break; }
        mbar_expect_tx(bar + Bz::K_FULL + 8 * s, C::KV_BYTES);
        for (int c = 0; c < C::NCH; ++c)
          tma_load_4d(sK + s * C::KV_BYTES + c * BN * 128, &tmK, c * 64, krow, kvh, g.bcoord, bar + Bz::K_FULL + 8 * s);
        if (j >= C::NS && !mbar_wait(bar + Bz::V_EMPTY + 8 * s, ((j / C::NS) - 1) & 1)) { record_error(1); break; }
        mbar_expect_tx(bar + Bz::V_FULL + 8 * s, C::KV_BYTES);
        for (int c = 0; c < C::NCH; ++c)
          tma_load_4d(sV + s * C::KV_BYTES + c * BN * 128, &tmV, c * 64, krow, kvh, g.bcoord, bar + Bz::V_FULL + 8 * s);
      }
      for (int j = max(0, ntiles - C::NS); j < ntiles; ++j) {
        mbar_wait(bar + Bz::K_FULL + 8 * (j % C::NS), (j / C::NS) & 1);
        mbar_wait(bar + Bz::V_FULL + 8 * (j % C::NS), (j / C::NS) & 1);
      }
    }
    __syncwarp();
  } else if (warp == WARP_MMA) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t ID_S = idesc_f16(BF16 ? 1 : 0, BM, BN, 0, 0);   // S, dP: 128 x 64
    constexpr uint32_t ID_Q = idesc_f16(BF16 ? 1 : 0, BM, D, 0, 1);    // dQ += dS K: 128 x D, K MN-major
    bool ok = ntiles == 0 || mbar_wait_warp(bar + Bz::Q_FULL, 0);
    auto issue_dq = [&](int i) -> bool {
      if (!mbar_wait_warp(bar + Bz::DS_FULL + 8 * (i & 1), (i >> 1) & 1)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t kt = sK + (i % C::NS) * C::KV_BYTES;
        // dS of keys [32 hf, 32 hf + 32) sits packed in the first 16 columns of half hf's own
        // S (hi) and dP (lo) columns
        const uint32_t hi = tmem + C::S_COL + (i & 1) * 64, lo = tmem + C::DP_COL + (i & 1) * 64;
        const uint64_t bd0 = desc_mnmajor(kt, BN, 0);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t bd = desc_add(bd0, kk * 128);
          const uint32_t off = (uint32_t)(32 * (kk / 2) + 8 * (kk % 2));
          mma_ts(tmem + C::DQ_COL, hi + off, bd, ID_Q, (i > 0 || kk > 0) ? 1u : 0u);
          mma_ts(tmem + C::DQ_COL, lo + off, bd, ID_Q, 1u);
        }
        mma_commit(bar + Bz::K_EMPTY + 8 * (i % C::NS));
      }
      __syncwarp();
      return true;
    };
    for (int j = 0; ok && j < ntiles; ++j) {
      const int s = j % C::NS;
      if (!mbar_wait_warp(bar + Bz::K_FULL + 8 * s, (j / C::NS) & 1) ||
          !mbar_wait_warp(bar + Bz::V_FULL + 8 * s, (j / C::NS) & 1)) { ok = false; break; }
      const int kb = (t0 + j) * BN;
      if (varlen && kb + BN > SK) {   // key rows past the sequence: zero (dQ += dS K reads K)
        zero_tile_rows<D>(sgen + C::OFF_K + s * C::KV_BYTES, BN, max(SK - kb, 0), lane);
        zero_tile_rows<D>(sgen + C::OFF_V + s * C::KV_BYTES, BN, max(SK - kb, 0), lane);
        fence_proxy_async_smem();
        __syncwarp();
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t kt = sK + s * C::KV_BYTES, vt = sV + s * C::KV_BYTES;
        const uint64_t aq = desc_kmajor(sQ, BM, 0), ado = desc_kmajor(sDO, BM, 0), bk = desc_kmajor(kt, BN, 0),
                       bv = desc_kmajor(vt, BN, 0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t oa = (uint32_t)(((kk / 4) * BM * 128 + (kk % 4) * 32) >> 4);
          const uint32_t ob = (uint32_t)(((kk / 4) * BN * 128 + (kk % 4) * 32) >> 4);
          mma_ss(tmem + C::S_COL + (j & 1) * 64, desc_add(aq, oa), desc_add(bk, ob), ID_S, kk > 0);
          mma_ss(tmem + C::DP_COL + (j & 1) * 64, desc_add(ado, oa), desc_add(bv, ob), ID_S, kk > 0);
        }
        mma_commit(bar + Bz::SP_FULL + 8 * (j & 1));
        mma_commit(bar + Bz::V_EMPTY + 8 * s);
      }
      __syncwarp();
      if (j >= 1 && !issue_dq(j - 1)) { ok = false; break; }
    }
    if (ok && ntiles > 0 && !issue_dq(ntiles - 1)) ok = false;
    if (!ok) record_error(2);
    if (lane == 0) { mma_commit(bar + Bz::DQ_DONE); mma_commit(bar + Bz::DRAIN); }
    __syncwarp();
    if (!mbar_wait_warp(bar + Bz::DRAIN, 0)) record_error(4);
  } else {
    // ------------------------------------------------------------ elementwise (thread = query row)
    // warps w and w + 4 share query rows 32 (w%4) .. + 31; w / 4 picks the half of the 64-key tile
    // (32 keys) and of the dQ row (D/2 columns) the thread owns
    const int qd = warp & 3, hf = warp >> 2;
    const int q = qb + qd * 32 + lane;
    const uint32_t la = tmem + ((uint32_t)(qd * 32) << 16);
    int rlo, rhi;
    fa_key_range(q, SQ, SK, p.causal, p.win_left, p.win_right, 0, rlo, rhi);
    float lse2 = 0.f, dsum = 0.f;
    if (q < SQ) {
      const long long li = fa_lse_index(varlen, z, h, p.Hq, p.SQ, g.qtok0, p.lse_total_q, q);
      lse2 = p.lse[li] * FA_LOG2E;
      dsum = p.dsum[li];
      if (!(lse2 > -INFINITY)) { rlo = 1; rhi = 0; }   // row saw no key in the forward
    } else {
      rlo = 1; rhi = 0;
    }
    const float slope = (FEAT && p.alibi) ? p.alibi[h] : 0.f;
    const bool drop = FEAT && p.dropout;
    const bool use_bits = drop && p.dropout_bits != nullptr;
    const int mask_w = (SK + 31) / 32;
    const uint32_t thresh = fa_drop_thresh(p.dropout_p);
    const bool cap_on = FEAT && p.softcap > 0.f;
    const float cap_in = cap_on ? p.scale / p.softcap : 0.f;
    // packed path (no softcap, no alibi): x = s * scale*log2e + nl2 with nl2 = -lse2, or -inf for a
    // row that saw no key (so its P is 0 without a test); key masks only on boundary tiles
    const bool fast = !cap_on && slope == 0.f;
    const float sl2 = p.scale * FA_LOG2E;
    const float nl2 = (rlo <= rhi) ? -lse2 : -INFINITY, nds = -dsum;
    int lo_last = 1, hi_first = 0;   // key tiles every row of the CTA sees in full
    {
      int a, b;
      fa_key_range(min(qb + BM, SQ) - 1, SQ, SK, p.causal, p.win_left, p.win_right, 0, lo_last, a);
      fa_key_range(qb, SQ, SK, p.causal, p.win_left, p.win_right, 0, b, hi_first);
    }
    const bool full_rows = qb + BM <= SQ;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int kb = (t0 + j) * BN + 32 * hf;   // first key of this thread's half
      // keep bits of this row for the half (bit b <-> key kb + b), prepared ahead of the wait:
      // loaded from the mask (coalesced over rows) or evaluated with Philox
      uint32_t dw[1];
      {
        const int kw = kb / 32;
        dw[0] = 0u;
        if (drop && q < SQ && kw < mask_w)
          dw[0] = use_bits ? __ldg(p.dropout_bits + fa_mask_word(h, SQ, SK, q, kw))
                           : fa_keep_word(p.drop_seed, ((uint64_t)h * SQ + q) * SK + 32 * kw, 1, thresh,
                                          SK - 32 * kw);
      }
      if (!mbar_wait_warp(bar + Bz::SP_FULL + 8 * (j & 1), (j >> 1) & 1)) { ok = false; break; }
      tc_fence_after();
      float s[32], dp[32];
      tmem_ld32(la + C::S_COL + (j & 1) * 64 + 32 * hf, s);
      tmem_ld32(la + C::DP_COL + (j & 1) * 64 + 32 * hf, dp);
      tc_wait_ld();
      const float d0 = (float)(kb - q);   // key - q = d0 + cc, exact in fp32
      // dS = P o (Z dP - dsum) o dlogit/ds, with Z the keep multiplier; one unrolled body per
      // softcap setting so that neither carries the other's code
      auto body = [&](auto cap_tag) {
        constexpr bool kCap = decltype(cap_tag)::value;
        {   // the half's 32 keys -> 16 packed columns of hi and of lo; inputs in registers
          constexpr int h32 = 0;
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            float dsv[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int cc = h32 + c + u, key = kb + cc;
              float logit, deriv = 1.f;
              if constexpr (kCap) {
                const float tn = fa_tanh_tc<BF16>(s[cc] * cap_in);
                logit = fmaf(p.softcap, tn, slope * (d0 + (float)cc));
                deriv = 1.f - tn * tn;
              } else if constexpr (FEAT) {
                logit = fmaf(s[cc], p.scale, slope * (d0 + (float)cc));
              } else {
                logit = s[cc] * p.scale;
              }
              const float pr = (key >= rlo && key <= rhi) ? ex2(fmaf(logit, FA_LOG2E, -lse2)) : 0.f;
              const float zm = drop ? (((dw[cc / 32] >> (cc % 32)) & 1u) ? p.keep_scale : 0.f) : 1.f;
              dsv[u] = pr * (zm * dp[cc] - dsum) * deriv;
            }
            split2<BF16>(dsv[0], dsv[1], hi[c / 2], lo[c / 2]);
          }
          tmem_st16(la + C::S_COL + (j & 1) * 64 + 32 * hf, hi);
          tmem_st16(la + C::DP_COL + (j & 1) * 64 + 32 * hf, lo);
        }
      };
      // packed body, one straight-line instantiation per (dropout, boundary tile) pair
      auto fast_body = [&](auto drop_tag, auto mask_tag) {
        constexpr bool kDrop = decltype(drop_tag)::value, kMask = decltype(mask_tag)::value;
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const float2 x = __ffma2_rn(make_float2(s[c], s[c + 1]), make_float2(sl2, sl2), make_float2(nl2, nl2));
          float a = ex2(x.x), b = ex2(x.y);
          if constexpr (kMask) {
            a = (kb + c >= rlo && kb + c <= rhi) ? a : 0.f;
            b = (kb + c + 1 >= rlo && kb + c + 1 <= rhi) ? b : 0.f;
          }
          const float2 dp2 = make_float2(dp[c], dp[c + 1]);
          float2 dsv;
          if constexpr (kDrop) {   // dS = P (Z dP - D) = (Z P) dP - P D, Z P by a sign-extended keep bit
            const uint32_t m0 = (uint32_t)((int32_t)(dw[0] << (31 - c)) >> 31);
            const uint32_t m1 = (uint32_t)((int32_t)(dw[0] << (30 - c)) >> 31);
            const float2 zp = __fmul2_rn(make_float2(__uint_as_float(__float_as_uint(a) & m0),
                                                     __uint_as_float(__float_as_uint(b) & m1)),
                                         make_float2(p.keep_scale, p.keep_scale));
            dsv = __ffma2_rn(make_float2(a, b), make_float2(nds, nds), __fmul2_rn(zp, dp2));
          } else {
            dsv = __fmul2_rn(make_float2(a, b), __fadd2_rn(dp2, make_float2(nds, nds)));
          }
          split2p<BF16>(dsv, hi[c / 2], lo[c / 2]);
        }
        tmem_st16(la + C::S_COL + (j & 1) * 64 + 32 * hf, hi);
        tmem_st16(la + C::DP_COL + (j & 1) * 64 + 32 * hf, lo);
      };
      if (fast) {
        const int kt = (t0 + j) * BN;
        const bool interior = full_rows && kt >= lo_last && kt + BN - 1 <= hi_first && kt + BN <= SK;
        if (drop) {
          if (interior) fast_body(std::true_type{}, std::false_type{});
          else fast_body(std::true_type{}, std::true_type{});
        } else {
          if (interior) fast_body(std::false_type{}, std::false_type{});
          else fast_body(std::false_type{}, std::true_type{});
        }
      } else if constexpr (FEAT) {
        if (cap_on) body(std::true_type{});
        else body(std::false_type{});
      }
      tc_wait_st();
      tc_fence_before();
      mbar_arrive(bar + Bz::DS_FULL + 8 * (j & 1));
    }
    if (!ok) record_error(8);
    const bool have = ok && ntiles > 0;
    if (have && !mbar_wait_warp(bar + Bz::DQ_DONE, 0)) record_error(16);
    tc_fence_after();
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    T* qrow = (T*)p.dQ + (varlen ? (long long)g.qtok0 * p.dqs.s : (long long)z * p.dqs.b) + (long long)h * p.dqs.h +
              (long long)q * p.dqs.s + hf * (D / 2);
#pragma unroll
    for (int c = 0; c < D / 2; c += 32) {
      float o[32];
      if (have) {
        tmem_ld32(la + C::DQ_COL + hf * (D / 2) + c, o);
        tc_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0.f;
      }
      if (q < SQ) {
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = pack2<BF16>(o[2 * i] * p.scale, o[2 * i + 1] * p.scale);
        uint4* dst = reinterpret_cast<uint4*>(qrow + c);
        // 8-column units; columns at or past the real head_dim are padding (never stored)
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (hf * (D / 2) + c + 8 * i < p.D) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// =====================================================================================
// dK / dV kernel
// =====================================================================================
template <int D>
struct DkvCfg {
  static constexpr int BK = 128, BQ = 64, NS = 3, NCH = D / 64;
  static constexpr int KV_BYTES = BK * D * 2, QT_BYTES = BQ * D * 2;
  static constexpr int OFF_K = 0, OFF_V = KV_BYTES, OFF_Q = 2 * KV_BYTES, OFF_DO = OFF_Q + NS * QT_BYTES;
  static constexpr int OFF_ST = OFF_DO + NS * QT_BYTES;      // lse2 / dsum per query tile: [2][2][64] f32
  static constexpr int OFF_BAR = OFF_ST + 2 * 2 * 64 * 4;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  // TMEM: dV [0,128), dK [128,256), S^T[2] at 256/320, dP^T[2] at 384/448
  static constexpr uint32_t DV_COL = 0, DK_COL = 128, S_COL = 256, DP_COL = 384;
};
struct DkvBars {
  static constexpr int KV_FULL = 0, Q_FULL = 8, Q_EMPTY = 40, SP_FULL = 72, DS_FULL = 88, DONE = 104,
                       DRAIN = 112, TMEM_ADDR = 120;
};

template <int D, bool BF16, bool FEAT>
__global__ void __launch_bounds__(NTHREADS, 1)
    bwd_dkdv_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                       const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                       const FaBwdParams p) {
  using C = DkvCfg<D>;
  using Bz = DkvBars;
  constexpr int BK = C::BK, BQ = C::BQ;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  const uint32_t sK = sbase + C::OFF_K, sV = sbase + C::OFF_V, sQ = sbase + C::OFF_Q, sDO = sbase + C::OFF_DO;
  float* st = reinterpret_cast<float*>(sgen + C::OFF_ST);   // [buf][lse2|dsum][64]
  const uint32_t bar = sbase + C::OFF_BAR;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + C::OFF_BAR + Bz::TMEM_ADDR);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int z = blockIdx.z, kvh = blockIdx.y;
  const bool varlen = p.cu_q != nullptr;
  const BwdGeom g = bwd_geom(p, z);
  const int SQ = g.SQ, SK = g.SK;
  const int kb = blockIdx.x * BK;
  if (kb >= SK) return;

  // query rows that can see a key of [kb, kb+BK): same bounds as the CUDA-core kernel
  const int delta = SK - SQ, kend = min(kb + BK, SK) - 1;
  int qstart = 0, qend = SQ - 1;
  if (p.causal) qstart = max(qstart, kb - delta);
  if (p.win_right >= 0) qstart = max(qstart, kb - delta - p.win_right);
  if (p.win_left >= 0) qend = min(qend, kend - delta + p.win_left);
  const int qt0 = qstart / BQ;
  const int nqt = (qend >= qstart) ? (qend / BQ - qt0 + 1) : 0;
  const int niter = nqt * p.gqa;   // (query head of the group, query tile) pairs, head-major

  if (tid == 0) {
    mbar_init(bar + Bz::KV_FULL, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(bar + Bz::Q_FULL + 8 * s, 1);
      mbar_init(bar + Bz::Q_EMPTY + 8 * s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar + Bz::SP_FULL + 8 * s, 1);
      mbar_init(bar + Bz::DS_FULL + 8 * s, NELEM);
    }
    mbar_init(bar + Bz::DONE, 1);
    mbar_init(bar + Bz::DRAIN, 1);
    fence_barrier_init();
  }
  if (warp == WARP_MMA) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == WARP_TMA) {
    if (lane == 0 && niter > 0) {
      mbar_expect_tx(bar + Bz::KV_FULL, 2 * C::KV_BYTES);
      for (int c = 0; c < C::NCH; ++c) {
        tma_load_4d(sK + c * BK * 128, &tmK, c * 64, g.ktok0 + kb, kvh, g.bcoord, bar + Bz::KV_FULL);
        tma_load_4d(sV + c * BK * 128, &tmV, c * 64, g.ktok0 + kb, kvh, g.bcoord, bar + Bz::KV_FULL);
      }
      for (int i = 0; i < niter; ++i) {
        const int s = i % C::NS, h = kvh * p.gqa + i / nqt, qrow = g.qtok0 + (qt0 + i % nqt) * BQ;
        if (i >= C::NS && !mbar_wait(bar + Bz::Q_EMPTY + 8 * s, ((i / C::NS) - 1) & 1)) { record_error(1); break; }
        mbar_expect_tx(bar + Bz::Q_FULL + 8 * s, 2 * C::QT_BYTES);
        for (int c = 0; c < C::NCH; ++c) {
          tma_load_4d(sQ + s * C::QT_BYTES + c * BQ * 128, &tmQ, c * 64, qrow, h, g.bcoord, bar + Bz::Q_FULL + 8 * s);
          tma_load_4d(sDO + s * C::QT_BYTES + c * BQ * 128, &tmDO, c * 64, qrow, h, g.bcoord, bar + Bz::Q_FULL + 8 * s);
        }
      }
      for (int i = max(0, niter - C::NS); i < niter; ++i) mbar_wait(bar + Bz::Q_FULL + 8 * (i % C::NS), (i / C::NS) & 1);
    }
    __syncwarp();
  } else if (warp == WARP_MMA) {
    constexpr uint32_t ID_S = idesc_f16(BF16 ? 1 : 0, BK, BQ, 0, 0);   // S^T, dP^T: 128 x 64
    constexpr uint32_t ID_O = idesc_f16(BF16 ? 1 : 0, BK, D, 0, 1);    // dV, dK: 128 x D, B MN-major
    bool ok = niter == 0 || mbar_wait_warp(bar + Bz::KV_FULL, 0);
    auto issue_kv = [&](int i) -> bool {
      if (!mbar_wait_warp(bar + Bz::DS_FULL + 8 * (i & 1), (i >> 1) & 1)) return false;
      tc_fence_after();
      if (lane == 0) {
        const int s = i % C::NS;
        const uint32_t qt = sQ + s * C::QT_BYTES, dot = sDO + s * C::QT_BYTES;
        // half hf (query rows [32 hf, 32 hf + 32)) keeps, in its own 32 S^T columns, P~^T packed at
        // [0,16) and dS^T hi at [16,32), and dS^T lo in the first 16 of its dP^T columns
        const uint32_t pb = tmem + C::S_COL + (i & 1) * 64, lo = tmem + C::DP_COL + (i & 1) * 64;
        const uint64_t mdo = desc_mnmajor(dot, BQ, 0), mq = desc_mnmajor(qt, BQ, 0);
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {
          const uint32_t off = (uint32_t)(32 * (kk / 2) + 8 * (kk % 2));
          const uint32_t step = (uint32_t)(kk * 128);
          mma_ts(tmem + C::DV_COL, pb + off, desc_add(mdo, step), ID_O, (i > 0 || kk > 0) ? 1u : 0u);
          mma_ts(tmem + C::DK_COL, pb + 16 + off, desc_add(mq, step), ID_O, (i > 0 || kk > 0) ? 1u : 0u);
          mma_ts(tmem + C::DK_COL, lo + off, desc_add(mq, step), ID_O, 1u);
        }
        mma_commit(bar + Bz::Q_EMPTY + 8 * s);
      }
      __syncwarp();
      return true;
    };
    for (int i = 0; ok && i < niter; ++i) {
      const int s = i % C::NS;
      if (!mbar_wait_warp(bar + Bz::Q_FULL + 8 * s, (i / C::NS) & 1)) { ok = false; break; }
      const int qbase = (qt0 + i % nqt) * BQ;
      if (varlen && qbase + BQ > SQ) {   // query rows past the sequence: zero (dV, dK sum over rows)
        zero_tile_rows<D>(sgen + C::OFF_Q + s * C::QT_BYTES, BQ, max(SQ - qbase, 0), lane);
        zero_tile_rows<D>(sgen + C::OFF_DO + s * C::QT_BYTES, BQ, max(SQ - qbase, 0), lane);
        fence_proxy_async_smem();
        __syncwarp();
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t qt = sQ + s * C::QT_BYTES, dot = sDO + s * C::QT_BYTES;
        const uint64_t ak = desc_kmajor(sK, BK, 0), av = desc_kmajor(sV, BK, 0), bq = desc_kmajor(qt, BQ, 0),
                       bdo = desc_kmajor(dot, BQ, 0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t oa = (uint32_t)(((kk / 4) * BK * 128 + (kk % 4) * 32) >> 4);
          const uint32_t ob = (uint32_t)(((kk / 4) * BQ * 128 + (kk % 4) * 32) >> 4);
          mma_ss(tmem + C::S_COL + (i & 1) * 64, desc_add(ak, oa), desc_add(bq, ob), ID_S, kk > 0);
          mma_ss(tmem + C::DP_COL + (i & 1) * 64, desc_add(av, oa), desc_add(bdo, ob), ID_S, kk > 0);
        }
        mma_commit(bar + Bz::SP_FULL + 8 * (i & 1));
      }
      __syncwarp();
      if (i >= 1 && !issue_kv(i - 1)) { ok = false; break; }
    }
    if (ok && niter > 0 && !issue_kv(niter - 1)) ok = false;
    if (!ok) record_error(32);
    if (lane == 0) { mma_commit(bar + Bz::DONE); mma_commit(bar + Bz::DRAIN); }
    __syncwarp();
    if (!mbar_wait_warp(bar + Bz::DRAIN, 0)) record_error(64);
  } else {
    // ------------------------------------------------------------ elementwise (thread = key row)
    // warps w and w + 4 share keys kb + 32 (w%4) .. + 31; w / 4 picks the half of the 64-row query
    // tile (32 rows) and of the dK / dV rows (D/2 columns) the thread owns
    const int qd = warp & 3, hf = warp >> 2;
    const int key = kb + qd * 32 + lane;
    const uint32_t la = tmem + ((uint32_t)(qd * 32) << 16);
    const bool drop = FEAT && p.dropout;
    const bool use_bits = drop && p.dropout_bits != nullptr;
    const bool use_bits_t = use_bits && p.dropout_bits_t != nullptr;   // key-major copy, no transpose
    const uint32_t thresh = fa_drop_thresh(p.dropout_p);
    const bool cap_on = FEAT && p.softcap > 0.f;
    const float cap_in = cap_on ? p.scale / p.softcap : 0.f;
    // the warp's 32 keys are one mask word column (kb is a multiple of 128)
    const int kw = kb / 32 + qd;
    const bool kw_ok = kw < (SK + 31) / 32;
    // query rows that see this key (empty for keys past SK)
    int qlo, qhi;
    fa_query_range(key, SQ, SK, p.causal, p.win_left, p.win_right, qlo, qhi);
    if (key >= SK) { qlo = 1; qhi = 0; }
    // query tiles every key of the CTA sees in full (the ranges grow with the key)
    int qlo_last, qhi_first, qd0, qd1;
    fa_query_range(min(kb + BK, SK) - 1, SQ, SK, p.causal, p.win_left, p.win_right, qlo_last, qd0);
    fa_query_range(kb, SQ, SK, p.causal, p.win_left, p.win_right, qd1, qhi_first);
    const bool full_keys = kb + BK <= SK;
    const float sl2 = p.scale * FA_LOG2E;
    bool ok = true;
    for (int i = 0; i < niter; ++i) {
      const int h = kvh * p.gqa + i / nqt, qbase = (qt0 + i % nqt) * BQ;
      // keep bits of this key over the half's query rows: cw[0] bit r <-> row qbase + 32hf + r.
      // From the mask, lane l loads the word of row qbase + 32hf + l (one line per warp) and a
      // ballot transpose after the wait turns rows-of-keys into keys-of-rows; without a mask,
      // Philox is evaluated here, down the key's column (counter stride SK).
      uint32_t cw[1];
      {
        constexpr int hq = 0;
        const int q0 = qbase + 32 * hf;
        cw[hq] = 0u;
        if (use_bits_t) {   // this key's word over the half's 32 rows (q0 is a multiple of 32)
          if (key < SK && q0 < SQ)
            cw[hq] = __ldg(p.dropout_bits_t + ((long long)h * ((SQ + 31) / 32) + q0 / 32) * SK + key);
        } else if (use_bits) {
          if (kw_ok && q0 + lane < SQ) cw[hq] = __ldg(p.dropout_bits + fa_mask_word(h, SQ, SK, q0 + lane, kw));
        } else if (drop && key < SK && q0 < SQ) {
          cw[hq] = fa_keep_word(p.drop_seed, ((uint64_t)h * SQ + q0) * SK + key, (uint64_t)SK, thresh, SQ - q0);
        }
      }
      float* stb = st + (i & 1) * 128;
      // this tile's lse2 / dsum (threads 0-63 and 64-127); the named barrier publishes them to the
      // 8 warps and AND-reduces the wait outcome, so a timeout ends every warp at the same point
      if (tid < 128) {
        const int qi = tid & 63, q = qbase + qi;
        float v = 0.f;
        if (q < SQ) {
          const long long li = fa_lse_index(varlen, z, h, p.Hq, p.SQ, g.qtok0, p.lse_total_q, q);
          if (tid < 64) {
            const float l = p.lse[li];
            v = (l > -INFINITY) ? -l * FA_LOG2E : -INFINITY;
          } else {
            v = -p.dsum[li];
          }
        } else if (tid < 64) {
          v = -INFINITY;
        }
        stb[(tid < 64 ? 0 : 64) + qi] = v;   // [nl2 = -lse2 or -inf | nds = -dsum]
      }
      const bool got = mbar_wait_warp(bar + Bz::SP_FULL + 8 * (i & 1), (i >> 1) & 1);
      if (!bar_and_elem(got)) { ok = false; break; }
      tc_fence_after();
      float s[32], dp[32];
      tmem_ld32(la + C::S_COL + (i & 1) * 64 + 32 * hf, s);
      tmem_ld32(la + C::DP_COL + (i & 1) * 64 + 32 * hf, dp);
      tc_wait_ld();
      if (use_bits && !use_bits_t) {   // warp-uniform: every lane takes part in the ballots
        {
          constexpr int hq = 0;
          uint32_t t = 0u;
#pragma unroll
          for (int b = 0; b < 32; ++b) {
            const uint32_t m = __ballot_sync(0xffffffffu, (cw[hq] >> b) & 1u);   // rows keeping key 32kw + b
            t = (lane == b) ? m : t;
          }
          cw[hq] = t;
        }
      }
      const float slope = (FEAT && p.alibi) ? p.alibi[h] : 0.f;
      const int qh = qbase + 32 * hf;          // first query row of this thread's half
      const float d0 = (float)(key - qh);      // key - q = d0 - cc, exact in fp32
      auto body = [&](auto cap_tag) {
        constexpr bool kCap = decltype(cap_tag)::value;
        {   // the half's 32 query rows; inputs are all in registers: in-place outputs are safe
          constexpr int h32 = 0;
          uint32_t pk[16], hi[16], lo[16];
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            float pv[2], dsv[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int cc = h32 + c + u, q = qh + cc;
              const float nl2 = stb[32 * hf + cc];
              const bool vis = q >= qlo && q <= qhi && nl2 > -INFINITY;
              float logit, deriv = 1.f;
              if constexpr (kCap) {
                const float tn = fa_tanh_tc<BF16>(s[cc] * cap_in);
                logit = fmaf(p.softcap, tn, slope * (d0 - (float)cc));
                deriv = 1.f - tn * tn;
              } else if constexpr (FEAT) {
                logit = fmaf(s[cc], p.scale, slope * (d0 - (float)cc));
              } else {
                logit = s[cc] * p.scale;
              }
              const float pr = vis ? ex2(fmaf(logit, FA_LOG2E, nl2)) : 0.f;
              const bool kept = !drop || ((cw[h32 / 32] >> (c + u)) & 1u);
              const float zm = drop ? (kept ? p.keep_scale : 0.f) : 1.f;
              pv[u] = kept ? pr : 0.f;   // Z P unscaled: dV gets 1/(1-p) in fp32 (epilogue)
              dsv[u] = pr * (zm * dp[cc] + stb[64 + 32 * hf + cc]) * deriv;
            }
            pk[c / 2] = pack2<BF16>(pv[0], pv[1]);
            split2<BF16>(dsv[0], dsv[1], hi[c / 2], lo[c / 2]);
          }
          tmem_st16(la + C::S_COL + (i & 1) * 64 + 32 * hf, pk);
          tmem_st16(la + C::S_COL + (i & 1) * 64 + 32 * hf + 16, hi);
          tmem_st16(la + C::DP_COL + (i & 1) * 64 + 32 * hf, lo);
        }
      };
      // packed path: nl2 = -inf for rows that saw no key, query masks only on boundary tiles; one
      // straight-line instantiation per (dropout, boundary tile) pair
      auto fast_body = [&](auto drop_tag, auto mask_tag) {
        constexpr bool kDrop = decltype(drop_tag)::value, kMask = decltype(mask_tag)::value;
        uint32_t pk[16], hi[16], lo[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const float2 nl2 = *reinterpret_cast<const float2*>(stb + 32 * hf + c);
          const float2 nds = *reinterpret_cast<const float2*>(stb + 64 + 32 * hf + c);
          const float2 x = __ffma2_rn(make_float2(s[c], s[c + 1]), make_float2(sl2, sl2), nl2);
          float a = ex2(x.x), b = ex2(x.y);
          if constexpr (kMask) {
            a = (qh + c >= qlo && qh + c <= qhi) ? a : 0.f;
            b = (qh + c + 1 >= qlo && qh + c + 1 <= qhi) ? b : 0.f;
          }
          const float2 pr = make_float2(a, b), dp2 = make_float2(dp[c], dp[c + 1]);
          float2 pm = pr, dsv;
          if constexpr (kDrop) {   // Z P by a sign-extended keep bit; dS = (Z P / (1-p)) dP - P D
            const uint32_t m0 = (uint32_t)((int32_t)(cw[0] << (31 - c)) >> 31);
            const uint32_t m1 = (uint32_t)((int32_t)(cw[0] << (30 - c)) >> 31);
            pm = make_float2(__uint_as_float(__float_as_uint(a) & m0), __uint_as_float(__float_as_uint(b) & m1));
            dsv = __ffma2_rn(pr, nds, __fmul2_rn(__fmul2_rn(pm, make_float2(p.keep_scale, p.keep_scale)), dp2));
          } else {
            dsv = __fmul2_rn(pr, __fadd2_rn(dp2, nds));
          }
          pk[c / 2] = pack2<BF16>(pm.x, pm.y);   // Z P unscaled: dV gets 1/(1-p) in fp32 (epilogue)
          split2p<BF16>(dsv, hi[c / 2], lo[c / 2]);
        }
        tmem_st16(la + C::S_COL + (i & 1) * 64 + 32 * hf, pk);
        tmem_st16(la + C::S_COL + (i & 1) * 64 + 32 * hf + 16, hi);
        tmem_st16(la + C::DP_COL + (i & 1) * 64 + 32 * hf, lo);
      };
      if (!cap_on && slope == 0.f) {
        const bool interior = full_keys && qbase >= qlo_last && qbase + BQ - 1 <= qhi_first && qbase + BQ <= SQ;
        if (drop) {
          if (interior) fast_body(std::true_type{}, std::false_type{});
          else fast_body(std::true_type{}, std::true_type{});
        } else {
          if (interior) fast_body(std::false_type{}, std::false_type{});
          else fast_body(std::false_type{}, std::true_type{});
        }
      } else if constexpr (FEAT) {
        if (cap_on) body(std::true_type{});
        else body(std::false_type{});
      }
      tc_wait_st();
      tc_fence_before();
      mbar_arrive(bar + Bz::DS_FULL + 8 * (i & 1));
    }
    if (!ok) record_error(128);
    const bool have = ok && niter > 0;
    if (have && !mbar_wait_warp(bar + Bz::DONE, 0)) record_error(256);
    tc_fence_after();
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    T* vrow = (T*)p.dV + (varlen ? (long long)g.ktok0 * p.dvs.s : (long long)z * p.dvs.b) + (long long)kvh * p.dvs.h +
              (long long)key * p.dvs.s + hf * (D / 2);
    T* krow = (T*)p.dK + (varlen ? (long long)g.ktok0 * p.dks.s : (long long)z * p.dks.b) + (long long)kvh * p.dks.h +
              (long long)key * p.dks.s + hf * (D / 2);
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      const uint32_t col = (part == 0 ? C::DV_COL : C::DK_COL) + hf * (D / 2);
      const float mul = part == 0 ? (drop ? p.keep_scale : 1.f) : p.scale;
      T* row = part == 0 ? vrow : krow;
#pragma unroll
      for (int c = 0; c < D / 2; c += 32) {
        float o[32];
        if (have) {
          tmem_ld32(la + col + c, o);
          tc_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (key < SK) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = pack2<BF16>(o[2 * i] * mul, o[2 * i + 1] * mul);
          uint4* dst = reinterpret_cast<uint4*>(row + c);
          // 8-column units; columns at or past the real head_dim are padding (never stored)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (hf * (D / 2) + c + 8 * i < p.D) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 bwd_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)ptr;
  }
  return fn;
}

bool map4(CUtensorMap* m, const void* base, bool bf16, long long D, long long S, long long H, long long B,
          const FaStrides& st, int box_rows) {
  auto enc = bwd_encode_fn();
  if (!enc || ((uintptr_t)base) % 16) return false;
  const long long sb = (B > 1) ? st.b : ((st.s * S > st.h * H ? st.s * S : st.h * H) + 7) / 8 * 8;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)st.s * 2, (cuuint64_t)st.h * 2, (cuuint64_t)sb * 2};
  for (int i = 0; i < 3; ++i)
    if (strides[i] % 16 || strides[i] >= (1ull << 40)) return false;
  const cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base),
             dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool out_ok(const void* ptr, const FaStrides& s, int B) {
  return ((uintptr_t)ptr) % 16 == 0 && s.s % 8 == 0 && s.h % 8 == 0 && (B <= 1 || s.b % 8 == 0);
}

template <int D, bool BF16, bool FEAT>
int launch_all(const FaBwdParams& p, cudaStream_t st, const CUtensorMap* maps) {
  const CUtensorMap &mq128 = maps[0], &mdo128 = maps[1], &mk64 = maps[2], &mv64 = maps[3];
  const CUtensorMap &mq64 = maps[4], &mdo64 = maps[5], &mk128 = maps[6], &mv128 = maps[7];
  using Cq = DqCfg<D>;
  using Ck = DkvCfg<D>;
  static unsigned long long done_q = 0, done_k = 0;
  if (int rc = fa::ensure_smem((const void*)bwd_dq_tc_kernel<D, BF16, FEAT>, Cq::SMEM, &done_q)) return rc;
  if (int rc = fa::ensure_smem((const void*)bwd_dkdv_tc_kernel<D, BF16, FEAT>, Ck::SMEM, &done_k)) return rc;
  bwd_dkdv_tc_kernel<D, BF16, FEAT><<<dim3((p.SK + Ck::BK - 1) / Ck::BK, p.Hk, p.B), NTHREADS, Ck::SMEM, st>>>(
      mq64, mdo64, mk128, mv128, p);
  bwd_dq_tc_kernel<D, BF16, FEAT><<<dim3((p.SQ + Cq::BM - 1) / Cq::BM, p.Hq, p.B), NTHREADS, Cq::SMEM, st>>>(
      mq128, mdo128, mk64, mv64, p);
  fa::count_launch(2);
  return fa::cuda_status(cudaGetLastError(), "bwd_sm100 launch");
}

template <bool BF16, bool FEAT>
int launch_d(const FaBwdParams& p, cudaStream_t st, const CUtensorMap* maps) {
  return p.D <= 64 ? launch_all<64, BF16, FEAT>(p, st, maps) : launch_all<128, BF16, FEAT>(p, st, maps);
}

}  // namespace

namespace fa {

// fp16/bf16, dense or varlen, head_dim a multiple of 16 up to 128 (tiles of 64 or 128 columns,
// the columns past head_dim zero-filled by the TMA), 16-byte aligned rows: dsum on the CUDA
// cores, then the dK/dV and dQ tensor-core kernels.  Anything else: *taken = false.
int bwd_sm100(const FaBwdParams& p, int dtype, cudaStream_t st, bool* taken) {
  *taken = false;
  if (p.D % 16 != 0 || p.D < 16 || p.D > 128 || dtype == FA_DTYPE_F32) return FA_OK;
  if (getenv("FABLE_ATTN_DISABLE_TC")) return FA_OK;
  int dev = current_device(), major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) return FA_OK;
  const bool bf16 = dtype == FA_DTYPE_BF16;
  const bool varlen = p.cu_q != nullptr;
  // varlen tensors are (total, H, D): 4-D maps with one batch entry whose rows are the packed
  // tokens, bounded by the true row counts (rows past the last token read as zeros)
  if (varlen && (p.lse_total_q <= 0 || p.total_k <= 0)) return FA_OK;
  const long long rq = varlen ? p.lse_total_q : p.SQ, rk = varlen ? p.total_k : p.SK;
  const int nb = varlen ? 1 : p.B;
  CUtensorMap maps[8];
  if (!map4(&maps[0], p.Q, bf16, p.D, rq, p.Hq, nb, p.qs, 128) ||
      !map4(&maps[1], p.dO, bf16, p.D, rq, p.Hq, nb, p.dos, 128) ||
      !map4(&maps[2], p.K, bf16, p.D, rk, p.Hk, nb, p.ks, 64) ||
      !map4(&maps[3], p.V, bf16, p.D, rk, p.Hk, nb, p.vs, 64) ||
      !map4(&maps[4], p.Q, bf16, p.D, rq, p.Hq, nb, p.qs, 64) ||
      !map4(&maps[5], p.dO, bf16, p.D, rq, p.Hq, nb, p.dos, 64) ||
      !map4(&maps[6], p.K, bf16, p.D, rk, p.Hk, nb, p.ks, 128) ||
      !map4(&maps[7], p.V, bf16, p.D, rk, p.Hk, nb, p.vs, 128))
    return FA_OK;
  if (!out_ok(p.dQ, p.dqs, nb) || !out_ok(p.dK, p.dks, nb) || !out_ok(p.dV, p.dvs, nb)) return FA_OK;
  *taken = true;
  if (int rc = bwd_dsum(p, dtype, st)) return rc;
  if (p.dropout && p.dropout_bits && p.dropout_bits_t)
    if (int rc = dropout_mask_transpose(p.dropout_bits, p.dropout_bits_t, p.Hq, p.SQ, p.SK, p.causal,
                                          p.win_left, p.win_right, st)) return rc;
  const bool feat = p.softcap > 0.f || p.alibi != nullptr || p.dropout;
  if (bf16) return feat ? launch_d<true, true>(p, st, maps) : launch_d<true, false>(p, st, maps);
  return feat ? launch_d<false, true>(p, st, maps) : launch_d<false, false>(p, st, maps);
}

int bwd_device_error(int clear) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_bwd_error, sizeof(int));
  if (clear) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_bwd_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace fa
