// fwd_sm100.cu — exact attention forward on the Blackwell tensor cores (tcgen05 + TMEM + TMA).
//
// Two kernels.  fwd_tc_kernel (below) works on one 128-row query tile at a time and takes every
// feature (softcap, alibi, dropout, varlen, paged K/V, in-kernel rotary of Q, every head_dim: tiles
// of 64, 128 or 256 columns with the columns past head_dim zero-filled by the TMA);
// fwd_pp_kernel (further down) takes two query tiles per CTA for dense head_dim-128 requests
// without softcap / alibi (dropout from a precomputed mask), and is chosen when its half-as-many
// CTAs do not cost whole waves (launch_d).
//
// fwd_tc_kernel: persistent, one CTA per SM walking the work items (a 128-row query tile of one
// head of one sequence) heavy first; the pipelines run on across items (short items, as under a
// sliding window, would otherwise pay their prologue and pipeline fill each time).  With rotary,
// the softmax warps first rotate each Q tile in shared memory.  Warp roles (320 threads):
//   warps 0-7  softmax: warps w and w+4 share query rows 32 (w%4) .. +31 (their TMEM lane
//              quadrant); w / 4 picks the half of each S row (64 keys) and of each O row (D/2
//              columns) the thread owns.  Each thread reads its half row of S from TMEM, applies
//              masks / softcap / alibi / dropout, agrees on the row max with its partner through
//              shared memory (a 64-thread named barrier per quadrant), keeps the online-softmax
//              state (lazy rescale: the reference max only moves when it grows by > 2^8), writes
//              P as packed 16-bit pairs into the first 32 columns of its own half, and finally
//              normalises its half of O and writes O and LSE.  Two softmax warps per scheduler
//              keep the exponentials of two half rows in flight; the scale / subtract and the
//              row sums run as packed fp32x2 operations.
//   warp 8     TMA producer: per item its Q tile (double-buffered), then its K and V tiles
//              (128 keys x D) into separate rings.
//   warp 9     MMA issuer: owns the TMEM allocation; S_j = Q K_j^T into one of two S buffers
//              (SS form), then O += P_j V_j with P read from TMEM (TS form).
// TMEM columns: S0 [0,128), S1 [128,256), O [256, 256+D).  K/V tiles are 128-byte swizzled
// (TMA SWIZZLE_128B, one 64-column box per 128-byte row chunk); S uses K-major Q and K operands,
// PV uses an MN-major V operand.  Every mbarrier wait is bounded: on timeout the CTA records an
// error (fa_device_error) and unwinds without touching TMEM or smem further.
//
// Semantics are identical to the CUDA-core kernel (fwd_simt.cu) and to the reference's forward
// (kernels/fa_forward.hip:52-313): bottom-right causal / window / chunk masks, softcap, signed
// alibi without diagonal offset, Philox dropout keyed (h*SQ+q)*SK+key, LSE in natural log,
// empty rows -> O = 0 and LSE = -inf.
#include <cudaTypedefs.h>
#include <algorithm>
#include <type_traits>
#include "fa_common.cuh"
#include "fa_launch.h"
#include "sm100_ptx.cuh"

namespace {

using namespace sm100;

constexpr int BM = 128, BN = 128;
constexpr int NSOFT = 256;                         // softmax threads: 8 warps, two per TMEM quadrant
constexpr int WARP_TMA = 8, WARP_MMA = 9, NTHREADS = 320;
constexpr float LAZY_THRESH = 8.0f;   // log2 units: rescale O only when the max grows by > 2^8
// named barrier `id` over the two softmax warps of one TMEM quadrant: AND of a predicate
// (uniform loop exits) and a plain sync (the row-max exchange)
__device__ __forceinline__ bool bar_and_pair(uint32_t id, bool v) {
  uint32_t r;
  asm volatile("{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %2, 0;\n\tbar.red.and.pred po, %1, 64, pi;\n\t"
               "selp.u32 %0, 1, 0, po;\n\t}"
               : "=r"(r) : "r"(id), "r"((uint32_t)v) : "memory");
  return r != 0;
}
__device__ __forceinline__ void bar_sync_pair(uint32_t id) { asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory"); }

__device__ int g_fwd_error = 0;       // non-zero after a pipeline wait timed out

// D is the tile width (64, 128 or 256); the request's head_dim p.HD may be smaller (a multiple of
// 16): the TMA maps span only p.HD columns, so the columns past it land as zeros (adding nothing
// to Q.K^T and giving zero O columns), and the epilogue stores only the real columns.
// D is the tile width (64, 128 or 256); the request's head_dim p.HD may be smaller (a multiple of
// 16): the TMA maps span only p.HD columns, so the columns past it land as zeros (adding nothing
// to Q.K^T and giving zero O columns), and the epilogue stores only the real columns.
template <int D>
struct Cfg {
  static constexpr int NQB = (D <= 128) ? 2 : 1;                   // Q buffers (next item's Q prefetched)
  static constexpr int NSK = (D <= 64) ? 4 : (D <= 128 ? 2 : 1);   // K ring depth (freed after S)
  static constexpr int NSV = (D <= 64) ? 4 : (D <= 128 ? 2 : 1);   // V ring depth (freed after PV)
  static constexpr int NCH = D / 64;                           // 64-column (128-byte) chunks per row
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;                  // one K (or V) tile
  static constexpr int CH_BYTES = BN * 128;                    // one 64-column chunk of a tile
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = NQB * Q_BYTES;
  static constexpr int OFF_V = OFF_K + NSK * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + NSV * KV_BYTES;
  static constexpr int OFF_X = OFF_BAR + 256;                  // row-max / row-sum exchange
  static constexpr int SMEM = OFF_X + 6 * BM * 4 + 1024;       // + alignment slack
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t O_COL = 256;
  static_assert(SMEM <= 232448, "shared memory per CTA");
  static_assert(O_COL + D <= TMEM_COLS, "S double buffer and O must fit in TMEM");
};

struct Bars {   // mbarrier offsets inside the barrier block (8 bytes each; rings of up to 4)
  static constexpr int Q_FULL = 0, Q_EMPTY = 16, Q_ROT = 32,   // [Q buffer]; Q_ROT: rotated (rotary only)
                       K_FULL = 48, K_EMPTY = 80, V_FULL = 112, V_EMPTY = 144, S_FULL = 176, P_FULL = 192,
                       O_DONE = 208, MMA_DRAIN = 216, TMEM_ADDR = 224;
};

__device__ __forceinline__ void record_error(int code) { atomicOr(&g_fwd_error, code); }

// One work item of the persistent forward: a 128-row query tile of one head of one sequence.
struct FwdItem {
  int z, h, SQ, SK, qtok0, ktok0, qb;   // sequence, head, lengths, token offsets, first row
  int t0, ntiles;                       // visible key tiles [t0, t0 + ntiles)
  bool live;                            // the tile holds rows of its sequence
};

// Geometry of item `idx` (warp-collective: every lane of the calling warp takes part).  Items are
// numbered heavy first: dense requests run every (head, batch) of the last query tile, then of
// the one before, ...; varlen requests enumerate the query tiles of all sequences back to back
// (sequence z owns ceil(SQ_z / BM) consecutive tile indices, its last tile first), each for
// every head, and a prefix sum over cu_seqlens finds the sequence of a tile index.
__device__ __forceinline__ FwdItem fwd_item(const FaFwdParams& p, int idx, int lane) {
  FwdItem it;
  it.live = false;
  it.ntiles = 0;
  it.t0 = 0;
  if (p.cu_q == nullptr) {
    const int nb = p.NH * p.batch, ntq = (p.SQ + BM - 1) / BM;
    const int trev = idx / nb, rest = idx % nb;
    it.h = rest % p.NH;
    it.z = rest / p.NH;
    it.SQ = p.SQ;
    it.SK = p.SK;
    it.qtok0 = it.ktok0 = 0;
    it.qb = (ntq - 1 - trev) * BM;
  } else {
    const int ft = idx / p.NH;
    it.h = idx % p.NH;
    int base = 0, zz = -1, loc = 0;
    for (int s0 = 0; s0 < p.batch; s0 += 32) {
      const int si = s0 + lane;
      int n = 0;
      if (si < p.batch) {
        int len = p.cu_q[si + 1] - p.cu_q[si];
        if (p.seqused_q && p.seqused_q[si] < len) len = p.seqused_q[si];
        n = (max(len, 0) + BM - 1) / BM;
      }
      int inc = n;   // inclusive warp scan of the tile counts
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
      }
      const int first = base + inc - n;
      const unsigned hit = __ballot_sync(0xffffffffu, n > 0 && ft >= first && ft < first + n);
      if (hit) {
        const int src = __ffs(hit) - 1;
        zz = s0 + src;
        loc = ft - __shfl_sync(0xffffffffu, first, src);
        break;
      }
      base += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (zz < 0) return it;   // past the last tile of the last sequence
    it.z = zz;
    it.qtok0 = p.cu_q[zz];
    it.ktok0 = p.cu_k[zz];
    it.SQ = p.cu_q[zz + 1] - it.qtok0;
    it.SK = p.cu_k[zz + 1] - it.ktok0;
    if (p.seqused_q && p.seqused_q[zz] < it.SQ) it.SQ = p.seqused_q[zz];
    if (p.seqused_k && p.seqused_k[zz] < it.SK) it.SK = p.seqused_k[zz];
    it.SQ = max(it.SQ, 0);
    it.SK = max(it.SK, 0);
    it.qb = ((it.SQ + BM - 1) / BM - 1 - loc) * BM;
  }
  if (it.qb < 0 || it.qb >= it.SQ) return it;
  it.live = true;
  int klo, khi, dmy;
  fa_key_range(it.qb, it.SQ, it.SK, p.causal, p.win_left, p.win_right, p.attn_chunk, klo, dmy);
  fa_key_range(min(it.qb + BM, it.SQ) - 1, it.SQ, it.SK, p.causal, p.win_left, p.win_right, p.attn_chunk, dmy, khi);
  klo = max(klo, 0);
  khi = min(khi, it.SK - 1);
  it.t0 = klo / BN;
  it.ntiles = (khi >= klo) ? (khi / BN - it.t0 + 1) : 0;
  return it;
}

// Persistent one-tile forward: each CTA (one per SM) walks the items blockIdx.x,
// blockIdx.x + gridDim.x, ...  The pipelines never drain between items: K/V ring slots, S
// buffers and their barrier phases follow a key-tile counter g that runs across the CTA's items,
// Q is double-buffered (the next item's tile is loaded while the current one computes; one buffer
// at D = 256), and the first P.V of an item overwrites O (which the softmax warps have read out
// before they release that item's first P).
template <int D, bool BF16, bool FEAT>
__global__ void __launch_bounds__(NTHREADS, 1)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const FaFwdParams p, int n_items) {
  using C = Cfg<D>;
  constexpr int HB = BN / 2;            // S columns (keys) per softmax thread
  constexpr int HD2 = D / 2;            // O columns per softmax thread
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  const uint32_t sK = sbase + C::OFF_K, sV = sbase + C::OFF_V;
  const uint32_t bar = sbase + C::OFF_BAR;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + C::OFF_BAR + Bars::TMEM_ADDR);
  float* xch = reinterpret_cast<float*>(sgen + C::OFF_X);   // [2 parity][2 halves][BM] row maxima, then l

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool varlen = p.cu_q != nullptr;
  const bool rot = p.rot_cos != nullptr;   // the softmax warps rotate each Q tile before its first MMA

  // ---- set-up: barriers (thread 0), TMEM (MMA warp)
  if (tid == 0) {
    for (int s = 0; s < C::NQB; ++s) {
      mbar_init(bar + Bars::Q_FULL + 8 * s, 1);
      mbar_init(bar + Bars::Q_EMPTY + 8 * s, 1);
      mbar_init(bar + Bars::Q_ROT + 8 * s, NSOFT);
    }
    for (int s = 0; s < C::NSK; ++s) {
      mbar_init(bar + Bars::K_FULL + 8 * s, 1);
      mbar_init(bar + Bars::K_EMPTY + 8 * s, 1);
    }
    for (int s = 0; s < C::NSV; ++s) {
      mbar_init(bar + Bars::V_FULL + 8 * s, 1);
      mbar_init(bar + Bars::V_EMPTY + 8 * s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar + Bars::S_FULL + 8 * s, 1);
      mbar_init(bar + Bars::P_FULL + 8 * s, NSOFT);
    }
    mbar_init(bar + Bars::O_DONE, 1);
    mbar_init(bar + Bars::MMA_DRAIN, 1);
    fence_barrier_init();
  }
  if (warp == WARP_MMA) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == WARP_TMA && lane == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == WARP_TMA) {
    // ======================= TMA producer: per item its Q tile, then its K and V tiles
    const bool paged = p.block_table != nullptr;
    const int R = paged ? min(p.page, BN) : BN;
    bool ok = true;
    int g = 0, w = 0;   // key tiles and items (with keys) issued so far
    for (int idx = blockIdx.x; ok && idx < n_items; idx += gridDim.x) {
      const FwdItem it = fwd_item(p, idx, lane);
      if (!it.live || it.ntiles == 0) continue;
      if (lane == 0) {
        const int kvh = it.h / p.gqa, bcoord = varlen ? 0 : it.z;
        const int qs = w % C::NQB;
        if (w >= C::NQB && !mbar_wait(bar + Bars::Q_EMPTY + 8 * qs, ((w / C::NQB) - 1) & 1)) {
          record_error(1);
          ok = false;
        }
        if (ok) {
          mbar_expect_tx(bar + Bars::Q_FULL + 8 * qs, C::Q_BYTES);
          for (int c = 0; c < C::NCH; ++c)
            tma_load_4d(sbase + C::OFF_Q + qs * C::Q_BYTES + c * (BM * 128), &tmQ, c * 64, it.qtok0 + it.qb, it.h,
                        bcoord, bar + Bars::Q_FULL + 8 * qs);
        }
        // paged K/V: a tile is loaded as page slices of R rows (3-D maps over the cache rows);
        // positions past the block table's row, and invalid entries, read page 0 (an invalid entry
        // for a real key also raises the error flag), so every slice lands and expect_tx is fixed
        auto page_row = [&](int pos) -> int {
          const int pi = pos / p.page;
          long long blk = 0;
          if (pi < p.max_blocks) {
            blk = p.block_table[(long long)it.z * p.max_blocks + pi];
            if (blk < 0 || blk >= p.num_blocks) {
              if (pos < it.SK) record_error(1024);
              blk = 0;
            }
          }
          return (int)(blk * p.page + pos % p.page);
        };
        auto load_tile = [&](uint32_t dst, const CUtensorMap* map, int kpos, uint32_t fb) {
          if (!paged) {
            for (int c = 0; c < C::NCH; ++c)
              tma_load_4d(dst + c * C::CH_BYTES, map, c * 64, it.ktok0 + kpos, kvh, bcoord, fb);
            return;
          }
          for (int sl = 0; sl < BN / R; ++sl) {
            const int row = page_row(kpos + sl * R);
            for (int c = 0; c < C::NCH; ++c) tma_load_3d(dst + c * C::CH_BYTES + sl * R * 128, map, c * 64, kvh, row, fb);
          }
        };
        for (int j = 0; ok && j < it.ntiles; ++j) {
          const int gg = g + j, kpos = (it.t0 + j) * BN;
          const int sk = gg % C::NSK, sv = gg % C::NSV;
          if (gg >= C::NSK && !mbar_wait(bar + Bars::K_EMPTY + 8 * sk, ((gg / C::NSK) - 1) & 1)) {
            record_error(1);
            ok = false;
            break;
          }
          mbar_expect_tx(bar + Bars::K_FULL + 8 * sk, C::KV_BYTES);
          load_tile(sK + sk * C::KV_BYTES, &tmK, kpos, bar + Bars::K_FULL + 8 * sk);
          if (gg >= C::NSV && !mbar_wait(bar + Bars::V_EMPTY + 8 * sv, ((gg / C::NSV) - 1) & 1)) {
            record_error(1);
            ok = false;
            break;
          }
          mbar_expect_tx(bar + Bars::V_FULL + 8 * sv, C::KV_BYTES);
          load_tile(sV + sv * C::KV_BYTES, &tmV, kpos, bar + Bars::V_FULL + 8 * sv);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      g += it.ntiles;
      ++w;
    }
    // do not leave while copies of this CTA are still landing in shared memory (a Q tile is only
    // ever in flight while the K/V loads behind it are)
    if (lane == 0) {
      for (int j = max(0, g - C::NSK); j < g; ++j) mbar_wait(bar + Bars::K_FULL + 8 * (j % C::NSK), (j / C::NSK) & 1);
      for (int j = max(0, g - C::NSV); j < g; ++j) mbar_wait(bar + Bars::V_FULL + 8 * (j % C::NSV), (j / C::NSV) & 1);
      for (int j = max(0, w - C::NQB); j < w; ++j) mbar_wait(bar + Bars::Q_FULL + 8 * (j % C::NQB), (j / C::NQB) & 1);
    }
    __syncwarp();
  } else if (warp == WARP_MMA) {
    // ======================= MMA issuer (whole warp follows; lane 0 issues)
    constexpr uint32_t IDESC_S = idesc_f16(BF16 ? 1 : 0, BM, BN, 0, 0);
    constexpr uint32_t IDESC_O = idesc_f16(BF16 ? 1 : 0, BM, D, 0, 1);
    bool ok = true;
    int g = 0, w = 0;
    // P.V of key tile gg (item tile t0 + jj of an item with SK keys): O (+)= P V, zero-initialised by
    // the item's first one
    auto issue_pv = [&](int gg, int jj, int t0, int SK) -> bool {
      const int s = gg % C::NSV;
      if (!mbar_wait_warp(bar + Bars::P_FULL + 8 * (gg & 1), (gg >> 1) & 1)) return false;
      if (!mbar_wait_warp(bar + Bars::V_FULL + 8 * s, (gg / C::NSV) & 1)) return false;
      const int kb = (t0 + jj) * BN;
      if (varlen && kb + BN > SK) {
        // rows past the sequence end belong to other sequences (or are unused): zero them so
        // that P = 0 never meets a non-finite value
        const int r0 = max(SK - kb, 0);
        for (int c = 0; c < C::NCH; ++c)   // rows [r0, BN) of every 64-column chunk, 16 bytes per lane
          for (int e = r0 * 8 + lane; e < BN * 8; e += 32)
            *reinterpret_cast<uint4*>(sgen + C::OFF_V + s * C::KV_BYTES + c * C::CH_BYTES + (e / 8) * 128 +
                                      (e % 8) * 16) = make_uint4(0, 0, 0, 0);
        fence_proxy_async_smem();
        __syncwarp();
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t pt = tmem + (uint32_t)(gg & 1) * 128u;
        const uint64_t vd0 = sdesc_sw128(sV + s * C::KV_BYTES, C::CH_BYTES, 1024);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          // A = P from TMEM: keys [64 hf, 64 hf + 64) sit packed in columns [64 hf, 64 hf + 32)
          // B = V tile, MN-major: 16 keys = 16 rows of 128 B; D spans NCH swizzle atoms (LBO apart)
          const uint32_t pa = pt + (uint32_t)((kk * 16) / HB) * 64u + (uint32_t)(((kk * 16) % HB) / 2);
          const uint64_t bd = desc_add(vd0, (uint32_t)(kk * 128));
          mma_ts(tmem + C::O_COL, pa, bd, IDESC_O, (jj > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(bar + Bars::V_EMPTY + 8 * s);
        mma_commit(bar + Bars::O_DONE);
      }
      __syncwarp();
      return true;
    };
    for (int idx = blockIdx.x; ok && idx < n_items; idx += gridDim.x) {
      const FwdItem it = fwd_item(p, idx, lane);
      if (!it.live || it.ntiles == 0) continue;
      const int qs = w % C::NQB;
      if (!mbar_wait_warp(bar + (rot ? Bars::Q_ROT : Bars::Q_FULL) + 8 * qs, (w / C::NQB) & 1)) {
        ok = false;
        break;
      }
      const uint32_t sQ = sbase + C::OFF_Q + qs * C::Q_BYTES;
      for (int j = 0; ok && j < it.ntiles; ++j) {
        const int gg = g + j, s = gg % C::NSK;
        if (!mbar_wait_warp(bar + Bars::K_FULL + 8 * s, (gg / C::NSK) & 1)) { ok = false; break; }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t st = tmem + (uint32_t)(gg & 1) * 128u;
          const uint64_t ad0 = sdesc_sw128(sQ, 16, 1024), bd0 = sdesc_sw128(sK + s * C::KV_BYTES, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int c = kk / 4, off = (kk % 4) * 32;   // 16 columns = 32 bytes inside a 128-byte chunk
            mma_ss(st, desc_add(ad0, (uint32_t)((c * (BM * 128) + off) >> 4)),
                   desc_add(bd0, (uint32_t)((c * C::CH_BYTES + off) >> 4)), IDESC_S, kk > 0 ? 1u : 0u);
          }
          mma_commit(bar + Bars::S_FULL + 8 * (gg & 1));
          mma_commit(bar + Bars::K_EMPTY + 8 * s);
          if (j == it.ntiles - 1) mma_commit(bar + Bars::Q_EMPTY + 8 * qs);   // the item's last read of Q
        }
        __syncwarp();
        if (j >= 1 && !issue_pv(gg - 1, j - 1, it.t0, it.SK)) { ok = false; break; }
      }
      if (ok && !issue_pv(g + it.ntiles - 1, it.ntiles - 1, it.t0, it.SK)) ok = false;
      g += it.ntiles;
      ++w;
    }
    if (!ok) record_error(4);
    // every MMA this warp issued has completed before TMEM can be released (also on error paths)
    if (lane == 0) mma_commit(bar + Bars::MMA_DRAIN);
    __syncwarp();
    if (!mbar_wait_warp(bar + Bars::MMA_DRAIN, 0)) record_error(32);
  } else {
    // ======================= softmax + epilogue (warps 0-7).  Warps w and w + 4 share TMEM lane
    // quadrant w % 4 (query rows 32 (w%4) .. + 31); half hf = w / 4 takes S columns (keys)
    // [64 hf, 64 hf + 64) and O columns [D/2 hf, D/2 hf + D/2).  The two halves of a row agree on
    // the row max through shared memory and a 64-thread named barrier per quadrant.
    const int qd = warp & 3, hf = warp >> 2;
    const int r = qd * 32 + lane;
    const uint32_t pair_bar = 1 + qd;
    const uint32_t lane_addr = tmem + ((uint32_t)(qd * 32) << 16);
    const float scale2 = p.scale * FA_LOG2E;
    const bool drop = FEAT && p.dropout_p > 0.f;
    const float inv_keep = drop ? 1.0f / (1.0f - p.dropout_p) : 1.f;
    const bool use_bits = drop && p.dropout_bits != nullptr;
    const uint32_t thresh = fa_drop_thresh(p.dropout_p);
    const bool cap_on = FEAT && p.softcap > 0.f;
    const float cap_in = cap_on ? p.scale / p.softcap : 0.f, cap2 = p.softcap * FA_LOG2E;
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    bool ok = true;
    int g = 0, w = 0;
    for (int idx = blockIdx.x; ok && idx < n_items; idx += gridDim.x) {
      const FwdItem it = fwd_item(p, idx, lane);
      if (!it.live) continue;
      const int z = it.z, h = it.h, SQ = it.SQ, SK = it.SK, qb = it.qb, q = qb + r, ntiles = it.ntiles;
      T* orow = (T*)p.O + (varlen ? (long long)it.qtok0 * p.sO.s : (long long)z * p.sO.b) + (long long)h * p.sO.h +
                (long long)q * p.sO.s + hf * HD2;
      if (ntiles == 0) {   // rows that see no key: O = 0, LSE = -inf (no pipeline work)
        if (q < SQ) {
          uint4* dst = reinterpret_cast<uint4*>(orow);
          for (int i = 0; i < HD2 / 8; ++i)
            if (hf * HD2 + 8 * i < p.HD) dst[i] = make_uint4(0, 0, 0, 0);
          if (hf == 0 && p.LSE) p.LSE[fa_lse_index(varlen, z, h, p.NH, p.SQ, it.qtok0, p.lse_total_q, q)] = -INFINITY;
        }
        continue;
      }
      const int qs = w % C::NQB;
      if (rot) {
        // rotary embedding of the Q tile in shared memory (before any MMA reads it): thread pair
        // (2 rr, 2 rr + 1) takes row rr, alternate rotary pairs; the roundings are the reference's
        // (cos / sin cast to the dtype, each product and the sum rounded, no fused multiply-add).
        // Element d of row rr sits in 64-column chunk d / 64 at 16-byte unit (d % 64) / 8 XOR rr % 8
        // (the TMA 128-byte swizzle).
        using RT = T;
        uint8_t* qbuf = sgen + C::OFF_Q + qs * C::Q_BYTES;
        auto rnd = [](float x) { return Elem<RT>::to_f(Elem<RT>::from_f(x)); };
        auto qel = [&](int rr, int d) -> RT* {
          const int e = d & 63;
          return reinterpret_cast<RT*>(qbuf + (d >> 6) * (BM * 128) + rr * 128 + (((e >> 3) ^ (rr & 7)) << 4) +
                                       ((e & 7) << 1));
        };
        // 16-byte unit of row rr holding elements d .. d + 7 (d a multiple of 8)
        auto qunit = [&](int rr, int d) -> uint4* {
          const int e = d & 63;
          return reinterpret_cast<uint4*>(qbuf + (d >> 6) * (BM * 128) + rr * 128 + (((e >> 3) ^ (rr & 7)) << 4));
        };
        auto rot1 = [&](float a, float b, float c, float sn, float& o1, float& o2) {
          c = rnd(c);
          sn = rnd(sn);
          o1 = Elem<RT>::to_f(Elem<RT>::from_f(__fsub_rn(rnd(__fmul_rn(a, c)), rnd(__fmul_rn(b, sn)))));
          o2 = Elem<RT>::to_f(Elem<RT>::from_f(__fadd_rn(rnd(__fmul_rn(b, c)), rnd(__fmul_rn(a, sn)))));
        };
        const int rr = tid >> 1, pos = qb + rr, half = p.rot_dim / 2;
        // cos / sin of this thread's pairs are loaded before the wait for Q: thread (2 rr + t) owns the
        // contiguous pairs [t * half/2, (t + 1) * half/2) of row rr, whole 16-byte units when
        // half/2 is a multiple of 8 (rot_dim 32, 64, 96, 128)
        const int per = half / 2, j0 = (tid & 1) * per;
        const bool vec = per % 8 == 0 && per <= 32 && ((uintptr_t)p.rot_cos | (uintptr_t)p.rot_sin) % 16 == 0;
        const bool row_ok = pos < SQ && pos < p.rot_seqlen_ro;
        float4 c4[8], s4[8];
#pragma unroll
        for (int gi = 0; gi < 8; ++gi) {
          c4[gi] = s4[gi] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (vec && row_ok && 4 * gi < per) {
            c4[gi] = __ldg(reinterpret_cast<const float4*>(p.rot_cos + (long long)pos * half + j0) + gi);
            s4[gi] = __ldg(reinterpret_cast<const float4*>(p.rot_sin + (long long)pos * half + j0) + gi);
          }
        }
        const bool got = mbar_wait(bar + Bars::Q_FULL + 8 * qs, (w / C::NQB) & 1);
        if (got && pos < SQ && pos >= p.rot_seqlen_ro) record_error(4096);
        if (got && row_ok && vec) {
          const float* cf = reinterpret_cast<const float*>(c4);
          const float* sf = reinterpret_cast<const float*>(s4);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (8 * u >= per) break;
            if (!p.rot_interleaved) {   // pairs (j, j + half): one unit of each side
              uint4* pa = qunit(rr, j0 + 8 * u);
              uint4* pb = qunit(rr, j0 + half + 8 * u);
              uint4 ua = *pa, ub = *pb;
              RT* xa = reinterpret_cast<RT*>(&ua);
              RT* xb = reinterpret_cast<RT*>(&ub);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                float o1, o2;
                rot1(Elem<RT>::to_f(xa[e]), Elem<RT>::to_f(xb[e]), cf[8 * u + e], sf[8 * u + e], o1, o2);
                xa[e] = Elem<RT>::from_f(o1);
                xb[e] = Elem<RT>::from_f(o2);
              }
              *pa = ua;
              *pb = ub;
            } else {   // pairs (2j, 2j + 1): 8 pairs = two units
              uint4* pa = qunit(rr, 2 * (j0 + 8 * u));
              uint4* pb = qunit(rr, 2 * (j0 + 8 * u) + 8);
              uint4 ua = *pa, ub = *pb;
              RT* x = reinterpret_cast<RT*>(&ua);
              RT* y = reinterpret_cast<RT*>(&ub);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                RT* wv = e < 4 ? x : y;
                const int o = 2 * (e & 3);
                float o1, o2;
                rot1(Elem<RT>::to_f(wv[o]), Elem<RT>::to_f(wv[o + 1]), cf[8 * u + e], sf[8 * u + e], o1, o2);
                wv[o] = Elem<RT>::from_f(o1);
                wv[o + 1] = Elem<RT>::from_f(o2);
              }
              *pa = ua;
              *pb = ub;
            }
          }
        } else if (got && row_ok) {
          for (int jr = tid & 1; jr < half; jr += 2) {
            const int d1 = p.rot_interleaved ? 2 * jr : jr, d2 = p.rot_interleaved ? 2 * jr + 1 : jr + half;
            RT* x1 = qel(rr, d1);
            RT* x2 = qel(rr, d2);
            const float a = Elem<RT>::to_f(*x1), b = Elem<RT>::to_f(*x2);
            const float c = rnd(p.rot_cos[(long long)pos * half + jr]), sn = rnd(p.rot_sin[(long long)pos * half + jr]);
            *x1 = Elem<RT>::from_f(__fsub_rn(rnd(__fmul_rn(a, c)), rnd(__fmul_rn(b, sn))));
            *x2 = Elem<RT>::from_f(__fadd_rn(rnd(__fmul_rn(b, c)), rnd(__fmul_rn(a, sn))));
          }
        }
        if (!got) record_error(8);
        fence_proxy_async_smem();   // generic-proxy stores, read next by the tensor core
        mbar_arrive(bar + Bars::Q_ROT + 8 * qs);
      }
      int rlo, rhi;
      fa_key_range(q, SQ, SK, p.causal, p.win_left, p.win_right, p.attn_chunk, rlo, rhi);
      if (q >= SQ) { rlo = 1; rhi = 0; }
      // tile-uniform bounds used to classify key tiles as fully visible
      int lo_last, hi_first;
      {
        int a, b;
        fa_key_range(min(qb + BM, SQ) - 1, SQ, SK, p.causal, p.win_left, p.win_right, p.attn_chunk, lo_last, a);
        fa_key_range(qb, SQ, SK, p.causal, p.win_left, p.win_right, p.attn_chunk, b, hi_first);
      }
      const bool full_rows = qb + BM <= SQ;
      const float slope2 = (FEAT && p.alibi_slopes) ? p.alibi_slopes[h] * FA_LOG2E : 0.f;
      const int mask_w = (SK + 31) / 32;
      float m_ref = -INFINITY, l = 0.f;
      float s[HB];
      for (int j = 0; j < ntiles; ++j) {
        const int gg = g + j;
        const int kb = (it.t0 + j) * BN, kh = kb + hf * HB;   // first key of this thread's half
        // this half's keep bits, one word per 32 keys (bit b <-> key kh + 32i + b), prepared before
        // the wait so that they overlap it: loaded from the mask (its layout puts the warp's 32 rows
        // on one line) or evaluated with Philox.  Mask words past the row's visible keys may be
        // unwritten: they only multiply probabilities that are already 0.
        uint32_t dw[HB / 32];
#pragma unroll
        for (int i = 0; i < HB / 32; ++i) {
          const int kw = kh / 32 + i;
          dw[i] = 0u;
          if (drop && q < SQ && kw < mask_w)
            dw[i] = use_bits ? __ldg(p.dropout_bits + fa_mask_word(h, SQ, SK, q, kw))
                             : fa_keep_word(p.philox_seed, ((uint64_t)h * SQ + q) * SK + 32 * kw, 1, thresh,
                                            SK - 32 * kw);
        }
        // both warps of the pair leave together (the exchange below is a barrier without timeout)
        const bool got = mbar_wait_warp(bar + Bars::S_FULL + 8 * (gg & 1), (gg >> 1) & 1);
        if (!bar_and_pair(pair_bar, got && ok)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = lane_addr + (uint32_t)(gg & 1) * 128u + (uint32_t)(hf * HB);
#pragma unroll
        for (int c = 0; c < HB; c += 32) tmem_ld32(sa + c, s + c);
        tc_wait_ld();
        // ---- scores (log2 domain) and masks
        float tmax = -INFINITY;
        if constexpr (FEAT) {
          // logits in log2 units; alibi adds slope2 * (key - q), and key - q = d0 + c exactly in
          // fp32.  Two tight loops (softcap or not) keep the unrolled code small.
          const float d0 = (float)(kh - q);
          if (cap_on) {
#pragma unroll
            for (int c = 0; c < HB; ++c) s[c] = fmaf(cap2, fa_tanh_tc<BF16>(s[c] * cap_in), slope2 * (d0 + (float)c));
          } else {
#pragma unroll
            for (int c = 0; c < HB; ++c) s[c] = fmaf(s[c], scale2, slope2 * (d0 + (float)c));
          }
        }
        const bool interior = full_rows && kb >= lo_last && kb + BN - 1 <= hi_first && kb + BN <= SK;
        if (!interior) {
#pragma unroll
          for (int c = 0; c < HB; ++c) {
            const int key = kh + c;
            if (key < rlo || key > rhi) s[c] = -INFINITY;
          }
        }
#pragma unroll
        for (int c = 0; c < HB; ++c) tmax = fmaxf(tmax, s[c]);
        if constexpr (!FEAT) tmax = (tmax == -INFINITY) ? -INFINITY : tmax * scale2;
        // ---- row max over both halves (slots alternate by key-tile parity, so a slot is rewritten
        //      only after the partner has passed the next exchange)
        float* xs = xch + (gg & 1) * (2 * BM);
        xs[hf * BM + r] = tmax;
        bar_sync_pair(pair_bar);
        tmax = fmaxf(tmax, xs[(1 - hf) * BM + r]);
        // ---- lazy online-softmax update: the reference max moves only when it grows by > 2^8
        const bool move = tmax > m_ref + LAZY_THRESH || (m_ref == -INFINITY && tmax != -INFINITY);
        float corr = 1.f;
        if (move) {
          corr = ex2(m_ref - tmax);   // 0 when the row had no visible key yet (its O row is 0)
          l *= corr;
          m_ref = tmax;
        }
        const float muse = (m_ref == -INFINITY) ? 0.f : m_ref;
        const float sc = FEAT ? 1.f : scale2;
        // ---- P = 2^(s - m): row sum (before dropout), dropout, 16-bit pairs into the first HB/2
        //      columns of this half's S range (already read into registers).
        // one straight-line instantiation per dropout setting (a runtime test inside the unrolled
        // pair loop would be compiled as predicated code that runs both sides)
        auto p_pass = [&](auto drop_tag) -> float2 {
          constexpr bool kDrop = decltype(drop_tag)::value;
          float2 lsum2 = make_float2(0.f, 0.f);
#pragma unroll
          for (int c0 = 0; c0 < HB; c0 += 32) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              // packed fp32x2 arithmetic (one FFMA2 / FADD2 per pair) around the two SFU exponentials
              const float2 x2 = __ffma2_rn(make_float2(s[c0 + 2 * i], s[c0 + 2 * i + 1]), make_float2(sc, sc),
                                           make_float2(-muse, -muse));
              float a = ex2(x2.x), b = ex2(x2.y);
              lsum2 = __fadd2_rn(lsum2, make_float2(a, b));
              if constexpr (kDrop) {   // keys kh + c0 + 2i, +1: bits 2i, 2i + 1 of word c0/32, sign-extended;
                // dropped scores become 0; 1/(1-p) is applied to O in fp32 (epilogue), so a kept
                // probability reaches the 16-bit P operand unscaled (1.0 stays exact)
                const uint32_t wd = dw[c0 / 32];
                const uint32_t m0 = (uint32_t)((int32_t)(wd << (31 - 2 * i)) >> 31);
                const uint32_t m1 = (uint32_t)((int32_t)(wd << (30 - 2 * i)) >> 31);
                a = __uint_as_float(__float_as_uint(a) & m0);
                b = __uint_as_float(__float_as_uint(b) & m1);
              }
              if constexpr (BF16) {
                const __nv_bfloat162 t2 = __floats2bfloat162_rn(a, b);
                pk[i] = *reinterpret_cast<const uint32_t*>(&t2);
              } else {
                const __half2 t2 = __floats2half2_rn(a, b);
                pk[i] = *reinterpret_cast<const uint32_t*>(&t2);
              }
            }
            tmem_st16(sa + c0 / 2, pk);
          }
          return lsum2;
        };
        float2 lsum2;
        if constexpr (FEAT) {
          lsum2 = drop ? p_pass(std::true_type{}) : p_pass(std::false_type{});
        } else {
          lsum2 = p_pass(std::false_type{});
        }
        // ---- O rescale of this half's columns.  Every key tile j >= 1 of an item waits exactly once
        //      for the P.V of the tile before (so the parity wait can never alias an older phase);
        //      that P.V normally finished while P_j was computed.  tcgen05.ld/st are warp-collective:
        //      rows that did not move scale by 1.
        if (j > 0) {
          if (!mbar_wait_warp(bar + Bars::O_DONE, (gg - 1) & 1)) ok = false;   // leaves at the next exchange
          if (ok && __any_sync(0xffffffffu, corr != 1.f)) {
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < HD2; c += 32) {
              float o[32];
              tmem_ld32(lane_addr + C::O_COL + hf * HD2 + c, o);
              tc_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] *= corr;
              tmem_st32(lane_addr + C::O_COL + hf * HD2 + c, reinterpret_cast<const uint32_t*>(o));
            }
          }
        }
        l += lsum2.x + lsum2.y;
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(bar + Bars::P_FULL + 8 * (gg & 1));
      }
      // ---- epilogue: row sum over both halves, this half's O columns / l, LSE (first half).  The
      //      TMEM reads complete before this warp releases the next item's first P, which is when
      //      the next item's first P.V may overwrite O.
      if (ok && !mbar_wait_warp(bar + Bars::O_DONE, (g + ntiles - 1) & 1)) {
        record_error(16);
        ok = false;
      }
      tc_fence_after();
      // the pair's exchanges AND-reduce `ok`: both warps of a quadrant go on to the next item or
      // both stop (their named barrier has no timeout, so they must never part ways)
      float* xl = xch + 4 * BM;
      xl[hf * BM + r] = l;
      ok = bar_and_pair(pair_bar, ok);
      l += xl[(1 - hf) * BM + r];
      ok = bar_and_pair(pair_bar, ok);   // both halves have read xl before either writes the next item's
      const float inv = l > 0.f ? inv_keep / l : 0.f;   // 1/(1-p) of the kept probabilities (1 without dropout)
#pragma unroll
      for (int c = 0; c < HD2; c += 32) {
        float o[32];
        if (ok) {
          tmem_ld32(lane_addr + C::O_COL + hf * HD2 + c, o);
          tc_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (q < SQ) {
          uint32_t wv[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if constexpr (BF16) {
              const __nv_bfloat162 t2 = __floats2bfloat162_rn(o[2 * i] * inv, o[2 * i + 1] * inv);
              wv[i] = *reinterpret_cast<const uint32_t*>(&t2);
            } else {
              const __half2 t2 = __floats2half2_rn(o[2 * i] * inv, o[2 * i + 1] * inv);
              wv[i] = *reinterpret_cast<const uint32_t*>(&t2);
            }
          }
          uint4* dst = reinterpret_cast<uint4*>(orow + c);
          // 8-column units; columns at or past the real head_dim are padding (never stored)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (hf * HD2 + c + 8 * i < p.HD) dst[i] = make_uint4(wv[4 * i], wv[4 * i + 1], wv[4 * i + 2], wv[4 * i + 3]);
        }
      }
      if (hf == 0 && q < SQ && p.LSE) {
        const long long li = fa_lse_index(varlen, z, h, p.NH, p.SQ, it.qtok0, p.lse_total_q, q);
        p.LSE[li] = l > 0.f ? m_ref * FA_LN2 + logf(l) : -INFINITY;
      }
      g += ntiles;
      ++w;
    }
    if (!ok) record_error(8);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// =====================================================================================
// Two query tiles per CTA ("ping-pong"), dense inputs without softcap / alibi; dropout only from a
// precomputed keep mask (DROP).
//
// One CTA = rows [qb, qb + 256) of one head: tile A = the first 128 rows, tile B = the next 128.
// The MMA warp alternates the tiles, so the tensor cores run one tile's S = Q K^T and O += P V
// while the other tile's softmax is in flight:
//   S_A(0) S_B(0) | PV_A(0) S_A(1) PV_B(0) S_B(1) | PV_A(1) S_A(2) PV_B(1) S_B(2) | ...
// Warp roles (384 threads, three warpgroups):
//   warps 0-3   softmax of tile A, warps 4-7 softmax of tile B: thread = query row (TMEM lane
//               32 (w % 4) + lane), the whole 128-key S row read into registers in one pass
//               (max, lazy online-softmax update, 2^(s - m), row sum, P as packed 16-bit pairs into
//               the first 64 columns of the same S buffer), then the O row of its tile.
//   warp 8      TMA producer (Q tiles once, K and V tiles into rings);
//   warp 9      MMA issuer (owns TMEM); warps 10-11 idle (they complete warpgroup 2).
// Registers: the kernel is compiled for 384 x 168; warpgroup 2 lowers itself to 56 per thread
// (setmaxnreg.dec) and the two softmax warpgroups raise themselves to 224, which holds a full S row.
// 2 * 224 + 56 = 3 * 168, so the raises are always satisfiable; the host launches this kernel only
// after checking that it really was built with 168 registers per thread.
// TMEM: S_A [0,128), S_B [128,256), O_A [256, 384), O_B [384, 512).
// Semantics are those of the single-tile kernel above (masks, lazy rescale, LSE, empty rows).
constexpr int PP_THREADS = 384, PP_REGS = 168, PP_REGS_SOFTMAX = 224, PP_REGS_OTHER = 56;
static_assert(2 * PP_REGS_SOFTMAX + PP_REGS_OTHER == 3 * PP_REGS, "register split must use the launch total");

struct PpCfg {   // D = 128
  static constexpr int D = 128, NSK = 2, NSV = 3, NCH = 2;
  static constexpr int Q_BYTES = BM * D * 2, KV_BYTES = BN * D * 2, CH_BYTES = BN * 128;
  static constexpr int OFF_Q = 0, OFF_K = 2 * Q_BYTES, OFF_V = OFF_K + NSK * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + NSV * KV_BYTES;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static constexpr uint32_t O_COL = 256;
  static_assert(SMEM <= 232448, "shared memory per CTA");
};
struct PpBars {   // S_FULL / P_FULL / O_DONE: [tile A, tile B]
  static constexpr int Q_FULL = 0, K_FULL = 8, K_EMPTY = 24, V_FULL = 40, V_EMPTY = 64, S_FULL = 88,
                       P_FULL = 104, O_DONE = 120, MMA_DRAIN = 136, TMEM_ADDR = 144;
};

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

template <bool BF16, bool DROP>
__global__ void __launch_bounds__(PP_THREADS, 1)
    fwd_pp_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const FaFwdParams p) {
  using C = PpCfg;
  using Bz = PpBars;
  constexpr int D = C::D;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  const uint32_t sQ = sbase + C::OFF_Q, sK = sbase + C::OFF_K, sV = sbase + C::OFF_V;
  const uint32_t bar = sbase + C::OFF_BAR;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + C::OFF_BAR + Bz::TMEM_ADDR);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int z = blockIdx.z, h = blockIdx.y, kvh = h / p.gqa;
  const int SQ = p.SQ, SK = p.SK;
  const int qb = (gridDim.x - 1 - blockIdx.x) * (2 * BM);   // heavy (late, causal) tiles first
  if (qb >= SQ) return;

  // key tiles: the union of what the CTA's 256 rows can see
  int klo, khi, dmy;
  fa_key_range(qb, SQ, SK, p.causal, p.win_left, p.win_right, p.attn_chunk, klo, dmy);
  fa_key_range(min(qb + 2 * BM, SQ) - 1, SQ, SK, p.causal, p.win_left, p.win_right, p.attn_chunk, dmy, khi);
  klo = max(klo, 0);
  khi = min(khi, SK - 1);
  const int t0 = klo / BN;
  const int ntiles = (khi >= klo) ? (khi / BN - t0 + 1) : 0;

  if (tid == 0) {
    mbar_init(bar + Bz::Q_FULL, 1);
    for (int s = 0; s < C::NSK; ++s) {
      mbar_init(bar + Bz::K_FULL + 8 * s, 1);
      mbar_init(bar + Bz::K_EMPTY + 8 * s, 1);
    }
    for (int s = 0; s < C::NSV; ++s) {
      mbar_init(bar + Bz::V_FULL + 8 * s, 1);
      mbar_init(bar + Bz::V_EMPTY + 8 * s, 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar + Bz::S_FULL + 8 * t, 1);
      mbar_init(bar + Bz::P_FULL + 8 * t, BM);
      mbar_init(bar + Bz::O_DONE + 8 * t, 1);
    }
    mbar_init(bar + Bz::MMA_DRAIN, 1);
    fence_barrier_init();
  }
  if (warp == WARP_MMA) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (warp == WARP_TMA && lane == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(PP_REGS_OTHER));
    if (warp == WARP_TMA) {
      // ======================= TMA producer
      if (lane == 0 && ntiles > 0) {
        mbar_expect_tx(bar + Bz::Q_FULL, 2 * C::Q_BYTES);
        for (int t = 0; t < 2; ++t)
          for (int c = 0; c < C::NCH; ++c)
            tma_load_4d(sQ + t * C::Q_BYTES + c * (BM * 128), &tmQ, c * 64, qb + t * BM, h, z, bar + Bz::Q_FULL);
        for (int j = 0; j < ntiles; ++j) {
          const int kpos = (t0 + j) * BN;
          const int sk = j % C::NSK, sv = j % C::NSV;
          if (j >= C::NSK && !mbar_wait(bar + Bz::K_EMPTY + 8 * sk, ((j / C::NSK) - 1) & 1)) {
            record_error(1);
            break;
          }
          mbar_expect_tx(bar + Bz::K_FULL + 8 * sk, C::KV_BYTES);
          for (int c = 0; c < C::NCH; ++c)
            tma_load_4d(sK + sk * C::KV_BYTES + c * C::CH_BYTES, &tmK, c * 64, kpos, kvh, z, bar + Bz::K_FULL + 8 * sk);
          if (j >= C::NSV && !mbar_wait(bar + Bz::V_EMPTY + 8 * sv, ((j / C::NSV) - 1) & 1)) {
            record_error(1);
            break;
          }
          mbar_expect_tx(bar + Bz::V_FULL + 8 * sv, C::KV_BYTES);
          for (int c = 0; c < C::NCH; ++c)
            tma_load_4d(sV + sv * C::KV_BYTES + c * C::CH_BYTES, &tmV, c * 64, kpos, kvh, z, bar + Bz::V_FULL + 8 * sv);
        }
        // do not leave while copies of this CTA are still landing in shared memory
        for (int j = max(0, ntiles - C::NSK); j < ntiles; ++j)
          mbar_wait(bar + Bz::K_FULL + 8 * (j % C::NSK), (j / C::NSK) & 1);
        for (int j = max(0, ntiles - C::NSV); j < ntiles; ++j)
          mbar_wait(bar + Bz::V_FULL + 8 * (j % C::NSV), (j / C::NSV) & 1);
      }
      __syncwarp();
    } else if (warp == WARP_MMA) {
      // ======================= MMA issuer (whole warp follows; lane 0 issues).  S_X(j+1) reuses
      // the TMEM columns PV_X(j) reads P_X(j) from; the tensor core executes one thread's MMAs in
      // issue order, so the overwrite follows the read.
      constexpr uint32_t IDESC_S = idesc_f16(BF16 ? 1 : 0, BM, BN, 0, 0);
      constexpr uint32_t IDESC_O = idesc_f16(BF16 ? 1 : 0, BM, D, 0, 1);
      bool ok = ntiles == 0 || mbar_wait_warp(bar + Bz::Q_FULL, 0);
      if (!ok) record_error(2);
      auto issue_s = [&](int j, int t) {   // lane 0; K tile j has landed
        const uint32_t kbase = sK + (j % C::NSK) * C::KV_BYTES, qbase = sQ + t * C::Q_BYTES;
        const uint64_t ad0 = sdesc_sw128(qbase, 16, 1024), bd0 = sdesc_sw128(kbase, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int c = kk / 4, off = (kk % 4) * 32;   // 16 columns = 32 bytes inside a 128-byte chunk
          mma_ss(tmem + (uint32_t)(t * BN), desc_add(ad0, (uint32_t)((c * (BM * 128) + off) >> 4)),
                 desc_add(bd0, (uint32_t)((c * C::CH_BYTES + off) >> 4)), IDESC_S, kk > 0 ? 1u : 0u);
        }
        mma_commit(bar + Bz::S_FULL + 8 * t);
      };
      auto wait_k = [&](int j) -> bool {
        if (!mbar_wait_warp(bar + Bz::K_FULL + 8 * (j % C::NSK), (j / C::NSK) & 1)) return false;
        tc_fence_after();
        return true;
      };
      auto issue_pv = [&](int j, int t) -> bool {
        const int s = j % C::NSV;
        if (!mbar_wait_warp(bar + Bz::P_FULL + 8 * t, j & 1)) return false;
        if (t == 0 && !mbar_wait_warp(bar + Bz::V_FULL + 8 * s, (j / C::NSV) & 1)) return false;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t pt = tmem + (uint32_t)(t * BN);
          const uint64_t vd0 = sdesc_sw128(sV + s * C::KV_BYTES, C::CH_BYTES, 1024);
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            // A = P from TMEM (keys packed two per column); B = V tile, MN-major
            const uint64_t bd = desc_add(vd0, (uint32_t)(kk * 128));
            mma_ts(tmem + C::O_COL + (uint32_t)(t * D), pt + kk * 8, bd, IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(bar + Bz::O_DONE + 8 * t);
          if (t == 1) mma_commit(bar + Bz::V_EMPTY + 8 * s);
        }
        __syncwarp();
        return true;
      };
      if (ok && ntiles > 0) {
        if (!wait_k(0)) ok = false;
        if (ok && lane == 0) {
          issue_s(0, 0);
          issue_s(0, 1);
          mma_commit(bar + Bz::K_EMPTY);
        }
        __syncwarp();
      }
      for (int j = 0; ok && j < ntiles; ++j) {
        const bool more = j + 1 < ntiles;
        if (!issue_pv(j, 0)) { ok = false; break; }
        if (more) {
          if (!wait_k(j + 1)) { ok = false; break; }
          if (lane == 0) issue_s(j + 1, 0);
          __syncwarp();
        }
        if (!issue_pv(j, 1)) { ok = false; break; }
        if (more) {
          if (lane == 0) {
            issue_s(j + 1, 1);
            mma_commit(bar + Bz::K_EMPTY + 8 * ((j + 1) % C::NSK));
          }
          __syncwarp();
        }
      }
      if (!ok) record_error(4);
      // every MMA this warp issued has completed before TMEM can be released (also on error paths)
      if (lane == 0) mma_commit(bar + Bz::MMA_DRAIN);
      __syncwarp();
      if (!mbar_wait_warp(bar + Bz::MMA_DRAIN, 0)) record_error(32);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(PP_REGS_SOFTMAX));
    // ======================= softmax + epilogue of tile tt
    const int tt = warp >> 2;
    const int r = (warp & 3) * 32 + lane, q = qb + tt * BM + r;
    const int qt = qb + tt * BM;   // first row of this tile
    const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t o_col = C::O_COL + (uint32_t)(tt * D);
    int rlo, rhi;
    fa_key_range(q, SQ, SK, p.causal, p.win_left, p.win_right, p.attn_chunk, rlo, rhi);
    if (q >= SQ) { rlo = 1; rhi = 0; }
    int lo_last = 1, hi_first = 0;   // tile-uniform bounds: key tiles every row sees in full
    if (qt < SQ) {
      int a, b;
      fa_key_range(min(qt + BM, SQ) - 1, SQ, SK, p.causal, p.win_left, p.win_right, p.attn_chunk, lo_last, a);
      fa_key_range(qt, SQ, SK, p.causal, p.win_left, p.win_right, p.attn_chunk, b, hi_first);
    }
    const bool full_rows = qt + BM <= SQ;
    const float scale2 = p.scale * FA_LOG2E;
    const float inv_keep = DROP ? 1.0f / (1.0f - p.dropout_p) : 1.f;
    const int mask_w = (SK + 31) / 32;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int kb = (t0 + j) * BN;
      // keep bits of this row for the tile (bit b of word i <-> key kb + 32 i + b), loaded ahead of
      // the wait; the mask layout puts the warp's 32 rows on one line.  Words past the row's visible
      // keys may be unwritten: they only meet probabilities that are already 0.
      uint32_t dw[BN / 32];
#pragma unroll
      for (int i = 0; i < BN / 32; ++i)
        dw[i] = (DROP && q < SQ && kb / 32 + i < mask_w) ? __ldg(p.dropout_bits + fa_mask_word(h, SQ, SK, q, kb / 32 + i)) : 0u;
      if (!mbar_wait_warp(bar + Bz::S_FULL + 8 * tt, j & 1)) { ok = false; break; }
      tc_fence_after();
      const uint32_t sa = lane_addr + (uint32_t)(tt * BN);
      float s[BN];
#pragma unroll
      for (int c0 = 0; c0 < BN; c0 += 32) tmem_ld32(sa + c0, s + c0);
      tc_wait_ld();
      if (!(full_rows && kb >= lo_last && kb + BN - 1 <= hi_first && kb + BN <= SK)) {
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          const int key = kb + c;
          if (key < rlo || key > rhi) s[c] = -INFINITY;
        }
      }
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < BN; c += 8) {
        mx[0] = fmax3(mx[0], s[c], s[c + 1]);
        mx[1] = fmax3(mx[1], s[c + 2], s[c + 3]);
        mx[2] = fmax3(mx[2], s[c + 4], s[c + 5]);
        mx[3] = fmax3(mx[3], s[c + 6], s[c + 7]);
      }
      float tmax = fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]);
      tmax = (tmax == -INFINITY) ? -INFINITY : tmax * scale2;
      // lazy online-softmax update: the reference max moves only when it grows by > 2^8
      const bool move = tmax > m_ref + LAZY_THRESH || (m_ref == -INFINITY && tmax != -INFINITY);
      float corr = 1.f;
      if (move) {
        corr = ex2(m_ref - tmax);   // 0 when the row had no visible key yet (its O row is 0)
        l *= corr;
        m_ref = tmax;
      }
      const float muse = (m_ref == -INFINITY) ? 0.f : m_ref;
      // P = 2^(s - m): row sum, 16-bit pairs into the first BN/2 columns of the same S buffer
      // (the whole row is already in registers)
      float2 lsum2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 x2 = __ffma2_rn(make_float2(s[c0 + 2 * i], s[c0 + 2 * i + 1]), make_float2(scale2, scale2),
                                       make_float2(-muse, -muse));
          float a = ex2(x2.x), b = ex2(x2.y);
          lsum2 = __fadd2_rn(lsum2, make_float2(a, b));   // the row sum is taken before dropout
          if constexpr (DROP) {   // keys kb + c0 + 2i, +1: bits 2i, 2i + 1 of word c0 / 32, sign-extended;
            // 1/(1-p) is applied to O in fp32 (epilogue), not to the 16-bit P operand
            const uint32_t w = dw[c0 / 32];
            const uint32_t m0 = (uint32_t)((int32_t)(w << (31 - 2 * i)) >> 31);
            const uint32_t m1 = (uint32_t)((int32_t)(w << (30 - 2 * i)) >> 31);
            a = __uint_as_float(__float_as_uint(a) & m0);
            b = __uint_as_float(__float_as_uint(b) & m1);
          }
          if constexpr (BF16) {
            const __nv_bfloat162 t2 = __floats2bfloat162_rn(a, b);
            pk[i] = *reinterpret_cast<const uint32_t*>(&t2);
          } else {
            const __half2 t2 = __floats2half2_rn(a, b);
            pk[i] = *reinterpret_cast<const uint32_t*>(&t2);
          }
        }
        tmem_st16(sa + c0 / 2, pk);
      }
      // O rescale.  Every tile j >= 1 waits exactly once for PV_{j-1} of this tile (so the parity
      // wait never aliases an older phase).  tcgen05.ld/st are warp-collective: rows that did not
      // move scale by 1.
      if (j > 0) {
        if (!mbar_wait_warp(bar + Bz::O_DONE + 8 * tt, (j - 1) & 1)) { ok = false; break; }
        if (__any_sync(0xffffffffu, corr != 1.f)) {
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < D; c += 32) {
            float o[32];
            tmem_ld32(lane_addr + o_col + c, o);
            tc_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= corr;
            tmem_st32(lane_addr + o_col + c, reinterpret_cast<const uint32_t*>(o));
          }
        }
      }
      l += lsum2.x + lsum2.y;
      tc_wait_st();
      tc_fence_before();
      mbar_arrive(bar + Bz::P_FULL + 8 * tt);
    }
    if (!ok) record_error(8);
    // epilogue: O / l, LSE (TMEM reads by whole warps; stores only for real rows)
    const bool have_o = ok && ntiles > 0;
    if (have_o && !mbar_wait_warp(bar + Bz::O_DONE + 8 * tt, (ntiles - 1) & 1)) record_error(16);
    tc_fence_after();
    const float inv = l > 0.f ? inv_keep / l : 0.f;   // 1/(1-p) of the kept probabilities (1 without dropout)
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    T* orow = (T*)p.O + (long long)z * p.sO.b + (long long)h * p.sO.h + (long long)q * p.sO.s;
#pragma unroll
    for (int c = 0; c < D; c += 32) {
      float o[32];
      if (have_o) {
        tmem_ld32(lane_addr + o_col + c, o);
        tc_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0.f;
      }
      if (q < SQ) {
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if constexpr (BF16) {
            const __nv_bfloat162 t2 = __floats2bfloat162_rn(o[2 * i] * inv, o[2 * i + 1] * inv);
            w[i] = *reinterpret_cast<const uint32_t*>(&t2);
          } else {
            const __half2 t2 = __floats2half2_rn(o[2 * i] * inv, o[2 * i + 1] * inv);
            w[i] = *reinterpret_cast<const uint32_t*>(&t2);
          }
        }
        uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
      }
    }
    if (q < SQ && p.LSE) {
      const long long li = fa_lse_index(false, z, h, p.NH, p.SQ, 0, p.lse_total_q, q);
      p.LSE[li] = l > 0.f ? m_ref * FA_LN2 + logf(l) : -INFINITY;
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
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// 4-D view [B][H][S][D] (dim 0 innermost) with 128-byte swizzled boxes of 64 x rows
bool make_map(CUtensorMap* m, const void* base, bool bf16, long long D, long long S, long long H, long long B,
              const FaStrides& st, int box_rows) {
  auto enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  // with a single batch entry the batch stride is never used: give it a valid (aligned) value
  const long long sb = (B > 1) ? st.b : ((st.s * S > st.h * H ? st.s * S : st.h * H) + 7) / 8 * 8;
  const cuuint64_t strides[3] = {(cuuint64_t)st.s * 2, (cuuint64_t)st.h * 2, (cuuint64_t)sb * 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  for (int i = 0; i < 3; ++i)
    if (strides[i] % 16 != 0 || strides[i] >= (1ull << 40)) return false;
  if (((uintptr_t)base) % 16 != 0) return false;
  const CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                         const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// paged cache rows [rows][H][D] as 3-D (D, H, rows) with 128-byte swizzled boxes of 64 x 1 x R
bool make_map3(CUtensorMap* m, const void* base, bool bf16, long long D, long long H, long long rows, int R) {
  auto enc = encode_fn();
  if (!enc || ((uintptr_t)base) % 16 != 0) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)rows};
  const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)(H * D) * 2};
  const cuuint32_t box[3] = {64, 1, (cuuint32_t)R};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base),
             dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D, bool BF16, bool FEAT>
int launch(const FaFwdParams& p, cudaStream_t st, const CUtensorMap& mq, const CUtensorMap& mk,
           const CUtensorMap& mv) {
  using C = Cfg<D>;
  static unsigned long long done = 0;
  if (int rc = fa::ensure_smem((const void*)fwd_tc_kernel<D, BF16, FEAT>, C::SMEM, &done)) return rc;
  // work items: (query tile, head, batch) for dense requests; varlen requests enumerate every
  // sequence's query tiles back to back (at most ceil(total_q / BM) + batch of them, each for every
  // head).  One persistent CTA per SM walks them.
  const long long tiles = p.cu_q ? (p.lse_total_q + BM - 1) / BM + p.batch : (long long)((p.SQ + BM - 1) / BM) * p.batch;
  const long long n_items = tiles * p.NH;
  if (n_items > 0x7fffffffLL) {
    fa::set_error("forward: %lld query tiles exceed the work-item range", n_items);
    return FA_ERR_SIZE;
  }
  const int grid = (int)std::min<long long>(n_items, fa::num_sms());
  fwd_tc_kernel<D, BF16, FEAT><<<grid, NTHREADS, C::SMEM, st>>>(mq, mk, mv, p, (int)n_items);
  fa::count_launch();
  return fa::cuda_status(cudaGetLastError(), "fwd_sm100 launch");
}

// The two-tile kernel, when it applies: D = 128, dense, no softcap / alibi / dropout, and the build
// gave it exactly the 168 registers per thread its register split is computed from (checked once;
// otherwise every request stays on the single-tile kernel).  Returns -1 when not taken.
template <bool BF16, bool DROP>
bool pp_ready() {
  static int regs = -1;
  if (regs < 0) {
    cudaFuncAttributes attr;
    regs = cudaFuncGetAttributes(&attr, (const void*)fwd_pp_kernel<BF16, DROP>) == cudaSuccess ? attr.numRegs : 0;
  }
  return regs == PP_REGS;
}

template <bool BF16, bool DROP>
int launch_pp(const FaFwdParams& p, cudaStream_t st, const CUtensorMap& mq, const CUtensorMap& mk,
              const CUtensorMap& mv) {
  if (!pp_ready<BF16, DROP>()) return -1;
  static unsigned long long done = 0;
  if (int rc = fa::ensure_smem((const void*)fwd_pp_kernel<BF16, DROP>, PpCfg::SMEM, &done)) return rc;
  dim3 grid((p.SQ + 2 * BM - 1) / (2 * BM), p.NH, p.batch);
  fwd_pp_kernel<BF16, DROP><<<grid, PP_THREADS, PpCfg::SMEM, st>>>(mq, mk, mv, p);
  fa::count_launch();
  return fa::cuda_status(cudaGetLastError(), "fwd_sm100 launch");
}

template <bool BF16, bool FEAT>
int launch_d(const FaFwdParams& p, cudaStream_t st, const CUtensorMap& mq, const CUtensorMap& mk,
             const CUtensorMap& mv) {
  // Two query tiles per CTA: ~1.1x the rows per second of the one-tile kernel, but half as many
  // CTAs, so the choice compares whole waves: two tiles when ceil(n2 / SMs) * 2 / 1.1 <=
  // ceil(n1 / SMs) (n1, n2 = CTAs of each kernel; a two-tile CTA takes ~2 / 1.1 one-tile CTAs).
  // FABLE_ATTN_FWD_TILES=1 / =2 forces one or two tiles per CTA wherever the two-tile kernel
  // applies (dropout qualifies when its keep mask is precomputed; softcap and alibi do not).
  const bool drop = p.dropout_p > 0.f;
  const bool eligible = p.HD == 128 && p.cu_q == nullptr && p.block_table == nullptr && p.softcap <= 0.f &&
                        p.alibi_slopes == nullptr && (!drop || p.dropout_bits != nullptr) && p.rot_cos == nullptr;
  const long long sms = fa::num_sms();
  const long long n2 = (long long)((p.SQ + 2 * BM - 1) / (2 * BM)) * p.NH * p.batch;
  const long long n1 = (long long)((p.SQ + BM - 1) / BM) * p.NH * p.batch;
  bool two = eligible && (double)((n2 + sms - 1) / sms) * (2.0 / 1.1) <= (double)((n1 + sms - 1) / sms);
  if (const char* force = getenv("FABLE_ATTN_FWD_TILES")) two = eligible && force[0] == '2';
  if (two) {
    const int rc = drop ? launch_pp<BF16, true>(p, st, mq, mk, mv) : launch_pp<BF16, false>(p, st, mq, mk, mv);
    if (rc >= 0) return rc;
  }
  if (p.HD <= 64) return launch<64, BF16, FEAT>(p, st, mq, mk, mv);
  if (p.HD <= 128) return launch<128, BF16, FEAT>(p, st, mq, mk, mv);
  return launch<256, BF16, FEAT>(p, st, mq, mk, mv);
}

}  // namespace

namespace fa {

// Takes fp16/bf16 requests with any head_dim that is a multiple of 16 up to 256 (tiles of 64, 128
// or 256 columns, zero-padded by the TMA), 16-byte aligned rows and strides; everything else is
// left to the CUDA-core kernel (*taken = false).
int fwd_sm100(const FaFwdParams& p, int dtype, cudaStream_t st, bool* taken) {
  *taken = false;
  if (p.HD % 16 != 0 || p.HD < 16 || p.HD > 256) return FA_OK;
  // the kernels scale the row max of the raw scores (the max commutes with a positive factor); a
  // zero or negative softmax scale runs on the CUDA-core kernel
  if (!(p.scale > 0.f)) return FA_OK;
  if (getenv("FABLE_ATTN_DISABLE_TC")) return FA_OK;
  int dev = current_device(), major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) return FA_OK;
  const bool bf16 = dtype == FA_DTYPE_BF16;
  const bool varlen = p.cu_q != nullptr;
  // varlen tensors are (total, H, D): a 4-D map with one batch entry whose rows are the packed
  // tokens, bounded by the tensors' true row counts so that no box reads past them (rows of the
  // next sequence are loaded but masked, rows past the last token read as zeros)
  long long rows_q, rows_k;
  if (varlen) {
    if (p.lse_total_q <= 0 || (p.total_k <= 0 && !p.block_table)) return FA_OK;
    rows_q = p.lse_total_q;
    rows_k = p.total_k;
  } else {
    rows_q = p.SQ;
    rows_k = p.SK;
  }
  const int NKV = p.NH / p.gqa;
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, p.Q, bf16, p.HD, rows_q, p.NH, varlen ? 1 : p.batch, p.sQ, BM)) return FA_OK;
  if (p.block_table) {
    // paged cache [num_blocks * page rows][NKV][HD]: boxes of one page slice (a power of two of at
    // least 8 rows, so each slice starts on a 1 KB swizzle atom)
    if (p.page < 8 || (p.page & (p.page - 1)) || p.num_blocks * (long long)p.page >= (1ll << 31)) return FA_OK;
    if (!make_map3(&mk, p.K, bf16, p.HD, NKV, p.num_blocks * (long long)p.page, std::min(p.page, BN)) ||
        !make_map3(&mv, p.V, bf16, p.HD, NKV, p.num_blocks * (long long)p.page, std::min(p.page, BN)))
      return FA_OK;
  } else {
    if (!make_map(&mk, p.K, bf16, p.HD, rows_k, NKV, varlen ? 1 : p.batch, p.sK, BN)) return FA_OK;
    if (!make_map(&mv, p.V, bf16, p.HD, rows_k, NKV, varlen ? 1 : p.batch, p.sV, BN)) return FA_OK;
  }
  if (((uintptr_t)p.O) % 16 || (p.sO.s % 8) || (p.sO.h % 8) || (!varlen && p.sO.b % 8)) return FA_OK;
  *taken = true;
  const bool feat = p.softcap > 0.f || p.alibi_slopes != nullptr || p.dropout_p > 0.f;
  if (bf16) return feat ? launch_d<true, true>(p, st, mq, mk, mv) : launch_d<true, false>(p, st, mq, mk, mv);
  return feat ? launch_d<false, true>(p, st, mq, mk, mv) : launch_d<false, false>(p, st, mq, mk, mv);
}

}  // namespace fa

extern "C" FA_API int fa_forward_two_tile_ready(int bf16) {
  int dev = fa::current_device(), major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
    return 0;
  if (major != 10 || minor != 0) return 0;
  return (bf16 ? (pp_ready<true, false>() && pp_ready<true, true>())
               : (pp_ready<false, false>() && pp_ready<false, true>())) ? 1 : 0;
}

// Self-test of the bounded mbarrier wait every pipeline uses: one thread waits on a barrier that
// nothing ever arrives on (no copy or MMA is in flight), gives up after limit_ns and records
// FA_DEVERR_WAIT_SELFTEST; the kernel then returns normally and the context stays usable.
__global__ void wait_selftest_kernel(unsigned long long limit_ns) {
  __shared__ __align__(8) unsigned long long slot;
  const uint32_t b = smem_u32(&slot);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    fence_barrier_init();
    if (!mbar_wait(b, 0, limit_ns)) record_error(FA_DEVERR_WAIT_SELFTEST);
  }
}

extern "C" FA_API int fa_wait_selftest(unsigned long long limit_ns, void* stream) {
  if (limit_ns == 0 || limit_ns > 10000000000ull) {
    fa::set_error("wait self-test: limit_ns=%llu outside (0, 1e10]", limit_ns);
    return FA_ERR_INVALID;
  }
  wait_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(limit_ns);
  fa::count_launch();
  return fa::cuda_status(cudaGetLastError(), "wait self-test launch");
}

extern "C" FA_API int fa_device_error(int clear) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_fwd_error, sizeof(int));
  if (clear) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_fwd_error, &zero, sizeof(int));
  }
  return v | (fa::dec_device_error(clear) ? 64 : 0) | (fa::bwd_device_error(clear) ? 128 : 0) |
         (fa::rot_device_error(clear) ? 256 : 0) | (fa::fwd_simt_device_error(clear) ? 1024 : 0);
}
