// decode_sm100.cu — paged-KV decode on the 5th-generation tensor cores (sm_100a): fp16/bf16 cache,
// head_dim 128, up to 16 query rows per kv head, a query row being one (new token, query head)
// pair of the kv head's group (one token with gqa <= 16, or several tokens of a speculative /
// multi-token step, each row with its own key range: causal among appended tokens, its own window
// start, alibi offset and rotary position).
//
// Decode streams every K/V byte of a sequence's context once per kv head; with GQA 4 that is
// two multiply-adds per streamed byte, more than the CUDA cores sustain next to HBM3e.  Both
// contractions therefore run on tcgen05, transposed so that the long dimension is M:
//   S^T = K Q^T    M = 128 positions (TMEM lanes), N = query rows, K = head dim
//   O^T = V^T P^T  M = 128 head dims (TMEM lanes), N = query rows, K = 128 positions
// K and V tiles arrive by TMA (128-byte swizzle; one box per page slice and 64-column chunk)
// in separate rings (K: 2 stages, freed as soon as S^T is computed; V: 4 stages, 3 for 16 query
// rows, held until P.V completes), each fed by its own producer warp; Q and P^T sit in shared
// memory; S^T and O^T are double-buffered in TMEM.  Q and P enter the MMAs as 16-bit hi + lo
// pairs (rows r and NRV + r of the N dimension, summed when S^T / O^T are read), so the
// contractions keep ~22 bits of q and p as the reference's fp32 arithmetic does; K and V are
// used exactly as stored.
// The 128 softmax threads own one position each for S^T and one head dim each for O^T.  Each
// tile's O^T is folded into register accumulators with the tile's max change, so TMEM is never
// rescaled.  The row max is lazy: a tile triggers a CTA-wide max only when a score exceeds the
// running reference by more than 2^8, otherwise probabilities are taken against the reference.
//
// Work split (stream-K): the contexts [lo, ctx) of all (sequence, kv head) groups, cut at
// absolute 128-position tile boundaries, form one sequence of tiles (sequence-major).  CTA c of
// the persistent grid (one per SM) takes tiles [c*Q, (c+1)*Q), Q = ceil(total / grid) (raised so
// that no group spans more than nsplit CTAs), so every CTA streams the same number of bytes.
// Each piece of a group a CTA covers is a segment; it writes split slot c - first CTA of the
// group (m in log2 units, l, acc[128]) for every query head of the group, and the CTA holding
// the group's last segment writes the remaining slots neutral (m = -inf) for the merge kernel,
// which handles empty contexts itself.  Semantics follow the FaDecParams contract of
// fable_attn.h (kernels/fa_decode.hip:57-252 of the reference).
//
// Warp roles (224 threads): 0-3 softmax / accumulate, 4 K producer, 5 MMA issuer, 6 V producer.
// Every wait is bounded (a timeout records an error and unwinds), and the softmax warps break
// out of their loops only together (bar.red.and), so no named barrier is left waiting.
#include <cudaTypedefs.h>
#include <algorithm>
#include <cstdlib>
#include <type_traits>
#include "fa_common.cuh"
#include "fa_launch.h"
#include "sm100_ptx.cuh"
#include "decode_common.cuh"

namespace {

using namespace sm100;
using fa_dec::page_of;

constexpr int TT = 128;            // positions per tile (M of S^T)
constexpr int HD = 128;            // head dim (M of O^T)
constexpr int NK = 2;              // K ring stages (a K tile is free once S^T is computed)
constexpr int NTH = 224;
constexpr int TILE_B = TT * HD * 2;             // one K or V tile, 32 KB
constexpr int CHUNK_B = TT * 128;               // one 64-column chunk of a tile
constexpr float LAZY = 8.f;                     // log2 headroom of the lazy row max

// NRV query rows (a power of two >= gqa); the MMAs' N = NQ rows hold hi rows [0, NRV), lo rows
// [NRV, 2 NRV) and zeros above
template <int NRV>
struct Lay {
  static constexpr int NV = NRV >= 16 ? 3 : 4;        // V ring stages (held until P.V completes)
  static constexpr int NQ = 2 * NRV < 16 ? 16 : 2 * NRV;
  static constexpr uint32_t S_COL = 0, O_COL = 2 * NQ, TMEM_COLS = 4 * NQ <= 64 ? 64 : 128;
  static constexpr int K = 0;                         // [NK][2 chunks][128 rows][128 B]
  static constexpr int V = NK * TILE_B;               // [NV][2 chunks][128 rows][128 B]
  static constexpr int Q = (NK + NV) * TILE_B;        // [2][2 chunks][NQ rows][128 B]
  static constexpr int QB = NQ * HD * 2;
  static constexpr int P = Q + 2 * QB;                // [2][2 chunks][NQ rows][128 B]
  static constexpr int PB = NQ * TT * 2;
  static constexpr int RED = P + 2 * PB;              // cross-warp reductions [4][NRV] fp32
  static constexpr int BAR = RED + 4 * NRV * 4;
  // barriers: KF[NK] KE[NK] VF[NV] VE[NV] SF[2] PF[2] OF[2] QF[2] QE[2] DRAIN
  static constexpr int KF = 0, KE = NK, VF = 2 * NK, VE = VF + NV, SF = VE + NV, PF = SF + 2, OF = PF + 2,
                       QFULL = OF + 2, QE = QFULL + 2, DRAIN = QE + 2, NBAR = DRAIN + 1;
  static constexpr int SMEM = BAR + 8 * NBAR + 1024;  // + 1 KB to align the base for SW128
  static_assert(Q % 1024 == 0 && P % 1024 == 0 && QB % 1024 == 0 && PB % 1024 == 0,
                "swizzled operand tiles must be 1 KB aligned");
  static_assert(SMEM <= 232448 - 2048, "shared memory per CTA");
};

__device__ int g_dectc_error = 0;
__device__ __forceinline__ void record_error(int code) { atomicOr(&g_dectc_error, code); }

// named barrier 1 over the 128 softmax threads, AND / OR of a predicate (uniform decisions)
__device__ __forceinline__ bool bar_and_128(bool v) {
  uint32_t r;
  asm volatile("{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\tbar.red.and.pred po, 1, 128, pi;\n\t"
               "selp.u32 %0, 1, 0, po;\n\t}"
               : "=r"(r) : "r"((uint32_t)v) : "memory");
  return r != 0;
}
__device__ __forceinline__ bool bar_or_128(bool v) {
  uint32_t r;
  asm volatile("{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\tbar.red.or.pred po, 1, 128, pi;\n\t"
               "selp.u32 %0, 1, 0, po;\n\t}"
               : "=r"(r) : "r"((uint32_t)v) : "memory");
  return r != 0;
}
__device__ __forceinline__ void bar_sync_128() { asm volatile("bar.sync 2, 128;" ::: "memory"); }

__device__ __forceinline__ uint64_t desc_kmajor(uint32_t tile, int rows, int kstep) {
  return sdesc_sw128(tile + (kstep / 4) * rows * 128 + (kstep % 4) * 32, 16, 1024);
}
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t tile, int rows, int kstep) {
  return sdesc_sw128(tile + kstep * 16 * 128, rows * 128, 1024);
}
// byte offset of element (row r, column c) of a [rows][64-column chunks] 16-bit tile, 128-B swizzle
__device__ __forceinline__ uint32_t swz_off(int rows, int r, int c) {
  return (uint32_t)((c / 64) * rows * 128 + r * 128 + ((((c % 64) >> 3) ^ (r & 7)) << 4) + (c % 8) * 2);
}

template <typename T>
__device__ __forceinline__ float round16(float a) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(__float2bfloat16_rn(a));
  else return __half2float(__float2half_rn(a));
}
template <typename T>
__device__ __forceinline__ unsigned short bits16(float a) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat16_as_ushort(__float2bfloat16_rn(a));
  else return __half_as_ushort(__float2half_rn(a));
}

// keys of sequence b's new tokens: the union [lo, ctx) of every token's range (token tk at
// position ctx0 + tk sees [max(leftpad, ctx0 + tk - window + 1), ctx0 + tk + 1) with append,
// [.., ctx0) without, so the union runs from the first token's start to the last token's end);
// returns its tile count (tiles lo/TT .. (ctx-1)/TT)
// A launch covers new tokens [tk0, tk0 + nqc) (groups of more than 16 query rows run in token
// chunks, one launch each); the range is that of its tokens.
__device__ __forceinline__ int seq_tiles(const FaDecParams& p, int b, int& lo, int& ctx, int tk0, int nqc) {
  const int ctx0 = p.ctx_len[b];
  ctx = ctx0 + (p.append ? tk0 + nqc : 0);
  int l = p.leftpad ? p.leftpad[b] : 0;
  if (p.window >= 0 && ctx0 + tk0 - p.window + 1 > l) l = ctx0 + tk0 - p.window + 1;
  lo = l > 0 ? l : 0;
  return ctx > lo ? (ctx - 1) / TT + 1 - lo / TT : 0;
}

// One CTA's walk over its tile range [start, end) of the global tile sequence
struct Seg {
  int b, kvh, slot, lo, ctx;
  int t0, t1;      // absolute tile indices [t0, t1)
  bool last;       // the group's last segment
};
struct Walk {
  long long start, end, Q, off;   // off: global tile offset of group (b, kvh)
  int b, kvh, c, tk0, nqc;
  __device__ bool next(const FaDecParams& p, int NKV, Seg& s) {
    while (b < p.batch) {
      int lo, ctx;
      const int n = seq_tiles(p, b, lo, ctx, tk0, nqc);
      if (n == 0) {   // empty context: no tiles, the merge handles it
        ++b;
        kvh = 0;
        continue;
      }
      if (off >= end) return false;
      const long long a0 = start > off ? start : off, a1 = end < off + n ? end : off + n;
      s.b = b; s.kvh = kvh; s.lo = lo; s.ctx = ctx;
      s.t0 = lo / TT + (int)(a0 - off);
      s.t1 = lo / TT + (int)(a1 - off);
      s.slot = c - (int)(off / Q);
      s.last = off + n <= end;
      off += n;
      if (++kvh == NKV) { kvh = 0; ++b; }
      return true;
    }
    return false;
  }
};

// NRV: query rows handled (a power of two >= gqa, <= 16)
template <typename T, int NRV>
__global__ void __launch_bounds__(NTH, 1)
    dec_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, const FaDecParams p,
                  const int tk0, const int nqc) {
  using L = Lay<NRV>;
  constexpr int NQ = L::NQ;
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smraw[];
  __shared__ uint32_t s_tmem;
  __shared__ long long s_part[NTH];   // per-thread tile sums, then their exclusive prefix
  __shared__ int s_maxn, s_b0;
  __shared__ int s_rlo[16], s_rhi[16];   // several new tokens: each query row's keys [rlo, rhi)
  __shared__ float s_rtk[16];            // and its token index
  __shared__ long long s_total, s_off0;
  const uint32_t sb = (smem_u32(smraw) + 1023u) & ~1023u;
  uint8_t* sg = smraw + (sb - smem_u32(smraw));
  auto bar = [&](int i) { return sb + (uint32_t)L::BAR + 8u * (uint32_t)i; };

  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int NKV = p.NH / p.gqa, nh = nqc * p.gqa;   // live query rows: (new token, head) pairs
  const int shift = __ffs(p.page) - 1, pmask = p.page - 1;
  const int R = p.page < TT ? p.page : TT;   // rows of one page-slice box
  const int c = blockIdx.x;

  // ---- schedule: per-sequence tile counts (each thread a chunk of sequences), their prefix
  const int CB = (p.batch + NTH - 1) / NTH;
  {
    long long sum = 0;
    int mx = 0;
    for (int b = t * CB; b < min(p.batch, (t + 1) * CB); ++b) {
      int lo, ctx;
      const int n = seq_tiles(p, b, lo, ctx, tk0, nqc);
      sum += n;
      mx = max(mx, n);
    }
    if (t == 0) { s_maxn = 0; s_b0 = p.batch; s_off0 = 0; }
    s_part[t] = sum;
    __syncthreads();
    atomicMax(&s_maxn, mx);
    if (t == 0) {
      long long a = 0;
      for (int i = 0; i < NTH; ++i) { const long long v = s_part[i]; s_part[i] = a; a += v; }
      s_total = a * NKV;
    }
  }
  if (t == 0) {
    for (int i = 0; i < L::NBAR; ++i) {
      uint32_t cnt = 1;
      if (i == L::PF || i == L::PF + 1 || i == L::QFULL || i == L::QFULL + 1) cnt = 128;
      mbar_init(bar(i), cnt);
    }
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(&s_tmem), L::TMEM_COLS);
    tmem_relinquish();
  }
  // Q and P^T rows >= 2 NRV stay zero for the whole kernel (16-byte units of the 4 buffers)
  for (int e = t; e < 2 * (L::QB + L::PB) / 16; e += NTH) {
    const int byte = e * 16, pair = L::QB + L::PB, bufi = byte / pair, in = byte % pair;
    const bool isq = in < L::QB;
    const int off = isq ? in : in - L::QB, row = (off % (NQ * 128)) / 128;
    if (row >= 2 * NRV)
      *reinterpret_cast<uint4*>(sg + (isq ? L::Q + bufi * L::QB : L::P + bufi * L::PB) + off) = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  const long long total = s_total;
  const int G = gridDim.x;
  long long Qt = (total + G - 1) / G;
  if (Qt < (long long)((s_maxn + p.nsplit - 2) / (p.nsplit - 1))) Qt = (s_maxn + p.nsplit - 2) / (p.nsplit - 1);
  if (Qt < 1) Qt = 1;
  const long long start = (long long)c * Qt, end = (c == G - 1) ? (1ll << 62) : start + Qt;
  // the thread whose chunk of sequences holds tile `start` finds the first sequence
  if (start < total) {
    const long long lo_t = s_part[t] * NKV;
    const long long hi_t = (t + 1 < NTH ? s_part[t + 1] * NKV : total);
    if (start >= lo_t && start < hi_t) {
      long long off = lo_t;
      for (int b = t * CB; b < min(p.batch, (t + 1) * CB); ++b) {
        int lo, ctx;
        const int n = seq_tiles(p, b, lo, ctx, tk0, nqc);
        if (start < off + (long long)n * NKV) {
          s_b0 = b;
          s_off0 = off;
          break;
        }
        off += (long long)n * NKV;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  auto walk0 = [&]() {
    Walk w;
    w.start = start; w.end = end; w.Q = Qt; w.c = c;
    w.b = s_b0; w.kvh = 0; w.off = s_off0; w.tk0 = tk0; w.nqc = nqc;
    if (w.b < p.batch) {   // the group of sequence b0 that holds tile `start`
      int lo, ctx;
      const int n = seq_tiles(p, w.b, lo, ctx, tk0, nqc);
      w.kvh = (int)((start - w.off) / n);
      w.off += (long long)w.kvh * n;
    }
    return w;
  };

  if (warp == 4 || warp == 6) {
    // ============================================================ TMA producers: warp 4 K, warp 6 V
    if (lane == 0) {
      const bool isk = warp == 4;
      const int NR = isk ? NK : L::NV;
      const int FULL = isk ? L::KF : L::VF, FREE = isk ? L::KE : L::VE;
      const CUtensorMap* map = isk ? &tmK : &tmV;
      const uint32_t ring = sb + (isk ? L::K : L::V);
      Walk w = walk0();
      Seg sgm;
      int g = 0;
      bool ok = true;
      while (ok && w.next(p, NKV, sgm)) {
        for (int tile = sgm.t0; tile < sgm.t1; ++tile, ++g) {
          const int s = g % NR;
          if (g >= NR && !mbar_wait(bar(FREE + s), ((g / NR) - 1) & 1)) { ok = false; break; }
          const int base = tile * TT;
          uint32_t bytes = 0;
          for (int k = 0; k < TT / R; ++k) {
            const int pos0 = base + k * R;
            if (pos0 + R <= sgm.lo || pos0 >= sgm.ctx) continue;
            bool okp;
            page_of(p, sgm.b, pos0, shift, okp);
            if (okp) bytes += (uint32_t)(R * HD * 2);
          }
          mbar_expect_tx(bar(FULL + s), bytes);
          const uint32_t dst = ring + s * TILE_B;
          for (int k = 0; k < TT / R; ++k) {
            const int pos0 = base + k * R;
            if (pos0 + R <= sgm.lo || pos0 >= sgm.ctx) continue;
            bool okp;
            const long long blk = page_of(p, sgm.b, pos0, shift, okp);
            if (!okp) continue;
            const int row = (int)(blk * p.page + (pos0 & pmask));
#pragma unroll
            for (int ch = 0; ch < HD / 64; ++ch)
              tma_load_3d(dst + ch * CHUNK_B + k * R * 128, map, 64 * ch, sgm.kvh, row, bar(FULL + s));
          }
        }
      }
      if (!ok) {
        record_error(1);
        // copies still in flight must land before the CTA's shared memory is released
        for (int j = max(0, g - NR); j < g; ++j) mbar_wait(bar(FULL + j % NR), (j / NR) & 1, 1000000000ull);
      }
    }
  } else if (warp == 5) {
    // ============================================================ MMA issuer (lane 0)
    constexpr uint32_t ID_S = idesc_f16(BF16 ? 1 : 0, TT, NQ, 0, 0);   // S^T = K Q^T
    constexpr uint32_t ID_O = idesc_f16(BF16 ? 1 : 0, HD, NQ, 1, 0);   // O^T = V^T P^T, V^T MN-major
    int g = 0, qi = 0;
    bool ok = true;
    auto issue_pv = [&](int gg) -> bool {
      const int s = gg % L::NV;
      if (!mbar_wait_warp(bar(L::PF + (gg & 1)), (gg >> 1) & 1)) return false;
      if (!mbar_wait_warp(bar(L::VF + s), (gg / L::NV) & 1)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t vt = sb + L::V + s * TILE_B, pt = sb + L::P + (gg & 1) * L::PB;
#pragma unroll
        for (int kk = 0; kk < TT / 16; ++kk)
          mma_ss(tmem + L::O_COL + (gg & 1) * NQ, desc_mnmajor(vt, TT, kk), desc_kmajor(pt, NQ, kk), ID_O, kk > 0);
        mma_commit(bar(L::OF + (gg & 1)));
        mma_commit(bar(L::VE + s));
      }
      __syncwarp();
      return true;
    };
    Walk w = walk0();
    Seg sgm;
    while (ok && w.next(p, NKV, sgm)) {
      if (!mbar_wait_warp(bar(L::QFULL + (qi & 1)), (qi >> 1) & 1)) { ok = false; break; }
      for (int tile = sgm.t0; tile < sgm.t1; ++tile, ++g) {
        const int s = g % NK;
        if (!mbar_wait_warp(bar(L::KF + s), (g / NK) & 1)) { ok = false; break; }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t kt = sb + L::K + s * TILE_B, qt = sb + L::Q + (qi & 1) * L::QB;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk)
            mma_ss(tmem + L::S_COL + (g & 1) * NQ, desc_kmajor(kt, TT, kk), desc_kmajor(qt, NQ, kk), ID_S, kk > 0);
          mma_commit(bar(L::SF + (g & 1)));
          mma_commit(bar(L::KE + s));
          if (tile == sgm.t1 - 1) mma_commit(bar(L::QE + (qi & 1)));
        }
        __syncwarp();
        // P.V of the previous tile of this segment overlaps the softmax of this one
        if (tile > sgm.t0 && !issue_pv(g - 1)) { ok = false; break; }
      }
      // the segment's last P.V goes out before the next segment's q is awaited
      if (ok && !issue_pv(g - 1)) ok = false;
      ++qi;
    }
    if (!ok) record_error(2);
    if (lane == 0) mma_commit(bar(L::DRAIN));
    __syncwarp();
    if (!mbar_wait_warp(bar(L::DRAIN), 0)) record_error(4);
  } else {
    // ============================================================ softmax / accumulate (warps 0-3)
    const uint32_t la = tmem + ((uint32_t)(warp * 32) << 16);
    const float scale2 = p.scale * FA_LOG2E;
    const bool cap_on = p.softcap > 0.f;
    const float cap_in = cap_on ? p.scale / p.softcap : 0.f, cap2 = p.softcap * FA_LOG2E;
    float* red = reinterpret_cast<float*>(sg + L::RED);
    float acc[NRV], mref[NRV], lt[NRV], cprev[NRV], slope2[NRV];
    int g = 0, qi = 0;
    bool ok = true;
    auto ld_cols = [&](uint32_t addr, float* v) {   // NQ columns of this thread's lane
      tmem_ld16(addr, v);
      if constexpr (NQ == 32) tmem_ld16(addr + 16, v + 16);
    };
    // q rows of a segment's group into Q buffer `buf`: rotary in fp32, then 16-bit hi / lo rows
    // (one job = one pair of dims that rotate together)
    auto write_q = [&](const Seg& sq, int buf) {
      const int hb = sq.kvh * p.gqa;
      const int mode = p.rotary, rdim = p.rotary_dim > 0 ? p.rotary_dim : HD, half = rdim / 2;
      const int rp0 = p.rotary_pos ? p.rotary_pos[sq.b] : p.ctx_len[sq.b];
      uint8_t* qs = sg + L::Q + buf * L::QB;
      for (int j = t; j < NRV * (HD / 2); j += 128) {
        const int r = j / (HD / 2), jj = j % (HD / 2);
        int d1, d2;
        bool rot = false;
        if (mode == 1) {
          if (jj < half) { d1 = jj; d2 = jj + half; rot = true; }
          else { d1 = rdim + 2 * (jj - half); d2 = d1 + 1; }
        } else {
          d1 = 2 * jj; d2 = d1 + 1;
          rot = mode == 2 && jj < half;
        }
        float x1 = 0.f, x2 = 0.f;
        if (r < nh) {   // row r = (new token r / gqa, head r % gqa of the group)
          const int tk = tk0 + r / p.gqa, rp = rp0 + tk;
          const T* qg = (const T*)p.q + (((long long)sq.b * p.nq + tk) * p.NH + hb + r % p.gqa) * HD;
          x1 = Elem<T>::to_f(qg[d1]);
          x2 = Elem<T>::to_f(qg[d2]);
          if (rot) {
            const float cs = p.cos[(long long)rp * half + jj], sn = p.sin[(long long)rp * half + jj];
            const float y1 = x1 * cs - x2 * sn, y2 = x2 * cs + x1 * sn;
            x1 = y1; x2 = y2;
          }
        }
        const float h1 = round16<T>(x1), h2 = round16<T>(x2);
        *reinterpret_cast<unsigned short*>(qs + swz_off(NQ, r, d1)) = bits16<T>(h1);
        *reinterpret_cast<unsigned short*>(qs + swz_off(NQ, r, d2)) = bits16<T>(h2);
        *reinterpret_cast<unsigned short*>(qs + swz_off(NQ, NRV + r, d1)) = bits16<T>(x1 - h1);
        *reinterpret_cast<unsigned short*>(qs + swz_off(NQ, NRV + r, d2)) = bits16<T>(x2 - h2);
      }
      fence_proxy_async_smem();
      mbar_arrive(bar(L::QFULL + buf));
    };
    Walk w = walk0();
    Seg cur, nxt;
    bool have = w.next(p, NKV, cur);
    if (have) write_q(cur, 0);
    while (ok && have) {
      // the next segment's q goes out now, so the MMAs can start it as soon as this one ends
      const bool have_n = w.next(p, NKV, nxt);
      if (have_n) {
        const int nb = (qi + 1) & 1;
        const bool qfree = (qi + 1 < 2) ? true : mbar_wait_warp(bar(L::QE + nb), (((qi + 1) >> 1) - 1) & 1);
        if (!bar_and_128(qfree)) { ok = false; break; }
        write_q(nxt, nb);
      }
      const int hbase = cur.kvh * p.gqa;
#pragma unroll
      for (int r = 0; r < NRV; ++r) {
        acc[r] = 0.f; mref[r] = -INFINITY; lt[r] = 0.f; cprev[r] = 1.f;
        slope2[r] = (p.alibi && r < nh) ? p.alibi[hbase + r % p.gqa] * FA_LOG2E : 0.f;
      }
      const int qpos = p.ctx_len[cur.b];
      // several new tokens: each row's own keys [rlo, rhi) and its offset from the first token
      const bool multi = p.nq > 1;
      if (multi) {
        if (t < NRV) {
          const int tk = tk0 + t / p.gqa, ctx0 = qpos;
          int l = p.leftpad ? p.leftpad[cur.b] : 0;
          if (p.window >= 0 && ctx0 + tk - p.window + 1 > l) l = ctx0 + tk - p.window + 1;
          s_rlo[t] = t < nh ? max(l, 0) : 0;
          s_rhi[t] = t < nh ? ctx0 + (p.append ? tk + 1 : 0) : 0;
          s_rtk[t] = (float)tk;
        }
        bar_sync_128();
      }
      // O^T of tile gg into the accumulators (thread = head dim), scaled by that tile's change
      auto consume = [&](int gg) -> bool {
        const bool got = mbar_wait_warp(bar(L::OF + (gg & 1)), (gg >> 1) & 1);
        if (!bar_and_128(got)) return false;
        tc_fence_after();
        float o[NQ];
        ld_cols(la + L::O_COL + (gg & 1) * NQ, o);
        tc_wait_ld();
#pragma unroll
        for (int r = 0; r < NRV; ++r) acc[r] = fmaf(acc[r], cprev[r], o[r] + o[NRV + r]);
        return true;
      };
      for (int tile = cur.t0; tile < cur.t1; ++tile, ++g) {
        // this thread's position and its page check, issued before the wait so that the
        // block-table load overlaps the S^T MMA
        const int pos = tile * TT + t;
        bool valid = pos >= cur.lo && pos < cur.ctx;
        if (valid) {
          bool okp;
          page_of(p, cur.b, pos, shift, okp);
          valid = okp;
        }
        const bool got = mbar_wait_warp(bar(L::SF + (g & 1)), (g >> 1) & 1);
        if (!bar_and_128(got)) { ok = false; break; }
        tc_fence_after();
        float s[NQ];
        ld_cols(la + L::S_COL + (g & 1) * NQ, s);
        tc_wait_ld();
        float v[NRV];
        bool need = false;
        const float dpos = (float)(pos - qpos);
        if (!multi) {
#pragma unroll
          for (int r = 0; r < NRV; ++r) {
            const float sr = s[r] + s[NRV + r];   // q_hi . k + q_lo . k
            float x = cap_on ? cap2 * fa_tanh(sr * cap_in) : sr * scale2;
            x = fmaf(slope2[r], dpos, x);
            v[r] = (valid && r < nh) ? x : -INFINITY;
            need |= v[r] > mref[r] + LAZY;
          }
        } else {
#pragma unroll
          for (int r = 0; r < NRV; ++r) {
            const float sr = s[r] + s[NRV + r];
            float x = cap_on ? cap2 * fa_tanh(sr * cap_in) : sr * scale2;
            x = fmaf(slope2[r], dpos - s_rtk[r], x);   // key - this row's position
            v[r] = (valid && r < nh && pos >= s_rlo[r] && pos < s_rhi[r]) ? x : -INFINITY;
            need |= v[r] > mref[r] + LAZY;
          }
        }
        float corr[NRV];
        if (bar_or_128(need)) {   // exact tile max per row, new reference
#pragma unroll
          for (int r = 0; r < NRV; ++r) {
            float x = v[r];
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
            if (lane == 0) red[warp * NRV + r] = x;
          }
          bar_sync_128();
#pragma unroll
          for (int r = 0; r < NRV; ++r) {
            const float tm = fmaxf(fmaxf(red[r], red[NRV + r]), fmaxf(red[2 * NRV + r], red[3 * NRV + r]));
            const float mn = fmaxf(mref[r], tm);
            corr[r] = (mn == -INFINITY) ? 1.f : ex2(mref[r] - mn);
            mref[r] = mn;
          }
        } else {
#pragma unroll
          for (int r = 0; r < NRV; ++r) corr[r] = 1.f;
        }
        // P^T column of this position as 16-bit hi / lo rows; row sums kept per thread in fp32
        uint8_t* pt = sg + L::P + (g & 1) * L::PB;
#pragma unroll
        for (int r = 0; r < NRV; ++r) {
          const float pr = ex2(v[r] - (mref[r] == -INFINITY ? 0.f : mref[r]));
          lt[r] = fmaf(lt[r], corr[r], pr);
          const float hi = round16<T>(pr);
          *reinterpret_cast<unsigned short*>(pt + swz_off(NQ, r, t)) = bits16<T>(hi);
          *reinterpret_cast<unsigned short*>(pt + swz_off(NQ, NRV + r, t)) = bits16<T>(pr - hi);
        }
        if (!valid) {
          // this position's V row may hold stale or unloaded bytes: P is 0 there, but 0 * NaN is
          // not, so the row is zeroed once its copy (if any) has landed
          const int s = g % L::NV;
          if (!mbar_wait(bar(L::VF + s), (g / L::NV) & 1)) record_error(8);
          uint8_t* vr = sg + L::V + s * TILE_B + t * 128;
#pragma unroll
          for (int ch = 0; ch < HD / 64; ++ch)
#pragma unroll
            for (int u = 0; u < 8; ++u) *reinterpret_cast<uint4*>(vr + ch * CHUNK_B + u * 16) = make_uint4(0, 0, 0, 0);
        }
        // P^T / zeroed V rows visible to the tensor core; S^T (and the last O^T read) ordered
        // before the MMAs that will overwrite those TMEM columns
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(bar(L::PF + (g & 1)));
        if (tile > cur.t0 && !consume(g - 1)) { ok = false; break; }
#pragma unroll
        for (int r = 0; r < NRV; ++r) cprev[r] = corr[r];
      }
      if (ok && !consume(g - 1)) ok = false;
      if (!ok) break;
      // ---- finalize: row sums over the 128 positions, then this segment's split slot of each
      // head; the group's last segment also clears the slots no CTA reaches
      float lsum[NRV];
#pragma unroll
      for (int r = 0; r < NRV; ++r) {
        float x = lt[r];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
        if (lane == 0) red[warp * NRV + r] = x;
      }
      bar_sync_128();
#pragma unroll
      for (int r = 0; r < NRV; ++r) lsum[r] = (red[r] + red[NRV + r]) + (red[2 * NRV + r] + red[3 * NRV + r]);
      // split slots of row r = (token tk, head g): scratch row ((b * nq + tk) * NH + hbase + g)
      auto slot_row = [&](int r) -> long long {
        return (((long long)cur.b * p.nq + tk0 + r / p.gqa) * p.NH + hbase + r % p.gqa) * p.nsplit;
      };
#pragma unroll
      for (int r = 0; r < NRV; ++r) {
        if (r < nh) {
          float* o = p.scratch + (slot_row(r) + cur.slot) * (HD + 2);
          o[2 + t] = acc[r];
          if (t == 0) { o[0] = mref[r]; o[1] = lsum[r]; }
        }
      }
      if (cur.last) {
        const int rest = p.nsplit - 1 - cur.slot;
        for (int e = t; e < nh * rest; e += 128) {
          float* o = p.scratch + (slot_row(e / rest) + cur.slot + 1 + e % rest) * (HD + 2);
          o[0] = -INFINITY;
          o[1] = 0.f;
        }
      }
      cur = nxt;
      have = have_n;
      ++qi;
    }
    if (!ok) record_error(16);
  }
  pdl_trigger();   // the merge kernel may start (it waits for this grid's completion before reading)
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

// cache [rows = num_blocks*page][NKV][HD] as 3-D (HD, NKV, rows); box = 64 columns x 1 head x R
// rows with the 128-byte swizzle (the canonical K-major / MN-major operand layout)
bool tc_map(CUtensorMap* m, const void* base, bool bf16, int NKV, long long rows, int R) {
  auto enc = encode_fn();
  if (!enc || ((uintptr_t)base) % 16) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)NKV, (cuuint64_t)rows};
  const cuuint64_t strides[2] = {(cuuint64_t)HD * 2, (cuuint64_t)NKV * HD * 2};
  const cuuint32_t box[3] = {64, 1, (cuuint32_t)R};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base),
             dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T, int NRV>
int launch(const FaDecParams& p, const CUtensorMap& mk, const CUtensorMap& mv, cudaStream_t st, int tk0, int nqc) {
  static unsigned long long done = 0;
  if (int rc = fa::ensure_smem((const void*)dec_tc_kernel<T, NRV>, Lay<NRV>::SMEM, &done)) return rc;
  dec_tc_kernel<T, NRV><<<fa::num_sms(), NTH, Lay<NRV>::SMEM, st>>>(mk, mv, p, tk0, nqc);
  fa::count_launch();
  return fa::cuda_status(cudaGetLastError(), "decode partial (tcgen05) launch");
}

}  // namespace

namespace fa {
// Split-K partials of the tensor-core decode, or *taken = false when the call is outside its
// envelope (then the CUDA-core kernels run).
int dec_tc_partial(const FaDecParams& p, int dtype, cudaStream_t st, bool* taken) {
  *taken = false;
  if (dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_BF16) return FA_OK;
  // query rows = new tokens x heads of a kv group, at most 16 per launch: larger groups run their
  // tokens in chunks of 16 / gqa, one launch (one pass over the cache) each, up to 8 launches
  if (p.HD != HD || p.nq < 1 || p.gqa > 16 || p.page < 8 || p.num_blocks <= 0 || p.nsplit < 2) return FA_OK;
  const int per = 16 / p.gqa;
  if ((p.nq + per - 1) / per > 8) return FA_OK;
  if (getenv("FABLE_ATTN_DECODE_NO_TC")) return FA_OK;
  const long long rows = p.num_blocks * (long long)p.page;
  if (rows >= (1ll << 31)) return FA_OK;
  const int NKV = p.NH / p.gqa;
  const bool bf16 = dtype == FA_DTYPE_BF16;
  const int R = p.page < TT ? p.page : TT;
  CUtensorMap mk, mv;
  if (!tc_map(&mk, p.Kc, bf16, NKV, rows, R) || !tc_map(&mv, p.Vc, bf16, NKV, rows, R)) return FA_OK;
  *taken = true;
  for (int tk0 = 0; tk0 < p.nq; tk0 += per) {
    const int nqc = std::min(per, p.nq - tk0), qrows = nqc * p.gqa;
    int rc;
    if (bf16) {
      rc = qrows <= 4 ? launch<__nv_bfloat16, 4>(p, mk, mv, st, tk0, nqc)
         : qrows <= 8 ? launch<__nv_bfloat16, 8>(p, mk, mv, st, tk0, nqc)
                      : launch<__nv_bfloat16, 16>(p, mk, mv, st, tk0, nqc);
    } else {
      rc = qrows <= 4 ? launch<__half, 4>(p, mk, mv, st, tk0, nqc)
         : qrows <= 8 ? launch<__half, 8>(p, mk, mv, st, tk0, nqc)
                      : launch<__half, 16>(p, mk, mv, st, tk0, nqc);
    }
    if (rc) return rc;
  }
  return FA_OK;
}

int dec_tc_device_error(int clear) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_dectc_error, sizeof(int));
  if (clear && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_dectc_error, &zero, sizeof(int));
  }
  return v;
}
}  // namespace fa
