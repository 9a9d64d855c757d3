// decode_sm100.cu — paged-KV decode on the 5th-generation tensor cores (sm_100a): one new token
// per sequence, fp16/bf16 cache, head_dim 128, up to 16 query heads per kv head.
//
// Decode streams every K/V byte of a sequence's context once per kv head; with GQA 4 that is
// two multiply-adds per streamed byte, more than the CUDA cores sustain next to HBM3e.  Both
// contractions therefore run on tcgen05, transposed so that the long dimension is M:
//   S^T = K Q^T    M = 128 positions (TMEM lanes), N = 16 query rows, K = head dim
//   O^T = V^T P^T  M = 128 head dims (TMEM lanes), N = 16 query rows, K = 128 positions
// K and V tiles arrive by TMA (128-byte swizzle; one box per page slice and 64-column chunk)
// in a 3-stage ring; Q and P^T sit in shared memory; S^T and O^T are double-buffered in TMEM.
// Q and P enter the MMAs as 16-bit hi + lo pairs (rows r and NRV + r of the N dimension, summed
// when S^T / O^T are read), so the contractions keep ~22 bits of q and p as the reference's fp32
// arithmetic does; K and V are used exactly as stored.
// The 128 softmax threads own one position each for S^T and one head dim each for O^T.  Each
// tile's O^T is folded into register accumulators with the tile's max change, so TMEM is never
// rescaled.  The row max is lazy: a tile triggers a CTA-wide max only when a score exceeds the
// running reference by more than 2^8, otherwise probabilities are taken against the reference.
//
// Work split: the context [lo, ctx) of every (sequence, kv head) is cut at absolute 128-position
// tile boundaries into items of TPI tiles, TPI the same for all sequences (from the longest
// context and nsplit), so items have equal cost.  A persistent grid of one CTA per SM takes items
// round-robin and streams them through one continuous pipeline; item (b, kvh, sp) writes split
// slot sp of each of its query heads (m in log2 units, l, acc[128]), and slots a sequence does
// not reach are written neutral (m = -inf) for the merge kernel.  Semantics follow the
// FaDecParams contract of fable_attn.h (kernels/fa_decode.hip:57-252 of the reference).
//
// Warp roles (192 threads): 0-3 softmax / accumulate, 4 TMA producer, 5 MMA issuer.  Every
// wait is bounded (a timeout records an error and unwinds), and the softmax warps break out
// of their loops only together (bar.red.and), so no named barrier is left waiting.
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
using fa_dec::rotate_row;

constexpr int TT = 128;            // positions per tile (M of S^T)
constexpr int HD = 128;            // head dim (M of O^T)
constexpr int NS = 3;              // K/V ring stages
constexpr int NTH = 192;
constexpr int TILE_B = TT * HD * 2;             // one K or V tile, 32 KB
constexpr int CHUNK_B = TT * 128;               // one 64-column chunk of a tile
constexpr float LAZY = 8.f;                     // log2 headroom of the lazy row max

// NRV query rows (a power of two >= gqa); the MMAs' N = NQ rows hold hi rows [0, NRV), lo rows
// [NRV, 2 NRV) and zeros above
template <int NRV>
struct Lay {
  static constexpr int NQ = 2 * NRV < 16 ? 16 : 2 * NRV;
  static constexpr uint32_t S_COL = 0, O_COL = 2 * NQ, TMEM_COLS = 4 * NQ <= 64 ? 64 : 128;
  static constexpr int K = 0;                         // [NS][2 chunks][128 rows][128 B]
  static constexpr int V = NS * TILE_B;
  static constexpr int Q = 2 * NS * TILE_B;           // [2][2 chunks][NQ rows][128 B]
  static constexpr int QB = NQ * HD * 2;
  static constexpr int P = Q + 2 * QB;                // [2][2 chunks][NQ rows][128 B]; also the
  static constexpr int PB = NQ * TT * 2;              //   fp32 q staging [NRV][HD] at item start
  static constexpr int RED = P + 2 * PB;              // cross-warp reductions [4][NRV] fp32
  static constexpr int BAR = RED + 4 * NRV * 4;
  // barriers: KF[NS] VF[NS] EMPTY[NS] SF[2] PF[2] OF[2] QF[2] QE[2] DRAIN
  static constexpr int KF = 0, VF = NS, EMPTY = 2 * NS, SF = 3 * NS, PF = SF + 2, OF = PF + 2, QFULL = OF + 2,
                       QE = QFULL + 2, DRAIN = QE + 2, NBAR = DRAIN + 1;
  static constexpr int SMEM = BAR + 8 * NBAR + 1024;  // + 1 KB to align the base for SW128
  static_assert(Q % 1024 == 0 && P % 1024 == 0 && QB % 1024 == 0 && PB % 1024 == 0,
                "swizzled operand tiles must be 1 KB aligned");
  static_assert(2 * PB >= NRV * HD * 4, "q staging must fit in the P^T buffers");
  static_assert(SMEM <= 232448 - 64, "shared memory per CTA");
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

// context of sequence b for its single new token: keys [lo, ctx)
__device__ __forceinline__ void seq_range(const FaDecParams& p, int b, int& lo, int& ctx) {
  const int ctx0 = p.ctx_len[b];
  ctx = ctx0 + (p.append ? 1 : 0);
  int l = p.leftpad ? p.leftpad[b] : 0;
  if (p.window >= 0 && ctx0 - p.window + 1 > l) l = ctx0 - p.window + 1;
  lo = l > 0 ? l : 0;
}

struct Item {
  int b, kvh, sp, lo, ctx, t0, t1;   // absolute tiles [t0, t1), positions [lo, ctx)
};
__device__ __forceinline__ bool item_of(const FaDecParams& p, int i, int NKV, int TPI, Item& it) {
  it.kvh = i % NKV;
  const int r = i / NKV;
  it.b = r % p.batch;
  it.sp = r / p.batch;
  seq_range(p, it.b, it.lo, it.ctx);
  if (it.ctx <= it.lo) return false;
  const int T0 = it.lo / TT, T1 = (it.ctx - 1) / TT + 1;
  it.t0 = T0 + it.sp * TPI;
  it.t1 = min(it.t0 + TPI, T1);
  return it.t0 < it.t1;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
  } else {
    const __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
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

// NRV: query rows handled (a power of two >= gqa, <= 16)
template <typename T, int NRV>
__global__ void __launch_bounds__(NTH, 1)
    dec_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, const FaDecParams p) {
  using L = Lay<NRV>;
  constexpr int NQ = L::NQ;
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smraw[];
  __shared__ uint32_t s_tmem;
  __shared__ int s_maxt;
  const uint32_t sb = (smem_u32(smraw) + 1023u) & ~1023u;
  uint8_t* sg = smraw + (sb - smem_u32(smraw));
  auto bar = [&](int i) { return sb + (uint32_t)L::BAR + 8u * (uint32_t)i; };

  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int NKV = p.NH / p.gqa, nh = p.gqa;
  const int shift = __ffs(p.page) - 1, pmask = p.page - 1;
  const int R = p.page < TT ? p.page : TT;   // rows of one page-slice box

  if (t == 0) s_maxt = 0;
  __syncthreads();
  for (int b = t; b < p.batch; b += NTH) {
    int lo, ctx;
    seq_range(p, b, lo, ctx);
    if (ctx > lo) atomicMax(&s_maxt, (ctx - 1) / TT + 1 - lo / TT);
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const int TPI = max(1, (s_maxt + p.nsplit - 1) / p.nsplit);
  const int nitems = p.nsplit * p.batch * NKV;

  if (warp == 4) {
    // ============================================================ TMA producer
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int i = blockIdx.x; ok && i < nitems; i += gridDim.x) {
        Item it;
        if (!item_of(p, i, NKV, TPI, it)) continue;
        for (int tile = it.t0; tile < it.t1; ++tile, ++g) {
          const int s = g % NS;
          if (g >= NS && !mbar_wait(bar(L::EMPTY + s), ((g / NS) - 1) & 1)) { ok = false; break; }
          const int base = tile * TT;
          uint32_t bytes = 0;
          for (int k = 0; k < TT / R; ++k) {
            const int pos0 = base + k * R;
            if (pos0 + R <= it.lo || pos0 >= it.ctx) continue;
            bool okp;
            page_of(p, it.b, pos0, shift, okp);
            if (okp) bytes += (uint32_t)(R * HD * 2);
          }
          mbar_expect_tx(bar(L::KF + s), bytes);
          mbar_expect_tx(bar(L::VF + s), bytes);
          const uint32_t kd = sb + L::K + s * TILE_B, vd = sb + L::V + s * TILE_B;
          for (int k = 0; k < TT / R; ++k) {
            const int pos0 = base + k * R;
            if (pos0 + R <= it.lo || pos0 >= it.ctx) continue;
            bool okp;
            const long long blk = page_of(p, it.b, pos0, shift, okp);
            if (!okp) continue;
            const int row = (int)(blk * p.page + (pos0 & pmask));
#pragma unroll
            for (int c = 0; c < HD / 64; ++c) {
              tma_load_3d(kd + c * CHUNK_B + k * R * 128, &tmK, 64 * c, it.kvh, row, bar(L::KF + s));
              tma_load_3d(vd + c * CHUNK_B + k * R * 128, &tmV, 64 * c, it.kvh, row, bar(L::VF + s));
            }
          }
        }
      }
      if (!ok) {
        record_error(1);
        // copies still in flight must land before the CTA's shared memory is released
        for (int j = max(0, g - NS); j < g; ++j) {
          mbar_wait(bar(L::KF + j % NS), (j / NS) & 1, 1000000000ull);
          mbar_wait(bar(L::VF + j % NS), (j / NS) & 1, 1000000000ull);
        }
      }
    }
  } else if (warp == 5) {
    // ============================================================ MMA issuer (lane 0)
    constexpr uint32_t ID_S = idesc_f16(BF16 ? 1 : 0, TT, NQ, 0, 0);   // S^T = K Q^T
    constexpr uint32_t ID_O = idesc_f16(BF16 ? 1 : 0, HD, NQ, 1, 0);   // O^T = V^T P^T, V^T MN-major
    int g = 0, qi = 0;
    bool ok = true;
    auto issue_pv = [&](int gg) -> bool {
      const int s = gg % NS;
      if (!mbar_wait_warp(bar(L::PF + (gg & 1)), (gg >> 1) & 1)) return false;
      if (!mbar_wait_warp(bar(L::VF + s), (gg / NS) & 1)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t vt = sb + L::V + s * TILE_B, pt = sb + L::P + (gg & 1) * L::PB;
#pragma unroll
        for (int kk = 0; kk < TT / 16; ++kk)
          mma_ss(tmem + L::O_COL + (gg & 1) * NQ, desc_mnmajor(vt, TT, kk), desc_kmajor(pt, NQ, kk), ID_O, kk > 0);
        mma_commit(bar(L::OF + (gg & 1)));
        mma_commit(bar(L::EMPTY + s));
      }
      __syncwarp();
      return true;
    };
    for (int i = blockIdx.x; ok && i < nitems; i += gridDim.x) {
      Item it;
      if (!item_of(p, i, NKV, TPI, it)) continue;
      if (!mbar_wait_warp(bar(L::QFULL + (qi & 1)), (qi >> 1) & 1)) { ok = false; break; }
      for (int tile = it.t0; tile < it.t1; ++tile, ++g) {
        const int s = g % NS;
        if (!mbar_wait_warp(bar(L::KF + s), (g / NS) & 1)) { ok = false; break; }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t kt = sb + L::K + s * TILE_B, qt = sb + L::Q + (qi & 1) * L::QB;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk)
            mma_ss(tmem + L::S_COL + (g & 1) * NQ, desc_kmajor(kt, TT, kk), desc_kmajor(qt, NQ, kk), ID_S, kk > 0);
          mma_commit(bar(L::SF + (g & 1)));
          if (tile == it.t1 - 1) mma_commit(bar(L::QE + (qi & 1)));
        }
        __syncwarp();
        // P.V of the previous tile of this item overlaps the softmax of this one
        if (tile > it.t0 && !issue_pv(g - 1)) { ok = false; break; }
      }
      // the item's last P.V goes out before the next item's q is awaited (the softmax warps
      // write that q only after consuming this O)
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
    float* qf = reinterpret_cast<float*>(sg + L::P);   // q staging aliases the (idle) P^T buffers
    float acc[NRV], mref[NRV], lt[NRV], cprev[NRV], slope2[NRV];
    int g = 0, qi = 0;
    bool ok = true;
    auto ld_cols = [&](uint32_t addr, float* v) {   // NQ columns of this thread's lane
      tmem_ld16(addr, v);
      if constexpr (NQ == 32) tmem_ld16(addr + 16, v + 16);
    };
    for (int i = blockIdx.x; ok && i < nitems; i += gridDim.x) {
      Item it;
      const bool live = item_of(p, i, NKV, TPI, it);
      const int hbase = it.kvh * p.gqa;
      if (!live) {   // a split this sequence does not reach: neutral slot for the merge
        if (t < nh) {
          float* o = p.scratch + ((long long)(it.b * p.NH + hbase + t) * p.nsplit + it.sp) * (HD + 2);
          o[0] = -INFINITY;
          o[1] = 0.f;
        }
        continue;
      }
      // ---- q of this item: fp32 staging (+ rotary), then 16-bit hi / lo rows, swizzled K-major.
      // Every P.V of earlier items has completed (their O^T were consumed), so the P^T buffers
      // are free for the staging; they are re-zeroed afterwards.
      const bool qfree = (qi < 2) ? true : mbar_wait_warp(bar(L::QE + (qi & 1)), ((qi >> 1) - 1) & 1);
      if (!bar_and_128(qfree)) { ok = false; break; }
      const T* qg = (const T*)p.q + ((long long)it.b * p.NH + hbase) * HD;
      for (int e = t; e < NRV * HD; e += 128) qf[e] = (e / HD < nh) ? Elem<T>::to_f(qg[e]) : 0.f;
      bar_sync_128();
      if (p.rotary && t < nh && t < NRV) {
        const int rdim = p.rotary_dim > 0 ? p.rotary_dim : HD;
        const int rp = p.rotary_pos ? p.rotary_pos[it.b] : p.ctx_len[it.b];
        rotate_row(qf + t * HD, rdim, p.rotary, p.cos + (long long)rp * (rdim / 2), p.sin + (long long)rp * (rdim / 2));
      }
      bar_sync_128();
      {
        uint8_t* qs = sg + L::Q + (qi & 1) * L::QB;
        for (int v = t; v < NQ * HD / 8; v += 128) {
          const int r = v / (HD / 8), c0 = (v % (HD / 8)) * 8;
          uint4 w = make_uint4(0, 0, 0, 0);
          if (r < 2 * NRV) {
            const bool lo = r >= NRV;
            const float* src = qf + (lo ? r - NRV : r) * HD + c0;
            float x[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float hi = round16<T>(src[j]);
              x[j] = lo ? src[j] - hi : hi;
            }
            w = make_uint4(pack2<T>(x[0], x[1]), pack2<T>(x[2], x[3]), pack2<T>(x[4], x[5]), pack2<T>(x[6], x[7]));
          }
          *reinterpret_cast<uint4*>(qs + swz_off(NQ, r, c0)) = w;
        }
      }
      bar_sync_128();   // staging reads done before the P^T buffers are cleared
      for (int e = t; e < 2 * L::PB / 16; e += 128) *reinterpret_cast<uint4*>(sg + L::P + e * 16) = make_uint4(0, 0, 0, 0);
      fence_proxy_async_smem();
      mbar_arrive(bar(L::QFULL + (qi & 1)));
#pragma unroll
      for (int r = 0; r < NRV; ++r) {
        acc[r] = 0.f; mref[r] = -INFINITY; lt[r] = 0.f; cprev[r] = 1.f;
        slope2[r] = (p.alibi && r < nh) ? p.alibi[hbase + r] * FA_LOG2E : 0.f;
      }
      const int qpos = p.ctx_len[it.b];
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
      for (int tile = it.t0; tile < it.t1; ++tile, ++g) {
        const bool got = mbar_wait_warp(bar(L::SF + (g & 1)), (g >> 1) & 1);
        if (!bar_and_128(got)) { ok = false; break; }
        tc_fence_after();
        float s[NQ];
        ld_cols(la + L::S_COL + (g & 1) * NQ, s);
        tc_wait_ld();
        const int pos = tile * TT + t;
        bool valid = pos >= it.lo && pos < it.ctx;
        if (valid) {
          bool okp;
          page_of(p, it.b, pos, shift, okp);
          valid = okp;
        }
        float v[NRV];
        bool need = false;
        const float dpos = (float)(pos - qpos);
#pragma unroll
        for (int r = 0; r < NRV; ++r) {
          const float sr = s[r] + s[NRV + r];   // q_hi . k + q_lo . k
          float x = cap_on ? cap2 * fa_tanh(sr * cap_in) : sr * scale2;
          x = fmaf(slope2[r], dpos, x);
          v[r] = (valid && r < nh) ? x : -INFINITY;
          need |= v[r] > mref[r] + LAZY;
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
          const int s = g % NS;
          if (!mbar_wait(bar(L::VF + s), (g / NS) & 1)) record_error(8);
          uint8_t* vr = sg + L::V + s * TILE_B + t * 128;
#pragma unroll
          for (int c = 0; c < HD / 64; ++c)
#pragma unroll
            for (int u = 0; u < 8; ++u) *reinterpret_cast<uint4*>(vr + c * CHUNK_B + u * 16) = make_uint4(0, 0, 0, 0);
        }
        // P^T / zeroed V rows visible to the tensor core; S^T (and the last O^T read) ordered
        // before the MMAs that will overwrite those TMEM columns
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(bar(L::PF + (g & 1)));
        if (tile > it.t0 && !consume(g - 1)) { ok = false; break; }
#pragma unroll
        for (int r = 0; r < NRV; ++r) cprev[r] = corr[r];
      }
      if (ok && !consume(g - 1)) ok = false;
      if (!ok) break;
      // ---- finalize: row sums over the 128 positions, then the split slot of each head
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
#pragma unroll
      for (int r = 0; r < NRV; ++r) {
        if (r < nh) {
          float* o = p.scratch + ((long long)(it.b * p.NH + hbase + r) * p.nsplit + it.sp) * (HD + 2);
          o[2 + t] = acc[r];
          if (t == 0) { o[0] = mref[r]; o[1] = lsum[r]; }
        }
      }
      ++qi;
    }
    if (!ok) record_error(16);
  }
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
int launch(const FaDecParams& p, const CUtensorMap& mk, const CUtensorMap& mv, cudaStream_t st) {
  static unsigned long long done = 0;
  if (int rc = fa::ensure_smem((const void*)dec_tc_kernel<T, NRV>, Lay<NRV>::SMEM, &done)) return rc;
  const long long items = (long long)p.nsplit * p.batch * (p.NH / p.gqa);
  const int grid = (int)std::min<long long>(items, (long long)fa::num_sms());
  dec_tc_kernel<T, NRV><<<grid, NTH, Lay<NRV>::SMEM, st>>>(mk, mv, p);
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
  if (p.HD != HD || p.nq != 1 || p.gqa > 16 || p.page < 8 || p.num_blocks <= 0) return FA_OK;
  if (getenv("FABLE_ATTN_DECODE_NO_TC")) return FA_OK;
  const long long rows = p.num_blocks * (long long)p.page;
  if (rows >= (1ll << 31) || (long long)p.nsplit * p.batch * (p.NH / p.gqa) >= (1ll << 31)) return FA_OK;
  const int NKV = p.NH / p.gqa;
  const bool bf16 = dtype == FA_DTYPE_BF16;
  const int R = p.page < TT ? p.page : TT;
  CUtensorMap mk, mv;
  if (!tc_map(&mk, p.Kc, bf16, NKV, rows, R) || !tc_map(&mv, p.Vc, bf16, NKV, rows, R)) return FA_OK;
  *taken = true;
#define FA_DEC_TC(TT_, N_) return launch<TT_, N_>(p, mk, mv, st);
  if (bf16) {
    if (p.gqa <= 4) FA_DEC_TC(__nv_bfloat16, 4)
    if (p.gqa <= 8) FA_DEC_TC(__nv_bfloat16, 8)
    FA_DEC_TC(__nv_bfloat16, 16)
  } else {
    if (p.gqa <= 4) FA_DEC_TC(__half, 4)
    if (p.gqa <= 8) FA_DEC_TC(__half, 8)
    FA_DEC_TC(__half, 16)
  }
#undef FA_DEC_TC
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
