// decode.cu — paged-KV decode: append, split-K partial attention, split merge; plus the
// standalone LSE-merge kernel behind flash_attn_combine.
//
// Cache layout is flash-attn's: Kc/Vc [num_blocks, page, NKV, HD], block_table [batch,
// max_blocks].  Position pos of sequence b lives in page block_table[b][pos / page], slot
// pos % page.  The decode is HBM-bound: one CTA streams the K/V rows of one (sequence, kv head,
// split) exactly once for all the query heads of its group (up to 8 per CTA; larger groups
// use several CTAs), so K/V bytes are read once per group.
//
// Work layout inside a CTA: a "row group" of HD/8 lanes owns one cache position at a time,
// each lane 8 contiguous dims (one 16-byte load for 2-byte types).  Every row group keeps its
// own online-softmax state (m, l, acc[g][8]) over the positions it visits, so the streaming
// loop has no block-wide synchronisation; the row groups are merged once at the end.  Scores
// are kept in the log2 domain; the scratch holds (m, l, acc[HD]) per (token, head, split)
// with m in log2 units.
#include <cudaTypedefs.h>
#include "fa_common.cuh"
#include "fa_launch.h"
#include "sm100_ptx.cuh"
#include "decode_common.cuh"

namespace {

using fa_dec::page_of;
using fa_dec::rotate_row;

constexpr int DEC_THREADS = 256;

template <typename T> struct Vec8;   // 8 elements of T, loaded as one (or two) 16-byte words
template <> struct Vec8<__half> {
  static __device__ __forceinline__ void load(const __half* p, float* f) {
    const uint4 r = __ldg(reinterpret_cast<const uint4*>(p));
    const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) { const float2 v = __half22float2(h[i]); f[2 * i] = v.x; f[2 * i + 1] = v.y; }
  }
};
template <> struct Vec8<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float* f) {
    const uint4 r = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) { f[2 * i] = __uint_as_float(w[i] << 16); f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u); }
  }
};
template <> struct Vec8<float> {
  static __device__ __forceinline__ void load(const float* p, float* f) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
};

// ---------------------------------------------------------------- append (new k/v -> cache)
template <typename T>
__global__ void dec_append_kernel(const FaDecParams p, const void* new_k, const void* new_v) {
  extern __shared__ float ks[];
  const int bx = blockIdx.x, kvh = blockIdx.y, t = threadIdx.x;
  const int b = bx / p.nq, tk = bx % p.nq, NKV = p.NH / p.gqa, HD = p.HD;
  const int pos = p.ctx_len[b] + tk;
  const int shift = __ffs(p.page) - 1;
  bool ok;
  const long long blk = page_of(p, b, pos, shift, ok);
  if (!ok) return;
  const long long src = ((long long)(b * p.nq + tk) * NKV + kvh) * HD;
  const long long dst = ((blk * p.page + (pos & (p.page - 1))) * NKV + kvh) * HD;
  const T* nk = (const T*)new_k + src;
  const T* nv = (const T*)new_v + src;
  for (int d = t; d < HD; d += blockDim.x) ks[d] = Elem<T>::to_f(nk[d]);
  __syncthreads();
  if (p.rotary && t == 0) {
    const int rdim = p.rotary_dim > 0 ? p.rotary_dim : HD;
    const int rp = (p.rotary_pos ? p.rotary_pos[b] : p.ctx_len[b]) + tk;
    rotate_row(ks, rdim, p.rotary, p.cos + (long long)rp * (rdim / 2), p.sin + (long long)rp * (rdim / 2));
  }
  __syncthreads();
  T* kc = (T*)p.Kc + dst;
  T* vc = (T*)p.Vc + dst;
  for (int d = t; d < HD; d += blockDim.x) {
    kc[d] = Elem<T>::from_f(ks[d]);
    vc[d] = nv[d];
  }
}

// ---------------------------------------------------------------- split-K partial attention
// grid (batch*nq, NKV*groups, nsplit); G = query heads handled per CTA
template <typename T, int HD, int G>
__global__ void __launch_bounds__(DEC_THREADS) dec_partial_kernel(const FaDecParams p, int groups) {
  // lanes per row group: HD/8 rounded up to a power of two (lanes past HD/8 stay idle)
  constexpr int LPR = (HD / 8 <= 2) ? 2 : (HD / 8 <= 4) ? 4 : (HD / 8 <= 8) ? 8 : (HD / 8 <= 16) ? 16 : 32;
  constexpr int RPW = 32 / LPR;               // row groups per warp
  constexpr int NRG = (DEC_THREADS / 32) * RPW;
  constexpr int U = 4;                        // positions in flight per row group
  __shared__ float qs[G][HD];
  __shared__ float ms[NRG][G], ls[NRG][G];
  __shared__ float red[NRG][8 * LPR];         // one head's accumulators of every row group

  const int bx = blockIdx.x, kvh = blockIdx.y / groups, grp = blockIdx.y % groups, sp = blockIdx.z;
  const int b = bx / p.nq, tk = bx % p.nq;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int rg = warp * RPW + lane / LPR, li = lane % LPR, d0 = li * 8;
  const bool dlive = d0 < HD;                 // this lane owns real dims
  const int NKV = p.NH / p.gqa;
  const int hbase = kvh * p.gqa + grp * G;
  const int nh = min(G, p.gqa - grp * G);     // heads of this CTA that exist

  const int ctx0 = p.ctx_len[b];
  const int qpos = ctx0 + tk;
  const int ctx = ctx0 + (p.append ? tk + 1 : 0);
  int lo = p.leftpad ? p.leftpad[b] : 0;
  if (p.window >= 0) lo = max(lo, qpos - p.window + 1);
  lo = max(lo, 0);
  const int n = max(ctx - lo, 0);
  const int chunk = (n + p.nsplit - 1) / p.nsplit;
  const int start = lo + sp * chunk, end = min(start + chunk, ctx);

  // q (+ rotary) into shared memory, fp32
  const T* qg = (const T*)p.q + ((long long)(b * p.nq + tk) * p.NH + hbase) * HD;
  for (int e = t; e < G * HD; e += DEC_THREADS) {
    const int g = e / HD, d = e % HD;
    qs[g][d] = (g < nh) ? Elem<T>::to_f(qg[(long long)g * HD + d]) : 0.f;
  }
  __syncthreads();
  if (p.rotary && t < G && t < nh) {
    const int rdim = p.rotary_dim > 0 ? p.rotary_dim : HD;
    const int rp = (p.rotary_pos ? p.rotary_pos[b] : ctx0) + tk;
    rotate_row(qs[t], rdim, p.rotary, p.cos + (long long)rp * (rdim / 2), p.sin + (long long)rp * (rdim / 2));
  }
  __syncthreads();

  const float scale2 = p.scale * FA_LOG2E;
  float qr[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < 8; ++i) qr[g][i] = dlive ? qs[g][d0 + i] : 0.f;
  float slope[G];
#pragma unroll
  for (int g = 0; g < G; ++g) slope[g] = (p.alibi && g < nh) ? p.alibi[hbase + g] : 0.f;

  float m[G], l[G], acc[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY; l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[g][i] = 0.f;
  }

  const int shift = __ffs(p.page) - 1, pmask = p.page - 1;
  const T* Kc = (const T*)p.Kc;
  const T* Vc = (const T*)p.Vc;
  // the trip count is the same for every lane of the CTA (the shuffles below are full-warp);
  // positions past the split end are simply invisible
  for (int base0 = start; base0 < end; base0 += NRG * U) {
    const int base = base0 + rg;
    float kf[U][8], vf[U][8];
    bool vis[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int pos = base + u * NRG;
      vis[u] = pos < end;
      if (vis[u]) {
        bool ok;
        const long long blk = page_of(p, b, pos, shift, ok);
        vis[u] = ok;
        const long long off = ((blk * p.page + (pos & pmask)) * NKV + kvh) * HD + d0;
        if (ok && dlive) {
          Vec8<T>::load(Kc + off, kf[u]);
          Vec8<T>::load(Vc + off, vf[u]);
        }
      }
      if (!vis[u] || !dlive) {
#pragma unroll
        for (int i = 0; i < 8; ++i) { kf[u][i] = 0.f; vf[u][i] = 0.f; }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int pos = base + u * NRG;
      float s[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) a = fmaf(qr[g][i], kf[u][i], a);
#pragma unroll
        for (int o = LPR / 2; o >= 1; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        s[g] = a;
      }
      if (!vis[u]) continue;   // uniform across the row group
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float v;
        if (p.softcap > 0.f) v = p.softcap * tanhf(s[g] * p.scale / p.softcap) * FA_LOG2E;
        else v = s[g] * scale2;
        v += slope[g] * (float)(pos - qpos) * FA_LOG2E;
        const float mn = fmaxf(m[g], v);
        const float corr = exp2f(m[g] - mn);
        const float pw = exp2f(v - mn);
        l[g] = l[g] * corr + pw;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[g][i] = fmaf(pw, vf[u][i], acc[g][i] * corr);
        m[g] = mn;
      }
    }
  }

  // merge the row groups: max, rescaled sums, then accumulators one head at a time
  if (li == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) { ms[rg][g] = m[g]; ls[rg][g] = l[g]; }
  }
  __syncthreads();
  float M[G], L[G], w[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float mx = -INFINITY;
    for (int r = 0; r < NRG; ++r) mx = fmaxf(mx, ms[r][g]);
    M[g] = mx;
    float sum = 0.f;
    if (mx != -INFINITY)
      for (int r = 0; r < NRG; ++r) sum += ls[r][g] * exp2f(ms[r][g] - mx);
    L[g] = sum;
    w[g] = (mx != -INFINITY) ? exp2f(m[g] - mx) : 0.f;
  }
  float* out_base = p.scratch + ((long long)(b * p.nq + tk) * p.NH) * (long long)p.nsplit * (HD + 2);
#pragma unroll
  for (int g = 0; g < G; ++g) {
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 8; ++i) red[rg][d0 + i] = acc[g][i] * w[g];
    __syncthreads();
    if (g < nh) {
      float* out = out_base + ((long long)(hbase + g) * p.nsplit + sp) * (HD + 2);
      if (t == 0) { out[0] = M[g]; out[1] = L[g]; }
      for (int d = t; d < HD; d += DEC_THREADS) {
        float a = 0.f;
        for (int r = 0; r < NRG; ++r) a += red[r][d];
        out[2 + d] = a;
      }
    }
  }
}

// ---------------------------------------------------------------- split merge -> O, LSE
constexpr int FA_DEC_MAX_SPLITS = 512;   // fa_decode_launch refuses nsplit above it
template <typename T>
__global__ void dec_merge_kernel(const FaDecParams p) {
  pdl_wait();      // the partials of the kernel before (a programmatic launch starts early)
  pdl_trigger();   // and the kernel after may start its own prologue
  const int row = blockIdx.x, h = blockIdx.y, HD = p.HD;
  {   // an empty context has no partials to read: O = 0, LSE = -inf
    const int b = row / p.nq, tk = row % p.nq, ctx0 = p.ctx_len[b];
    const int ctx = ctx0 + (p.append ? tk + 1 : 0);
    int lo = p.leftpad ? p.leftpad[b] : 0;
    if (p.window >= 0) lo = max(lo, ctx0 + tk - p.window + 1);
    if (ctx <= max(lo, 0)) {
      for (int d = threadIdx.x; d < HD; d += blockDim.x) {
        if (p.o_f32) ((float*)p.o)[((long long)row * p.NH + h) * HD + d] = 0.f;
        else ((T*)p.o)[((long long)row * p.NH + h) * HD + d] = Elem<T>::from_f(0.f);
      }
      if (p.lse_out && threadIdx.x == 0) p.lse_out[(long long)row * p.NH + h] = -INFINITY;
      return;
    }
  }
  // split weights: the first warp loads every split's (m, l) at once (lane s, s + 32, ...), reduces
  // the max and the weighted sum by shuffles, and leaves w_s = 2^(m_s - M) in shared memory
  __shared__ float wsh[FA_DEC_MAX_SPLITS];
  __shared__ float lsh[2];
  const float* base = p.scratch + ((long long)row * p.NH + h) * (long long)p.nsplit * (HD + 2);
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float M = -INFINITY;
    for (int s = lane; s < p.nsplit; s += 32) M = fmaxf(M, base[(long long)s * (HD + 2)]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.f;
    for (int s = lane; s < p.nsplit; s += 32) {
      const float ms = base[(long long)s * (HD + 2)];
      const float w = (M != -INFINITY && ms != -INFINITY) ? exp2f(ms - M) : 0.f;
      wsh[s] = w;
      if (w > 0.f) L += base[(long long)s * (HD + 2) + 1] * w;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    if (lane == 0) {
      lsh[0] = M;
      lsh[1] = L;
    }
  }
  __syncthreads();
  const float M = lsh[0], L = lsh[1];
  const float invL = L > 0.f ? 1.f / L : 0.f;
  const long long obase = ((long long)row * p.NH + h) * HD;
  for (int d = threadIdx.x; d < HD; d += blockDim.x) {
    float a = 0.f;
    for (int s = 0; s < p.nsplit; ++s) {
      const float w = wsh[s];
      if (w > 0.f) a = fmaf(base[(long long)s * (HD + 2) + 2 + d], w, a);
    }
    if (p.o_f32) ((float*)p.o)[obase + d] = a * invL;
    else ((T*)p.o)[obase + d] = Elem<T>::from_f(a * invL);
  }
  if (p.lse_out && threadIdx.x == 0)
    p.lse_out[(long long)row * p.NH + h] = L > 0.f ? M * FA_LN2 + logf(L) : -INFINITY;
}


// ---------------------------------------------------------------- split-K partial, TMA-fed
// fp16/bf16 caches.  The page slices of K and V of one kv head (rows of HD elements, NKV*HD
// apart) are streamed by the TMA engine into an NS-stage shared-memory ring, 64 positions per
// tile, while the 8 warps work on the previous tile in three phases:
//   A  scores s[g][pos] = q_g . k_pos (row groups of HD/8 lanes, 16-byte smem reads, shuffle sums)
//   B  per-head online softmax of the tile (warp g owns head g: tile max, rescale factor,
//      2^(s - m) once per score)
//   C  O_g += p[g][pos] * V[pos] (thread = head x 8-dim chunk x position group)
// Positions outside the split are never read, so stale or unloaded rows cannot leak in.
constexpr int DEC_TILE = 64;

template <int HD>
struct DecTmaCfg {
  static constexpr int NS = (HD <= 128) ? 4 : 3;
  static constexpr int ROW = HD * 2;                     // bytes per cached row (2-byte types)
  static constexpr int TILE = DEC_TILE * ROW;            // one K (or V) tile
  static constexpr int STAGE = 2 * TILE;
  static constexpr int OFF_S = NS * STAGE;               // scores     [8][64] f32
  static constexpr int OFF_P = OFF_S + 8 * 64 * 4;       // 2^(s - m)  [8][64] f32
  static constexpr int OFF_Q = OFF_P + 8 * 64 * 4;       // q          [8][HD] f32
  static constexpr int OFF_C = OFF_Q + 8 * HD * 4;       // rescale    [8] f32
  static constexpr int OFF_BAR = OFF_C + 64;
  static constexpr int SMEM = OFF_BAR + 8 * NS + 256;    // + alignment slack
};

template <typename T>
__device__ __forceinline__ void cvt8(const uint4& r, float* f) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) { f[2 * i] = __uint_as_float(w[i] << 16); f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u); }
  } else {
    const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) { const float2 v = __half22float2(h[i]); f[2 * i] = v.x; f[2 * i + 1] = v.y; }
  }
}

__device__ int g_dec_error = 0;

template <typename T, int HD, int G>
__global__ void __launch_bounds__(DEC_THREADS, 1)
    dec_tma_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                   const FaDecParams p, int groups) {
  using C = DecTmaCfg<HD>;
  constexpr int LPR = (HD / 8 <= 2) ? 2 : (HD / 8 <= 4) ? 4 : (HD / 8 <= 8) ? 8 : (HD / 8 <= 16) ? 16 : 32;
  constexpr int RPW = 32 / LPR, NRG = (DEC_THREADS / 32) * RPW;
  constexpr int D8 = HD / 8, TPH = DEC_THREADS / G, NPG = TPH / D8;   // PV: threads per head, position groups
  extern __shared__ uint8_t dsm_raw[];
  const uint32_t sbase = (sm100::smem_u32(dsm_raw) + 127u) & ~127u;
  uint8_t* sg = dsm_raw + (sbase - sm100::smem_u32(dsm_raw));
  float* s_sc = reinterpret_cast<float*>(sg + C::OFF_S);
  float* s_p = reinterpret_cast<float*>(sg + C::OFF_P);
  float* s_q = reinterpret_cast<float*>(sg + C::OFF_Q);
  float* s_corr = reinterpret_cast<float*>(sg + C::OFF_C);
  const uint32_t bar0 = sbase + C::OFF_BAR;

  const int bx = blockIdx.x, kvh = blockIdx.y / groups, grp = blockIdx.y % groups, sp = blockIdx.z;
  const int b = bx / p.nq, tk = bx % p.nq;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int hbase = kvh * p.gqa + grp * G;
  const int nh = min(G, p.gqa - grp * G);

  const int ctx0 = p.ctx_len[b];
  const int qpos = ctx0 + tk;
  const int ctx = ctx0 + (p.append ? tk + 1 : 0);
  int lo = p.leftpad ? p.leftpad[b] : 0;
  if (p.window >= 0) lo = max(lo, qpos - p.window + 1);
  lo = max(lo, 0);
  const int n = max(ctx - lo, 0);
  const int chunk = (((n + p.nsplit - 1) / p.nsplit) + DEC_TILE - 1) / DEC_TILE * DEC_TILE;
  const int start = lo + sp * chunk, end = min(start + chunk, ctx);
  float* out_base = p.scratch + ((long long)(b * p.nq + tk) * p.NH) * (long long)p.nsplit * (HD + 2);
  if (start >= end) {   // empty split (CTA-uniform): neutral partial
    for (int e = t; e < nh * (HD + 2); e += DEC_THREADS) {
      const int g = e / (HD + 2), k = e % (HD + 2);
      out_base[((long long)(hbase + g) * p.nsplit + sp) * (HD + 2) + k] = (k == 0) ? -INFINITY : 0.f;
    }
    return;
  }
  const int start_al = start & ~(DEC_TILE - 1);
  const int ntile = (end - start_al + DEC_TILE - 1) / DEC_TILE;
  const int shift = __ffs(p.page) - 1, pmask = p.page - 1;
  const int R = p.page < DEC_TILE ? p.page : DEC_TILE;     // rows per TMA box (one page slice)

  if (t == 0) {
    for (int s = 0; s < C::NS; ++s) sm100::mbar_init(bar0 + 8 * s, 1);
    sm100::fence_barrier_init();
  }
  // q (+ rotary) -> fp32 smem
  const T* qg = (const T*)p.q + ((long long)(b * p.nq + tk) * p.NH + hbase) * HD;
  for (int e = t; e < G * HD; e += DEC_THREADS) {
    const int g = e / HD, d = e % HD;
    s_q[g * HD + d] = (g < nh) ? Elem<T>::to_f(qg[(long long)g * HD + d]) : 0.f;
  }
  __syncthreads();
  if (p.rotary && t < nh) {
    const int rdim = p.rotary_dim > 0 ? p.rotary_dim : HD;
    const int rp = (p.rotary_pos ? p.rotary_pos[b] : ctx0) + tk;
    rotate_row(s_q + t * HD, rdim, p.rotary, p.cos + (long long)rp * (rdim / 2), p.sin + (long long)rp * (rdim / 2));
  }

  // one tile = up to 64/R page slices of K and V; slices wholly outside [start, end) or with an
  // invalid page are not loaded (their rows are never read)
  auto issue = [&](int ti) {
    const int s = ti % C::NS;
    const int base = start_al + ti * DEC_TILE;
    const uint32_t kdst = sbase + s * C::STAGE, vdst = kdst + C::TILE;
    uint32_t bytes = 0;
    for (int i = 0; i < DEC_TILE / R; ++i) {
      const int pos0 = base + i * R;
      if (pos0 >= end || pos0 + R <= start) continue;
      bool ok;
      page_of(p, b, pos0, shift, ok);
      if (ok) bytes += 2u * R * C::ROW;
    }
    sm100::mbar_expect_tx(bar0 + 8 * s, bytes);
    for (int i = 0; i < DEC_TILE / R; ++i) {
      const int pos0 = base + i * R;
      if (pos0 >= end || pos0 + R <= start) continue;
      bool ok;
      const long long blk = page_of(p, b, pos0, shift, ok);
      if (!ok) continue;
      const int row = (int)(blk * p.page + (pos0 & pmask));
      sm100::tma_load_3d(kdst + i * R * C::ROW, &tmK, 0, kvh, row, bar0 + 8 * s);
      sm100::tma_load_3d(vdst + i * R * C::ROW, &tmV, 0, kvh, row, bar0 + 8 * s);
    }
  };
  __syncthreads();   // barriers initialised, q rotated
  int issued = 0;   // tiles whose loads thread 0 has issued
  if (t == 0)
    for (; issued < min(ntile, C::NS); ++issued) issue(issued);

  // ---- per-thread roles
  const int rg = warp * RPW + lane / LPR, li = lane % LPR, d0 = li * 8;
  const bool dlive = d0 < HD;
  float qr[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < 8; ++i) qr[g][i] = dlive ? s_q[g * HD + d0 + i] : 0.f;
  const float scale2 = p.scale * FA_LOG2E;
  const int gp = t / TPH, cchunk = (t % TPH) % D8, pg = (t % TPH) / D8;   // PV role
  const bool pv_live = (t % TPH) < NPG * D8;   // HD/8 need not divide the threads of a head
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;   // softmax stats, meaningful in warp g < G
  bool ok = true;

  for (int ti = 0; ti < ntile; ++ti) {
    const int s = ti % C::NS;
    const bool got = sm100::mbar_wait(bar0 + 8 * s, (ti / C::NS) & 1);
    if (!__syncthreads_and(got)) { ok = false; break; }
    // every thread is past phase C of tile ti-1: its stage can be refilled
    if (t == 0 && ti >= 1 && ti - 1 + C::NS < ntile) issue(issued++);
    const uint8_t* Kt = sg + s * C::STAGE;
    const uint8_t* Vt = Kt + C::TILE;
    const int base = start_al + ti * DEC_TILE;
    const int v0 = max(start - base, 0), v1 = min(end - base, DEC_TILE);
    // phase A: scores (trip count uniform: the shuffles are full-warp)
    for (int pp = 0; pp < DEC_TILE; pp += NRG) {
      const int pr = pp + rg;
      const bool vis = pr < DEC_TILE && pr >= v0 && pr < v1;
      float kf[8];
      if (vis && dlive) cvt8<T>(*reinterpret_cast<const uint4*>(Kt + pr * C::ROW + d0 * 2), kf);
      else {
#pragma unroll
        for (int i = 0; i < 8; ++i) kf[i] = 0.f;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) a = fmaf(qr[g][i], kf[i], a);
#pragma unroll
        for (int o = LPR / 2; o >= 1; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (li == 0 && pr < DEC_TILE) {
          float v = -INFINITY;
          if (vis && g < nh) {
            v = (p.softcap > 0.f) ? p.softcap * tanhf(a * p.scale / p.softcap) * FA_LOG2E : a * scale2;
            if (p.alibi) v += p.alibi[hbase + g] * (float)(base + pr - qpos) * FA_LOG2E;
          }
          s_sc[g * DEC_TILE + pr] = v;
        }
      }
    }
    __syncthreads();
    // phase B: per-head tile softmax (warp g = head g)
    if (warp < G) {
      const int g = warp;
      const float a = s_sc[g * DEC_TILE + lane], c = s_sc[g * DEC_TILE + lane + 32];
      float tm = fmaxf(a, c);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, o));
      const float mn = fmaxf(m_run, tm);
      const float muse = (mn == -INFINITY) ? 0.f : mn;
      const float corr = (mn == -INFINITY) ? 1.f : exp2f(m_run - mn);
      const float pa = exp2f(a - muse), pc = exp2f(c - muse);
      float sum = pa + pc;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      l_run = l_run * corr + sum;
      m_run = mn;
      s_p[g * DEC_TILE + lane] = pa;
      s_p[g * DEC_TILE + lane + 32] = pc;
      if (lane == 0) s_corr[g] = corr;
    }
    __syncthreads();
    // phase C: O += p V over the visible positions of this thread's group
    if (pv_live) {
      const float corr = s_corr[gp];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] *= corr;
      for (int pr = v0 + ((pg - v0 % NPG) + NPG) % NPG; pr < v1; pr += NPG) {
        const float w = s_p[gp * DEC_TILE + pr];
        float vf[8];
        cvt8<T>(*reinterpret_cast<const uint4*>(Vt + pr * C::ROW + cchunk * 16), vf);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = fmaf(w, vf[i], acc[i]);
      }
    }
  }
  if (!ok && t == 0) {
    atomicOr(&g_dec_error, 1);
    // no copy of this CTA may still be landing when its shared memory is reused or released
    for (int tj = 0; tj < issued; ++tj) sm100::mbar_wait(bar0 + 8 * (tj % C::NS), (tj / C::NS) & 1, 1000000000ull);
  }
  __syncthreads();
  // reduce the position groups (stage 0 is free: every issued tile was consumed or timed out)
  float* red = reinterpret_cast<float*>(sg);   // [G][NPG][HD]
  if (pv_live) {
#pragma unroll
    for (int i = 0; i < 8; ++i) red[(gp * NPG + pg) * HD + cchunk * 8 + i] = acc[i];
  }
  if (warp < G && lane == 0) {
    s_sc[warp] = ok ? m_run : -INFINITY;
    s_sc[8 + warp] = ok ? l_run : 0.f;
  }
  __syncthreads();
  for (int e = t; e < nh * HD; e += DEC_THREADS) {
    const int g = e / HD, d = e % HD;
    float a = 0.f;
    for (int r = 0; r < NPG; ++r) a += red[(g * NPG + r) * HD + d];
    float* out = out_base + ((long long)(hbase + g) * p.nsplit + sp) * (HD + 2);
    out[2 + d] = ok ? a : 0.f;
    if (d == 0) { out[0] = s_sc[g]; out[1] = s_sc[8 + g]; }
  }
}

PFN_cuTensorMapEncodeTiled_v12000 dec_encode_fn() {
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

// cache [num_blocks*page rows][NKV][HD] viewed as 3-D (HD, NKV, rows); box = one page slice
bool dec_map(CUtensorMap* m, const void* base, bool bf16, int HD, int NKV, long long rows, int box_rows) {
  auto enc = dec_encode_fn();
  if (!enc || ((uintptr_t)base) % 16) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)NKV, (cuuint64_t)rows};
  const cuuint64_t strides[2] = {(cuuint64_t)HD * 2, (cuuint64_t)NKV * HD * 2};
  const cuuint32_t box[3] = {(cuuint32_t)HD, 1, (cuuint32_t)box_rows};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base),
             dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T, int HD>
int launch_tma(const FaDecParams& p, cudaStream_t st, bool* taken) {
  *taken = false;
  const int NKV = p.NH / p.gqa;
  const long long rows = p.num_blocks * (long long)p.page;
  if (p.num_blocks <= 0 || rows >= (1ll << 31) || getenv("FABLE_ATTN_DECODE_NO_TMA")) return FA_OK;
  CUtensorMap mk, mv;
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  const int R = p.page < DEC_TILE ? p.page : DEC_TILE;
  if (!dec_map(&mk, p.Kc, bf16, HD, NKV, rows, R) || !dec_map(&mv, p.Vc, bf16, HD, NKV, rows, R)) return FA_OK;
  *taken = true;
  using Cf = DecTmaCfg<HD>;
  dim3 grid(p.batch * p.nq, 1, p.nsplit);
#define FA_DEC_TMA(GG)                                                                       \
  {                                                                                          \
    const int groups = (p.gqa + GG - 1) / GG;                                                \
    grid.y = NKV * groups;                                                                   \
    static unsigned long long done = 0;                                                      \
    if (int rc = fa::ensure_smem((const void*)dec_tma_kernel<T, HD, GG>, Cf::SMEM, &done)) return rc; \
    dec_tma_kernel<T, HD, GG><<<grid, DEC_THREADS, Cf::SMEM, st>>>(mk, mv, p, groups);       \
  }
  if (p.gqa <= 1) FA_DEC_TMA(1)
  else if (p.gqa <= 2) FA_DEC_TMA(2)
  else if (p.gqa <= 4) FA_DEC_TMA(4)
  else FA_DEC_TMA(8)
#undef FA_DEC_TMA
  fa::count_launch();
  return fa::cuda_status(cudaGetLastError(), "decode partial (TMA) launch");
}

template <typename T, int HD>
int launch_partial(const FaDecParams& p, cudaStream_t st) {
  if constexpr (!std::is_same<T, float>::value) {
    bool taken = false;
    const int rc = launch_tma<T, HD>(p, st, &taken);
    if (taken || rc) return rc;
  }
  const int NKV = p.NH / p.gqa;
  const int gq = p.gqa;
  dim3 grid(p.batch * p.nq, 1, p.nsplit);
#define FA_DEC_G(GG)                                                                  \
  {                                                                                   \
    const int groups = (gq + GG - 1) / GG;                                            \
    grid.y = NKV * groups;                                                            \
    dec_partial_kernel<T, HD, GG><<<grid, DEC_THREADS, 0, st>>>(p, groups);           \
  }
  if (gq <= 1) FA_DEC_G(1)
  else if (gq <= 2) FA_DEC_G(2)
  else if (gq <= 4) FA_DEC_G(4)
  else FA_DEC_G(8)
#undef FA_DEC_G
  fa::count_launch();
  return fa::cuda_status(cudaGetLastError(), "decode partial launch");
}

template <typename T>
int launch_t(const FaDecParams& p, cudaStream_t st, const void* nk, const void* nv) {
  if (nk) {
    const int NKV = p.NH / p.gqa;
    const int thr = p.HD < 32 ? 32 : p.HD;
    dec_append_kernel<T><<<dim3(p.batch * p.nq, NKV), thr, p.HD * sizeof(float), st>>>(p, nk, nv);
    fa::count_launch();
    if (int rc = fa::cuda_status(cudaGetLastError(), "decode append launch")) return rc;
  }
  int rc = FA_OK;
  bool tc = false;
  if constexpr (!std::is_same<T, float>::value) {
    rc = fa::dec_tc_partial(p, std::is_same<T, __half>::value ? FA_DTYPE_F16 : FA_DTYPE_BF16, st, &tc);
    if (rc) return rc;
  }
  if (!tc) switch (p.HD) {
    case 16: rc = launch_partial<T, 16>(p, st); break;
    case 32: rc = launch_partial<T, 32>(p, st); break;
    case 48: rc = launch_partial<T, 48>(p, st); break;
    case 64: rc = launch_partial<T, 64>(p, st); break;
    case 80: rc = launch_partial<T, 80>(p, st); break;
    case 96: rc = launch_partial<T, 96>(p, st); break;
    case 112: rc = launch_partial<T, 112>(p, st); break;
    case 128: rc = launch_partial<T, 128>(p, st); break;
    case 160: rc = launch_partial<T, 160>(p, st); break;
    case 192: rc = launch_partial<T, 192>(p, st); break;
    case 224: rc = launch_partial<T, 224>(p, st); break;
    case 256: rc = launch_partial<T, 256>(p, st); break;
    default:
      fa::set_error("decode: head_dim=%d not instantiated", p.HD);
      return FA_ERR_UNSUPPORTED;
  }
  if (rc) return rc;
  const int thr = p.HD < 32 ? 32 : p.HD;
  // programmatic launch: the merge's CTAs start while the partial kernel drains (they wait in
  // pdl_wait for its results)
  const cudaError_t le = fa::launch_pdl(dec_merge_kernel<T>, dim3(p.batch * p.nq, p.NH), dim3(thr), 0, st, p);
  fa::count_launch();
  return fa::cuda_status(le != cudaSuccess ? le : cudaGetLastError(), "decode merge launch");
}

// ---------------------------------------------------------------- flash_attn_combine
template <typename TI, typename TO>
__global__ void combine_kernel(const FaCombineParams p) {
  // one CTA per (b, s, h) row; threads over D
  const long long row = blockIdx.x;   // ((b*S)+s)*H + h
  const int h = (int)(row % p.H);
  const long long bs = row / p.H;
  const int s = (int)(bs % p.S);
  const int b = (int)(bs / p.S);
  const long long rows = (long long)p.B * p.S * p.H;
  const long long ostride = p.out_split_stride ? p.out_split_stride : rows * p.D;
  const long long lstride = p.lse_split_stride ? p.lse_split_stride : rows;
  const long long lrow = p.lse_bsh ? row : ((long long)b * p.H + h) * p.S + s;
  float M = -INFINITY;
  for (int k = 0; k < p.nsplit; ++k) M = fmaxf(M, p.lse_partial[k * lstride + lrow]);
  float W = 0.f;
  if (M != -INFINITY)
    for (int k = 0; k < p.nsplit; ++k) W += expf(p.lse_partial[k * lstride + lrow] - M);
  const float invW = W > 0.f ? 1.f / W : 0.f;
  for (int d = threadIdx.x; d < p.D; d += blockDim.x) {
    float a = 0.f;
    if (M != -INFINITY)
      for (int k = 0; k < p.nsplit; ++k) {
        const float w = expf(p.lse_partial[k * lstride + lrow] - M);
        a += w * Elem<TI>::to_f(((const TI*)p.out_partial)[k * ostride + row * p.D + d]);
      }
    ((TO*)p.out)[row * p.D + d] = Elem<TO>::from_f(a * invW);
  }
  if (p.lse_out && threadIdx.x == 0)
    p.lse_out[((long long)b * p.H + h) * p.S + s] = W > 0.f ? M + logf(W) : -INFINITY;
}

template <typename TI>
int combine_out(const FaCombineParams& p, cudaStream_t st) {
  const long long rows = (long long)p.B * p.S * p.H;
  const int thr = p.D < 32 ? 32 : (p.D > 256 ? 256 : p.D);
  if (p.out_dtype == FA_DTYPE_F16) combine_kernel<TI, __half><<<(unsigned)rows, thr, 0, st>>>(p);
  else if (p.out_dtype == FA_DTYPE_BF16) combine_kernel<TI, __nv_bfloat16><<<(unsigned)rows, thr, 0, st>>>(p);
  else combine_kernel<TI, float><<<(unsigned)rows, thr, 0, st>>>(p);
  fa::count_launch();
  return fa::cuda_status(cudaGetLastError(), "combine launch");
}

}  // namespace

namespace fa {
int dec_device_error(int clear) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_dec_error, sizeof(int));
  if (clear) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_dec_error, &zero, sizeof(int));
  }
  return v | (dec_tc_device_error(clear) ? 1 : 0);
}
int dec_run(const FaDecParams& p, int dtype, cudaStream_t st, const void* nk, const void* nv) {
  if (dtype == FA_DTYPE_F16) return launch_t<__half>(p, st, nk, nv);
  if (dtype == FA_DTYPE_BF16) return launch_t<__nv_bfloat16>(p, st, nk, nv);
  return launch_t<float>(p, st, nk, nv);
}
int combine_run(const FaCombineParams& p, cudaStream_t st) {
  if (p.in_dtype == FA_DTYPE_F16) return combine_out<__half>(p, st);
  if (p.in_dtype == FA_DTYPE_BF16) return combine_out<__nv_bfloat16>(p, st);
  return combine_out<float>(p, st);
}
}  // namespace fa

// ---------------------------------------------------------------- decode without allocation
// Split-K scratch for fa_decode_launch_noalloc: a fixed device array (16 MiB) owned by the
// library, so callers that cannot allocate device memory can still decode.  Device code could
// name it directly; host code only holds a stand-in symbol, so the launcher passes the real
// device address, looked up with the call's device current.
static __device__ __align__(256) float g_noalloc_scratch[FA_DECODE_NOALLOC_MAX_SCRATCH_FLOATS];

extern "C" FA_API int fa_decode_launch_noalloc(const FaDecParams* pp, int dtype, void* stream, const void* new_k,
                                               const void* new_v) {
  if (!pp) {
    fa::set_error("decode (no-alloc): null parameter block");
    return FA_ERR_INVALID;
  }
  if (pp->struct_size != sizeof(FaDecParams)) {
    fa::set_error("decode (no-alloc): struct_size %u != %zu", pp->struct_size, sizeof(FaDecParams));
    return FA_ERR_ABI;
  }
  FaDecParams p = *pp;
  const long long need = fa_decode_scratch_floats(p.batch, p.nq < 1 ? 1 : p.nq, p.NH, p.HD, p.nsplit);
  if (need > FA_DECODE_NOALLOC_MAX_SCRATCH_FLOATS || need < 0) {
    fa::set_error("decode (no-alloc): needs %lld scratch floats for batch=%d nq=%d NH=%d HD=%d nsplit=%d, above the "
                  "fixed maximum %lld; lower nsplit", need, p.batch, p.nq, p.NH, p.HD, p.nsplit,
                  (long long)FA_DECODE_NOALLOC_MAX_SCRATCH_FLOATS);
    return FA_ERR_SIZE;
  }
  // the array's address on the current device, looked up on every call: nothing cached can go
  // stale after a context reset, and concurrent first calls from several threads share no state
  void* ptr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (e != cudaSuccess) return fa::cuda_status(e, "decode (no-alloc): cudaGetSymbolAddress");
  p.scratch = (float*)ptr;
  return fa_decode_launch(&p, dtype, stream, new_k, new_v);
}
