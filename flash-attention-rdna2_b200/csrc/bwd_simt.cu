// bwd_simt.cu — exact attention backward on the CUDA cores, fp32 arithmetic, no atomics.
//
// Same decomposition as the reference (kernels/backward.hip:86-387), so the result is
// bit-reproducible run to run:
//   1. preprocess: dsum[row] = sum_d O*dO                       (one warp per 4 rows)
//   2. dK/dV     : one CTA per 32-key tile; loops over every query head of the kv group and
//                  every 32-row query tile that can see the keys; dK, dV live in registers
//   3. dQ        : one CTA per 32-row query tile; loops over the visible key tiles
// In each tile P = exp(logit - LSE) is recomputed, Z is the forward's Philox keep multiplier,
// dP = dO.V^T, dS = P*(Z*dP - dsum)*(1 - tanh^2) (softcap), dV += (Z*P)^T dO,
// dK += scale*dS^T Q, dQ += scale*dS K.  Masks: causal/window (no attn_chunk, as in the
// reference's fwd_ok, kernels/backward.hip:76-83).  Varlen via cu_seqlens like the forward.
#include "fa_common.cuh"
#include "fa_launch.h"

#include <type_traits>

namespace {

constexpr int BQ = 32, BK = 32;

__device__ __forceinline__ SeqGeom bwd_geom(const FaBwdParams& p, int z) {
  SeqGeom g = fa_seq_geom(z, p.SQ, p.SK, p.cu_q, p.cu_k, p.seqused_q, p.seqused_k, p.qs, p.ks, p.vs, p.os);
  return g;
}
// dO / dQ / dK / dV offsets of row 0 for sequence z (their strides may differ from q/k/v/o)
__device__ __forceinline__ long long row0(const FaBwdParams& p, int z, const FaStrides& s, bool is_q) {
  if (p.cu_q) return (long long)(is_q ? p.cu_q[z] : p.cu_k[z]) * s.s;
  return (long long)z * s.b;
}

// dsum rows per warp: their loads are all issued before the first multiply, so each lane has
// 2 * DSUM_ROWS loads in flight (a lone 128-dim row per warp left HBM at 40 % of its bandwidth)
constexpr int DSUM_ROWS = 4;

template <typename T>
__global__ void __launch_bounds__(256) bwd_pre_kernel(const FaBwdParams p) {
  const int z = blockIdx.z, h = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = (blockIdx.x * 8 + warp) * DSUM_ROWS;
  const SeqGeom g = bwd_geom(p, z);
  if (q0 >= g.SQ) return;
  const T* O = (const T*)p.O + g.o0 + (long long)h * p.os.h + (long long)q0 * p.os.s;
  const T* dO = (const T*)p.dO + row0(p, z, p.dos, true) + (long long)h * p.dos.h + (long long)q0 * p.dos.s;
  const int nr = min(DSUM_ROWS, g.SQ - q0);
  float acc[DSUM_ROWS];
#pragma unroll
  for (int r = 0; r < DSUM_ROWS; ++r) acc[r] = 0.f;
  // 4 elements per lane in one vector load (8 bytes of a 16-bit type, 16 of fp32) when every row
  // start allows it, so a row of up to 128 dims is one load per tensor and lane
  constexpr int VB = 4 * (int)sizeof(T);
  if ((p.D & 3) == 0 && ((uintptr_t)O % VB) == 0 && ((uintptr_t)dO % VB) == 0 && (p.os.s & 3) == 0 &&
      (p.dos.s & 3) == 0) {
    using V = typename std::conditional<sizeof(T) == 2, uint2, float4>::type;
    for (int d = 4 * lane; d < p.D; d += 128) {
      V va[DSUM_ROWS], vb[DSUM_ROWS];
#pragma unroll
      for (int r = 0; r < DSUM_ROWS; ++r)
        if (r < nr) {
          va[r] = *reinterpret_cast<const V*>(O + (long long)r * p.os.s + d);
          vb[r] = *reinterpret_cast<const V*>(dO + (long long)r * p.dos.s + d);
        }
#pragma unroll
      for (int r = 0; r < DSUM_ROWS; ++r) {
        if (r >= nr) continue;
        const T* ea = reinterpret_cast<const T*>(&va[r]);
        const T* eb = reinterpret_cast<const T*>(&vb[r]);
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[r] += Elem<T>::to_f(ea[i]) * Elem<T>::to_f(eb[i]);
      }
    }
  } else {
    for (int r = 0; r < nr; ++r)
#pragma unroll 4
      for (int d = lane; d < p.D; d += 32)
        acc[r] += Elem<T>::to_f(O[(long long)r * p.os.s + d]) * Elem<T>::to_f(dO[(long long)r * p.dos.s + d]);
  }
#pragma unroll
  for (int r = 0; r < DSUM_ROWS; ++r) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
    if (lane == 0 && r < nr)
      p.dsum[fa_lse_index(p.cu_q != nullptr, z, h, p.Hq, p.SQ, g.tok_q, p.lse_total_q, q0 + r)] = acc[r];
  }
}

// Shared tile computation: given Q/dO rows [BQ] and K/V rows [BK] in smem, write
// Pt[i][j] = Z*P and dS[i][j] (unscaled by softmax scale) into smem.
template <int HD>
__device__ __forceinline__ void fill_pds(const FaBwdParams& p, const float* Qs, const float* dOs,
                                         const float* Ks, const float* Vs, const float* lse,
                                         const float* dsum, float* Pt, float* dS, int h, int qbase,
                                         int kbase, int SQ, int SK, float slope, float inv_keep) {
  constexpr int LD = HD + 1;
  const int t = threadIdx.x, tx = t & 15, ty = t >> 4;
  float s[2][2], dp[2][2];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int b = 0; b < 2; ++b) { s[a][b] = 0.f; dp[a][b] = 0.f; }
#pragma unroll 4
  for (int d = 0; d < HD; ++d) {
    const float q0 = Qs[(ty * 2) * LD + d], q1 = Qs[(ty * 2 + 1) * LD + d];
    const float o0 = dOs[(ty * 2) * LD + d], o1 = dOs[(ty * 2 + 1) * LD + d];
    const float k0 = Ks[tx * LD + d], k1 = Ks[(tx + 16) * LD + d];
    const float v0 = Vs[tx * LD + d], v1 = Vs[(tx + 16) * LD + d];
    s[0][0] = fmaf(q0, k0, s[0][0]); s[0][1] = fmaf(q0, k1, s[0][1]);
    s[1][0] = fmaf(q1, k0, s[1][0]); s[1][1] = fmaf(q1, k1, s[1][1]);
    dp[0][0] = fmaf(o0, v0, dp[0][0]); dp[0][1] = fmaf(o0, v1, dp[0][1]);
    dp[1][0] = fmaf(o1, v0, dp[1][0]); dp[1][1] = fmaf(o1, v1, dp[1][1]);
  }
#pragma unroll
  for (int a = 0; a < 2; ++a) {
    const int i = ty * 2 + a, q = qbase + i;
    int lo, hi;
    fa_key_range(q, SQ, SK, p.causal, p.win_left, p.win_right, 0, lo, hi);
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      const int j = tx + 16 * b, k = kbase + j;
      float pv = 0.f, dsv = 0.f;
      if (q < SQ && k >= lo && k <= hi) {
        const float g0 = p.scale * s[a][b];
        float logit, deriv = 1.f;
        if (p.softcap > 0.f) {
          const float tn = tanhf(g0 / p.softcap);
          logit = p.softcap * tn;
          deriv = 1.f - tn * tn;
        } else {
          logit = g0;
        }
        logit += slope * (float)(k - q);
        const float pr = exp2f((logit - lse[i]) * FA_LOG2E);
        float zm = 1.f;
        if (p.dropout) {
          zm = fa_keep_mul(p.dropout_bits, p.drop_seed, h, SQ, SK, q, k, p.dropout_p, inv_keep);
        }
        pv = zm * pr;
        dsv = pr * (zm * dp[a][b] - dsum[i]) * deriv;
      }
      Pt[i * (BK + 1) + j] = pv;
      dS[i * (BK + 1) + j] = dsv;
    }
  }
}

template <typename T, int HD>
__device__ __forceinline__ void load_rows(float* dst, const T* src, long long stride, int row0, int nrows,
                                          int limit) {
  constexpr int LD = HD + 1;
  for (int e = threadIdx.x; e < nrows * HD; e += 256) {
    const int r = e / HD, d = e % HD, rr = row0 + r;
    dst[r * LD + d] = (rr < limit) ? Elem<T>::to_f(src[(long long)rr * stride + d]) : 0.f;
  }
}

template <typename T, int HD>
__global__ void __launch_bounds__(256) bwd_dkdv_kernel(const FaBwdParams p) {
  constexpr int LD = HD + 1, DPT = HD / 16;
  extern __shared__ float smem[];
  float* Ks = smem;
  float* Vs = Ks + BK * LD;
  float* Qs = Vs + BK * LD;
  float* dOs = Qs + BQ * LD;
  float* Pt = dOs + BQ * LD;
  float* dS = Pt + BQ * (BK + 1);
  float* lse = dS + BQ * (BK + 1);
  float* dsum = lse + BQ;

  const int t = threadIdx.x, tx = t & 15, ty = t >> 4;
  const int z = blockIdx.z, kvh = blockIdx.y, kbase = blockIdx.x * BK;
  const bool varlen = p.cu_q != nullptr;
  const SeqGeom g = bwd_geom(p, z);
  const int SQ = g.SQ, SK = g.SK;
  if (kbase >= SK) return;
  const float inv_keep = p.dropout ? p.keep_scale : 1.f;

  const T* Kg = (const T*)p.K + g.k0 + (long long)kvh * p.ks.h;
  const T* Vg = (const T*)p.V + g.v0 + (long long)kvh * p.vs.h;
  load_rows<T, HD>(Ks, Kg, p.ks.s, kbase, BK, SK);
  load_rows<T, HD>(Vs, Vg, p.vs.s, kbase, BK, SK);

  float accK[2][DPT], accV[2][DPT];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int e = 0; e < DPT; ++e) { accK[r][e] = 0.f; accV[r][e] = 0.f; }

  // query rows that can see any key of [kbase, kbase+BK-1]
  const int delta = SK - SQ, kend = min(kbase + BK, SK) - 1;
  int qstart = 0, qend = SQ - 1;
  if (p.causal) qstart = max(qstart, kbase - delta);
  if (p.win_right >= 0) qstart = max(qstart, kbase - delta - p.win_right);
  if (p.win_left >= 0) qend = min(qend, kend - delta + p.win_left);

  const long long dq0 = row0(p, z, p.dos, true);
  for (int hg = 0; hg < p.gqa; ++hg) {
    const int h = kvh * p.gqa + hg;
    const float slope = p.alibi ? p.alibi[h] : 0.f;
    const T* Qg = (const T*)p.Q + g.q0 + (long long)h * p.qs.h;
    const T* dOg = (const T*)p.dO + dq0 + (long long)h * p.dos.h;
    for (int qb = (qstart / BQ) * BQ; qb <= qend; qb += BQ) {
      __syncthreads();
      load_rows<T, HD>(Qs, Qg, p.qs.s, qb, BQ, SQ);
      load_rows<T, HD>(dOs, dOg, p.dos.s, qb, BQ, SQ);
      for (int i = t; i < BQ; i += 256) {
        const int q = qb + i;
        if (q < SQ) {
          const long long li = fa_lse_index(varlen, z, h, p.Hq, p.SQ, g.tok_q, p.lse_total_q, q);
          lse[i] = p.lse[li];
          dsum[i] = p.dsum[li];
        } else {
          lse[i] = 0.f; dsum[i] = 0.f;
        }
      }
      __syncthreads();
      fill_pds<HD>(p, Qs, dOs, Ks, Vs, lse, dsum, Pt, dS, h, qb, kbase, SQ, SK, slope, inv_keep);
      __syncthreads();
#pragma unroll 4
      for (int i = 0; i < BQ; ++i) {
        const float p0 = Pt[i * (BK + 1) + ty * 2], p1 = Pt[i * (BK + 1) + ty * 2 + 1];
        const float s0 = dS[i * (BK + 1) + ty * 2], s1 = dS[i * (BK + 1) + ty * 2 + 1];
#pragma unroll
        for (int e = 0; e < DPT; ++e) {
          const float o = dOs[i * LD + tx + 16 * e], qv = Qs[i * LD + tx + 16 * e];
          accV[0][e] = fmaf(p0, o, accV[0][e]); accV[1][e] = fmaf(p1, o, accV[1][e]);
          accK[0][e] = fmaf(s0, qv, accK[0][e]); accK[1][e] = fmaf(s1, qv, accK[1][e]);
        }
      }
    }
  }
  T* dKg = (T*)p.dK + row0(p, z, p.dks, false) + (long long)kvh * p.dks.h;
  T* dVg = (T*)p.dV + row0(p, z, p.dvs, false) + (long long)kvh * p.dvs.h;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int k = kbase + ty * 2 + r;
    if (k >= SK) continue;
#pragma unroll
    for (int e = 0; e < DPT; ++e) {
      const int d = tx + 16 * e;
      dKg[(long long)k * p.dks.s + d] = Elem<T>::from_f(accK[r][e] * p.scale);
      dVg[(long long)k * p.dvs.s + d] = Elem<T>::from_f(accV[r][e]);
    }
  }
}

template <typename T, int HD>
__global__ void __launch_bounds__(256) bwd_dq_kernel(const FaBwdParams p) {
  constexpr int LD = HD + 1, DPT = HD / 16;
  extern __shared__ float smem[];
  float* Ks = smem;
  float* Vs = Ks + BK * LD;
  float* Qs = Vs + BK * LD;
  float* dOs = Qs + BQ * LD;
  float* Pt = dOs + BQ * LD;
  float* dS = Pt + BQ * (BK + 1);
  float* lse = dS + BQ * (BK + 1);
  float* dsum = lse + BQ;

  const int t = threadIdx.x, tx = t & 15, ty = t >> 4;
  const int z = blockIdx.z, h = blockIdx.y, kvh = h / p.gqa, qbase = blockIdx.x * BQ;
  const bool varlen = p.cu_q != nullptr;
  const SeqGeom g = bwd_geom(p, z);
  const int SQ = g.SQ, SK = g.SK;
  if (qbase >= SQ) return;
  const float inv_keep = p.dropout ? p.keep_scale : 1.f;
  const float slope = p.alibi ? p.alibi[h] : 0.f;

  const T* Qg = (const T*)p.Q + g.q0 + (long long)h * p.qs.h;
  const T* dOg = (const T*)p.dO + row0(p, z, p.dos, true) + (long long)h * p.dos.h;
  load_rows<T, HD>(Qs, Qg, p.qs.s, qbase, BQ, SQ);
  load_rows<T, HD>(dOs, dOg, p.dos.s, qbase, BQ, SQ);
  for (int i = t; i < BQ; i += 256) {
    const int q = qbase + i;
    if (q < SQ) {
      const long long li = fa_lse_index(varlen, z, h, p.Hq, p.SQ, g.tok_q, p.lse_total_q, q);
      lse[i] = p.lse[li];
      dsum[i] = p.dsum[li];
    } else {
      lse[i] = 0.f; dsum[i] = 0.f;
    }
  }
  int klo, khi, dummy;
  fa_key_range(qbase, SQ, SK, p.causal, p.win_left, p.win_right, 0, klo, dummy);
  fa_key_range(min(qbase + BQ, SQ) - 1, SQ, SK, p.causal, p.win_left, p.win_right, 0, dummy, khi);
  if (klo < 0) klo = 0;

  float accQ[2][DPT];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int e = 0; e < DPT; ++e) accQ[a][e] = 0.f;

  const T* Kg = (const T*)p.K + g.k0 + (long long)kvh * p.ks.h;
  const T* Vg = (const T*)p.V + g.v0 + (long long)kvh * p.vs.h;
  for (int kb = (klo / BK) * BK; kb <= khi; kb += BK) {
    __syncthreads();
    load_rows<T, HD>(Ks, Kg, p.ks.s, kb, BK, SK);
    load_rows<T, HD>(Vs, Vg, p.vs.s, kb, BK, SK);
    __syncthreads();
    fill_pds<HD>(p, Qs, dOs, Ks, Vs, lse, dsum, Pt, dS, h, qbase, kb, SQ, SK, slope, inv_keep);
    __syncthreads();
#pragma unroll 4
    for (int j = 0; j < BK; ++j) {
      const float s0 = dS[(ty * 2) * (BK + 1) + j], s1 = dS[(ty * 2 + 1) * (BK + 1) + j];
#pragma unroll
      for (int e = 0; e < DPT; ++e) {
        const float kv = Ks[j * LD + tx + 16 * e];
        accQ[0][e] = fmaf(s0, kv, accQ[0][e]);
        accQ[1][e] = fmaf(s1, kv, accQ[1][e]);
      }
    }
  }
  T* dQg = (T*)p.dQ + row0(p, z, p.dqs, true) + (long long)h * p.dqs.h;
#pragma unroll
  for (int a = 0; a < 2; ++a) {
    const int q = qbase + ty * 2 + a;
    if (q >= SQ) continue;
#pragma unroll
    for (int e = 0; e < DPT; ++e) dQg[(long long)q * p.dqs.s + tx + 16 * e] = Elem<T>::from_f(accQ[a][e] * p.scale);
  }
}

template <typename T, int HD>
int launch_hd(const FaBwdParams& p, cudaStream_t st) {
  const int LD = HD + 1;
  const size_t smem = sizeof(float) * (size_t)(2 * BK * LD + 2 * BQ * LD + 2 * BQ * (BK + 1) + 2 * BQ);
  static unsigned long long done_kv = 0, done_q = 0;
  if (int rc = fa::ensure_smem((const void*)bwd_dkdv_kernel<T, HD>, (int)smem, &done_kv)) return rc;
  if (int rc = fa::ensure_smem((const void*)bwd_dq_kernel<T, HD>, (int)smem, &done_q)) return rc;
  bwd_pre_kernel<T><<<dim3((p.SQ + 8 * DSUM_ROWS - 1) / (8 * DSUM_ROWS), p.Hq, p.B), 256, 0, st>>>(p);
  bwd_dkdv_kernel<T, HD><<<dim3((p.SK + BK - 1) / BK, p.Hk, p.B), 256, smem, st>>>(p);
  bwd_dq_kernel<T, HD><<<dim3((p.SQ + BQ - 1) / BQ, p.Hq, p.B), 256, smem, st>>>(p);
  fa::count_launch(3);
  return fa::cuda_status(cudaGetLastError(), "bwd_simt launch");
}

template <typename T>
int launch_t(const FaBwdParams& p, cudaStream_t st) {
  switch (p.D) {
    case 16: return launch_hd<T, 16>(p, st);
    case 32: return launch_hd<T, 32>(p, st);
    case 48: return launch_hd<T, 48>(p, st);
    case 64: return launch_hd<T, 64>(p, st);
    case 80: return launch_hd<T, 80>(p, st);
    case 96: return launch_hd<T, 96>(p, st);
    case 112: return launch_hd<T, 112>(p, st);
    case 128: return launch_hd<T, 128>(p, st);
    case 160: return launch_hd<T, 160>(p, st);
    case 192: return launch_hd<T, 192>(p, st);
    case 224: return launch_hd<T, 224>(p, st);
    case 256: return launch_hd<T, 256>(p, st);
  }
  fa::set_error("backward: head_dim=%d not instantiated", p.D);
  return FA_ERR_UNSUPPORTED;
}

}  // namespace

namespace fa {
int bwd_dsum(const FaBwdParams& p, int dtype, cudaStream_t st) {
  const dim3 grid((p.SQ + 8 * DSUM_ROWS - 1) / (8 * DSUM_ROWS), p.Hq, p.B);
  if (dtype == FA_DTYPE_F16) bwd_pre_kernel<__half><<<grid, 256, 0, st>>>(p);
  else if (dtype == FA_DTYPE_BF16) bwd_pre_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(p);
  else bwd_pre_kernel<float><<<grid, 256, 0, st>>>(p);
  count_launch();
  return cuda_status(cudaGetLastError(), "bwd dsum launch");
}
int bwd_simt(const FaBwdParams& p, int dtype, cudaStream_t st) {
  if (dtype == FA_DTYPE_F16) return launch_t<__half>(p, st);
  if (dtype == FA_DTYPE_BF16) return launch_t<__nv_bfloat16>(p, st);
  return launch_t<float>(p, st);
}
}  // namespace fa
