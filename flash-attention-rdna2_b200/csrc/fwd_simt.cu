// fwd_simt.cu — exact attention forward on the CUDA cores, fp32 arithmetic.
//
// Serves the fp32 dtype (the reference's fp32 path, kernels/fa_forward.hip:317-400) and every
// fp16/bf16 configuration the tensor-core kernel (fwd_sm100.cu) does not take.  One CTA owns
// a 32-row query tile of one head of one sequence and streams 64-key tiles of K/V through
// shared memory with an online softmax (log2 domain); for head dims up to 64 the next tile's K/V
// are loaded into registers while the current one computes.  Every mask, softcap, alibi, Philox
// dropout, varlen/seqused and LSE output follows the FaFwdParams contract in fable_attn.h.
#include "fa_common.cuh"
#include "fa_launch.h"

namespace {

constexpr int BR = 32, BC = 64;
__device__ int g_simt_error = 0;   // bit 0: an invalid block-table entry of a real key

template <typename T, int HD>
__global__ void __launch_bounds__(256, 2) fwd_simt_kernel(const FaFwdParams p) {
  // rows of Q and K padded to HD + 4 floats (16-byte aligned float4 reads along the head dim);
  // P rows to BC + 4.  With DPT a multiple of 4 a thread owns the 4-dim groups 64 g + 4 tx .. + 3
  // (float4 reads of V and P; the 16 threads of a row read consecutive 16-byte units), else the
  // dims tx, tx + 16, ...
  constexpr int DPT = HD / 16, LDQ = HD + 4, LDP = BC + 4;
  constexpr bool VEC = DPT % 4 == 0;
  extern __shared__ float smem[];
  float* Qs = smem;                 // [BR][HD+4]
  float* Ks = Qs + BR * LDQ;        // [BC][HD+4]
  float* Vs = Ks + BC * LDQ;        // [BC][HD]
  float* Ps = Vs + BC * HD;         // [BR][BC+4]
  auto dim = [&](int e) { return VEC ? 64 * (e / 4) + 4 * (threadIdx.x & 15) + e % 4 : (threadIdx.x & 15) + 16 * e; };

  const int t = threadIdx.x, tx = t & 15, ty = t >> 4;
  const int z = blockIdx.z, h = blockIdx.y, kvh = h / p.gqa;
  const bool varlen = p.cu_q != nullptr;
  const SeqGeom g = fa_seq_geom(z, p.SQ, p.SK, p.cu_q, p.cu_k, p.seqused_q, p.seqused_k, p.sQ, p.sK,
                                p.sV, p.sO);
  const int qb = blockIdx.x * BR;
  if (qb >= g.SQ) return;
  const int SQ = g.SQ, SK = g.SK;

  const T* Qg = (const T*)p.Q + g.q0 + (long long)h * p.sQ.h;
  const T* Kg = (const T*)p.K + g.k0 + (long long)kvh * p.sK.h;
  const T* Vg = (const T*)p.V + g.v0 + (long long)kvh * p.sV.h;

  for (int e = t; e < BR * HD; e += 256) {
    const int r = e / HD, d = e % HD, q = qb + r;
    Qs[r * LDQ + d] = (q < SQ) ? Elem<T>::to_f(Qg[(long long)q * p.sQ.s + d]) : 0.f;
  }

  // per-row key windows; the tile loop covers their union
  int rlo[2], rhi[2];
#pragma unroll
  for (int i = 0; i < 2; ++i)
    fa_key_range(qb + ty * 2 + i, SQ, SK, p.causal, p.win_left, p.win_right, p.attn_chunk, rlo[i],
                 rhi[i]);
  int klo, khi, dummy;
  fa_key_range(qb, SQ, SK, p.causal, p.win_left, p.win_right, p.attn_chunk, klo, dummy);
  fa_key_range(min(qb + BR, SQ) - 1, SQ, SK, p.causal, p.win_left, p.win_right, p.attn_chunk, dummy,
               khi);
  if (klo < 0) klo = 0;
  if (khi > SK - 1) khi = SK - 1;

  const float slope = p.alibi_slopes ? p.alibi_slopes[h] : 0.f;
  const float scale2 = p.scale * FA_LOG2E;
  const bool drop = p.dropout_p > 0.f;
  const float inv_keep = drop ? 1.0f / (1.0f - p.dropout_p) : 1.f;

  float acc[2][DPT], m[2], l[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    m[i] = -INFINITY; l[i] = 0.f;
#pragma unroll
    for (int e = 0; e < DPT; ++e) acc[i][e] = 0.f;
  }

  // element e of a K/V tile (thread t takes e = t, t + 256, ...): K and V of key kb + e / HD, dim
  // e % HD, as fp32 (0 past SK)
  auto fetch = [&](int kb, int e, float& kx, float& vx) {
    const int r = e / HD, d = e % HD, k = kb + r;
    const bool ok = k < SK;
    if (p.block_table) {   // paged cache [num_blocks * page rows][NKV][HD]
      bool bad = false;
      const long long row = ok ? fa_paged_row(p, z, k, SK, bad) : 0;
      if (bad && d == 0) atomicOr(&g_simt_error, 1);
      const long long off = (row * (p.NH / p.gqa) + kvh) * HD + d;
      kx = ok ? Elem<T>::to_f(((const T*)p.K)[off]) : 0.f;
      vx = ok ? Elem<T>::to_f(((const T*)p.V)[off]) : 0.f;
    } else {
      kx = ok ? Elem<T>::to_f(Kg[(long long)k * p.sK.s + d]) : 0.f;
      vx = ok ? Elem<T>::to_f(Vg[(long long)k * p.sV.s + d]) : 0.f;
    }
  };
  // head dims up to 64: the next tile's K/V are loaded into registers while this tile computes
  constexpr int NE = BC * HD / 256;
  constexpr bool PF = NE <= 16;
  float kpf[PF ? NE : 1], vpf[PF ? NE : 1];
  const int kb0 = (klo / BC) * BC;
  if constexpr (PF) {
    if (kb0 <= khi) {
#pragma unroll
      for (int i = 0; i < NE; ++i) fetch(kb0, t + 256 * i, kpf[i], vpf[i]);
    }
  }
  for (int kb = kb0; kb <= khi; kb += BC) {
    __syncthreads();
    if constexpr (PF) {
#pragma unroll
      for (int i = 0; i < NE; ++i) {
        const int e = t + 256 * i, r = e / HD, d = e % HD;
        Ks[r * LDQ + d] = kpf[i];
        Vs[r * HD + d] = vpf[i];
      }
      if (kb + BC <= khi) {
#pragma unroll
        for (int i = 0; i < NE; ++i) fetch(kb + BC, t + 256 * i, kpf[i], vpf[i]);
      }
    } else {
      for (int e = t; e < BC * HD; e += 256) {
        float kx, vx;
        fetch(kb, e, kx, vx);
        Ks[(e / HD) * LDQ + e % HD] = kx;
        Vs[(e / HD) * HD + e % HD] = vx;
      }
    }
    __syncthreads();

    constexpr int KJ = BC / 16;   // keys per thread: tx, tx + 16, ...
    float s[2][KJ];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < KJ; ++j) s[i][j] = 0.f;
#pragma unroll 2
    for (int d = 0; d < HD; d += 4) {
      const float4 q0 = *reinterpret_cast<const float4*>(Qs + (ty * 2) * LDQ + d);
      const float4 q1 = *reinterpret_cast<const float4*>(Qs + (ty * 2 + 1) * LDQ + d);
#pragma unroll
      for (int j = 0; j < KJ; ++j) {
        const float4 kv = *reinterpret_cast<const float4*>(Ks + (tx + 16 * j) * LDQ + d);
        s[0][j] = fmaf(q0.x, kv.x, fmaf(q0.y, kv.y, fmaf(q0.z, kv.z, fmaf(q0.w, kv.w, s[0][j]))));
        s[1][j] = fmaf(q1.x, kv.x, fmaf(q1.y, kv.y, fmaf(q1.z, kv.z, fmaf(q1.w, kv.w, s[1][j]))));
      }
    }

#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int q = qb + ty * 2 + i;
      float sv[KJ], tmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < KJ; ++j) {
        const int key = kb + tx + 16 * j;
        float v;
        if (p.softcap > 0.f) v = p.softcap * tanhf(s[i][j] * p.scale / p.softcap) * FA_LOG2E;
        else v = s[i][j] * scale2;
        if (p.alibi_slopes) v += slope * (float)(key - q) * FA_LOG2E;
        if (q >= SQ || key < rlo[i] || key > rhi[i]) v = -INFINITY;
        sv[j] = v;
        tmax = fmaxf(tmax, v);
      }
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      const float mnew = fmaxf(m[i], tmax);
      // a row that has seen no visible key yet keeps m = -inf and contributes nothing
      const float muse = (mnew == -INFINITY) ? 0.f : mnew;
      float pj[KJ], ls = 0.f;
#pragma unroll
      for (int j = 0; j < KJ; ++j) { pj[j] = exp2f(sv[j] - muse); ls += pj[j]; }
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
      if (mnew != -INFINITY) {
        const float corr = exp2f(m[i] - mnew);
        l[i] = l[i] * corr + ls;
#pragma unroll
        for (int e = 0; e < DPT; ++e) acc[i][e] *= corr;
        m[i] = mnew;
        if (drop) {
#pragma unroll
          for (int j = 0; j < KJ; ++j) {
            const int key = kb + tx + 16 * j;
            if (q < SQ && key < SK)
              pj[j] *= fa_keep_mul(p.dropout_bits, p.philox_seed, h, SQ, SK, q, key, p.dropout_p, inv_keep);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < KJ; ++j) Ps[(ty * 2 + i) * LDP + tx + 16 * j] = pj[j];
    }
    __syncthreads();
    if constexpr (VEC) {
#pragma unroll 2
      for (int c = 0; c < BC; c += 4) {
        const float4 p0 = *reinterpret_cast<const float4*>(Ps + (ty * 2) * LDP + c);
        const float4 p1 = *reinterpret_cast<const float4*>(Ps + (ty * 2 + 1) * LDP + c);
        const float pa[4] = {p0.x, p0.y, p0.z, p0.w}, pb[4] = {p1.x, p1.y, p1.z, p1.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
#pragma unroll
          for (int e = 0; e < DPT; e += 4) {
            const float4 v = *reinterpret_cast<const float4*>(Vs + (c + u) * HD + 16 * e + 4 * tx);
            acc[0][e] = fmaf(pa[u], v.x, acc[0][e]);
            acc[0][e + 1] = fmaf(pa[u], v.y, acc[0][e + 1]);
            acc[0][e + 2] = fmaf(pa[u], v.z, acc[0][e + 2]);
            acc[0][e + 3] = fmaf(pa[u], v.w, acc[0][e + 3]);
            acc[1][e] = fmaf(pb[u], v.x, acc[1][e]);
            acc[1][e + 1] = fmaf(pb[u], v.y, acc[1][e + 1]);
            acc[1][e + 2] = fmaf(pb[u], v.z, acc[1][e + 2]);
            acc[1][e + 3] = fmaf(pb[u], v.w, acc[1][e + 3]);
          }
        }
      }
    } else {
#pragma unroll 4
      for (int c = 0; c < BC; ++c) {
        const float p0 = Ps[(ty * 2) * LDP + c], p1 = Ps[(ty * 2 + 1) * LDP + c];
#pragma unroll
        for (int e = 0; e < DPT; ++e) {
          const float v = Vs[c * HD + tx + 16 * e];
          acc[0][e] = fmaf(p0, v, acc[0][e]);
          acc[1][e] = fmaf(p1, v, acc[1][e]);
        }
      }
    }
  }

  T* Og = (T*)p.O + g.o0 + (long long)h * p.sO.h;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int q = qb + ty * 2 + i;
    if (q >= SQ) continue;
    const float inv = l[i] > 0.f ? 1.f / l[i] : 0.f;
#pragma unroll
    for (int e = 0; e < DPT; ++e) Og[(long long)q * p.sO.s + dim(e)] = Elem<T>::from_f(acc[i][e] * inv);
    if (p.LSE && tx == 0) {
      const long long li = fa_lse_index(varlen, z, h, p.NH, p.SQ, g.tok_q, p.lse_total_q, q);
      p.LSE[li] = l[i] > 0.f ? m[i] * FA_LN2 + logf(l[i]) : -INFINITY;
    }
  }
}

template <typename T, int HD>
int launch_hd(const FaFwdParams& p, cudaStream_t st) {
  const size_t smem = sizeof(float) * (size_t)(BR * (HD + 4) + BC * (HD + 4) + BC * HD + BR * (BC + 4));
  static unsigned long long done = 0;
  if (int rc = fa::ensure_smem((const void*)fwd_simt_kernel<T, HD>, (int)smem, &done)) return rc;
  dim3 grid((p.SQ + BR - 1) / BR, p.NH, p.batch);
  fwd_simt_kernel<T, HD><<<grid, 256, smem, st>>>(p);
  fa::count_launch();
  return fa::cuda_status(cudaGetLastError(), "fwd_simt launch");
}

template <typename T>
int launch_t(const FaFwdParams& p, cudaStream_t st) {
  switch (p.HD) {
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
  fa::set_error("forward: head_dim=%d not instantiated (valid: multiples of 16 up to 256 "
                "from the list 16,32,48,64,80,96,112,128,160,192,224,256)", p.HD);
  return FA_ERR_UNSUPPORTED;
}

}  // namespace

namespace fa {
int fwd_simt_device_error(int clear) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_simt_error, sizeof(int));
  if (clear && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_simt_error, &zero, sizeof(int));
  }
  return v;
}
int fwd_simt(const FaFwdParams& p, int dtype, cudaStream_t st) {
  if (dtype == FA_DTYPE_F16) return launch_t<__half>(p, st);
  if (dtype == FA_DTYPE_BF16) return launch_t<__nv_bfloat16>(p, st);
  return launch_t<float>(p, st);
}
}  // namespace fa
