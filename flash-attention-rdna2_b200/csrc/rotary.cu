// rotary.cu — rotary position embedding of q / k in one HBM pass (see fa_rotary_launch in
// fable_attn.h).
//
// The reference rotates with torch ops in the tensor's dtype (layers/rotary.py:20-68): cos/sin
// are cast to x's dtype, then a*cos - b*sin and b*cos + a*sin are evaluated op by op, each
// product and the difference rounded to that dtype.  This kernel performs the same roundings in
// the same order, so its output equals the reference's bit for bit, in one read and one write of
// the rotated dims (plus a copy of the rest when the output is a new tensor).
//
// One thread per (row, head, pair): NeoX pairs (j, j + rd/2), interleaved pairs (2j, 2j + 1).
// Positions: dense rows b*seqlen + s sit at s + offset[b]; packed varlen rows at t - cu[seq(t)]
// + offset[seq] with seq(t) found by binary search over cu_seqlens.  A position past the cos/sin
// table leaves the row unrotated and raises the device error flag (fa_device_error bit 256).
#include <algorithm>
#include "fa_common.cuh"
#include "fa_launch.h"

namespace {

__device__ int g_rot_error = 0;

template <typename T>
__device__ __forceinline__ float rnd(float x) {
  return Elem<T>::to_f(Elem<T>::from_f(x));
}

template <typename T>
__global__ void __launch_bounds__(256) rotary_kernel(const FaRotaryParams p) {
  const int half = p.rotary_dim / 2;
  const long long items = p.rows * p.heads * (long long)half;
  const T* x = (const T*)p.x;
  T* out = (T*)p.out;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < items; i += (long long)gridDim.x * blockDim.x) {
    const int j = (int)(i % half);
    const long long rh = i / half;
    const int h = (int)(rh % p.heads);
    const long long row = rh / p.heads;
    int pos, seq;
    if (p.cu_seqlens) {   // last sequence whose start <= row
      int lo = 0, hi = p.batch - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (p.cu_seqlens[mid] <= row) lo = mid;
        else hi = mid - 1;
      }
      seq = lo;
      pos = (int)(row - p.cu_seqlens[seq]);
    } else {
      seq = (int)(row / p.seqlen);
      pos = (int)(row % p.seqlen);
    }
    pos += p.offsets ? p.offsets[seq] : p.offset;
    const int d1 = p.interleaved ? 2 * j : j, d2 = p.interleaved ? 2 * j + 1 : j + half;
    const T* xr = x + row * p.x_row_stride + (long long)h * p.x_head_stride;
    T* orow = out + row * p.out_row_stride + (long long)h * p.out_head_stride;
    const float a = Elem<T>::to_f(xr[d1]), b = Elem<T>::to_f(xr[d2]);
    if (pos < 0 || pos >= p.seqlen_ro) {
      atomicOr(&g_rot_error, 1);
      orow[d1] = xr[d1];
      orow[d2] = xr[d2];
      continue;
    }
    const float c = rnd<T>(p.cos[(long long)pos * half + j]), s = rnd<T>(p.sin[(long long)pos * half + j]);
    // explicit roundings: no fused multiply-add, exactly torch's separate elementwise ops
    orow[d1] = Elem<T>::from_f(__fsub_rn(rnd<T>(__fmul_rn(a, c)), rnd<T>(__fmul_rn(b, s))));
    orow[d2] = Elem<T>::from_f(__fadd_rn(rnd<T>(__fmul_rn(b, c)), rnd<T>(__fmul_rn(a, s))));
  }
}

// Vectorised form for 16-byte aligned rows: one thread per 16-byte unit of U elements.  NeoX:
// a unit of the first half and its partner unit rd/2 further (U pairs); interleaved: one unit
// (U/2 pairs); out of place, units past rotary_dim are copied in the same pass.
__device__ __forceinline__ void pos_of(const FaRotaryParams& p, long long row, int& pos) {
  int seq;
  if (p.cu_seqlens) {
    int lo = 0, hi = p.batch - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.cu_seqlens[mid] <= row) lo = mid;
      else hi = mid - 1;
    }
    seq = lo;
    pos = (int)(row - p.cu_seqlens[seq]);
  } else {
    seq = (int)(row / p.seqlen);
    pos = (int)(row % p.seqlen);
  }
  pos += p.offsets ? p.offsets[seq] : p.offset;
}

template <typename T>
__device__ __forceinline__ void rot2(float a, float b, float c, float s, float& o1, float& o2) {
  o1 = __fsub_rn(rnd<T>(__fmul_rn(a, c)), rnd<T>(__fmul_rn(b, s)));
  o2 = __fadd_rn(rnd<T>(__fmul_rn(b, c)), rnd<T>(__fmul_rn(a, s)));
}

template <typename T>
__global__ void __launch_bounds__(256) rotary_vec_kernel(const FaRotaryParams p) {
  constexpr int U = 16 / sizeof(T);
  union Vec { uint4 u; T e[U]; };
  const int half = p.rotary_dim / 2;
  const int rot_units = p.interleaved ? p.rotary_dim / U : half / U;
  const int copy_units = (p.out != p.x) ? (p.dim - p.rotary_dim) / U : 0;
  const int W = rot_units + copy_units;
  const long long items = p.rows * p.heads * (long long)W;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < items; i += (long long)gridDim.x * blockDim.x) {
    const int w = (int)(i % W);
    const long long rh = i / W;
    const int h = (int)(rh % p.heads);
    const long long row = rh / p.heads;
    const T* xr = (const T*)p.x + row * p.x_row_stride + (long long)h * p.x_head_stride;
    T* orow = (T*)p.out + row * p.out_row_stride + (long long)h * p.out_head_stride;
    if (w >= rot_units) {   // copy of a unit past rotary_dim
      const int d = p.rotary_dim + (w - rot_units) * U;
      *reinterpret_cast<uint4*>(orow + d) = __ldg(reinterpret_cast<const uint4*>(xr + d));
      continue;
    }
    int pos;
    pos_of(p, row, pos);
    const bool inside = pos >= 0 && pos < p.seqlen_ro;
    if (!inside) atomicOr(&g_rot_error, 1);
    const float* cr = p.cos + (long long)(inside ? pos : 0) * half;
    const float* sr = p.sin + (long long)(inside ? pos : 0) * half;
    if (p.interleaved) {
      const int d = w * U;
      Vec v, o;
      v.u = __ldg(reinterpret_cast<const uint4*>(xr + d));
#pragma unroll
      for (int k = 0; k < U; k += 2) {
        const int j = (d + k) / 2;
        float o1 = Elem<T>::to_f(v.e[k]), o2 = Elem<T>::to_f(v.e[k + 1]);
        if (inside) rot2<T>(o1, o2, rnd<T>(cr[j]), rnd<T>(sr[j]), o1, o2);
        o.e[k] = Elem<T>::from_f(o1);
        o.e[k + 1] = Elem<T>::from_f(o2);
      }
      *reinterpret_cast<uint4*>(orow + d) = o.u;
    } else {
      const int d = w * U;
      Vec va, vb, oa, ob;
      va.u = __ldg(reinterpret_cast<const uint4*>(xr + d));
      vb.u = __ldg(reinterpret_cast<const uint4*>(xr + d + half));
#pragma unroll
      for (int k = 0; k < U; ++k) {
        float o1 = Elem<T>::to_f(va.e[k]), o2 = Elem<T>::to_f(vb.e[k]);
        if (inside) rot2<T>(o1, o2, rnd<T>(cr[d + k]), rnd<T>(sr[d + k]), o1, o2);
        oa.e[k] = Elem<T>::from_f(o1);
        ob.e[k] = Elem<T>::from_f(o2);
      }
      *reinterpret_cast<uint4*>(orow + d) = oa.u;
      *reinterpret_cast<uint4*>(orow + d + half) = ob.u;
    }
  }
}

// dims past rotary_dim, for an out-of-place rotation
template <typename T>
__global__ void __launch_bounds__(256) rotary_copy_kernel(const FaRotaryParams p) {
  const int rest = p.dim - p.rotary_dim;
  const long long items = p.rows * p.heads * (long long)rest;
  const T* x = (const T*)p.x;
  T* out = (T*)p.out;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < items; i += (long long)gridDim.x * blockDim.x) {
    const int d = p.rotary_dim + (int)(i % rest);
    const long long rh = i / rest;
    const int h = (int)(rh % p.heads);
    const long long row = rh / p.heads;
    out[row * p.out_row_stride + (long long)h * p.out_head_stride + d] =
        x[row * p.x_row_stride + (long long)h * p.x_head_stride + d];
  }
}

template <typename T>
int run(const FaRotaryParams& p, cudaStream_t st) {
  constexpr int U = 16 / sizeof(T);
  const bool vec = ((uintptr_t)p.x % 16 == 0) && ((uintptr_t)p.out % 16 == 0) && p.dim % U == 0 &&
                   (p.interleaved ? p.rotary_dim % U == 0 : (p.rotary_dim / 2) % U == 0) &&
                   p.x_row_stride % U == 0 && p.x_head_stride % U == 0 && p.out_row_stride % U == 0 &&
                   p.out_head_stride % U == 0;
  if (vec) {
    const int W = (p.interleaved ? p.rotary_dim / U : p.rotary_dim / 2 / U) + (p.out != p.x ? (p.dim - p.rotary_dim) / U : 0);
    const long long items = p.rows * p.heads * (long long)W;
    if (items > 0) {
      rotary_vec_kernel<T><<<(int)std::min<long long>((items + 255) / 256, 32LL * fa::num_sms()), 256, 0, st>>>(p);
      fa::count_launch();
      return fa::cuda_status(cudaGetLastError(), "rotary launch");
    }
    return FA_OK;
  }
  const long long items = p.rows * p.heads * (long long)(p.rotary_dim / 2);
  const int grid = (int)std::min<long long>((items + 255) / 256, 64LL * fa::num_sms());
  if (items > 0) {
    rotary_kernel<T><<<grid, 256, 0, st>>>(p);
    fa::count_launch();
    if (int rc = fa::cuda_status(cudaGetLastError(), "rotary launch")) return rc;
  }
  if (p.out != p.x && p.dim > p.rotary_dim) {
    const long long rest = p.rows * p.heads * (long long)(p.dim - p.rotary_dim);
    rotary_copy_kernel<T><<<(int)std::min<long long>((rest + 255) / 256, 64LL * fa::num_sms()), 256, 0, st>>>(p);
    fa::count_launch();
    if (int rc = fa::cuda_status(cudaGetLastError(), "rotary copy launch")) return rc;
  }
  return FA_OK;
}

}  // namespace

namespace fa {
int rot_device_error(int clear) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_rot_error, sizeof(int));
  if (clear && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_rot_error, &zero, sizeof(int));
  }
  return v;
}
}  // namespace fa

extern "C" FA_API int fa_rotary_launch(const FaRotaryParams* pp, int dtype, void* stream) {
  if (!pp) {
    fa::set_error("FaRotaryParams: null parameter block");
    return FA_ERR_INVALID;
  }
  if (pp->struct_size != sizeof(FaRotaryParams)) {
    fa::set_error("FaRotaryParams: struct_size %u != %zu", pp->struct_size, sizeof(FaRotaryParams));
    return FA_ERR_ABI;
  }
  const FaRotaryParams& p = *pp;
  FA_CHECK_ARG(p.x && p.out && p.cos && p.sin, "rotary: x, out, cos, sin must be non-null");
  FA_CHECK_ARG(p.rows >= 0 && p.heads > 0 && p.dim > 0, "rotary: rows=%lld heads=%d dim=%d", p.rows, p.heads, p.dim);
  FA_CHECK_ARG(p.rotary_dim > 0 && p.rotary_dim % 2 == 0 && p.rotary_dim <= p.dim,
               "rotary: rotary_dim=%d must be even and <= dim=%d", p.rotary_dim, p.dim);
  FA_CHECK_ARG(p.seqlen_ro > 0, "rotary: seqlen_ro=%d", p.seqlen_ro);
  if (p.cu_seqlens) FA_CHECK_ARG(p.batch > 0, "rotary: varlen needs batch > 0");
  else FA_CHECK_ARG(p.seqlen > 0, "rotary: dense rows need seqlen > 0");
  FA_CHECK_ARG(dtype == FA_DTYPE_F16 || dtype == FA_DTYPE_BF16 || dtype == FA_DTYPE_F32, "rotary: dtype code %d", dtype);
  if (p.rows == 0) return FA_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == FA_DTYPE_F16) return run<__half>(p, st);
  if (dtype == FA_DTYPE_BF16) return run<__nv_bfloat16>(p, st);
  return run<float>(p, st);
}
