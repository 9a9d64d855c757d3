// decode_peer.cu — the exchange and LSE merge of a decode whose KV range is split across GPUs, as one
// kernel over peer memory (NVLink P2P loads), in place of an all-gather followed by a merge.
//
// Every rank's decode writes its partial result (rows = batch * new tokens * heads rows of D fp32
// values, then the rows' fp32 LSE in the same order) into its own buffer of a symmetric
// allocation; every rank can load every other rank's buffer through a peer pointer.  Per decode
// step s (a device counter, so a captured CUDA graph replays correctly):
//   merge kernel : publishes ready = s into every peer's signal words (system-scope release after a
//                  system fence: the rank's partial, written by the kernel before, is visible),
//                  waits until every peer's ready word is >= s (system-scope acquire, bounded),
//                  then merges each row from all ranks' buffers: out = sum_r w_r out_r / sum_r w_r,
//                  w_r = exp(lse_r - max_r lse_r) (flash_attn_combine's rule).
//   end kernel   : publishes done = s to every peer, waits for every peer's done >= s (nobody reads
//                  this rank's buffer any more, so the next step may overwrite it), advances the
//                  counter.
// Waits give up after a bound and record FA_PEER_ERR_WAIT in the caller's error word instead of
// hanging; the merge then still writes every row.  Signal words: ready from rank r at word r,
// done from rank r at word world + r.
#include <stdint.h>
#include <algorithm>
#include "fa_common.cuh"
#include "fa_launch.h"

namespace {

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// wait until every peer's word at base + r (r != rank) reaches `step`; false when the bound ran out
__device__ __forceinline__ bool wait_words(const unsigned int* base, int rank, int world, unsigned int step,
                                           uint64_t limit_ns) {
  const uint64_t t0 = gtimer();
  for (int r = 0; r < world; ++r) {
    if (r == rank) continue;
    while ((int)(ld_acquire_sys(base + r) - step) < 0) {
      if (gtimer() - t0 > limit_ns) return false;
      __nanosleep(64);
    }
  }
  return true;
}

template <typename TO>
__global__ void peer_merge_kernel(const FaPeerMergeParams p) {
  pdl_wait();   // this rank's partial (written by the kernels before) is complete and visible
  const unsigned int step = (unsigned int)(*p.step) + 1u;
  const uint64_t limit = p.wait_ns ? p.wait_ns : 2000000000ull;
  const long long slot = p.slot_floats ? (long long)((step - 1u) & 1u) * p.slot_floats : 0;
  // publish: every CTA's threads 0 .. world-1 store this rank's ready word into each peer (same
  // value, so the redundancy is harmless, and no CTA depends on another being resident)
  if (threadIdx.x < (unsigned)p.world && (int)threadIdx.x != p.rank) {
    __threadfence_system();
    st_release_sys(p.peer_signals[threadIdx.x] + p.rank, step);
  }
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    const bool ok = wait_words(p.peer_signals[p.rank], p.rank, p.world, step, limit);
    if (!ok && p.err_flag) atomicOr(p.err_flag, FA_PEER_ERR_WAIT);
    ok_s = ok;
  }
  __syncthreads();
  const bool ok = ok_s;
  const long long rows = (long long)p.B * p.S * p.H;
  const int warps = blockDim.x / 32, lane = threadIdx.x % 32;
  for (long long row = (long long)blockIdx.x * warps + threadIdx.x / 32; row < rows; row += (long long)gridDim.x * warps) {
    // row = (b * S + s) * H + h; LSE of rank r at buffer r + rows * D + row
    float M = -INFINITY;
    float lse[FA_PEER_MAX_WORLD];
#pragma unroll
    for (int r = 0; r < FA_PEER_MAX_WORLD; ++r) {
      lse[r] = (ok && r < p.world) ? __ldcg(p.peer_bufs[r] + slot + rows * p.D + row) : -INFINITY;
      M = fmaxf(M, lse[r]);
    }
    float W = 0.f;
#pragma unroll
    for (int r = 0; r < FA_PEER_MAX_WORLD; ++r) {
      lse[r] = (M != -INFINITY && r < p.world) ? __expf(lse[r] - M) : 0.f;
      W += lse[r];
    }
    const float invW = W > 0.f ? 1.f / W : 0.f;
    for (int d = 4 * lane; d < p.D; d += 128) {   // 16-byte loads from each rank's row
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int r = 0; r < FA_PEER_MAX_WORLD; ++r) {
        if (r < p.world && lse[r] > 0.f) {
          const float4 v = __ldcg(reinterpret_cast<const float4*>(p.peer_bufs[r] + slot + row * p.D + d));
          a.x = fmaf(lse[r], v.x, a.x);
          a.y = fmaf(lse[r], v.y, a.y);
          a.z = fmaf(lse[r], v.z, a.z);
          a.w = fmaf(lse[r], v.w, a.w);
        }
      }
      TO* o = (TO*)p.out + row * p.D + d;
      o[0] = Elem<TO>::from_f(a.x * invW);
      o[1] = Elem<TO>::from_f(a.y * invW);
      o[2] = Elem<TO>::from_f(a.z * invW);
      o[3] = Elem<TO>::from_f(a.w * invW);
    }
    if (p.lse_out && lane == 0) {
      const long long h = row % p.H, bs = row / p.H, s = bs % p.S, b = bs / p.S;
      p.lse_out[(b * p.H + h) * p.S + s] = W > 0.f ? M + logf(W) : -INFINITY;
    }
  }
  if (p.slot_floats) {
    // two-slot mode: the last CTA to finish advances the step (every CTA read it when it started)
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      if (atomicAdd(p.done_ctas, 1) == (int)gridDim.x - 1) {
        *p.done_ctas = 0;
        *p.step = (int)step;
        __threadfence();
      }
    }
  }
}

__global__ void peer_end_kernel(const FaPeerMergeParams p) {
  const unsigned int step = (unsigned int)(*p.step) + 1u;
  const uint64_t limit = p.wait_ns ? p.wait_ns : 2000000000ull;
  if (threadIdx.x < (unsigned)p.world && (int)threadIdx.x != p.rank) {
    __threadfence_system();
    st_release_sys(p.peer_signals[threadIdx.x] + p.world + p.rank, step);
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    if (!wait_words(p.peer_signals[p.rank] + p.world, p.rank, p.world, step, limit) && p.err_flag)
      atomicOr(p.err_flag, FA_PEER_ERR_WAIT);
    *p.step = (int)step;
  }
}

}  // namespace

extern "C" FA_API int fa_peer_merge_launch(const FaPeerMergeParams* pp, void* stream) {
  if (!pp) {
    fa::set_error("peer merge: null parameter block");
    return FA_ERR_INVALID;
  }
  if (pp->struct_size != sizeof(FaPeerMergeParams)) {
    fa::set_error("peer merge: struct_size %u != %zu", pp->struct_size, sizeof(FaPeerMergeParams));
    return FA_ERR_ABI;
  }
  const FaPeerMergeParams& p = *pp;
  FA_CHECK_ARG(p.peer_bufs && p.peer_signals && p.out && p.step, "peer merge: peer_bufs, peer_signals, out, step "
               "must be non-null");
  FA_CHECK_ARG(p.world >= 1 && p.world <= FA_PEER_MAX_WORLD && p.rank >= 0 && p.rank < p.world,
               "peer merge: rank %d / world %d (world at most %d)", p.rank, p.world, FA_PEER_MAX_WORLD);
  FA_CHECK_ARG(p.B >= 0 && p.S >= 0 && p.H >= 0 && p.D > 0 && p.D % 4 == 0, "peer merge: bad sizes (D a multiple of 4)");
  FA_CHECK_ARG(p.out_dtype == FA_DTYPE_F16 || p.out_dtype == FA_DTYPE_BF16 || p.out_dtype == FA_DTYPE_F32,
               "peer merge: out_dtype %d", p.out_dtype);
  FA_CHECK_ARG(p.slot_floats >= 0 && (p.slot_floats == 0 || p.done_ctas),
               "peer merge: two-slot mode needs done_ctas");
  FA_CHECK_ARG(p.slot_floats == 0 || p.slot_floats >= (long long)p.B * p.S * p.H * (p.D + 1),
               "peer merge: slot_floats %lld below one packed partial", p.slot_floats);
  const long long rows = (long long)p.B * p.S * p.H;
  cudaStream_t st = (cudaStream_t)stream;
  // one warp per row, 8 warps per CTA, at most two CTAs per SM's worth
  const long long ctas = std::min<long long>(std::max<long long>((rows + 7) / 8, 1), 2LL * fa::num_sms());
  cudaError_t le;
  if (p.out_dtype == FA_DTYPE_F16) le = fa::launch_pdl(peer_merge_kernel<__half>, dim3((unsigned)ctas), dim3(256), 0, st, p);
  else if (p.out_dtype == FA_DTYPE_BF16)
    le = fa::launch_pdl(peer_merge_kernel<__nv_bfloat16>, dim3((unsigned)ctas), dim3(256), 0, st, p);
  else le = fa::launch_pdl(peer_merge_kernel<float>, dim3((unsigned)ctas), dim3(256), 0, st, p);
  fa::count_launch();
  return fa::cuda_status(le != cudaSuccess ? le : cudaGetLastError(), "peer merge launch");
}

extern "C" FA_API int fa_peer_step_end_launch(const FaPeerMergeParams* pp, void* stream) {
  if (!pp || pp->struct_size != sizeof(FaPeerMergeParams)) {
    fa::set_error("peer step end: null parameter block or struct_size mismatch");
    return pp ? FA_ERR_ABI : FA_ERR_INVALID;
  }
  const FaPeerMergeParams& p = *pp;
  FA_CHECK_ARG(p.peer_signals && p.step && p.world >= 1 && p.world <= FA_PEER_MAX_WORLD && p.rank >= 0 &&
                   p.rank < p.world,
               "peer step end: peer_signals / step / rank / world");
  peer_end_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(p);
  fa::count_launch();
  return fa::cuda_status(cudaGetLastError(), "peer step end launch");
}
