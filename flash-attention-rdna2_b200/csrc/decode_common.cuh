// decode_common.cuh — helpers shared by the decode kernels (CUDA-core and tensor-core paths):
// rotary rotation of one row and the bounds-checked page lookup of a cache position.
#pragma once
#include "fa_common.cuh"

namespace fa_dec {

// Rotates the first rdim dims of v in place: mode 1 = NeoX halves (d, d + rdim/2), mode 2 =
// interleaved pairs (2d, 2d+1); c / s are the table row of the position (rdim/2 entries).
__device__ __forceinline__ void rotate_row(float* v, int rdim, int mode, const float* c, const float* s) {
  const int half = rdim / 2;
  for (int d = 0; d < half; ++d) {
    if (mode == 1) {
      const float x = v[d], y = v[d + half];
      v[d] = x * c[d] - y * s[d];
      v[d + half] = y * c[d] + x * s[d];
    } else {
      const float x = v[2 * d], y = v[2 * d + 1];
      v[2 * d] = x * c[d] - y * s[d];
      v[2 * d + 1] = y * c[d] + x * s[d];
    }
  }
}

// Page lookup with a bounds check; an invalid page index marks the position invisible and
// raises the caller's error flag (the cache is never read out of bounds).
__device__ __forceinline__ long long page_of(const FaDecParams& p, int b, int pos, int shift, bool& ok) {
  const int slot = pos >> shift;
  if (pos < 0 || slot >= p.max_blocks) {   // position past the block table's row
    ok = false;
    if (p.err_flag) atomicExch(p.err_flag, 1);
    return 0;
  }
  const int blk = p.block_table[(long long)b * p.max_blocks + slot];
  ok = blk >= 0 && (p.num_blocks <= 0 || blk < p.num_blocks);
  if (!ok && p.err_flag) atomicExch(p.err_flag, 1);
  return ok ? (long long)blk : 0;
}

}  // namespace fa_dec
