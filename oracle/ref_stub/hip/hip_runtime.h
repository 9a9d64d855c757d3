/* Host-only stand-in for <hip/hip_runtime.h>, just enough for the reference's
 * kernels/fa_common.hpp to compile with g++ so its CPU oracle (ref_attention) and Philox can be
 * called from tests.  Device-only helpers in that header are compiled but never called. */
#pragma once
#include <stdint.h>
#define __device__
#define __host__
#define __global__
#define __forceinline__ inline
typedef int hipError_t;
#define hipSuccess 0
static inline const char* hipGetErrorString(hipError_t) { return "hip stub"; }
struct uint2 { unsigned int x, y; };
static inline uint2 make_uint2(unsigned int x, unsigned int y) { uint2 r; r.x = x; r.y = y; return r; }
static inline unsigned int __umulhi(unsigned int a, unsigned int b) { return (unsigned int)(((unsigned long long)a * b) >> 32); }
static inline int __builtin_amdgcn_update_dpp(int, int v, int, int, int, bool) { return v; }
