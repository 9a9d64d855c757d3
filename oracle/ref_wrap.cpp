// ref_wrap.cpp — exports the reference's OWN CPU oracle (kernels/fa_common.hpp:71-139, compiled
// from the reference sources at build time, never copied) through a C ABI for the tests and for
// bench.py's reference arm.  Test infrastructure only.
#include <hip/hip_runtime.h>
#include FA_REF_COMMON
extern "C" {
// ref_attention: Q/O [SQ][NH][HD], K/V [NKV][SK][HD], LSE [NH][SQ] (reference layouts)
void ref_attention_c(const float* Q, const float* K, const float* V, float* O, float* LSE, int SQ, int SK, int HD,
                     int NH, int gqa, float scale, float softcap, int win_left, int win_right, int causal,
                     int alibi_on, const float* slopes, int attn_chunk) {
  RefCfg c{SQ, SK, HD, NH, gqa, scale, softcap, win_left, win_right, causal != 0, alibi_on != 0, slopes, attn_chunk};
  ref_attention(Q, K, V, O, LSE, c);
}
void ref_philox_c(unsigned long long seed, unsigned long long idx, unsigned int* out2) {
  uint2 r = philox(seed, idx);
  out2[0] = r.x;
  out2[1] = r.y;
}
float ref_dropout_mul_c(unsigned long long seed, unsigned long long idx, float p) {
  return dropout_mul(seed, idx, p, 1.0f / (1.0f - p));
}
}
