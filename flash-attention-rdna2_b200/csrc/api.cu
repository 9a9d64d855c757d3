// api.cu — the extern "C" entry points declared in include/fable_attn.h: argument validation,
// error reporting (status codes + thread-local message, never abort), kernel selection.
#include <algorithm>
#include <stdarg.h>
#include <stdio.h>
#include <atomic>
#include "fa_common.cuh"
#include "fa_launch.h"

namespace fa {

static thread_local char g_err[512] = "";
static std::atomic<unsigned long long> g_launches{0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return FA_OK;
  set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  return FA_ERR_CUDA;
}

void count_launch(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

int num_sms() {
  static int cached[64] = {0};
  const int d = current_device();
  if (d < 0 || d >= 64) return 148;
  if (!cached[d]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || v <= 0) v = 148;
    cached[d] = v;
  }
  return cached[d];
}

// FABLE_ATTN_REQUIRE_TC=1: fp16/bf16 forward / backward requests that the tensor-core kernels do
// not take fail with FA_ERR_UNSUPPORTED instead of running on the CUDA-core kernels (lets a caller,
// or a test, be sure which kernels ran)
bool require_tc() {
  const char* v = getenv("FABLE_ATTN_REQUIRE_TC");
  return v && v[0] && v[0] != '0';
}

bool pdl_enabled() {
  const char* v = getenv("FABLE_ATTN_NO_PDL");
  return !(v && v[0] && v[0] != '0');
}

int ensure_smem(const void* func, int bytes, unsigned long long* done_mask) {
  const int d = current_device();
  const unsigned long long bit = 1ull << (d & 63);
  if (*done_mask & bit) return FA_OK;
  const cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
  *done_mask |= bit;
  return FA_OK;
}

static bool valid_hd(int d) {
  switch (d) {
    case 16: case 32: case 48: case 64: case 80: case 96: case 112: case 128:
    case 160: case 192: case 224: case 256: return true;
  }
  return false;
}

}  // namespace fa

using fa::set_error;

#define FA_ABI_GUARD(p, T)                                                                   \
  do {                                                                                       \
    if (!(p)) { set_error(#T ": null parameter block"); return FA_ERR_INVALID; }              \
    if ((p)->struct_size != sizeof(T)) {                                                     \
      set_error(#T ": struct_size %u != %zu (caller built against another fable_attn.h)",     \
                (p)->struct_size, sizeof(T));                                                \
      return FA_ERR_ABI;                                                                     \
    }                                                                                        \
  } while (0)

static bool dtype_ok(int dt) { return dt == FA_DTYPE_F16 || dt == FA_DTYPE_BF16 || dt == FA_DTYPE_F32; }

extern "C" int fa_abi_version(void) { return FA_ABI_VERSION; }
extern "C" const char* fa_last_error(void) { return fa::g_err; }
extern "C" unsigned long long fa_kernel_launch_count(void) { return fa::g_launches.load(); }

extern "C" int fa_forward_launch(const FaFwdParams* pp, int dtype, void* stream) {
  FA_ABI_GUARD(pp, FaFwdParams);
  const FaFwdParams& p = *pp;
  FA_CHECK_ARG(dtype_ok(dtype), "forward: dtype code %d (0=fp16, 1=bf16, 2=fp32)", dtype);
  FA_CHECK_ARG(p.Q && p.K && p.V && p.O, "forward: Q/K/V/O must be non-null");
  FA_CHECK_ARG(p.batch >= 0 && p.SQ >= 0 && p.SK >= 0 && p.NH > 0 && p.gqa > 0 && p.NH % p.gqa == 0,
               "forward: bad sizes batch=%d SQ=%d SK=%d NH=%d gqa=%d", p.batch, p.SQ, p.SK, p.NH, p.gqa);
  FA_CHECK_ARG((p.cu_q == nullptr) == (p.cu_k == nullptr), "forward: cu_q and cu_k must both be set or both null");
  FA_CHECK_ARG(!(p.dropout_p < 0.f) && p.dropout_p < 1.f, "forward: dropout_p=%f outside [0,1)", p.dropout_p);
  FA_CHECK_ARG(p.attn_chunk >= 0, "forward: attn_chunk=%d < 0", p.attn_chunk);
  if (!fa::valid_hd(p.HD)) {
    set_error("forward: head_dim=%d not instantiated (16,32,48,64,80,96,112,128,160,192,224,256)", p.HD);
    return FA_ERR_UNSUPPORTED;
  }
  if (p.cu_q && p.LSE) FA_CHECK_ARG(p.lse_total_q > 0, "forward: varlen LSE needs lse_total_q");
  FA_CHECK_ARG(!(p.dropout_bits && p.cu_q), "forward: dropout_bits is for dense layouts only");
  if (p.block_table) {
    FA_CHECK_ARG(p.cu_q != nullptr, "forward: a block table needs the varlen layout (cu_q / cu_k)");
    FA_CHECK_ARG(p.page > 0 && p.max_blocks > 0 && p.num_blocks > 0, "forward: paged K/V needs page=%d > 0, "
                 "max_blocks=%d > 0, num_blocks=%lld > 0", p.page, p.max_blocks, p.num_blocks);
  }
  if (p.rot_cos) {
    FA_CHECK_ARG(p.rot_sin != nullptr && p.rot_dim > 0 && p.rot_dim % 2 == 0 && p.rot_dim <= p.HD &&
                     p.rot_seqlen_ro > 0,
                 "forward: rotary needs rot_sin, an even rot_dim=%d in (0, head_dim], rot_seqlen_ro=%d > 0",
                 p.rot_dim, p.rot_seqlen_ro);
  }
  if (p.batch == 0 || p.SQ == 0) return FA_OK;
  cudaStream_t st = (cudaStream_t)stream;
  bool taken = false;
  if (dtype != FA_DTYPE_F32) {
    const int rc = fa::fwd_sm100(p, dtype, st, &taken);
    if (taken || rc) return rc;
    if (fa::require_tc()) {
      set_error("forward: FABLE_ATTN_REQUIRE_TC is set and the tensor-core kernels do not take this request "
                "(head_dim=%d, alignment or strides)", p.HD);
      return FA_ERR_UNSUPPORTED;
    }
  }
  if (p.rot_cos) {
    set_error("forward: in-kernel rotary needs the tensor-core path (fp16/bf16, head_dim a multiple of 16 up to "
              "256, 16-byte aligned rows); rotate q with fa_rotary_launch instead");
    return FA_ERR_UNSUPPORTED;
  }
  return fa::fwd_simt(p, dtype, st);
}

extern "C" int fable_attn_backward_launch(const FaBwdParams* pp, int dtype, void* stream) {
  FA_ABI_GUARD(pp, FaBwdParams);
  const FaBwdParams& p = *pp;
  FA_CHECK_ARG(dtype_ok(dtype), "backward: dtype code %d", dtype);
  FA_CHECK_ARG(p.Q && p.K && p.V && p.O && p.dO && p.dQ && p.dK && p.dV && p.lse && p.dsum,
               "backward: every tensor pointer (Q,K,V,O,dO,dQ,dK,dV,lse,dsum) must be non-null");
  FA_CHECK_ARG(p.B >= 0 && p.SQ >= 0 && p.SK >= 0 && p.Hq > 0 && p.Hk > 0 && p.Hq % p.Hk == 0 &&
                   p.gqa == p.Hq / p.Hk,
               "backward: bad sizes B=%d Hq=%d Hk=%d gqa=%d", p.B, p.Hq, p.Hk, p.gqa);
  FA_CHECK_ARG((p.cu_q == nullptr) == (p.cu_k == nullptr), "backward: cu_q and cu_k must both be set or both null");
  FA_CHECK_ARG(!p.dropout || (p.dropout_p > 0.f && p.dropout_p < 1.f), "backward: dropout_p=%f", p.dropout_p);
  if (!fa::valid_hd(p.D)) {
    set_error("backward: head_dim=%d not instantiated", p.D);
    return FA_ERR_UNSUPPORTED;
  }
  if (p.cu_q) FA_CHECK_ARG(p.lse_total_q > 0, "backward: varlen needs lse_total_q");
  FA_CHECK_ARG(!(p.dropout_bits && p.cu_q), "backward: dropout_bits is for dense layouts only");
  FA_CHECK_ARG(!(p.dropout_bits_t && !p.dropout_bits), "backward: dropout_bits_t is the workspace of dropout_bits");
  if (p.B == 0 || p.SQ == 0 || p.SK == 0) return FA_OK;
  bool taken = false;
  const int rc = fa::bwd_sm100(p, dtype, (cudaStream_t)stream, &taken);
  if (taken || rc) return rc;
  if (dtype != FA_DTYPE_F32 && fa::require_tc()) {
    set_error("backward: FABLE_ATTN_REQUIRE_TC is set and the tensor-core kernels do not take this request "
              "(head_dim=%d, alignment or strides)", p.D);
    return FA_ERR_UNSUPPORTED;
  }
  return fa::bwd_simt(p, dtype, (cudaStream_t)stream);
}

extern "C" int fa_decode_num_splits(int batch, int nq, int nheads_kv, long long ctx_bound, int num_splits) {
  int n;
  if (num_splits > 0) {
    n = num_splits;
  } else {
    // enough work items to cover every SM ~8 times over, and splits of at most ~1024 positions
    // so that the persistent tensor-core decode can balance them; each split keeps >= 256
    // positions
    const long long groups = (long long)(batch > 0 ? batch : 1) * (nq > 0 ? nq : 1) * (nheads_kv > 0 ? nheads_kv : 1);
    const long long target = 8LL * fa::num_sms();
    n = (int)((target + groups - 1) / groups);
    const long long by_len = (ctx_bound + 1023) / 1024;
    if (by_len > n) n = (int)std::min<long long>(by_len, 512);
    long long maxn = (ctx_bound + 255) / 256;
    if (maxn < 1) maxn = 1;
    if (n > maxn) n = (int)maxn;
  }
  if (n < 1) n = 1;
  if (n > 512) n = 512;
  return n;
}

extern "C" long long fa_decode_scratch_floats(int batch, int nq, int NH, int HD, int nsplit) {
  return (long long)batch * nq * NH * nsplit * (HD + 2);
}

extern "C" int fa_decode_launch(const FaDecParams* pp, int dtype, void* stream, const void* new_k,
                                const void* new_v) {
  FA_ABI_GUARD(pp, FaDecParams);
  FaDecParams p = *pp;
  FA_CHECK_ARG(dtype_ok(dtype), "decode: dtype code %d", dtype);
  FA_CHECK_ARG(p.q && p.Kc && p.Vc && p.block_table && p.o && p.scratch && p.ctx_len,
               "decode: q, Kc, Vc, block_table, o, scratch, ctx_len must be non-null");
  FA_CHECK_ARG(p.batch >= 0 && p.NH > 0 && p.gqa > 0 && p.NH % p.gqa == 0, "decode: NH=%d gqa=%d", p.NH, p.gqa);
  FA_CHECK_ARG(p.page > 0 && (p.page & (p.page - 1)) == 0, "decode: page=%d must be a power of two", p.page);
  FA_CHECK_ARG(p.max_blocks > 0, "decode: max_blocks=%d", p.max_blocks);
  FA_CHECK_ARG(p.nsplit >= 1 && p.nsplit <= 512, "decode: nsplit=%d outside [1,512]", p.nsplit);
  FA_CHECK_ARG((new_k == nullptr) == (new_v == nullptr), "decode: new_k and new_v go together");
  FA_CHECK_ARG(p.rotary >= 0 && p.rotary <= 2, "decode: rotary mode %d", p.rotary);
  if (p.rotary) {
    FA_CHECK_ARG(p.cos && p.sin, "decode: rotary needs cos/sin tables");
    const int rd = p.rotary_dim > 0 ? p.rotary_dim : p.HD;
    FA_CHECK_ARG(rd % 2 == 0 && rd <= p.HD, "decode: rotary_dim=%d", rd);
  }
  if (p.nq < 1) p.nq = 1;
  if (!fa::valid_hd(p.HD)) {
    set_error("decode: head_dim=%d not instantiated", p.HD);
    return FA_ERR_UNSUPPORTED;
  }
  p.append = new_k ? 1 : 0;
  if (p.batch == 0) return FA_OK;
  return fa::dec_run(p, dtype, (cudaStream_t)stream, new_k, new_v);
}

extern "C" int fa_combine_launch(const FaCombineParams* pp, void* stream) {
  FA_ABI_GUARD(pp, FaCombineParams);
  const FaCombineParams& p = *pp;
  FA_CHECK_ARG(dtype_ok(p.in_dtype) && dtype_ok(p.out_dtype), "combine: dtype codes %d/%d", p.in_dtype, p.out_dtype);
  FA_CHECK_ARG(p.out_partial && p.lse_partial && p.out, "combine: out_partial, lse_partial, out must be non-null");
  FA_CHECK_ARG(p.nsplit >= 1 && p.B >= 0 && p.S >= 0 && p.H >= 0 && p.D > 0, "combine: bad sizes");
  if ((long long)p.B * p.S * p.H == 0) return FA_OK;
  FA_CHECK_ARG((long long)p.B * p.S * p.H < (1LL << 31), "combine: too many rows");
  FA_CHECK_ARG(p.out_split_stride >= 0 && p.lse_split_stride >= 0 && (p.lse_bsh == 0 || p.lse_bsh == 1),
               "combine: split strides %lld / %lld must be >= 0 and lse_bsh 0 or 1", p.out_split_stride,
               p.lse_split_stride);
  return fa::combine_run(p, (cudaStream_t)stream);
}
