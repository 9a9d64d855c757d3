// dispatch.cpp — torch extension fable_attn._C: turns tensors into the C-ABI parameter blocks of
// include/fable_attn.h and enqueues the launch on torch's current stream for the tensor's device.
// Same function names and argument order as the reference's extension
// (package/csrc/dispatch.cpp:239-267): fwd, bwd, fwd_varlen, dec; plus bwd_varlen (native varlen
// backward), combine (flash_attn_combine on the GPU) and kernel_launch_count.
// Outputs and workspaces (out, lse, dq/dk/dv, dsum, decode scratch) are allocated here by torch,
// as in the reference; kernels own nothing.  No host synchronisation anywhere.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cmath>
#include "fable_attn.h"

namespace {

int dt_of(const torch::Tensor& t) {
  if (t.scalar_type() == torch::kHalf) return FA_DTYPE_F16;
  if (t.scalar_type() == torch::kBFloat16) return FA_DTYPE_BF16;
  if (t.scalar_type() == torch::kFloat32) return FA_DTYPE_F32;
  TORCH_CHECK_VALUE(false, "fable_attn: dtype ", t.scalar_type(), " not supported; need fp16/bf16/fp32");
  return -1;
}

void* cur_stream(const torch::Tensor& t) {
  return (void*)at::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

void check(int rc, const char* what) {
  if (rc == FA_OK) return;
  const std::string msg = std::string("fable_attn ") + what + ": " + fa_last_error();
  if (rc == FA_ERR_UNSUPPORTED) TORCH_CHECK_NOT_IMPLEMENTED(false, msg);
  if (rc == FA_ERR_INVALID || rc == FA_ERR_SIZE) TORCH_CHECK_VALUE(false, msg);
  TORCH_CHECK(false, msg);
}

FaStrides S4(const torch::Tensor& x) { return FaStrides{x.stride(0), x.stride(1), x.stride(2)}; }
// (total, H, D) varlen tensors: token stride = stride(0), head stride = stride(1)
FaStrides S3(const torch::Tensor& x) { return FaStrides{0, x.stride(1), x.stride(0)}; }

void need_cuda_lastdim(const torch::Tensor& t, const char* name) {
  TORCH_CHECK_VALUE(t.is_cuda(), "fable_attn: ", name, " must be a CUDA tensor");
  TORCH_CHECK_VALUE(t.stride(-1) == 1, "fable_attn: ", name, " must have a contiguous last dimension");
}

const float* opt_f32(const c10::optional<torch::Tensor>& t) {
  if (!t.has_value() || !t->defined()) return nullptr;
  TORCH_CHECK_VALUE(t->scalar_type() == torch::kFloat32 && t->is_contiguous(), "fable_attn: expected contiguous fp32");
  return t->data_ptr<float>();
}
const int* opt_i32(const c10::optional<torch::Tensor>& t) {
  if (!t.has_value() || !t->defined()) return nullptr;
  TORCH_CHECK_VALUE(t->scalar_type() == torch::kInt32 && t->is_contiguous(), "fable_attn: expected contiguous int32");
  return t->data_ptr<int>();
}

// ------------------------------------------------------------------ dropout keep mask
// The keep mask (one bit per score, O(H*SQ*SK/8) bytes) saves the backward from evaluating Philox
// again, but autograd keeps it alive until the backward: above this many bytes per call it is not
// built and every kernel evaluates Philox itself (the reference's O(S) memory).  Default 256 MiB
// (config 3's mask is 64 MiB), FABLE_ATTN_DROPOUT_MASK_MAX_MB overrides it (0 = never build one).
long long max_mask_bytes() {
  const char* v = getenv("FABLE_ATTN_DROPOUT_MASK_MAX_MB");
  if (v && *v) {
    char* end = nullptr;
    const long long mb = strtoll(v, &end, 10);
    if (end != v && mb >= 0) return mb << 20;
  }
  return 256ll << 20;
}

c10::optional<torch::Tensor> make_mask(const torch::Tensor& like, int64_t seed, double dropout_p, int NH, int SQ,
                                       int SK, bool causal, int64_t wl, int64_t wr) {
  const long long words = fa_dropout_mask_words(NH, SQ, SK);
  if (!(dropout_p > 0) || words * 4 > max_mask_bytes() || words == 0) return c10::nullopt;
  auto bits = torch::empty({words}, like.options().dtype(torch::kInt32));
  check(fa_dropout_mask_launch((unsigned long long)seed, (float)dropout_p, NH, SQ, SK, causal ? 1 : 0, (int)wl,
                               (int)wr, (unsigned int*)bits.data_ptr<int>(), cur_stream(like)),
        "dropout mask");
  return bits;
}

torch::Tensor dropout_mask(torch::Tensor like, int64_t seed, double dropout_p, int64_t NH, int64_t SQ, int64_t SK,
                           bool causal, int64_t wl, int64_t wr) {
  const c10::cuda::CUDAGuard guard(like.device());
  auto m = make_mask(like, seed, dropout_p, (int)NH, (int)SQ, (int)SK, causal, wl, wr);
  return m.has_value() ? *m : torch::empty({0}, like.options().dtype(torch::kInt32));
}

// the kernels index the mask as [NH][SQ][ceil(SK/32)] words: a mask of any other size is refused
const unsigned int* mask_ptr(const c10::optional<torch::Tensor>& m, int NH, int SQ, int SK) {
  if (!m.has_value() || !m->defined() || m->numel() == 0) return nullptr;
  TORCH_CHECK_VALUE(m->scalar_type() == torch::kInt32 && m->is_contiguous(), "fable_attn: dropout_bits must be int32");
  TORCH_CHECK_VALUE(m->numel() == fa_dropout_mask_words(NH, SQ, SK),
                    "fable_attn: dropout_bits has ", m->numel(), " words, expected ", fa_dropout_mask_words(NH, SQ, SK),
                    " for nheads=", NH, " seqlen_q=", SQ, " seqlen_k=", SK);
  return (const unsigned int*)m->data_ptr<int>();
}

// ------------------------------------------------------------------ forward (dense)
// In-kernel rotary of q (fa_forward_launch rotates each Q tile as it lands) and a one-pass rotary
// of k into a new tensor (k is read by many CTAs, so it is rotated once).  rows of k: dense
// (B, Hk, SK, D) view -> B*SK rows at positions 0..SK-1 per batch entry; varlen (total, Hk, D) with
// cu_k -> positions restart per sequence.  Returns the rotated k; fills p's rot_* fields.
struct RotaryArgs {
  torch::Tensor cos, sin;
  bool interleaved = false;
  bool on() const { return cos.defined(); }
};
RotaryArgs rotary_args(const c10::optional<torch::Tensor>& cos, const c10::optional<torch::Tensor>& sin,
                       bool interleaved, int D) {
  RotaryArgs r;
  const bool has_c = cos.has_value() && cos->defined(), has_s = sin.has_value() && sin->defined();
  TORCH_CHECK_VALUE(has_c == has_s, "fable_attn: rotary_cos and rotary_sin go together");
  if (!has_c) return r;
  r.cos = cos->to(torch::kFloat32).contiguous();
  r.sin = sin->to(torch::kFloat32).contiguous();
  TORCH_CHECK_VALUE(r.cos.dim() == 2 && r.sin.sizes() == r.cos.sizes() && 2 * r.cos.size(1) <= D,
                    "fable_attn: rotary_cos / rotary_sin must be (seqlen_ro, rotary_dim / 2) with rotary_dim <= head_dim");
  r.interleaved = interleaved;
  return r;
}
torch::Tensor rotate_k_rows(const torch::Tensor& k, const RotaryArgs& r, const int* cu_k, int batch, bool varlen) {
  torch::Tensor src = k;
  // dense rows (b, s) must form one strided dimension: batch stride = SK * row stride
  if (!varlen && k.size(0) > 1 && k.stride(0) != k.size(2) * k.stride(2)) src = k.contiguous();
  auto out = torch::empty_like(src);
  FaRotaryParams rp{};
  rp.struct_size = sizeof(FaRotaryParams);
  rp.x = src.data_ptr(); rp.out = out.data_ptr();
  if (varlen) {
    rp.rows = src.size(0); rp.heads = (int)src.size(1); rp.dim = (int)src.size(2);
    rp.x_row_stride = src.stride(0); rp.x_head_stride = src.stride(1);
    rp.out_row_stride = out.stride(0); rp.out_head_stride = out.stride(1);
    rp.cu_seqlens = cu_k; rp.batch = batch;
  } else {   // (B, Hk, SK, D) view
    rp.rows = src.size(0) * src.size(2); rp.heads = (int)src.size(1); rp.dim = (int)src.size(3);
    rp.x_row_stride = src.stride(2); rp.x_head_stride = src.stride(1);
    rp.out_row_stride = out.stride(2); rp.out_head_stride = out.stride(1);
    rp.seqlen = (int)src.size(2); rp.batch = (int)src.size(0);
  }
  rp.rotary_dim = (int)r.cos.size(1) * 2;
  rp.cos = r.cos.data_ptr<float>(); rp.sin = r.sin.data_ptr<float>(); rp.seqlen_ro = (int)r.cos.size(0);
  rp.interleaved = r.interleaved ? 1 : 0;
  check(fa_rotary_launch(&rp, dt_of(src), cur_stream(src)), "rotary (k)");
  return out;
}
void set_q_rotary(FaFwdParams& p, const RotaryArgs& r) {
  p.rot_cos = r.cos.data_ptr<float>(); p.rot_sin = r.sin.data_ptr<float>();
  p.rot_dim = (int)r.cos.size(1) * 2; p.rot_seqlen_ro = (int)r.cos.size(0);
  p.rot_interleaved = r.interleaved ? 1 : 0;
}

std::vector<torch::Tensor> fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, double scale, bool causal,
                               int64_t win_left, int64_t win_right, double softcap,
                               c10::optional<torch::Tensor> alibi, double dropout_p, int64_t seed,
                               int64_t attn_chunk, c10::optional<torch::Tensor> out_opt,
                               c10::optional<torch::Tensor> dropout_bits, c10::optional<torch::Tensor> rotary_cos,
                               c10::optional<torch::Tensor> rotary_sin, bool rotary_interleaved) {
  need_cuda_lastdim(q, "q"); need_cuda_lastdim(k, "k"); need_cuda_lastdim(v, "v");
  TORCH_CHECK_VALUE(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "fable_attn: fwd expects [B,H,S,D]");
  const c10::cuda::CUDAGuard guard(q.device());
  const RotaryArgs rot = rotary_args(rotary_cos, rotary_sin, rotary_interleaved, (int)q.size(3));
  if (rot.on()) k = rotate_k_rows(k, rot, nullptr, 0, false);
  const int B = q.size(0), Hq = q.size(1), SQ = q.size(2), D = q.size(3), Hk = k.size(1), SK = k.size(2);
  TORCH_CHECK_VALUE(Hq % Hk == 0, "fable_attn: Hq must be a multiple of Hk (GQA)");
  TORCH_CHECK_VALUE(k.scalar_type() == q.scalar_type() && v.scalar_type() == q.scalar_type(), "fable_attn: q/k/v dtypes differ");
  torch::Tensor out = out_opt.has_value() ? *out_opt : torch::empty_like(q);
  if (out_opt.has_value()) {
    TORCH_CHECK_VALUE(out.sizes() == q.sizes() && out.scalar_type() == q.scalar_type() && out.stride(3) == 1,
                      "fable_attn: out must match q's shape/dtype with a contiguous last dim");
  }
  auto lse = torch::empty({B, Hq, SQ}, q.options().dtype(torch::kFloat32));
  FaFwdParams p{};
  p.struct_size = sizeof(FaFwdParams);
  p.Q = q.data_ptr(); p.K = k.data_ptr(); p.V = v.data_ptr(); p.O = out.data_ptr(); p.LSE = lse.data_ptr<float>();
  p.sQ = S4(q); p.sK = S4(k); p.sV = S4(v); p.sO = S4(out);
  p.batch = B; p.SQ = SQ; p.SK = SK; p.HD = D; p.NH = Hq; p.gqa = Hq / Hk;
  p.scale = (float)scale; p.softcap = (float)softcap;
  p.causal = causal ? 1 : 0; p.win_left = (int)win_left; p.win_right = (int)win_right;
  p.attn_chunk = (int)attn_chunk; p.alibi_slopes = opt_f32(alibi);
  p.dropout_p = (float)dropout_p; p.philox_seed = (unsigned long long)seed;
  c10::optional<torch::Tensor> bits = dropout_bits;
  if (dropout_p > 0 && !mask_ptr(bits, Hq, SQ, SK))
    bits = make_mask(q, seed, dropout_p, Hq, SQ, SK, causal, win_left, win_right);
  p.dropout_bits = mask_ptr(bits, Hq, SQ, SK);
  if (rot.on()) set_q_rotary(p, rot);
  check(fa_forward_launch(&p, dt_of(q), cur_stream(q)), "forward");
  return {out, lse};
}

// ------------------------------------------------------------------ forward (varlen)
py::object fwd_varlen(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor cu_q, torch::Tensor cu_k,
                      int64_t max_sq, int64_t max_sk, double scale, bool causal, int64_t win_left,
                      int64_t win_right, double softcap, c10::optional<torch::Tensor> alibi, double dropout_p,
                      int64_t seed, int64_t attn_chunk, c10::optional<torch::Tensor> seqused_q,
                      c10::optional<torch::Tensor> seqused_k, bool return_lse,
                      c10::optional<torch::Tensor> block_table, c10::optional<torch::Tensor> rotary_cos,
                      c10::optional<torch::Tensor> rotary_sin, bool rotary_interleaved) {
  need_cuda_lastdim(q, "q"); need_cuda_lastdim(k, "k"); need_cuda_lastdim(v, "v");
  const bool paged = block_table.has_value() && block_table->defined();
  if (paged) {
    TORCH_CHECK_VALUE(q.dim() == 3 && k.dim() == 4 && v.dim() == 4 && k.is_contiguous() && v.is_contiguous() &&
                          k.sizes() == v.sizes(),
                      "fable_attn: paged varlen expects q (total, H, D) and contiguous k/v (num_blocks, page, Hk, D)");
  } else {
    TORCH_CHECK_VALUE(q.dim() == 3 && k.dim() == 3 && v.dim() == 3, "fable_attn: varlen expects (total, H, D)");
  }
  const c10::cuda::CUDAGuard guard(q.device());
  const RotaryArgs rot = rotary_args(rotary_cos, rotary_sin, rotary_interleaved, (int)q.size(2));
  TORCH_CHECK_VALUE(!(rot.on() && paged), "fable_attn: in-kernel rotary takes packed k/v, not a paged cache");
  if (rot.on()) k = rotate_k_rows(k, rot, opt_i32(cu_k), (int)cu_k.numel() - 1, true);
  const int Hq = q.size(1), D = q.size(2), Hk = paged ? k.size(2) : k.size(1);
  TORCH_CHECK_VALUE(Hq % Hk == 0, "fable_attn: Hq must be a multiple of Hk (GQA)");
  const int batch = (int)cu_q.numel() - 1;
  // rows past seqused_q are not written by the kernel: zero them so nothing uninitialised leaks
  auto out = seqused_q.has_value() ? torch::zeros_like(q) : torch::empty_like(q);
  torch::Tensor lse;
  if (return_lse) lse = torch::full({Hq, q.size(0)}, -INFINITY, q.options().dtype(torch::kFloat32));
  FaFwdParams p{};
  p.struct_size = sizeof(FaFwdParams);
  p.Q = q.data_ptr(); p.K = k.data_ptr(); p.V = v.data_ptr(); p.O = out.data_ptr();
  p.LSE = return_lse ? lse.data_ptr<float>() : nullptr;
  p.sQ = S3(q); p.sK = S3(k); p.sV = S3(v); p.sO = S3(out);
  p.batch = batch; p.SQ = (int)max_sq; p.SK = (int)max_sk; p.HD = D; p.NH = Hq; p.gqa = Hq / Hk;
  p.scale = (float)scale; p.softcap = (float)softcap;
  p.causal = causal ? 1 : 0; p.win_left = (int)win_left; p.win_right = (int)win_right;
  p.attn_chunk = (int)attn_chunk; p.alibi_slopes = opt_f32(alibi);
  p.dropout_p = (float)dropout_p; p.philox_seed = (unsigned long long)seed;
  p.cu_q = opt_i32(cu_q); p.cu_k = opt_i32(cu_k);
  p.seqused_q = opt_i32(seqused_q); p.seqused_k = opt_i32(seqused_k);
  p.lse_total_q = q.size(0);
  p.total_k = paged ? 0 : k.size(0);
  torch::Tensor bt;
  if (paged) {
    bt = block_table->to(torch::kInt32).contiguous();
    TORCH_CHECK_VALUE(bt.dim() == 2 && bt.size(0) == batch, "fable_attn: block_table must be (batch, max_blocks)");
    p.block_table = bt.data_ptr<int>();
    p.page = (int)k.size(1);
    p.max_blocks = (int)bt.size(1);
    p.num_blocks = k.size(0);
  }
  if (rot.on()) set_q_rotary(p, rot);
  check(fa_forward_launch(&p, dt_of(q), cur_stream(q)), "forward (varlen)");
  if (return_lse) return py::make_tuple(out, lse);
  return py::cast(out);
}

// ------------------------------------------------------------------ backward
FaBwdParams bwd_common(torch::Tensor& dout, torch::Tensor& q, torch::Tensor& k, torch::Tensor& v,
                       torch::Tensor& out, torch::Tensor& lse, double scale, bool causal, int64_t win_left,
                       int64_t win_right, double softcap, const c10::optional<torch::Tensor>& alibi,
                       double dropout_p, int64_t seed) {
  FaBwdParams p{};
  p.struct_size = sizeof(FaBwdParams);
  p.Q = q.data_ptr(); p.K = k.data_ptr(); p.V = v.data_ptr(); p.O = out.data_ptr(); p.dO = dout.data_ptr();
  p.lse = lse.data_ptr<float>();
  p.scale = (float)scale; p.softcap = (float)softcap; p.alibi = opt_f32(alibi);
  p.causal = causal ? 1 : 0; p.win_left = (int)win_left; p.win_right = (int)win_right;
  p.dropout = dropout_p > 0 ? 1 : 0; p.drop_seed = (unsigned long long)seed; p.dropout_p = (float)dropout_p;
  p.keep_scale = dropout_p > 0 ? (float)(1.0 / (1.0 - dropout_p)) : 1.f;
  return p;
}

std::vector<torch::Tensor> bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                               torch::Tensor out, torch::Tensor lse, double scale, bool causal, int64_t win_left,
                               int64_t win_right, double softcap, c10::optional<torch::Tensor> alibi,
                               double dropout_p, int64_t seed, c10::optional<torch::Tensor> dropout_bits) {
  for (auto* t : {&dout, &q, &k, &v, &out}) need_cuda_lastdim(*t, "backward input");
  TORCH_CHECK_VALUE(lse.is_contiguous() && lse.scalar_type() == torch::kFloat32, "fable_attn: lse must be contiguous fp32");
  const c10::cuda::CUDAGuard guard(q.device());
  const int B = q.size(0), Hq = q.size(1), SQ = q.size(2), D = q.size(3), Hk = k.size(1), SK = k.size(2);
  auto dq = torch::empty_like(q), dk = torch::empty_like(k), dv = torch::empty_like(v);
  auto dsum = torch::empty({B, Hq, SQ}, q.options().dtype(torch::kFloat32));
  FaBwdParams p = bwd_common(dout, q, k, v, out, lse, scale, causal, win_left, win_right, softcap, alibi, dropout_p, seed);
  p.dQ = dq.data_ptr(); p.dK = dk.data_ptr(); p.dV = dv.data_ptr(); p.dsum = dsum.data_ptr<float>();
  p.qs = S4(q); p.ks = S4(k); p.vs = S4(v); p.os = S4(out); p.dos = S4(dout);
  p.dqs = S4(dq); p.dks = S4(dk); p.dvs = S4(dv);
  p.B = B; p.Hq = Hq; p.Hk = Hk; p.SQ = SQ; p.SK = SK; p.D = D; p.gqa = Hq / Hk;
  c10::optional<torch::Tensor> bits = dropout_bits;
  if (dropout_p > 0 && !mask_ptr(bits, Hq, SQ, SK))
    bits = make_mask(q, seed, dropout_p, Hq, SQ, SK, causal, win_left, win_right);
  p.dropout_bits = mask_ptr(bits, Hq, SQ, SK);
  torch::Tensor bits_t;   // key-major copy of the mask for the dK/dV kernel (filled by the backward)
  if (p.dropout_bits) {
    bits_t = torch::empty({fa_dropout_mask_words(Hq, SK, SQ)}, q.options().dtype(torch::kInt32));
    p.dropout_bits_t = reinterpret_cast<unsigned int*>(bits_t.data_ptr<int32_t>());
  }
  check(fable_attn_backward_launch(&p, dt_of(q), cur_stream(q)), "backward");
  return {dq, dk, dv};
}

std::vector<torch::Tensor> bwd_varlen(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                      torch::Tensor out, torch::Tensor lse, torch::Tensor cu_q, torch::Tensor cu_k,
                                      int64_t max_sq, int64_t max_sk, double scale, bool causal, int64_t win_left,
                                      int64_t win_right, double softcap, c10::optional<torch::Tensor> alibi,
                                      double dropout_p, int64_t seed, c10::optional<torch::Tensor> seqused_q,
                                      c10::optional<torch::Tensor> seqused_k) {
  for (auto* t : {&dout, &q, &k, &v, &out}) need_cuda_lastdim(*t, "backward input");
  TORCH_CHECK_VALUE(lse.is_contiguous() && lse.scalar_type() == torch::kFloat32, "fable_attn: lse must be contiguous fp32");
  const c10::cuda::CUDAGuard guard(q.device());
  const int Hq = q.size(1), D = q.size(2), Hk = k.size(1);
  auto dq = torch::zeros_like(q), dk = torch::zeros_like(k), dv = torch::zeros_like(v);
  auto dsum = torch::empty({Hq, q.size(0)}, q.options().dtype(torch::kFloat32));
  FaBwdParams p = bwd_common(dout, q, k, v, out, lse, scale, causal, win_left, win_right, softcap, alibi, dropout_p, seed);
  p.dQ = dq.data_ptr(); p.dK = dk.data_ptr(); p.dV = dv.data_ptr(); p.dsum = dsum.data_ptr<float>();
  p.qs = S3(q); p.ks = S3(k); p.vs = S3(v); p.os = S3(out); p.dos = S3(dout);
  p.dqs = S3(dq); p.dks = S3(dk); p.dvs = S3(dv);
  p.B = (int)cu_q.numel() - 1; p.Hq = Hq; p.Hk = Hk; p.SQ = (int)max_sq; p.SK = (int)max_sk; p.D = D;
  p.gqa = Hq / Hk;
  p.cu_q = opt_i32(cu_q); p.cu_k = opt_i32(cu_k);
  p.seqused_q = opt_i32(seqused_q); p.seqused_k = opt_i32(seqused_k);
  p.lse_total_q = q.size(0);
  p.total_k = k.size(0);
  check(fable_attn_backward_launch(&p, dt_of(q), cur_stream(q)), "backward (varlen)");
  return {dq, dk, dv};
}

// ------------------------------------------------------------------ decode
std::vector<torch::Tensor> dec(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_table,
                               torch::Tensor cache_seqlens, c10::optional<torch::Tensor> new_k,
                               c10::optional<torch::Tensor> new_v, c10::optional<torch::Tensor> rotary_cos,
                               c10::optional<torch::Tensor> rotary_sin, bool rotary_interleaved, double scale,
                               int64_t window, int64_t num_splits, c10::optional<torch::Tensor> cache_leftpad,
                               bool return_lse, double softcap, c10::optional<torch::Tensor> alibi,
                               int64_t rotary_dim, c10::optional<torch::Tensor> rotary_pos, bool out_fp32,
                               c10::optional<torch::Tensor> out_opt, c10::optional<torch::Tensor> lse_opt) {
  TORCH_CHECK_VALUE(q.is_cuda() && k_cache.is_cuda() && v_cache.is_cuda(), "fable_attn: decode needs CUDA tensors");
  TORCH_CHECK_VALUE(q.dim() == 4 && q.is_contiguous(), "fable_attn: decode q must be contiguous [B,nq,Hq,D]");
  TORCH_CHECK_VALUE(k_cache.dim() == 4 && k_cache.is_contiguous() && v_cache.is_contiguous(),
                    "fable_attn: k_cache/v_cache must be contiguous [num_blocks, page, Hk, D]");
  const c10::cuda::CUDAGuard guard(q.device());
  const int B = q.size(0), NQ = q.size(1), Hq = q.size(2), D = q.size(3);
  const int page = k_cache.size(1), Hk = k_cache.size(2);
  TORCH_CHECK_VALUE(Hq % Hk == 0, "fable_attn: Hq must be a multiple of nheads_k (GQA)");
  TORCH_CHECK_VALUE((page & (page - 1)) == 0, "fable_attn: page size must be a power of two");
  // split count from shapes only (no .item(): no host sync)
  const long long ctx_bound = (long long)block_table.size(1) * page;
  const int nsplit = fa_decode_num_splits(B, NQ, Hk, ctx_bound, (int)num_splits);
  // optional caller-owned destinations (e.g. views of one packed buffer that a single all-gather
  // sends): out [B, NQ, Hq, D] and lse [B, NQ, Hq], contiguous
  const auto odt = out_fp32 ? torch::kFloat32 : q.scalar_type();
  torch::Tensor out;
  if (out_opt.has_value() && out_opt->defined()) {
    out = *out_opt;
    TORCH_CHECK_VALUE(out.is_contiguous() && out.scalar_type() == odt && out.sizes() == q.sizes() &&
                          out.device() == q.device(),
                      "fable_attn: decode out must be a contiguous [B, nq, H, D] tensor of the output dtype");
  } else {
    out = torch::empty({B, NQ, Hq, D}, q.options().dtype(odt));
  }
  auto scratch = torch::empty({fa_decode_scratch_floats(B, NQ, Hq, D, nsplit)}, q.options().dtype(torch::kFloat32));
  torch::Tensor lse;
  if (lse_opt.has_value() && lse_opt->defined()) {
    lse = *lse_opt;
    TORCH_CHECK_VALUE(return_lse && lse.is_contiguous() && lse.scalar_type() == torch::kFloat32 &&
                          lse.numel() == (int64_t)B * NQ * Hq && lse.device() == q.device(),
                      "fable_attn: decode lse must be a contiguous fp32 [B, nq, H] tensor (with return_lse)");
  } else {
    lse = return_lse ? torch::empty({B, NQ, Hq}, q.options().dtype(torch::kFloat32))
                     : torch::empty({0}, q.options().dtype(torch::kFloat32));
  }
  FaDecParams p{};
  p.struct_size = sizeof(FaDecParams);
  p.q = q.data_ptr(); p.Kc = k_cache.data_ptr(); p.Vc = v_cache.data_ptr();
  p.block_table = opt_i32(block_table); p.o = out.data_ptr(); p.scratch = scratch.data_ptr<float>();
  p.ctx_len = opt_i32(cache_seqlens);
  p.cos = opt_f32(rotary_cos); p.sin = opt_f32(rotary_sin);
  p.batch = B; p.NH = Hq; p.gqa = Hq / Hk; p.HD = D; p.page = page; p.max_blocks = (int)block_table.size(1);
  p.nsplit = nsplit; p.window = (int)window;
  p.rotary = rotary_cos.has_value() ? (rotary_interleaved ? 2 : 1) : 0;
  p.scale = (float)scale; p.leftpad = opt_i32(cache_leftpad);
  p.lse_out = return_lse ? lse.data_ptr<float>() : nullptr;
  p.softcap = (float)softcap; p.alibi = opt_f32(alibi); p.nq = NQ;
  p.rotary_dim = (int)rotary_dim; p.rotary_pos = opt_i32(rotary_pos);
  p.num_blocks = k_cache.size(0);
  p.o_f32 = out_fp32 ? 1 : 0;
  const void* nk = nullptr; const void* nv = nullptr;
  if (new_k.has_value()) {
    TORCH_CHECK_VALUE(new_v.has_value() && new_k->is_contiguous() && new_v->is_contiguous(),
                      "fable_attn: new k/v must be contiguous and given together");
    nk = new_k->data_ptr(); nv = new_v->data_ptr();
  }
  check(fa_decode_launch(&p, dt_of(q), cur_stream(q), nk, nv), "decode");
  return {out, lse};
}

// ------------------------------------------------------------------ combine
std::vector<torch::Tensor> combine(torch::Tensor out_partial, torch::Tensor lse_partial, c10::ScalarType out_dtype,
                                   bool return_lse) {
  TORCH_CHECK_VALUE(out_partial.is_cuda() && out_partial.dim() == 5 && out_partial.is_contiguous(),
                    "fable_attn: out_partial must be contiguous CUDA (nsplit, B, S, H, D)");
  TORCH_CHECK_VALUE(lse_partial.dim() == 4 && lse_partial.is_contiguous() && lse_partial.scalar_type() == torch::kFloat32,
                    "fable_attn: lse_partial must be contiguous fp32 (nsplit, B, H, S)");
  const c10::cuda::CUDAGuard guard(out_partial.device());
  const int ns = out_partial.size(0), B = out_partial.size(1), S = out_partial.size(2), H = out_partial.size(3),
            D = out_partial.size(4);
  auto out = torch::empty({B, S, H, D}, out_partial.options().dtype(out_dtype));
  auto lse = return_lse ? torch::empty({B, H, S}, lse_partial.options()) : torch::empty({0}, lse_partial.options());
  FaCombineParams p{};
  p.struct_size = sizeof(FaCombineParams);
  p.out_partial = out_partial.data_ptr(); p.in_dtype = dt_of(out_partial);
  p.lse_partial = lse_partial.data_ptr<float>(); p.out = out.data_ptr(); p.out_dtype = dt_of(out);
  p.lse_out = return_lse ? lse.data_ptr<float>() : nullptr;
  p.nsplit = ns; p.B = B; p.S = S; p.H = H; p.D = D;
  check(fa_combine_launch(&p, cur_stream(out_partial)), "combine");
  return {out, lse};
}

// LSE-merge of `nsplit` packed partials: buf holds, per split, rows = B*S*H output rows of D fp32
// values followed by the rows' fp32 LSE in the same (b, s, h) order (one rank's decode partial, as
// multigpu.decode_kv_split sends it); the merge reads that layout in place.  Returns out (B, S, H, D).
torch::Tensor combine_packed(torch::Tensor buf, int64_t nsplit, int64_t B, int64_t S, int64_t H, int64_t D,
                             c10::ScalarType out_dtype) {
  TORCH_CHECK_VALUE(buf.is_cuda() && buf.is_contiguous() && buf.scalar_type() == torch::kFloat32,
                    "fable_attn: packed partials must be a contiguous fp32 CUDA tensor");
  const int64_t rows = B * S * H, per = rows * (D + 1);
  TORCH_CHECK_VALUE(nsplit >= 1 && buf.numel() == nsplit * per, "fable_attn: packed partials hold ", buf.numel(),
                    " floats, expected nsplit * B*S*H*(D+1) = ", nsplit * per);
  const c10::cuda::CUDAGuard guard(buf.device());
  auto out = torch::empty({B, S, H, D}, buf.options().dtype(out_dtype));
  FaCombineParams p{};
  p.struct_size = sizeof(FaCombineParams);
  p.out_partial = buf.data_ptr(); p.in_dtype = FA_DTYPE_F32;
  p.lse_partial = buf.data_ptr<float>() + rows * D; p.out = out.data_ptr(); p.out_dtype = dt_of(out);
  p.nsplit = (int)nsplit; p.B = (int)B; p.S = (int)S; p.H = (int)H; p.D = (int)D;
  p.out_split_stride = per; p.lse_split_stride = per; p.lse_bsh = 1;
  check(fa_combine_launch(&p, cur_stream(buf)), "combine (packed)");
  return out;
}

// Multi-GPU decode exchange over peer memory (fa_peer_merge_launch / fa_peer_step_end_launch):
// peer_bufs / peer_signals are int64 CUDA tensors [world] holding the ranks' device addresses of
// their packed partials and signal words; step / err are int32 CUDA tensors [1] of this rank.
FaPeerMergeParams peer_params(torch::Tensor peer_bufs, torch::Tensor peer_signals, int64_t rank, int64_t world,
                              int64_t B, int64_t S, int64_t H, int64_t D, torch::Tensor step, torch::Tensor err,
                              int64_t slot_floats = 0, c10::optional<torch::Tensor> done_ctas = c10::nullopt) {
  TORCH_CHECK_VALUE(peer_bufs.is_cuda() && peer_signals.is_cuda() && peer_bufs.scalar_type() == torch::kInt64 &&
                        peer_signals.scalar_type() == torch::kInt64 && peer_bufs.numel() == world &&
                        peer_signals.numel() == world,
                    "fable_attn: peer_bufs / peer_signals must be int64 CUDA tensors of `world` addresses");
  TORCH_CHECK_VALUE(step.is_cuda() && step.scalar_type() == torch::kInt32 && err.is_cuda() &&
                        err.scalar_type() == torch::kInt32,
                    "fable_attn: step and err must be int32 CUDA tensors");
  FaPeerMergeParams p{};
  p.struct_size = sizeof(FaPeerMergeParams);
  p.peer_bufs = reinterpret_cast<const float* const*>(peer_bufs.data_ptr<int64_t>());
  p.peer_signals = reinterpret_cast<unsigned int* const*>(peer_signals.data_ptr<int64_t>());
  p.rank = (int)rank; p.world = (int)world;
  p.B = (int)B; p.S = (int)S; p.H = (int)H; p.D = (int)D;
  p.step = step.data_ptr<int>(); p.err_flag = err.data_ptr<int>();
  p.slot_floats = slot_floats;
  if (done_ctas.has_value() && done_ctas->defined()) {
    TORCH_CHECK_VALUE(done_ctas->is_cuda() && done_ctas->scalar_type() == torch::kInt32,
                      "fable_attn: done_ctas must be an int32 CUDA tensor");
    p.done_ctas = done_ctas->data_ptr<int>();
  }
  return p;
}

torch::Tensor peer_merge(torch::Tensor peer_bufs, torch::Tensor peer_signals, int64_t rank, int64_t world, int64_t B,
                         int64_t S, int64_t H, int64_t D, torch::Tensor step, torch::Tensor err,
                         c10::ScalarType out_dtype, c10::optional<torch::Tensor> lse_out, int64_t slot_floats,
                         c10::optional<torch::Tensor> done_ctas) {
  const c10::cuda::CUDAGuard guard(step.device());
  FaPeerMergeParams p = peer_params(peer_bufs, peer_signals, rank, world, B, S, H, D, step, err, slot_floats,
                                    done_ctas);
  auto out = torch::empty({B, S, H, D}, step.options().dtype(out_dtype));
  p.out = out.data_ptr(); p.out_dtype = dt_of(out);
  p.lse_out = const_cast<float*>(opt_f32(lse_out));
  check(fa_peer_merge_launch(&p, cur_stream(step)), "peer merge");
  return out;
}

void peer_step_end(torch::Tensor peer_bufs, torch::Tensor peer_signals, int64_t rank, int64_t world, int64_t B,
                   int64_t S, int64_t H, int64_t D, torch::Tensor step, torch::Tensor err) {
  const c10::cuda::CUDAGuard guard(step.device());
  FaPeerMergeParams p = peer_params(peer_bufs, peer_signals, rank, world, B, S, H, D, step, err);
  check(fa_peer_step_end_launch(&p, cur_stream(step)), "peer step end");
}

}  // namespace

// ------------------------------------------------------------------ rotary (q / k, one pass)
// x (batch, seqlen, heads, dim) or, with cu_seqlens, (total, heads, dim); dim contiguous.
// offsets: int or per-sequence int32 tensor.  Returns the rotated tensor (x itself if inplace).
torch::Tensor rotary(torch::Tensor x, torch::Tensor cos, torch::Tensor sin, bool interleaved, bool inplace,
                     py::object offsets, c10::optional<torch::Tensor> cu_seqlens) {
  TORCH_CHECK_VALUE(x.is_cuda(), "fable_attn: rotary expects a CUDA tensor");
  TORCH_CHECK_VALUE(x.stride(-1) == 1, "fable_attn: rotary needs a contiguous last dim");
  const c10::cuda::CUDAGuard guard(x.device());
  const bool varlen = cu_seqlens.has_value() && cu_seqlens->defined();
  TORCH_CHECK_VALUE(x.dim() == (varlen ? 3 : 4), "fable_attn: rotary expects ", varlen ? "(total, heads, dim)" :
                    "(batch, seqlen, heads, dim)");
  // rows must be one strided dimension: (batch, seqlen) merge when batch stride = seqlen * row stride
  torch::Tensor src = x;
  if (!varlen && x.size(0) > 1 && x.stride(0) != x.size(1) * x.stride(1)) src = x.contiguous();
  auto c = cos.to(torch::kFloat32).contiguous(), s = sin.to(torch::kFloat32).contiguous();
  TORCH_CHECK_VALUE(c.dim() == 2 && s.sizes() == c.sizes(), "fable_attn: cos/sin must be (seqlen_ro, rotary_dim/2)");
  torch::Tensor out = (inplace && src.is_same(x)) ? x : torch::empty_like(src);
  FaRotaryParams p{};
  p.struct_size = sizeof(FaRotaryParams);
  p.x = src.data_ptr(); p.out = out.data_ptr();
  const int hd = varlen ? 1 : 2;
  p.rows = varlen ? src.size(0) : src.size(0) * src.size(1);
  p.heads = (int)src.size(hd); p.dim = (int)src.size(hd + 1); p.rotary_dim = (int)c.size(1) * 2;
  p.x_row_stride = src.stride(hd - 1); p.x_head_stride = src.stride(hd);
  p.out_row_stride = out.stride(hd - 1); p.out_head_stride = out.stride(hd);
  torch::Tensor cu, offs;
  if (varlen) {
    cu = cu_seqlens->to(torch::kInt32).contiguous();
    p.cu_seqlens = cu.data_ptr<int>();
    p.batch = (int)cu.numel() - 1;
  } else {
    p.seqlen = (int)src.size(1);
    p.batch = (int)src.size(0);
  }
  if (py::isinstance<py::int_>(offsets)) {
    p.offset = offsets.cast<int>();
  } else {
    offs = offsets.cast<torch::Tensor>().to(x.device(), torch::kInt32).contiguous();
    TORCH_CHECK_VALUE(offs.numel() == p.batch, "fable_attn: seqlen_offsets needs one entry per sequence");
    p.offsets = offs.data_ptr<int>();
  }
  p.cos = c.data_ptr<float>(); p.sin = s.data_ptr<float>(); p.seqlen_ro = (int)c.size(0);
  p.interleaved = interleaved ? 1 : 0;
  check(fa_rotary_launch(&p, dt_of(src), cur_stream(src)), "rotary");
  if (inplace && !out.is_same(x)) {
    x.copy_(out);
    return x;
  }
  return out;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "fable_attn sm_100a attention kernels (binds the C ABI of include/fable_attn.h)";
  m.def("fwd", &fwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("scale"), py::arg("causal"),
        py::arg("win_left"), py::arg("win_right"), py::arg("softcap"), py::arg("alibi"), py::arg("dropout_p"),
        py::arg("seed"), py::arg("attn_chunk") = 0, py::arg("out") = c10::optional<torch::Tensor>(),
        py::arg("dropout_bits") = c10::optional<torch::Tensor>(), py::arg("rotary_cos") = c10::optional<torch::Tensor>(),
        py::arg("rotary_sin") = c10::optional<torch::Tensor>(), py::arg("rotary_interleaved") = false);
  m.def("bwd", &bwd, py::arg("dout"), py::arg("q"), py::arg("k"), py::arg("v"), py::arg("out"), py::arg("lse"),
        py::arg("scale"), py::arg("causal"), py::arg("win_left"), py::arg("win_right"), py::arg("softcap"),
        py::arg("alibi"), py::arg("dropout_p"), py::arg("seed"), py::arg("dropout_bits") = c10::optional<torch::Tensor>());
  m.def("rotary", &rotary, py::arg("x"), py::arg("cos"), py::arg("sin"), py::arg("interleaved"), py::arg("inplace"),
        py::arg("offsets"), py::arg("cu_seqlens") = c10::optional<torch::Tensor>());
  m.def("dropout_mask", &dropout_mask, py::arg("like"), py::arg("seed"), py::arg("dropout_p"), py::arg("nheads"),
        py::arg("seqlen_q"), py::arg("seqlen_k"), py::arg("causal"), py::arg("win_left"), py::arg("win_right"));
  m.def("fwd_varlen", &fwd_varlen, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("cu_q"), py::arg("cu_k"),
        py::arg("max_sq"), py::arg("max_sk"), py::arg("scale"), py::arg("causal"), py::arg("win_left"),
        py::arg("win_right"), py::arg("softcap"), py::arg("alibi"), py::arg("dropout_p"), py::arg("seed"),
        py::arg("attn_chunk") = 0, py::arg("seqused_q") = c10::optional<torch::Tensor>(),
        py::arg("seqused_k") = c10::optional<torch::Tensor>(), py::arg("return_lse") = false,
        py::arg("block_table") = c10::optional<torch::Tensor>(), py::arg("rotary_cos") = c10::optional<torch::Tensor>(),
        py::arg("rotary_sin") = c10::optional<torch::Tensor>(), py::arg("rotary_interleaved") = false);
  m.def("bwd_varlen", &bwd_varlen, py::arg("dout"), py::arg("q"), py::arg("k"), py::arg("v"), py::arg("out"),
        py::arg("lse"), py::arg("cu_q"), py::arg("cu_k"), py::arg("max_sq"), py::arg("max_sk"), py::arg("scale"),
        py::arg("causal"), py::arg("win_left"), py::arg("win_right"), py::arg("softcap"), py::arg("alibi"),
        py::arg("dropout_p"), py::arg("seed"), py::arg("seqused_q") = c10::optional<torch::Tensor>(),
        py::arg("seqused_k") = c10::optional<torch::Tensor>());
  m.def("dec", &dec, py::arg("q"), py::arg("k_cache"), py::arg("v_cache"), py::arg("block_table"),
        py::arg("cache_seqlens"), py::arg("new_k"), py::arg("new_v"), py::arg("rotary_cos"), py::arg("rotary_sin"),
        py::arg("rotary_interleaved"), py::arg("scale"), py::arg("window"), py::arg("num_splits"),
        py::arg("cache_leftpad") = c10::optional<torch::Tensor>(), py::arg("return_lse") = false,
        py::arg("softcap") = 0.0, py::arg("alibi") = c10::optional<torch::Tensor>(), py::arg("rotary_dim") = 0,
        py::arg("rotary_pos") = c10::optional<torch::Tensor>(), py::arg("out_fp32") = false,
        py::arg("out") = c10::optional<torch::Tensor>(), py::arg("lse_out") = c10::optional<torch::Tensor>());
  m.def("combine", &combine, py::arg("out_partial"), py::arg("lse_partial"), py::arg("out_dtype"),
        py::arg("return_lse") = false);
  m.def("combine_packed", &combine_packed, py::arg("buf"), py::arg("nsplit"), py::arg("B"), py::arg("S"),
        py::arg("H"), py::arg("D"), py::arg("out_dtype"));
  m.def("peer_merge", &peer_merge, py::arg("peer_bufs"), py::arg("peer_signals"), py::arg("rank"), py::arg("world"),
        py::arg("B"), py::arg("S"), py::arg("H"), py::arg("D"), py::arg("step"), py::arg("err"),
        py::arg("out_dtype"), py::arg("lse_out") = c10::optional<torch::Tensor>(), py::arg("slot_floats") = 0,
        py::arg("done_ctas") = c10::optional<torch::Tensor>());
  m.def("peer_step_end", &peer_step_end, py::arg("peer_bufs"), py::arg("peer_signals"), py::arg("rank"),
        py::arg("world"), py::arg("B"), py::arg("S"), py::arg("H"), py::arg("D"), py::arg("step"), py::arg("err"));
  m.def("kernel_launch_count", []() { return fa_kernel_launch_count(); });
  m.def("device_error", [](bool clear) { return fa_device_error(clear ? 1 : 0); }, py::arg("clear") = false);
  m.def("wait_selftest", [](int64_t limit_ns) {
    check(fa_wait_selftest((unsigned long long)limit_ns, (void*)at::cuda::getCurrentCUDAStream().stream()),
          "wait self-test");
  }, py::arg("limit_ns"));
  m.def("abi_version", []() { return fa_abi_version(); });
}
