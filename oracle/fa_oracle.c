/*
 * fa_oracle.c — CPU oracle for the exact-attention path.  TEST INFRASTRUCTURE ONLY: called by
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as the checker; nothing in the
 * product path links or calls it.
 *
 * Plain-C fp64 restatement of the reference's arithmetic (MatafakaRespect/flash-attention-rdna2):
 *   fa_oracle_philox_r0 / fa_oracle_dropout_mul  <- kernels/fa_common.hpp:71-88 (Philox4x32-10,
 *                                                  first output word, keep iff (r0>>8)/2^24 >= p)
 *   fa_oracle_forward                            <- kernels/fa_common.hpp:102-134 (ref_attention)
 *                                                  + dropout as in kernels/backward.hip:570-582
 *   fa_oracle_backward                           <- kernels/backward.hip:583-597
 *   fa_oracle_decode                             <- kernels/fa_decode_gate.inc:66-96 (+ rot_at :20-25)
 *   fa_oracle_combine                            <- package/fable_attn/flash_attn_interface.py:567-580
 * Pinned against the reference's own ref_attention/philox compiled from its sources
 * (oracle/Makefile -> oracle/_ref) and against the committed golden vectors in tests/golden.
 *
 * Layouts (all contiguous, float inputs already rounded to the tested dtype):
 *   Q, O, dO, dQ : [B][SQ][NH][HD]      K, V, dK, dV : [B][SK][NKV][HD]     LSE : [B][NH][SQ]
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

uint32_t fa_oracle_philox_r0(uint64_t seed, uint64_t idx) {
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
  uint32_t c0 = (uint32_t)idx, c1 = (uint32_t)(idx >> 32), c2 = 0, c3 = 0;
  for (int r = 0; r < 10; ++r) {
    const uint64_t m0 = (uint64_t)0xD2511F53u * c0, m1 = (uint64_t)0xCD9E8D57u * c2;
    const uint32_t n0 = (uint32_t)(m1 >> 32) ^ c1 ^ k0;
    const uint32_t n2 = (uint32_t)(m0 >> 32) ^ c3 ^ k1;
    c1 = (uint32_t)m1;
    c3 = (uint32_t)m0;
    c0 = n0;
    c2 = n2;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c0;
}

/* keep multiplier: inv_keep (computed in float as 1/(1-p)) when kept, else 0 */
float fa_oracle_dropout_mul(uint64_t seed, uint64_t idx, float p) {
  const float inv_keep = 1.0f / (1.0f - p);
  const float u = (float)(fa_oracle_philox_r0(seed, idx) >> 8) * (1.0f / 16777216.0f);
  return (u >= p) ? inv_keep : 0.0f;
}

/* keep bits for rows [0,SQ) x keys [0,SK) of query head h: out[q*SK+k] = 1 kept / 0 dropped */
void fa_oracle_dropout_mask(uint64_t seed, int h, int SQ, int SK, float p, uint8_t* out) {
  for (int q = 0; q < SQ; ++q)
    for (int k = 0; k < SK; ++k) {
      const uint64_t idx = ((uint64_t)h * SQ + q) * SK + k;
      out[(size_t)q * SK + k] = fa_oracle_dropout_mul(seed, idx, p) != 0.0f;
    }
}

/* keep bits for the block rows [q0,q1) x keys [k0,k1) of query head h (problem SQ x SK):
 * out[(q-q0)*(k1-k0) + (k-k0)] = 1 kept / 0 dropped */
void fa_oracle_dropout_block(uint64_t seed, int h, int SQ, int SK, float p, int q0, int q1, int k0, int k1,
                             uint8_t* out) {
  const int w = k1 - k0;
  for (int q = q0; q < q1; ++q)
    for (int k = k0; k < k1; ++k) {
      const uint64_t idx = ((uint64_t)h * SQ + q) * SK + k;
      out[(size_t)(q - q0) * w + (k - k0)] = fa_oracle_dropout_mul(seed, idx, p) != 0.0f;
    }
}

static int visible(int q, int k, int SQ, int SK, int causal, int wl, int wr, int chunk) {
  const int diag = q + SK - SQ;
  if (k < 0 || k >= SK) return 0;
  if (causal && k > diag) return 0;
  if (wl >= 0 && k < diag - wl) return 0;
  if (wr >= 0 && k > diag + wr) return 0;
  if (chunk > 0) {
    const int pp = diag < 0 ? 0 : diag;
    const int cs = (pp / chunk) * chunk;
    if (k < cs || k >= cs + chunk) return 0;
  }
  return 1;
}

/* one (b, h, q) row: writes O row (HD doubles) and returns LSE (or -inf for an empty row) */
static double fwd_row(const float* Q, const float* K, const float* V, double* orow, double* prob, int b, int h,
                      int q, int SQ, int SK, int NH, int NKV, int HD, double scale, double softcap, int causal,
                      int wl, int wr, int chunk, const float* alibi, float dropout_p, uint64_t seed) {
  const int kvh = h / (NH / NKV);
  const float* qr = Q + (((size_t)b * SQ + q) * NH + h) * HD;
  double mx = -INFINITY;
  int cnt = 0;
  for (int k = 0; k < SK; ++k) {
    if (!visible(q, k, SQ, SK, causal, wl, wr, chunk)) { prob[k] = -INFINITY; continue; }
    const float* kr = K + (((size_t)b * SK + k) * NKV + kvh) * HD;
    double s = 0;
    for (int d = 0; d < HD; ++d) s += (double)qr[d] * (double)kr[d];
    s *= scale;
    if (softcap > 0) s = softcap * tanh(s / softcap);
    if (alibi) s += (double)alibi[h] * (double)(k - q);
    prob[k] = s;
    if (s > mx) mx = s;
    ++cnt;
  }
  for (int d = 0; d < HD; ++d) orow[d] = 0;
  if (!cnt) return -INFINITY;
  double sum = 0;
  for (int k = 0; k < SK; ++k) {
    if (prob[k] == -INFINITY) { prob[k] = 0; continue; }
    prob[k] = exp(prob[k] - mx);
    sum += prob[k];
  }
  for (int k = 0; k < SK; ++k) {
    if (prob[k] == 0) continue;
    double w = prob[k] / sum;
    if (dropout_p > 0) w *= fa_oracle_dropout_mul(seed, ((uint64_t)h * SQ + q) * SK + k, dropout_p);
    if (w == 0) continue;
    const float* vr = V + (((size_t)b * SK + k) * NKV + kvh) * HD;
    for (int d = 0; d < HD; ++d) orow[d] += w * (double)vr[d];
  }
  return mx + log(sum);
}

/* Forward for rows [row_begin, row_end) of every (b, h); row_end < 0 means SQ. */
void fa_oracle_forward(const float* Q, const float* K, const float* V, float* O, float* LSE, int B, int SQ, int SK,
                       int NH, int NKV, int HD, double scale, double softcap, int causal, int wl, int wr, int chunk,
                       const float* alibi, float dropout_p, uint64_t seed, int row_begin, int row_end) {
  if (row_end < 0 || row_end > SQ) row_end = SQ;
  double* prob = (double*)malloc(sizeof(double) * (SK > 0 ? SK : 1));
  double* orow = (double*)malloc(sizeof(double) * HD);
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < NH; ++h)
      for (int q = row_begin; q < row_end; ++q) {
        const double lse = fwd_row(Q, K, V, orow, prob, b, h, q, SQ, SK, NH, NKV, HD, scale, softcap, causal, wl,
                                   wr, chunk, alibi, dropout_p, seed);
        float* o = O + (((size_t)b * SQ + q) * NH + h) * HD;
        for (int d = 0; d < HD; ++d) o[d] = (float)orow[d];
        if (LSE) LSE[((size_t)b * NH + h) * SQ + q] = (float)lse;
      }
  free(prob);
  free(orow);
}

/* Backward (no attn_chunk, as the reference).  Outputs dQ [B][SQ][NH][HD], dK/dV [B][SK][NKV][HD]. */
void fa_oracle_backward(const float* Q, const float* K, const float* V, const float* dO, float* dQ, float* dK,
                        float* dV, int B, int SQ, int SK, int NH, int NKV, int HD, double scale, double softcap,
                        int causal, int wl, int wr, const float* alibi, float dropout_p, uint64_t seed) {
  const int gqa = NH / NKV;
  const size_t nq = (size_t)B * SQ * NH * HD, nk = (size_t)B * SK * NKV * HD;
  double* gQ = (double*)calloc(nq, sizeof(double));
  double* gK = (double*)calloc(nk, sizeof(double));
  double* gV = (double*)calloc(nk, sizeof(double));
  double* prob = (double*)malloc(sizeof(double) * (SK > 0 ? SK : 1));
  double* orow = (double*)malloc(sizeof(double) * HD);
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < NH; ++h) {
      const int kvh = h / gqa;
      for (int q = 0; q < SQ; ++q) {
        const double lse = fwd_row(Q, K, V, orow, prob, b, h, q, SQ, SK, NH, NKV, HD, scale, softcap, causal, wl, wr,
                                   0, alibi, dropout_p, seed);
        if (lse == -INFINITY) continue;
        const float* qr = Q + (((size_t)b * SQ + q) * NH + h) * HD;
        const float* gr = dO + (((size_t)b * SQ + q) * NH + h) * HD;
        double Di = 0;
        for (int d = 0; d < HD; ++d) Di += orow[d] * (double)gr[d];
        for (int k = 0; k < SK; ++k) {
          if (!visible(q, k, SQ, SK, causal, wl, wr, 0)) continue;
          const float* kr = K + (((size_t)b * SK + k) * NKV + kvh) * HD;
          const float* vr = V + (((size_t)b * SK + k) * NKV + kvh) * HD;
          double s = 0, dp = 0;
          for (int d = 0; d < HD; ++d) {
            s += (double)qr[d] * (double)kr[d];
            dp += (double)gr[d] * (double)vr[d];
          }
          const double g0 = scale * s;
          double logit, deriv = 1;
          if (softcap > 0) {
            const double t = tanh(g0 / softcap);
            logit = softcap * t;
            deriv = 1 - t * t;
          } else {
            logit = g0;
          }
          if (alibi) logit += (double)alibi[h] * (double)(k - q);
          const double p = exp(logit - lse);
          const double z = dropout_p > 0 ? (double)fa_oracle_dropout_mul(seed, ((uint64_t)h * SQ + q) * SK + k, dropout_p) : 1.0;
          const double dS = p * (z * dp - Di) * deriv;
          double* gq = gQ + (((size_t)b * SQ + q) * NH + h) * HD;
          double* gk = gK + (((size_t)b * SK + k) * NKV + kvh) * HD;
          double* gv = gV + (((size_t)b * SK + k) * NKV + kvh) * HD;
          for (int d = 0; d < HD; ++d) {
            gv[d] += z * p * (double)gr[d];
            gk[d] += scale * dS * (double)qr[d];
            gq[d] += scale * dS * (double)kr[d];
          }
        }
      }
    }
  for (size_t i = 0; i < nq; ++i) dQ[i] = (float)gQ[i];
  for (size_t i = 0; i < nk; ++i) { dK[i] = (float)gK[i]; dV[i] = (float)gV[i]; }
  free(gQ); free(gK); free(gV); free(prob); free(orow);
}

/* rotate one row in place: mode 1 NeoX halves, 2 interleaved pairs; table row `pos` */
static void rot_row(double* v, int rdim, int mode, const float* cs, const float* sn, int pos) {
  const int half = rdim / 2;
  const float* c = cs + (size_t)pos * half;
  const float* s = sn + (size_t)pos * half;
  for (int d = 0; d < half; ++d) {
    if (mode == 1) {
      const double x = v[d], y = v[d + half];
      v[d] = x * c[d] - y * s[d];
      v[d + half] = y * c[d] + x * s[d];
    } else {
      const double x = v[2 * d], y = v[2 * d + 1];
      v[2 * d] = x * c[d] - y * s[d];
      v[2 * d + 1] = y * c[d] + x * s[d];
    }
  }
}

/*
 * Decode against a paged cache.  q [B][nq][NH][HD]; Kc/Vc [num_blocks][page][NKV][HD] (the cache
 * BEFORE the call); block_table [B][max_blocks]; ctx_len [B]; new_k/new_v [B][nq][NKV][HD] or NULL.
 * Token tk is at qpos = ctx+tk and sees positions [lo, ctx + (append ? tk+1 : 0)) with
 * lo = max(0, leftpad, qpos-window+1).  Appended keys are rotated by table row
 * (rotary_pos ? rotary_pos[b] : ctx) + j.  O [B][nq][NH][HD], LSE [B][nq][NH].
 */
void fa_oracle_decode(const float* q, const float* Kc, const float* Vc, const int* block_table, const int* ctx_len,
                      const float* new_k, const float* new_v, const float* cs, const float* sn, int rotary,
                      int rotary_dim, const int* rotary_pos, const int* leftpad, const float* alibi, float* O,
                      float* LSE, int B, int nq, int NH, int NKV, int HD, int page, int max_blocks, int window,
                      double scale, double softcap) {
  const int gqa = NH / NKV;
  const int rdim = rotary_dim > 0 ? rotary_dim : HD;
  double* qr = (double*)malloc(sizeof(double) * HD);
  double* kk = (double*)malloc(sizeof(double) * HD);
  for (int b = 0; b < B; ++b) {
    const int ctx = ctx_len[b];
    const int cend_max = ctx + (new_k ? nq : 0);
    double* sc = (double*)malloc(sizeof(double) * (cend_max > 0 ? cend_max : 1));
    for (int tk = 0; tk < nq; ++tk) {
      const int qpos = ctx + tk;
      const int cend = ctx + (new_k ? tk + 1 : 0);
      int lo = 0;
      if (window >= 0 && qpos - window + 1 > lo) lo = qpos - window + 1;
      if (leftpad && leftpad[b] > lo) lo = leftpad[b];
      const int rp_q = (rotary_pos ? rotary_pos[b] : ctx) + tk;
      for (int h = 0; h < NH; ++h) {
        const int kvh = h / gqa;
        const float* qg = q + (((size_t)b * nq + tk) * NH + h) * HD;
        for (int d = 0; d < HD; ++d) qr[d] = qg[d];
        if (rotary) rot_row(qr, rdim, rotary, cs, sn, rp_q);
        double mx = -INFINITY;
        for (int pos = 0; pos < cend; ++pos) {
          sc[pos] = -INFINITY;
          if (pos < lo) continue;
          if (new_k && pos >= ctx) {
            const int j = pos - ctx;
            const float* nk = new_k + (((size_t)b * nq + j) * NKV + kvh) * HD;
            for (int d = 0; d < HD; ++d) kk[d] = nk[d];
            if (rotary) rot_row(kk, rdim, rotary, cs, sn, (rotary_pos ? rotary_pos[b] : ctx) + j);
          } else {
            const int blk = block_table[(size_t)b * max_blocks + pos / page];
            const float* kr = Kc + (((size_t)blk * page + pos % page) * NKV + kvh) * HD;
            for (int d = 0; d < HD; ++d) kk[d] = kr[d];
          }
          double s = 0;
          for (int d = 0; d < HD; ++d) s += qr[d] * kk[d];
          s *= scale;
          if (softcap > 0) s = softcap * tanh(s / softcap);
          if (alibi) s += (double)alibi[h] * (double)(pos - qpos);
          sc[pos] = s;
          if (s > mx) mx = s;
        }
        double sum = 0;
        for (int pos = 0; pos < cend; ++pos) {
          if (sc[pos] == -INFINITY) { sc[pos] = 0; continue; }
          sc[pos] = exp(sc[pos] - mx);
          sum += sc[pos];
        }
        float* o = O + (((size_t)b * nq + tk) * NH + h) * HD;
        for (int d = 0; d < HD; ++d) {
          double acc = 0;
          for (int pos = 0; pos < cend; ++pos) {
            if (sc[pos] == 0) continue;
            float vv;
            if (new_v && pos >= ctx) vv = new_v[(((size_t)b * nq + (pos - ctx)) * NKV + kvh) * HD + d];
            else {
              const int blk = block_table[(size_t)b * max_blocks + pos / page];
              vv = Vc[(((size_t)blk * page + pos % page) * NKV + kvh) * HD + d];
            }
            acc += sc[pos] * vv;
          }
          o[d] = (float)(sum > 0 ? acc / sum : 0.0);
        }
        if (LSE) LSE[((size_t)b * nq + tk) * NH + h] = (float)(sum > 0 ? mx + log(sum) : -INFINITY);
      }
    }
    free(sc);
  }
  free(qr);
  free(kk);
}

/* flash_attn_combine: out_partial [ns][rows][D] (rows = B*S*H in (b,s,h) order), lse [ns][B][H][S] */
void fa_oracle_combine(const float* out_partial, const float* lse, float* out, float* lse_out, int ns, int B, int S,
                       int H, int D) {
  const size_t rows = (size_t)B * S * H;
  for (int b = 0; b < B; ++b)
    for (int s = 0; s < S; ++s)
      for (int h = 0; h < H; ++h) {
        const size_t row = ((size_t)b * S + s) * H + h;
        double m = -INFINITY;
        for (int k = 0; k < ns; ++k) {
          const double l = lse[(((size_t)k * B + b) * H + h) * S + s];
          if (l > m) m = l;
        }
        double w = 0;
        if (m != -INFINITY)
          for (int k = 0; k < ns; ++k) w += exp(lse[(((size_t)k * B + b) * H + h) * S + s] - m);
        for (int d = 0; d < D; ++d) {
          double a = 0;
          if (m != -INFINITY)
            for (int k = 0; k < ns; ++k)
              a += exp(lse[(((size_t)k * B + b) * H + h) * S + s] - m) * out_partial[((size_t)k * rows + row) * D + d];
          out[row * D + d] = (float)(w > 0 ? a / w : 0.0);
        }
        if (lse_out) lse_out[((size_t)b * H + h) * S + s] = (float)(w > 0 ? m + log(w) : -INFINITY);
      }
}
