"""ctypes bindings of the CPU oracle — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs use this module,
as the checker or the timed CPU baseline; the product path never imports it.

  lib()      -> oracle/_build/libfa_oracle.so  (fa_oracle.c, plain-C fp64 restatement)
  ref_lib()  -> oracle/_ref/libfa_ref.so       (the reference's own fp64 oracle compiled from its
                sources by oracle/Makefile), or None when it was not built
Both are built by `make -C oracle REF_DIR=<reference checkout>` (and by __graft_entry__.build()).
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None

f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True, capture_output=True)


def _opt(arr):
    return None if arr is None else arr.ctypes.data_as(C.c_void_p)


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "_build", "libfa_oracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        L.fa_oracle_philox_r0.restype = C.c_uint32
        L.fa_oracle_philox_r0.argtypes = [C.c_uint64, C.c_uint64]
        L.fa_oracle_dropout_mul.restype = C.c_float
        L.fa_oracle_dropout_mul.argtypes = [C.c_uint64, C.c_uint64, C.c_float]
        L.fa_oracle_dropout_mask.argtypes = [C.c_uint64, C.c_int, C.c_int, C.c_int, C.c_float, u8p]
        L.fa_oracle_forward.argtypes = [f32p, f32p, f32p, f32p, C.c_void_p] + [C.c_int] * 6 + [
            C.c_double, C.c_double] + [C.c_int] * 4 + [C.c_void_p, C.c_float, C.c_uint64, C.c_int, C.c_int]
        L.fa_oracle_backward.argtypes = [f32p] * 7 + [C.c_int] * 6 + [C.c_double, C.c_double] + [C.c_int] * 3 + [
            C.c_void_p, C.c_float, C.c_uint64]
        L.fa_oracle_decode.argtypes = [f32p, f32p, f32p, i32p, i32p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                       C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, f32p, f32p] + [
            C.c_int] * 8 + [C.c_double, C.c_double]
        L.fa_oracle_combine.argtypes = [f32p, f32p, f32p, f32p] + [C.c_int] * 5
        L.fa_oracle_dropout_block.argtypes = [C.c_uint64, C.c_int, C.c_int, C.c_int, C.c_float] + [C.c_int] * 4 + [u8p]
        _LIB = L
    return _LIB


def ref_lib():
    """The reference's own oracle, or None if oracle/_ref was not built."""
    global _REF
    if _REF is None:
        path = os.path.join(HERE, "_ref", "libfa_ref.so")
        if not os.path.exists(path):
            return None
        L = C.CDLL(path)
        L.ref_attention_c.argtypes = [f32p, f32p, f32p, f32p, f32p] + [C.c_int] * 5 + [C.c_float, C.c_float] + [
            C.c_int] * 4 + [C.c_void_p, C.c_int]
        L.ref_philox_c.argtypes = [C.c_uint64, C.c_uint64, np.ctypeslib.ndpointer(dtype=np.uint32)]
        L.ref_dropout_mul_c.restype = C.c_float
        L.ref_dropout_mul_c.argtypes = [C.c_uint64, C.c_uint64, C.c_float]
        _REF = L
    return _REF


# ------------------------------------------------------------------ numpy-level helpers
def dropout_block(seed, h, SQ, SK, p, q0, q1, k0, k1):
    """Keep bits (1 kept) of rows [q0,q1) x keys [k0,k1) of query head h, as uint8 (q1-q0, k1-k0)."""
    out = np.empty((max(q1 - q0, 0), max(k1 - k0, 0)), dtype=np.uint8)
    if out.size:
        lib().fa_oracle_dropout_block(seed, h, SQ, SK, p, q0, q1, k0, k1, out)
    return out


def philox_r0(seed, idx):
    return int(lib().fa_oracle_philox_r0(seed, idx))


def dropout_mask(seed, h, SQ, SK, p):
    out = np.empty((SQ, SK), dtype=np.uint8)
    lib().fa_oracle_dropout_mask(seed, h, SQ, SK, p, out)
    return out


def forward(q, k, v, scale, causal=False, wl=-1, wr=-1, softcap=0.0, alibi=None, chunk=0, dropout_p=0.0, seed=0,
            rows=None):
    """q (B,SQ,NH,D), k/v (B,SK,NKV,D) float32 -> (O (B,SQ,NH,D), LSE (B,NH,SQ)); optional row range."""
    q, k, v = (np.ascontiguousarray(x, dtype=np.float32) for x in (q, k, v))
    B, SQ, NH, D = q.shape
    SK, NKV = k.shape[1], k.shape[2]
    O = np.zeros_like(q)
    L = np.full((B, NH, SQ), -np.inf, dtype=np.float32)
    al = None if alibi is None else np.ascontiguousarray(alibi, dtype=np.float32)
    r0, r1 = rows if rows is not None else (0, -1)
    lib().fa_oracle_forward(q, k, v, O, L.ctypes.data_as(C.c_void_p), B, SQ, SK, NH, NKV, D, scale, softcap,
                            int(causal), wl, wr, chunk, _opt(al), dropout_p, seed, r0, r1)
    return O, L


def backward(q, k, v, do, scale, causal=False, wl=-1, wr=-1, softcap=0.0, alibi=None, dropout_p=0.0, seed=0):
    q, k, v, do = (np.ascontiguousarray(x, dtype=np.float32) for x in (q, k, v, do))
    B, SQ, NH, D = q.shape
    SK, NKV = k.shape[1], k.shape[2]
    dq, dk, dv = np.zeros_like(q), np.zeros_like(k), np.zeros_like(v)
    al = None if alibi is None else np.ascontiguousarray(alibi, dtype=np.float32)
    lib().fa_oracle_backward(q, k, v, do, dq, dk, dv, B, SQ, SK, NH, NKV, D, scale, softcap, int(causal), wl, wr,
                             _opt(al), dropout_p, seed)
    return dq, dk, dv


def decode(q, k_cache, v_cache, block_table, ctx_len, new_k=None, new_v=None, cos=None, sin=None, rotary=0,
           rotary_dim=0, rotary_pos=None, leftpad=None, alibi=None, window=-1, scale=None, softcap=0.0):
    """q (B,nq,NH,D); caches (num_blocks,page,NKV,D) BEFORE the call -> (O (B,nq,NH,D), LSE (B,nq,NH))."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    kc = np.ascontiguousarray(k_cache, dtype=np.float32)
    vc = np.ascontiguousarray(v_cache, dtype=np.float32)
    bt = np.ascontiguousarray(block_table, dtype=np.int32)
    cl = np.ascontiguousarray(ctx_len, dtype=np.int32)
    B, nq, NH, D = q.shape
    page, NKV = kc.shape[1], kc.shape[2]
    if scale is None:
        scale = D ** -0.5
    keep = []

    def arr(x, dt):
        if x is None:
            return None
        a = np.ascontiguousarray(x, dtype=dt)
        keep.append(a)
        return a.ctypes.data_as(C.c_void_p)

    O = np.zeros_like(q)
    L = np.zeros((B, nq, NH), dtype=np.float32)
    lib().fa_oracle_decode(q, kc, vc, bt, cl, arr(new_k, np.float32), arr(new_v, np.float32), arr(cos, np.float32),
                           arr(sin, np.float32), rotary, rotary_dim, arr(rotary_pos, np.int32),
                           arr(leftpad, np.int32), arr(alibi, np.float32), O, L, B, nq, NH, NKV, D, page,
                           bt.shape[1], window, scale, softcap)
    return O, L


def combine(out_partial, lse_partial):
    """out_partial (ns,B,S,H,D), lse (ns,B,H,S) -> (out (B,S,H,D), lse (B,H,S))."""
    op = np.ascontiguousarray(out_partial, dtype=np.float32)
    lp = np.ascontiguousarray(lse_partial, dtype=np.float32)
    ns, B, S, H, D = op.shape
    out = np.zeros((B, S, H, D), dtype=np.float32)
    lo = np.zeros((B, H, S), dtype=np.float32)
    lib().fa_oracle_combine(op, lp, out, lo, ns, B, S, H, D)
    return out, lo


def _key_bounds(rows, SQ, SK, causal, wl, wr, chunk):
    """Visible key range [lo, hi] of each query row (bottom-right aligned masks), int64 arrays."""
    diag = rows + (SK - SQ)
    lo = np.zeros_like(rows)
    hi = np.full_like(rows, SK - 1)
    if causal:
        hi = np.minimum(hi, diag)
    if wl >= 0:
        lo = np.maximum(lo, diag - wl)
    if wr >= 0:
        hi = np.minimum(hi, diag + wr)
    if chunk > 0:
        cs = (np.maximum(diag, 0) // chunk) * chunk
        lo = np.maximum(lo, cs)
        hi = np.minimum(hi, cs + chunk - 1)
    return lo, hi


def attention_head(q, k, v, scale, causal=False, wl=-1, wr=-1, softcap=0.0, slope=None, chunk=0, dropout_p=0.0,
                   seed=0, h=0, do=None, rows=None, block=512):
    """One (sequence, query head) in float64, vectorised over row blocks: the arithmetic of
    fa_oracle.c (fwd_row / fa_oracle_backward, i.e. kernels/fa_common.hpp:102-134 and
    kernels/backward.hip:570-597) for problems too large for the scalar loops.
      q (SQ, D), k / v (SK, D) float32 holding the tested dtype's values; h = the global query
      head (the Philox counter is (h*SQ + q)*SK + key); slope = alibi slope of h or None.
    Returns dict(O (SQ, D), LSE (SQ,)) and, with do (SQ, D), dQ / dK / dV (dK / dV of this query
    head only: sum them over the heads of a kv group).  rows=(r0, r1) restricts the forward to a
    row range (no backward then).  Only keys a row block can see are touched, so banded masks
    (sliding windows) cost O(rows x window)."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    SQ, D = q.shape
    SK = k.shape[0]
    r_begin, r_end = rows if rows is not None else (0, SQ)
    if do is not None and rows is not None:
        raise ValueError("attention_head: the backward needs every row")
    O = np.zeros((SQ, D))
    LSE = np.full(SQ, -np.inf)
    res = {"O": O, "LSE": LSE}
    if do is not None:
        do = np.asarray(do, np.float64)
        dQ, dK, dV = np.zeros((SQ, D)), np.zeros((SK, D)), np.zeros((SK, D))
        res.update(dQ=dQ, dK=dK, dV=dV)
    for r0 in range(r_begin, r_end, block):
        r1 = min(r0 + block, r_end)
        rr = np.arange(r0, r1, dtype=np.int64)
        lo, hi = _key_bounds(rr, SQ, SK, causal, wl, wr, chunk)
        lo, hi = np.maximum(lo, 0), np.minimum(hi, SK - 1)
        if not (lo <= hi).any():
            continue
        k0 = int(lo[lo <= hi].min())
        k1 = int(hi[lo <= hi].max()) + 1
        kk = np.arange(k0, k1, dtype=np.int64)
        vis = (kk[None, :] >= lo[:, None]) & (kk[None, :] <= hi[:, None])
        g0 = scale * (q[r0:r1] @ k[k0:k1].T)
        if softcap > 0:
            t = np.tanh(g0 / softcap)
            logit, deriv = softcap * t, 1.0 - t * t
        else:
            logit, deriv = g0, None
        if slope is not None:
            logit = logit + float(slope) * (kk[None, :] - rr[:, None]).astype(np.float64)
        logit = np.where(vis, logit, -np.inf)
        mx = logit.max(axis=1, keepdims=True)
        live = np.isfinite(mx[:, 0])
        e = np.where(vis, np.exp(logit - np.where(live[:, None], mx, 0.0)), 0.0)
        ssum = e.sum(axis=1)
        lse = np.where(live, mx[:, 0] + np.log(np.where(live, ssum, 1.0)), -np.inf)
        LSE[r0:r1] = lse
        p = np.where(live[:, None], e / np.where(live, ssum, 1.0)[:, None], 0.0)
        if dropout_p > 0:
            z = dropout_block(seed, h, SQ, SK, dropout_p, r0, r1, k0, k1).astype(np.float64)
            z *= np.float64(np.float32(1.0) / (np.float32(1.0) - np.float32(dropout_p)))
        else:
            z = None
        pz = p * z if z is not None else p
        O[r0:r1] = pz @ v[k0:k1]
        if do is None:
            continue
        dob = do[r0:r1]
        Di = (O[r0:r1] * dob).sum(axis=1, keepdims=True)
        dp = dob @ v[k0:k1].T
        zdp = dp * z if z is not None else dp
        ds = p * (zdp - Di)
        if deriv is not None:
            ds = ds * deriv
        ds = np.where(vis, ds, 0.0)
        dV[k0:k1] += pz.T @ dob
        dK[k0:k1] += scale * (ds.T @ q[r0:r1])
        dQ[r0:r1] = scale * (ds @ k[k0:k1])
    return res


def ref_forward(q, k, v, scale, causal=False, wl=-1, wr=-1, softcap=0.0, alibi=None, chunk=0):
    """The reference's own ref_attention on one batch element: q (SQ,NH,D), k/v (SK,NKV,D) in the
    public layout (converted to its [NKV][SK][D] K/V layout here) -> (O (SQ,NH,D), LSE (NH,SQ))."""
    R = ref_lib()
    if R is None:
        raise RuntimeError("oracle/_ref/libfa_ref.so not built (reference sources absent)")
    q = np.ascontiguousarray(q, dtype=np.float32)
    kt = np.ascontiguousarray(np.transpose(k, (1, 0, 2)), dtype=np.float32)
    vt = np.ascontiguousarray(np.transpose(v, (1, 0, 2)), dtype=np.float32)
    SQ, NH, D = q.shape
    NKV, SK = kt.shape[0], kt.shape[1]
    O = np.zeros_like(q)
    L = np.zeros((NH, SQ), dtype=np.float32)
    al = None if alibi is None else np.ascontiguousarray(alibi, dtype=np.float32)
    R.ref_attention_c(q, kt, vt, O, L, SQ, SK, D, NH, NH // NKV, scale, softcap, wl, wr, int(causal),
                      int(al is not None), _opt(al), chunk)
    return O, L


def ref_philox(seed, idx):
    out = np.zeros(2, dtype=np.uint32)
    ref_lib().ref_philox_c(seed, idx, out)
    return int(out[0]), int(out[1])


# ------------------------------------------------------------------ dtype rounding and metrics
def round_to(x, dtype):
    """Round float32 data to fp16 / bf16 (round-to-nearest-even) and back, as the GPU sees it."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "fp16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        b = x.view(np.uint32).astype(np.uint64)
        r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
        return r.astype(np.uint32).view(np.float32)
    return x


def rel_rms(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    e = np.sum((got - ref) ** 2)
    r = np.sum(ref ** 2)
    return float(np.sqrt(e / r)) if r > 0 else float(np.sqrt(e))
