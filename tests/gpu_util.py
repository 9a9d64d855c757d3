"""Helpers for the GPU parity tests: seeded inputs rounded to the tested dtype (so the oracle sees
exactly what the GPU sees), C-ABI launches through tests/fa_abi.py, and tolerances."""
import ctypes as C

import numpy as np
import torch

import fa_abi as A
from oracle import oracle as O

TDT = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}
# rel_rms bars: fp16 / bf16 from the path's contract, fp32 from the reference's fp32 gate
TOL = {"fp16": 3e-4, "bf16": 2.5e-3, "fp32": 1e-5}


def randn(rng, shape, dt):
    """N(0,1) float32 numpy array rounded to dt, plus the matching CUDA tensor."""
    x = O.round_to(rng.standard_normal(shape).astype(np.float32), dt)
    return x, torch.from_numpy(x).to("cuda", TDT[dt])


def to_np(t):
    return t.float().cpu().numpy()


def stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def fwd_params(q, k, v, o, lse, *, scale, causal=False, wl=-1, wr=-1, softcap=0.0, chunk=0, alibi=None,
               dropout_p=0.0, seed=0, k_layout="bshd"):
    """Dense forward on (B,S,H,D) q/o; k/v either (B,S,Hk,D) or (B,Hk,S,D) (k_layout='bhsd')."""
    p = A.FaFwdParams()
    p.struct_size = C.sizeof(A.FaFwdParams)
    p.Q, p.K, p.V, p.O = A.ptr(q), A.ptr(k), A.ptr(v), A.ptr(o)
    p.LSE = A.ptr(lse)
    p.sQ, p.sO = A.strides_bshd(q), A.strides_bshd(o)
    if k_layout == "bshd":
        p.sK, p.sV = A.strides_bshd(k), A.strides_bshd(v)
        SK, Hk = k.shape[1], k.shape[2]
    else:
        p.sK, p.sV = A.strides4(k), A.strides4(v)
        SK, Hk = k.shape[2], k.shape[1]
    p.batch, p.SQ, p.SK, p.HD, p.NH = q.shape[0], q.shape[1], SK, q.shape[3], q.shape[2]
    p.gqa = q.shape[2] // Hk
    p.scale, p.softcap = scale, softcap
    p.causal, p.win_left, p.win_right, p.attn_chunk = int(causal), wl, wr, chunk
    p.alibi_slopes = A.ptr(alibi)
    p.dropout_p, p.philox_seed = dropout_p, seed
    return p


def run_fwd(p, dt):
    A.check(A.lib().fa_forward_launch(C.byref(p), A.DT[dt], stream()))
    torch.cuda.synchronize()


def lse_close(got, ref, tol):
    """-inf pattern identical; finite entries within rel_rms tol."""
    got, ref = np.asarray(got), np.asarray(ref)
    fr, fg = np.isfinite(ref), np.isfinite(got)
    if not np.array_equal(fr, fg):
        return False, "empty-row pattern differs"
    if not fr.any():
        return True, 0.0
    e = O.rel_rms(got[fr], ref[fr])
    return e < tol, e
