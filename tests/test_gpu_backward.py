"""GPU parity of the backward against the fp64 oracle (kernels/backward.hip:583-597 restated),
through the C ABI, on the reference's backward case table (kernels/backward.hip:710-730), plus
bit-determinism (two runs compared with memcmp semantics, :628-631) and native varlen.
As in the reference gate, O and LSE fed to the kernel come from the oracle (O rounded to dtype),
which isolates the backward kernels.  rel_rms bars: fp16 3e-4, bf16 2.5e-3, fp32 1e-5."""
import ctypes as C
import zlib

import numpy as np
import pytest
import torch

import fa_abi as A
from gpu_util import TDT, TOL, randn, stream, to_np
from oracle import oracle as O

pytestmark = pytest.mark.gpu

# (name, B, Hq, Hk, SQ, SK, D, causal, wl, wr, softcap, alibi, pdrop)
CASES = [
    ("base", 1, 4, 4, 64, 64, 64, False, -1, -1, 0.0, False, 0.0),
    ("causal", 1, 4, 4, 64, 64, 64, True, -1, -1, 0.0, False, 0.0),
    ("causal_gqa", 2, 8, 2, 128, 128, 64, True, -1, -1, 0.0, False, 0.0),
    ("causal_tail", 1, 4, 4, 100, 100, 64, True, -1, -1, 0.0, False, 0.0),
    ("cross_sq_lt_sk", 1, 4, 4, 96, 128, 64, True, -1, -1, 0.0, False, 0.0),
    ("cross_sq_gt_sk", 1, 4, 4, 128, 96, 64, True, -1, -1, 0.0, False, 0.0),
    ("window_47_0", 1, 4, 4, 128, 128, 64, False, 47, 0, 0.0, False, 0.0),
    ("window_24_24", 1, 4, 4, 128, 128, 64, False, 24, 24, 0.0, False, 0.0),
    ("window_open_0", 1, 4, 4, 128, 128, 64, False, -1, 0, 0.0, False, 0.0),
    ("d192", 1, 4, 4, 64, 64, 192, False, -1, -1, 0.0, False, 0.0),
    ("d256_causal", 1, 4, 4, 64, 64, 256, True, -1, -1, 0.0, False, 0.0),
    ("d160_causal", 1, 4, 4, 64, 64, 160, True, -1, -1, 0.0, False, 0.0),
    ("d224", 1, 4, 4, 64, 64, 224, False, -1, -1, 0.0, False, 0.0),
    ("softcap30", 1, 4, 4, 128, 128, 64, False, -1, -1, 30.0, False, 0.0),
    ("alibi_causal", 1, 4, 4, 128, 128, 64, True, -1, -1, 0.0, True, 0.0),
    ("dropout0.2", 1, 4, 4, 128, 128, 64, False, -1, -1, 0.0, False, 0.2),
    ("d16", 1, 4, 4, 64, 64, 16, False, -1, -1, 0.0, False, 0.0),
    ("d128", 1, 4, 4, 64, 64, 128, False, -1, -1, 0.0, False, 0.0),
    ("d96_causal", 1, 4, 4, 80, 80, 96, True, -1, -1, 0.0, False, 0.0),
    ("d128_window_dropout_gqa", 1, 4, 2, 160, 256, 128, False, 40, 24, 0.0, False, 0.1),
    ("d128_causal_dropout_gqa", 2, 8, 2, 192, 192, 128, True, -1, -1, 0.0, False, 0.1),
]


def _bwd_params(q, k, v, o, do, dq, dk, dv, lse, dsum, *, scale, causal, wl, wr, softcap, alibi, pdrop, seed):
    p = A.FaBwdParams()
    p.struct_size = C.sizeof(A.FaBwdParams)
    p.Q, p.K, p.V, p.O, p.dO = A.ptr(q), A.ptr(k), A.ptr(v), A.ptr(o), A.ptr(do)
    p.dQ, p.dK, p.dV, p.lse, p.dsum = A.ptr(dq), A.ptr(dk), A.ptr(dv), A.ptr(lse), A.ptr(dsum)
    for f, t in (("qs", q), ("ks", k), ("vs", v), ("os", o), ("dos", do), ("dqs", dq), ("dks", dk), ("dvs", dv)):
        setattr(p, f, A.strides_bshd(t))
    p.B, p.SQ, p.Hq, p.D = q.shape[0], q.shape[1], q.shape[2], q.shape[3]
    p.SK, p.Hk = k.shape[1], k.shape[2]
    p.gqa = p.Hq // p.Hk
    p.scale, p.softcap, p.alibi = scale, softcap, A.ptr(alibi)
    p.causal, p.win_left, p.win_right = int(causal), wl, wr
    p.dropout = int(pdrop > 0)
    p.drop_seed, p.dropout_p = seed, pdrop
    p.keep_scale = 1.0 / (1.0 - pdrop) if pdrop > 0 else 1.0
    return p


def _run_case(case, dt):
    name, B, Hq, Hk, SQ, SK, D, causal, wl, wr, sc, al, pd = case
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    qn, q = randn(rng, (B, SQ, Hq, D), dt)
    kn, k = randn(rng, (B, SK, Hk, D), dt)
    vn, v = randn(rng, (B, SK, Hk, D), dt)
    don, do = randn(rng, (B, SQ, Hq, D), dt)
    slopes = (-0.1 * (np.arange(Hq) + 1)).astype(np.float32) if al else None
    scale, seed = D ** -0.5, 777
    on, ln = O.forward(qn, kn, vn, scale, causal, wl, wr, sc, slopes, 0, pd, seed)
    o = torch.from_numpy(O.round_to(on, dt)).to("cuda", TDT[dt])
    lse = torch.from_numpy(ln).cuda()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dsum = torch.empty((B, Hq, SQ), device="cuda", dtype=torch.float32)
    al_t = torch.from_numpy(slopes).cuda() if al else None
    p = _bwd_params(q, k, v, o, do, dq, dk, dv, lse, dsum, scale=scale, causal=causal, wl=wl, wr=wr, softcap=sc,
                    alibi=al_t, pdrop=pd, seed=seed)
    A.check(A.lib().fable_attn_backward_launch(C.byref(p), A.DT[dt], stream()))
    torch.cuda.synchronize()
    refs = O.backward(qn, kn, vn, don, scale, causal, wl, wr, sc, slopes, pd, seed)
    # the parameter block holds raw pointers: keep every tensor it names alive with it
    p._keep = (q, k, v, o, do, lse, dsum, al_t, dq, dk, dv)
    return p, (dq, dk, dv), refs


@pytest.mark.parametrize("dt", ["fp16", "bf16", "fp32"])
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_backward_gate_table(case, dt):
    p, got, refs = _run_case(case, dt)
    for nm, g, r in zip(("dQ", "dK", "dV"), got, refs):
        t = to_np(g)
        assert np.isfinite(t).all(), nm
        e = O.rel_rms(t, r)
        assert e < TOL[dt], f"{nm} rel_rms {e:.3e}"


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_backward_bit_deterministic(dt):
    case = CASES[-1]
    p, got, _ = _run_case(case, dt)
    first = [g.clone() for g in got]
    for _ in range(2):
        A.check(A.lib().fable_attn_backward_launch(C.byref(p), A.DT[dt], stream()))
        torch.cuda.synchronize()
        for a, b in zip(first, got):
            assert torch.equal(a.view(torch.int16), b.view(torch.int16))


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_backward_varlen_native(dt):
    """Native varlen backward (one launch for all sequences) vs per-sequence oracle."""
    rng = np.random.default_rng(31)
    lens = [70, 128, 33]
    Hq, Hk, D = 4, 2, 64
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    tot = int(cu[-1])
    qn, q = randn(rng, (tot, Hq, D), dt)
    kn, k = randn(rng, (tot, Hk, D), dt)
    vn, v = randn(rng, (tot, Hk, D), dt)
    don, do = randn(rng, (tot, Hq, D), dt)
    on = np.zeros_like(qn)
    ln = np.full((Hq, tot), -np.inf, np.float32)
    for i in range(3):
        a, b = int(cu[i]), int(cu[i + 1])
        oo, ll = O.forward(qn[a:b][None], kn[a:b][None], vn[a:b][None], D ** -0.5, True)
        on[a:b], ln[:, a:b] = oo[0], ll[0]
    o = torch.from_numpy(O.round_to(on, dt)).to("cuda", TDT[dt])
    lse = torch.from_numpy(ln).cuda()
    dq, dk, dv = torch.zeros_like(q), torch.zeros_like(k), torch.zeros_like(v)
    dsum = torch.empty((Hq, tot), device="cuda", dtype=torch.float32)
    cu_t = torch.from_numpy(cu).cuda()
    p = A.FaBwdParams()
    p.struct_size = C.sizeof(A.FaBwdParams)
    p.Q, p.K, p.V, p.O, p.dO = A.ptr(q), A.ptr(k), A.ptr(v), A.ptr(o), A.ptr(do)
    p.dQ, p.dK, p.dV, p.lse, p.dsum = A.ptr(dq), A.ptr(dk), A.ptr(dv), A.ptr(lse), A.ptr(dsum)
    for f, t in (("qs", q), ("ks", k), ("vs", v), ("os", o), ("dos", do), ("dqs", dq), ("dks", dk), ("dvs", dv)):
        setattr(p, f, A.FaStrides(0, t.stride(1), t.stride(0)))
    p.B, p.Hq, p.Hk, p.SQ, p.SK, p.D, p.gqa = 3, Hq, Hk, max(lens), max(lens), D, Hq // Hk
    p.scale, p.causal, p.win_left, p.win_right = D ** -0.5, 1, -1, 0
    p.keep_scale = 1.0
    p.cu_q = p.cu_k = A.ptr(cu_t)
    p.lse_total_q = tot
    A.check(A.lib().fable_attn_backward_launch(C.byref(p), A.DT[dt], stream()))
    torch.cuda.synchronize()
    for i in range(3):
        a, b = int(cu[i]), int(cu[i + 1])
        rq, rk, rv = O.backward(qn[a:b][None], kn[a:b][None], vn[a:b][None], don[a:b][None], D ** -0.5, True)
        for g, r in ((dq, rq), (dk, rk), (dv, rv)):
            assert O.rel_rms(to_np(g)[a:b], r[0]) < TOL[dt]


@pytest.mark.parametrize("dt", ["fp16", "bf16", "fp32"])
@pytest.mark.parametrize("name", ["dropout0.2", "d128_causal_dropout_gqa", "d128_window_dropout_gqa"])
def test_backward_with_bitmask_equals_inkernel_philox(dt, name):
    """Backward reading the precomputed keep bits gives bitwise the same gradients as Philox in-kernel."""
    case = next(c for c in CASES if c[0] == name)
    p, got, _ = _run_case(case, dt)
    first = [g.clone() for g in got]
    bits = torch.zeros(A.lib().fa_dropout_mask_words(p.Hq, p.SQ, p.SK), dtype=torch.int32, device="cuda")
    A.check(A.lib().fa_dropout_mask_launch(p.drop_seed, p.dropout_p, p.Hq, p.SQ, p.SK, p.causal, p.win_left,
                                           p.win_right, A.ptr(bits), stream()))
    p.dropout_bits = A.ptr(bits)
    for g in got:
        g.zero_()
    A.check(A.lib().fable_attn_backward_launch(C.byref(p), A.DT[dt], stream()))
    torch.cuda.synchronize()
    for nm, a, b in zip(("dQ", "dK", "dV"), first, got):
        assert torch.equal(a, b), nm
    # with the key-major workspace (pre-filled with all-ones words, so a word the backward failed
    # to write would show up as kept scores)
    bits_t = torch.full((A.lib().fa_dropout_mask_words(p.Hq, p.SK, p.SQ),), -1, dtype=torch.int32, device="cuda")
    p.dropout_bits_t = A.ptr(bits_t)
    for g in got:
        g.zero_()
    A.check(A.lib().fable_attn_backward_launch(C.byref(p), A.DT[dt], stream()))
    torch.cuda.synchronize()
    for nm, a, b in zip(("dQ", "dK", "dV"), first, got):
        assert torch.equal(a, b), nm + " (key-major mask copy)"
    if dt != "fp32" and p.D == 128:   # the tensor-core backward wrote the copy: check its layout
        QW = (p.SQ + 31) // 32
        row = bits.view(p.Hq, (p.SK + 31) // 32, p.SQ).cpu().numpy().view(np.uint32)
        col = bits_t.view(p.Hq, QW, p.SK).cpu().numpy().view(np.uint32)
        for h, q, k in [(0, 0, 0), (1, 37, 5), (p.Hq - 1, p.SQ - 1, p.SK - 1), (2, 100, 64),
                        (0, min(100, p.SQ - 1), min(200, p.SK - 1))]:
            diag = q + p.SK - p.SQ
            hi = min(p.SK - 1, diag) if p.causal else p.SK - 1
            lo = max(0, diag - p.win_left) if p.win_left >= 0 else 0
            hi = min(hi, diag + p.win_right) if p.win_right >= 0 else hi
            if lo <= k <= hi:   # words of keys the row cannot see are never read
                assert (row[h, k // 32, q] >> (k % 32)) & 1 == (col[h, q // 32, k] >> (q % 32)) & 1
