"""GPU parity of the forward kernels against the CPU oracle, called through the C ABI.

Case table: the reference's forward gate (kernels/fa_forward_gate.inc:170-205) — causal, full,
SQ != SK bottom-right, empty rows, seven window shapes, softcap, alibi, head dims 32..256,
attention_chunk aligned and unaligned — plus varlen/seqused (:85-138), bit-exact dropout, the
reference's golden outputs, and determinism.  Tolerances (rel_rms): fp16 3e-4, bf16 2.5e-3,
fp32 1e-5, for both O and LSE.
"""
import os
import zlib

import numpy as np
import pytest
import torch

import fa_abi as A
from gpu_util import TOL, TDT, fwd_params, lse_close, randn, run_fwd, to_np
from oracle import oracle as O

pytestmark = pytest.mark.gpu

# (name, SQ, SK, HD, NH, gqa, causal, alibi, wl, wr, softcap, chunk)
CASES = [
    ("d128_causal_gqa4", 256, 256, 128, 16, 4, True, False, -1, -1, 0.0, 0),
    ("d128_causal_mha", 256, 256, 128, 8, 1, True, False, -1, -1, 0.0, 0),
    ("d128_full", 192, 192, 128, 16, 4, False, False, -1, -1, 0.0, 0),
    ("d128_sq_lt_sk", 128, 320, 128, 16, 4, True, False, -1, -1, 0.0, 0),
    ("d128_sq_gt_sk_empty_rows", 256, 64, 128, 16, 4, True, False, -1, -1, 0.0, 0),
    ("win_63_0", 256, 256, 128, 16, 4, True, False, 63, 0, 0.0, 0),
    ("win_32_32", 256, 256, 128, 16, 4, False, False, 32, 32, 0.0, 0),
    ("win_0_0_diag", 256, 256, 128, 16, 4, False, False, 0, 0, 0.0, 0),
    ("win_open_0_causal", 256, 256, 128, 16, 4, False, False, -1, 0, 0.0, 0),
    ("win_0_open", 256, 256, 128, 16, 4, False, False, 0, -1, 0.0, 0),
    ("win_16_48", 192, 192, 128, 16, 4, False, False, 16, 48, 0.0, 0),
    ("win_32_32_sq_lt_sk", 128, 320, 128, 16, 4, False, False, 32, 32, 0.0, 0),
    ("softcap30", 200, 200, 128, 16, 4, True, False, -1, -1, 30.0, 0),
    ("alibi", 200, 200, 128, 16, 4, True, True, -1, -1, 0.0, 0),
    ("d64", 200, 200, 64, 16, 4, True, False, -1, -1, 0.0, 0),
    ("d80", 200, 200, 80, 16, 4, True, False, -1, -1, 0.0, 0),
    ("d96", 160, 160, 96, 16, 4, True, False, -1, -1, 0.0, 0),
    ("d256", 160, 160, 256, 8, 4, True, False, -1, -1, 0.0, 0),
    ("d32", 160, 160, 32, 16, 4, True, False, -1, -1, 0.0, 0),
    ("d112", 160, 160, 112, 16, 4, True, False, -1, -1, 0.0, 0),
    ("d160", 160, 160, 160, 8, 4, True, False, -1, -1, 0.0, 0),
    ("d192", 160, 160, 192, 8, 4, True, False, -1, -1, 0.0, 0),
    ("d224", 160, 160, 224, 8, 4, True, False, -1, -1, 0.0, 0),
    ("d192_full_gqa2", 128, 192, 192, 8, 2, False, False, -1, -1, 0.0, 0),
    ("chunk64_causal", 256, 256, 128, 16, 4, True, False, -1, -1, 0.0, 64),
    ("chunk100_causal", 256, 256, 128, 16, 4, True, False, -1, -1, 0.0, 100),
    ("chunk128_full", 256, 256, 128, 16, 4, False, False, -1, -1, 0.0, 128),
    ("chunk64_sq_lt_sk", 128, 320, 128, 16, 4, True, False, -1, -1, 0.0, 64),
]


def _slopes(NH):
    return (-(2.0 ** (-(8.0 * (np.arange(NH) + 1) / NH)))).astype(np.float32)


@pytest.mark.parametrize("dt", ["fp16", "bf16", "fp32"])
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_forward_gate_table(case, dt):
    name, SQ, SK, D, NH, g, causal, al, wl, wr, sc, ch = case
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    B = 2 if SQ <= 200 else 1
    qn, q = randn(rng, (B, SQ, NH, D), dt)
    kn, k = randn(rng, (B, SK, NH // g, D), dt)
    vn, v = randn(rng, (B, SK, NH // g, D), dt)
    slopes = _slopes(NH) if al else None
    o = torch.empty_like(q)
    lse = torch.empty((B, NH, SQ), device="cuda", dtype=torch.float32)
    al_t = torch.from_numpy(slopes).cuda() if al else None
    run_fwd(fwd_params(q, k, v, o, lse, scale=D ** -0.5, causal=causal, wl=wl, wr=wr, softcap=sc, chunk=ch,
                       alibi=al_t), dt)
    ro, rl = O.forward(qn, kn, vn, D ** -0.5, causal, wl, wr, sc, slopes, ch)
    e = O.rel_rms(to_np(o), ro)
    assert e < TOL[dt], f"O rel_rms {e:.3e}"
    ok, el = lse_close(lse.cpu().numpy(), rl, TOL[dt])
    assert ok, f"LSE {el}"
    if causal and SQ > SK:   # rows that see no key are exactly zero
        assert torch.all(o[:, : SQ - SK] == 0)


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_forward_kv_bhsd_layout(dt):
    """Q/O in (B,S,H,D), K/V in (B,H,S,D): mixed strides as in the reference gate."""
    rng = np.random.default_rng(3)
    B, SQ, SK, NH, Hk, D = 1, 256, 384, 16, 4, 128
    qn, q = randn(rng, (B, SQ, NH, D), dt)
    kn, k = randn(rng, (B, Hk, SK, D), dt)
    vn, v = randn(rng, (B, Hk, SK, D), dt)
    o = torch.empty_like(q)
    lse = torch.empty((B, NH, SQ), device="cuda", dtype=torch.float32)
    run_fwd(fwd_params(q, k, v, o, lse, scale=D ** -0.5, causal=True, k_layout="bhsd"), dt)
    ro, rl = O.forward(qn, kn.transpose(0, 2, 1, 3), vn.transpose(0, 2, 1, 3), D ** -0.5, True)
    assert O.rel_rms(to_np(o), ro) < TOL[dt]
    assert lse_close(lse.cpu().numpy(), rl, TOL[dt])[0]


@pytest.mark.parametrize("dt", ["fp16", "bf16", "fp32"])
@pytest.mark.parametrize("seqused", [False, True])
def test_forward_varlen(dt, seqused):
    """3 packed sequences (100, 64, 200), GQA4, causal; seqused clips to (70,64,150)/(90,30,180)."""
    import ctypes as C
    rng = np.random.default_rng(9)
    lens, used_q, used_k = [100, 64, 200], [70, 64, 150], [90, 30, 180]
    NH, Hk, D = 8, 2, 128
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    tot = int(cu[-1])
    qn, q = randn(rng, (tot, NH, D), dt)
    kn, k = randn(rng, (tot, Hk, D), dt)
    vn, v = randn(rng, (tot, Hk, D), dt)
    o = torch.zeros_like(q)
    lse = torch.full((NH, tot), -np.inf, device="cuda", dtype=torch.float32)
    cu_t = torch.from_numpy(cu).cuda()
    uq = torch.tensor(used_q, dtype=torch.int32, device="cuda")
    uk = torch.tensor(used_k, dtype=torch.int32, device="cuda")
    p = A.FaFwdParams()
    p.struct_size = C.sizeof(A.FaFwdParams)
    p.Q, p.K, p.V, p.O, p.LSE = A.ptr(q), A.ptr(k), A.ptr(v), A.ptr(o), A.ptr(lse)
    p.sQ = A.FaStrides(0, q.stride(1), q.stride(0))
    p.sK = A.FaStrides(0, k.stride(1), k.stride(0))
    p.sV = A.FaStrides(0, v.stride(1), v.stride(0))
    p.sO = A.FaStrides(0, o.stride(1), o.stride(0))
    p.batch, p.SQ, p.SK, p.HD, p.NH, p.gqa = 3, max(lens), max(lens), D, NH, NH // Hk
    p.scale, p.causal, p.win_left, p.win_right = D ** -0.5, 1, -1, 0
    p.cu_q = p.cu_k = A.ptr(cu_t)
    if seqused:
        p.seqused_q, p.seqused_k = A.ptr(uq), A.ptr(uk)
    p.lse_total_q = p.total_k = tot
    run_fwd(p, dt)
    ref_o = np.zeros_like(qn)
    ref_l = np.full((NH, tot), -np.inf, dtype=np.float32)
    for i in range(3):
        a = int(cu[i])
        LQ = used_q[i] if seqused else lens[i]
        LK = used_k[i] if seqused else lens[i]
        oo, ll = O.forward(qn[a:a + LQ][None], kn[a:a + LK][None], vn[a:a + LK][None], D ** -0.5, True)
        ref_o[a:a + LQ] = oo[0]
        ref_l[:, a:a + LQ] = ll[0]
    assert O.rel_rms(to_np(o), ref_o) < TOL[dt]
    assert lse_close(lse.cpu().numpy(), ref_l, TOL[dt])[0]


@pytest.mark.parametrize("dt", ["fp16", "bf16", "fp32"])
def test_dropout_mask_bit_exact(dt):
    """Q = 0 makes every visible key weigh 1/SK; V = identity (SK = HD = 64) exposes the kept
    multiplier of each (row, key) in O: O[q, h, d] = keep(h, q, d) * (1/(1-p)) / SK.  The zero
    pattern must equal the oracle's Philox mask bit for bit, for every head."""
    B, SQ, SK, NH, D, p_drop, seed = 2, 96, 64, 4, 64, 0.2, 0x1234_5678_9ABC
    q = torch.zeros((B, SQ, NH, D), device="cuda", dtype=TDT[dt])
    eye = torch.eye(SK, D, device="cuda", dtype=TDT[dt])
    k = torch.zeros((B, SK, NH, D), device="cuda", dtype=TDT[dt])
    v = eye[None, :, None, :].expand(B, SK, NH, D).contiguous()
    o = torch.empty_like(q)
    run_fwd(fwd_params(q, k, v, o, None, scale=D ** -0.5, dropout_p=p_drop, seed=seed), dt)
    got = to_np(o)
    for h in range(NH):
        ref = O.dropout_mask(seed, h, SQ, SK, p_drop).astype(bool)
        for b in range(B):   # the mask has no batch term (reference kernels/fa_forward.hip:258)
            assert np.array_equal(got[b, :, h, :] != 0, ref), f"head {h} batch {b}"
    kept = got[got != 0]
    assert np.allclose(kept, (1.0 / (1.0 - np.float32(p_drop))) / SK, rtol=1e-2)


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_dropout_forward_values(dt):
    rng = np.random.default_rng(21)
    B, S, NH, D = 1, 192, 8, 128
    qn, q = randn(rng, (B, S, NH, D), dt)
    kn, k = randn(rng, (B, S, NH, D), dt)
    vn, v = randn(rng, (B, S, NH, D), dt)
    o = torch.empty_like(q)
    lse = torch.empty((B, NH, S), device="cuda", dtype=torch.float32)
    run_fwd(fwd_params(q, k, v, o, lse, scale=D ** -0.5, causal=True, dropout_p=0.1, seed=777), dt)
    ro, rl = O.forward(qn, kn, vn, D ** -0.5, True, dropout_p=0.1, seed=777)
    assert O.rel_rms(to_np(o), ro) < TOL[dt]
    assert lse_close(lse.cpu().numpy(), rl, TOL[dt])[0]


def test_forward_on_reference_golden_outputs():
    """The kernels on the reference's own fixture inputs (fp16) against its oracle outputs."""
    gold = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_oracle.npz"))
    names = sorted({k.split("/")[1] for k in gold.files if k.startswith("fwd/")})
    for name in names:
        pfx = f"fwd/{name}/"
        SQ, SK, D, NH, g, causal, al, wl, wr, sc, ch = gold[pfx + "cfg"].tolist()
        q = torch.from_numpy(gold[pfx + "q"]).cuda()[None]
        k = torch.from_numpy(gold[pfx + "k"]).cuda()[None]
        v = torch.from_numpy(gold[pfx + "v"]).cuda()[None]
        o = torch.empty_like(q)
        lse = torch.empty((1, int(NH), int(SQ)), device="cuda", dtype=torch.float32)
        al_t = torch.from_numpy(gold[pfx + "slopes"]).cuda() if al else None
        run_fwd(fwd_params(q, k, v, o, lse, scale=int(D) ** -0.5, causal=bool(causal), wl=int(wl), wr=int(wr),
                           softcap=sc, chunk=int(ch), alibi=al_t), "fp16")
        assert O.rel_rms(to_np(o)[0], gold[pfx + "o"]) < TOL["fp16"], name
        assert lse_close(lse.cpu().numpy()[0], gold[pfx + "lse"], TOL["fp16"])[0], name


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_forward_deterministic(dt):
    rng = np.random.default_rng(4)
    _, q = randn(rng, (1, 512, 8, 128), dt)
    _, k = randn(rng, (1, 512, 8, 128), dt)
    _, v = randn(rng, (1, 512, 8, 128), dt)
    outs = []
    for _ in range(2):
        o = torch.empty_like(q)
        lse = torch.empty((1, 8, 512), device="cuda", dtype=torch.float32)
        run_fwd(fwd_params(q, k, v, o, lse, scale=128 ** -0.5, causal=True), dt)
        outs.append((o, lse))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


@pytest.mark.parametrize("wide", [False, True])
@pytest.mark.parametrize("causal,wl,wr", [(False, -1, -1), (True, -1, -1), (False, 40, 8)])
def test_dropout_bitmask_matches_oracle(causal, wl, wr, wide, monkeypatch):
    """fa_dropout_mask_launch writes exactly the oracle's keep bits for every word a row can see,
    with 32-bit counters and with the 64-bit counter form that masks past 2^32 draws use."""
    import ctypes as C
    if wide:
        monkeypatch.setenv("FABLE_ATTN_MASK_WIDE", "1")
    NH, SQ, SK, p_drop, seed = 3, 77, 150, 0.3, 0xABCDEF0123
    W = (SK + 31) // 32
    words = A.lib().fa_dropout_mask_words(NH, SQ, SK)
    assert words == NH * SQ * W
    bits = torch.zeros(words, dtype=torch.int32, device="cuda")
    A.check(A.lib().fa_dropout_mask_launch(seed, p_drop, NH, SQ, SK, int(causal), wl, wr, A.ptr(bits),
                                           C.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    got = bits.cpu().numpy().view(np.uint32).reshape(NH, W, SQ)   # [h][key word][query row]
    for h in range(NH):
        ref = O.dropout_mask(seed, h, SQ, SK, p_drop)
        for q in range(SQ):
            diag = q + SK - SQ
            lo = max(0, diag - wl) if wl >= 0 else 0
            hi = min(SK - 1, diag if causal else SK - 1, diag + wr if wr >= 0 else SK - 1)
            for w in range(W):
                if hi < w * 32 or lo > w * 32 + 31 or lo > hi:
                    continue            # words no row reads are not written
                want = 0
                for b in range(32):
                    k = w * 32 + b
                    if k < SK and ref[q, k]:
                        want |= 1 << b
                assert int(got[h, w, q]) == want, (h, q, w)


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("D", [64, 128])
def test_forward_with_bitmask_equals_inkernel_philox(dt, D):
    import ctypes as C
    rng = np.random.default_rng(33)
    B, S, NH = 2, 320, 4
    _, q = randn(rng, (B, S, NH, D), dt)
    _, k = randn(rng, (B, S, NH, D), dt)
    _, v = randn(rng, (B, S, NH, D), dt)
    seed, pd = 4242, 0.15
    outs = []
    for use_bits in (False, True):
        o = torch.empty_like(q)
        lse = torch.empty((B, NH, S), device="cuda", dtype=torch.float32)
        p = fwd_params(q, k, v, o, lse, scale=D ** -0.5, causal=True, dropout_p=pd, seed=seed)
        if use_bits:
            bits = torch.zeros(A.lib().fa_dropout_mask_words(NH, S, S), dtype=torch.int32, device="cuda")
            A.check(A.lib().fa_dropout_mask_launch(seed, pd, NH, S, S, 1, -1, 0, A.ptr(bits),
                                                   C.c_void_p(torch.cuda.current_stream().cuda_stream)))
            p.dropout_bits = A.ptr(bits)
        run_fwd(p, dt)
        outs.append((o, lse))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("total_k_known", [True, False])
def test_forward_varlen_swa_softcap_gqa8(dt, total_k_known):
    """Config-5 shape in miniature: packed sequences, GQA 8, causal sliding window (512, 0),
    softcap 30, keys longer than queries (cu_seqlens_k != cu_seqlens_q).  With total_k the
    tensor-core kernel runs; without it (an older caller) the CUDA-core kernel does."""
    import ctypes as C
    rng = np.random.default_rng(41)
    lq, lk = [700, 130, 1000, 257, 1], [900, 130, 1000, 300, 1]
    NH, Hk, D = 16, 2, 128
    cq = np.concatenate([[0], np.cumsum(lq)]).astype(np.int32)
    ck = np.concatenate([[0], np.cumsum(lk)]).astype(np.int32)
    tq, tk = int(cq[-1]), int(ck[-1])
    qn, q = randn(rng, (tq, NH, D), dt)
    kn, k = randn(rng, (tk, Hk, D), dt)
    vn, v = randn(rng, (tk, Hk, D), dt)
    o = torch.zeros_like(q)
    lse = torch.full((NH, tq), -np.inf, device="cuda", dtype=torch.float32)
    cq_t, ck_t = torch.from_numpy(cq).cuda(), torch.from_numpy(ck).cuda()
    p = A.FaFwdParams()
    p.struct_size = C.sizeof(A.FaFwdParams)
    p.Q, p.K, p.V, p.O, p.LSE = A.ptr(q), A.ptr(k), A.ptr(v), A.ptr(o), A.ptr(lse)
    p.sQ = A.FaStrides(0, q.stride(1), q.stride(0))
    p.sK = A.FaStrides(0, k.stride(1), k.stride(0))
    p.sV = A.FaStrides(0, v.stride(1), v.stride(0))
    p.sO = A.FaStrides(0, o.stride(1), o.stride(0))
    p.batch, p.SQ, p.SK, p.HD, p.NH, p.gqa = len(lq), max(lq), max(lk), D, NH, NH // Hk
    p.scale, p.causal, p.win_left, p.win_right, p.softcap = D ** -0.5, 1, 512, 0, 30.0
    p.cu_q, p.cu_k = A.ptr(cq_t), A.ptr(ck_t)
    p.lse_total_q = tq
    p.total_k = tk if total_k_known else 0
    run_fwd(p, dt)
    ref_o = np.zeros_like(qn)
    ref_l = np.full((NH, tq), -np.inf, dtype=np.float32)
    for i in range(len(lq)):
        a, b = int(cq[i]), int(ck[i])
        oo, ll = O.forward(qn[a:a + lq[i]][None], kn[b:b + lk[i]][None], vn[b:b + lk[i]][None], D ** -0.5, True,
                           512, 0, 30.0)
        ref_o[a:a + lq[i]] = oo[0]
        ref_l[:, a:a + lq[i]] = ll[0]
    assert O.rel_rms(to_np(o), ref_o) < TOL[dt]
    assert lse_close(lse.cpu().numpy(), ref_l, TOL[dt])[0]


# cases the two-query-tile kernel takes (head_dim 128, no softcap / alibi / dropout), plus row
# counts that leave the second tile of the last CTA partly or wholly past the sequence end
TWO_TILE_CASES = [c for c in CASES if c[3] == 128 and c[10] == 0.0 and not c[7]] + [
    ("d128_sq300_full", 300, 300, 128, 8, 2, False, False, -1, -1, 0.0, 0),
    ("d128_sq100_causal", 100, 100, 128, 8, 1, True, False, -1, -1, 0.0, 0),
    ("d128_sq640_sk200_causal", 640, 200, 128, 8, 4, True, False, -1, -1, 0.0, 0),
    ("d128_sq384_win_100_20", 384, 384, 128, 8, 2, False, False, 100, 20, 0.0, 0),
    ("d128_gqa8_sq1000_causal", 1000, 1000, 128, 16, 8, True, False, -1, -1, 0.0, 0),
    ("d128_sq700_win_256_64", 700, 700, 128, 8, 4, False, False, 256, 64, 0.0, 0),
    ("d128_chunk96_causal", 520, 520, 128, 8, 2, True, False, -1, -1, 0.0, 96),
    ("d128_sq200_sk900_full", 200, 900, 128, 8, 1, False, False, -1, -1, 0.0, 0),
]


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("case", TWO_TILE_CASES, ids=[c[0] for c in TWO_TILE_CASES])
def test_forward_two_tile_kernel(case, dt, monkeypatch):
    """The two-query-tile kernel (forced on small shapes with FABLE_ATTN_FWD_TILES=2) against the
    oracle: masks, windows, chunks, empty rows, partial and empty second tiles."""
    assert A.lib().fa_forward_two_tile_ready(int(dt == "bf16")) == 1, "two-tile kernel unavailable"
    monkeypatch.setenv("FABLE_ATTN_FWD_TILES", "2")
    name, SQ, SK, D, NH, g, causal, al, wl, wr, sc, ch = case
    rng = np.random.default_rng(zlib.crc32(name.encode()) + 7)
    B = 2
    qn, q = randn(rng, (B, SQ, NH, D), dt)
    kn, k = randn(rng, (B, SK, NH // g, D), dt)
    vn, v = randn(rng, (B, SK, NH // g, D), dt)
    o = torch.full_like(q, float("nan"))
    lse = torch.full((B, NH, SQ), float("nan"), device="cuda", dtype=torch.float32)
    run_fwd(fwd_params(q, k, v, o, lse, scale=D ** -0.5, causal=causal, wl=wl, wr=wr, chunk=ch), dt)
    ro, rl = O.forward(qn, kn, vn, D ** -0.5, causal, wl, wr, 0.0, None, ch)
    e = O.rel_rms(to_np(o), ro)
    assert e < TOL[dt], f"O rel_rms {e:.3e}"
    ok, el = lse_close(lse.cpu().numpy(), rl, TOL[dt])
    assert ok, f"LSE {el}"
    if causal and SQ > SK:
        assert torch.all(o[:, : SQ - SK] == 0)


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_forward_two_tile_matches_one_tile(dt, monkeypatch):
    """Both forward kernels on the same dense causal input: equal within the dtype's tolerance, and
    the two-tile kernel is the default at this size (config 3's shape: 1024 two-tile CTAs, 7 waves
    on 148 SMs, against 14 waves of one-tile CTAs)."""
    rng = np.random.default_rng(11)
    B, S, H, D = 2, 4096, 32, 128
    _, q = randn(rng, (B, S, H, D), dt)
    _, k = randn(rng, (B, S, H, D), dt)
    _, v = randn(rng, (B, S, H, D), dt)
    outs = {}
    for tiles in ("1", "2", None):
        if tiles is None:
            monkeypatch.delenv("FABLE_ATTN_FWD_TILES", raising=False)
        else:
            monkeypatch.setenv("FABLE_ATTN_FWD_TILES", tiles)
        o = torch.empty_like(q)
        lse = torch.empty((B, H, S), device="cuda", dtype=torch.float32)
        run_fwd(fwd_params(q, k, v, o, lse, scale=D ** -0.5, causal=True), dt)
        outs[tiles] = (o.float(), lse.clone())
    o1, l1 = outs["1"]
    o2, l2 = outs["2"]
    assert ((o1 - o2).norm() / o1.norm()).item() < TOL[dt]
    assert ((l1 - l2).abs().max()).item() < 1e-3
    assert torch.equal(outs[None][0], o2), "the default at this size is the two-tile kernel"


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("causal,wl,wr,SQ", [(True, -1, -1, 300), (False, -1, -1, 256), (False, 70, 10, 384)])
def test_forward_two_tile_dropout_bits(dt, causal, wl, wr, SQ, monkeypatch):
    """The two-query-tile kernel with a precomputed keep mask against the oracle's dropout forward,
    and bitwise equal to itself run twice."""
    import ctypes as C
    monkeypatch.setenv("FABLE_ATTN_FWD_TILES", "2")
    rng = np.random.default_rng(SQ + 5)
    B, NH, D, seed, pd = 2, 4, 128, 9090, 0.2
    qn, q = randn(rng, (B, SQ, NH, D), dt)
    kn, k = randn(rng, (B, SQ, NH, D), dt)
    vn, v = randn(rng, (B, SQ, NH, D), dt)
    bits = torch.zeros(A.lib().fa_dropout_mask_words(NH, SQ, SQ), dtype=torch.int32, device="cuda")
    A.check(A.lib().fa_dropout_mask_launch(seed, pd, NH, SQ, SQ, int(causal), wl, wr, A.ptr(bits),
                                           C.c_void_p(torch.cuda.current_stream().cuda_stream)))
    outs = []
    for _ in range(2):
        o = torch.empty_like(q)
        lse = torch.empty((B, NH, SQ), device="cuda", dtype=torch.float32)
        p = fwd_params(q, k, v, o, lse, scale=D ** -0.5, causal=causal, wl=wl, wr=wr, dropout_p=pd, seed=seed)
        p.dropout_bits = A.ptr(bits)
        run_fwd(p, dt)
        outs.append((o, lse))
    ro, rl = O.forward(qn, kn, vn, D ** -0.5, causal, wl, wr, dropout_p=pd, seed=seed)
    assert O.rel_rms(to_np(outs[0][0]), ro) < TOL[dt]
    assert lse_close(outs[0][1].cpu().numpy(), rl, TOL[dt])[0]
    assert torch.equal(outs[0][0], outs[1][0])
