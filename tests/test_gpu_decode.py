"""GPU parity of paged-KV decode (append + split-K partial + merge) and of the combine kernel,
through the C ABI, against the oracle (kernels/fa_decode_gate.inc:66-96 restated).

Case table: the reference's decode gate (kernels/fa_decode_gate.inc:159-192) — paged GQA, NeoX
and interleaved rotary, window, append(+rotary), leftpad(+window), softcap, alibi, nq = 3..8,
every head dim — on a 2-sequence batch with a RANDOM permutation block table (the reference uses
the identity), plus gqa values the reference's kernel cannot map (3, 6, 16), bit-exact append
placement, split-count invariance, and out-of-range page detection."""
import ctypes as C
import zlib

import numpy as np
import pytest
import torch

import fa_abi as A
from gpu_util import TDT, TOL, randn, stream, to_np
from oracle import oracle as O

pytestmark = pytest.mark.gpu

# (name, HD, NH, gqa, ctx, window, rotary, append, leftpad, nq, softcap, alibi)
CASES = [
    ("paged_gqa4_ctx333", 128, 32, 4, 333, -1, 0, False, 0, 1, 0.0, False),
    ("paged_gqa1_ctx200", 128, 8, 1, 200, -1, 0, False, 0, 1, 0.0, False),
    ("rotary_neox", 128, 32, 4, 256, -1, 1, False, 0, 1, 0.0, False),
    ("rotary_interleaved", 128, 32, 4, 256, -1, 2, False, 0, 1, 0.0, False),
    ("window64", 128, 32, 4, 500, 64, 0, False, 0, 1, 0.0, False),
    ("append_rotary", 128, 32, 4, 257, -1, 1, True, 0, 1, 0.0, False),
    ("leftpad100", 128, 32, 4, 400, -1, 0, False, 100, 1, 0.0, False),
    ("leftpad37_gqa1", 128, 8, 1, 333, -1, 0, False, 37, 1, 0.0, False),
    ("leftpad_window", 128, 32, 4, 500, 64, 0, False, 50, 1, 0.0, False),
    ("softcap30", 128, 32, 4, 333, -1, 0, False, 0, 1, 30.0, False),
    ("softcap50_append", 128, 32, 4, 257, -1, 0, True, 0, 1, 50.0, False),
    ("alibi", 128, 32, 4, 333, -1, 0, False, 0, 1, 0.0, True),
    ("alibi_window", 128, 32, 4, 500, 128, 0, False, 0, 1, 0.0, True),
    ("nq4_no_append", 128, 32, 4, 300, -1, 0, False, 0, 4, 0.0, False),
    ("nq4_append", 128, 32, 4, 300, -1, 0, True, 0, 4, 0.0, False),
    ("nq8_append_rotary", 128, 32, 4, 257, -1, 1, True, 0, 8, 0.0, False),
    ("nq5_gqa1_window", 128, 8, 1, 400, 96, 0, True, 0, 5, 0.0, False),
    ("nq3_softcap_alibi", 128, 32, 4, 300, -1, 0, True, 0, 3, 30.0, True),
    ("hd64", 64, 32, 4, 300, -1, 0, False, 0, 1, 0.0, False),
    ("hd256", 256, 8, 4, 300, -1, 0, False, 0, 1, 0.0, False),
    ("hd16", 16, 32, 4, 200, -1, 0, False, 0, 1, 0.0, False),
    ("hd32", 32, 32, 4, 200, -1, 0, False, 0, 1, 0.0, False),
    ("hd48", 48, 32, 4, 200, -1, 0, False, 0, 1, 0.0, False),
    ("hd80", 80, 32, 4, 200, -1, 0, False, 0, 1, 0.0, False),
    ("hd96", 96, 32, 4, 200, -1, 0, False, 0, 1, 0.0, False),
    ("hd112", 112, 32, 4, 200, -1, 0, False, 0, 1, 0.0, False),
    ("hd160", 160, 8, 4, 200, -1, 0, False, 0, 1, 0.0, False),
    ("hd192", 192, 8, 4, 200, -1, 0, False, 0, 1, 0.0, False),
    ("hd224", 224, 8, 4, 200, -1, 0, False, 0, 1, 0.0, False),
    ("gqa3", 64, 12, 3, 300, -1, 0, False, 0, 1, 0.0, False),
    ("gqa6_append", 64, 12, 6, 300, -1, 0, True, 0, 2, 0.0, False),
    ("gqa16_mqa", 64, 16, 16, 300, -1, 0, False, 0, 1, 0.0, False),
]

PAGE = 16


def _setup(case, dt, nsplit=0, batch=2, page=None, ctxs=None):
    name, HD, NH, gqa, ctx, window, rotary, append, leftpad, nq, sc, al = case
    PAGE = page or globals()["PAGE"]
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    NKV = NH // gqa
    if ctxs is None:
        ctxs = np.array([ctx, max(ctx // 2 + 7, 1)][:batch], dtype=np.int32)
    else:
        ctxs = np.asarray(ctxs, dtype=np.int32)
        batch = len(ctxs)
    total = ctxs + (nq if append else 0)
    max_blocks = int((total.max() + PAGE - 1) // PAGE)
    nblocks = batch * max_blocks + 3
    bt = rng.permutation(nblocks)[: batch * max_blocks].astype(np.int32).reshape(batch, max_blocks)
    kcn, kc = randn(rng, (nblocks, PAGE, NKV, HD), dt)
    vcn, vc = randn(rng, (nblocks, PAGE, NKV, HD), dt)
    qn, q = randn(rng, (batch, nq, NH, HD), dt)
    nkn = nvn = nk = nv = None
    if append:
        nkn, nk = randn(rng, (batch, nq, NKV, HD), dt)
        nvn, nv = randn(rng, (batch, nq, NKV, HD), dt)
    seqro = int(total.max()) + 8
    ang = np.arange(seqro)[:, None] * (10000.0 ** (-2.0 * np.arange(HD // 2) / HD))[None]
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    slopes = (-(2.0 ** (-(8.0 * (np.arange(NH) + 1) / NH)))).astype(np.float32) if al else None
    lp = np.full(batch, leftpad, np.int32) if leftpad else None
    if nsplit <= 0:
        nsplit = A.lib().fa_decode_num_splits(batch, nq, NKV, max_blocks * PAGE, 0)
    o = torch.empty_like(q)
    lse = torch.empty((batch, nq, NH), device="cuda", dtype=torch.float32)
    scratch = torch.empty(A.lib().fa_decode_scratch_floats(batch, nq, NH, HD, nsplit), device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    keep = dict(bt=torch.from_numpy(bt).cuda(), ctx=torch.from_numpy(ctxs).cuda(),
                cos=torch.from_numpy(cos).cuda(), sin=torch.from_numpy(sin).cuda(),
                al=torch.from_numpy(slopes).cuda() if al else None,
                lp=torch.from_numpy(lp).cuda() if lp is not None else None)
    p = A.FaDecParams()
    p.struct_size = C.sizeof(A.FaDecParams)
    p.q, p.Kc, p.Vc, p.block_table, p.o = A.ptr(q), A.ptr(kc), A.ptr(vc), A.ptr(keep["bt"]), A.ptr(o)
    p.scratch, p.ctx_len = A.ptr(scratch), A.ptr(keep["ctx"])
    if rotary:
        p.cos, p.sin = A.ptr(keep["cos"]), A.ptr(keep["sin"])
    p.batch, p.NH, p.gqa, p.HD, p.page, p.max_blocks, p.nsplit, p.window = (batch, NH, gqa, HD, PAGE, max_blocks,
                                                                             nsplit, window)
    p.rotary, p.scale, p.leftpad, p.lse_out = rotary, HD ** -0.5, A.ptr(keep["lp"]), A.ptr(lse)
    p.softcap, p.alibi, p.nq = sc, A.ptr(keep["al"]), nq
    p.num_blocks, p.err_flag = nblocks, A.ptr(err)
    ref = O.decode(qn, kcn, vcn, bt, ctxs, nkn, nvn, cos if rotary else None, sin if rotary else None, rotary, 0,
                   None, lp, slopes, window, HD ** -0.5, sc)
    keep["scratch"] = scratch   # the parameter block holds raw pointers: keep them alive
    return dict(p=p, keep=keep, q=q, kc=kc, vc=vc, nk=nk, nv=nv, o=o, lse=lse, err=err, ref=ref, bt=bt, ctxs=ctxs,
                nkn=nkn, nvn=nvn, kcn=kcn, vcn=vcn)


def _launch(s, dt):
    A.check(A.lib().fa_decode_launch(C.byref(s["p"]), A.DT[dt], stream(), A.ptr(s["nk"]), A.ptr(s["nv"])))
    torch.cuda.synchronize()


@pytest.mark.parametrize("dt", ["fp16", "bf16", "fp32"])
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_decode_gate_table(case, dt):
    s = _setup(case, dt)
    _launch(s, dt)
    ro, rl = s["ref"]
    e = O.rel_rms(to_np(s["o"]), ro)
    assert e < TOL[dt], f"O rel_rms {e:.3e}"
    el = O.rel_rms(s["lse"].cpu().numpy(), rl)
    assert el < TOL[dt], f"LSE rel_rms {el:.3e}"
    assert int(s["err"].item()) == 0


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_decode_append_placement_bit_exact(dt):
    """New V rows land verbatim at block_table[b][pos//page], slot pos%page, pos = ctx+tk;
    un-rotated K rows likewise; every other cache byte is untouched."""
    case = ("placement", 64, 8, 2, 45, -1, 0, True, 0, 4, 0.0, False)
    s = _setup(case, dt)
    kc0, vc0 = s["kc"].clone(), s["vc"].clone()
    _launch(s, dt)
    kexp, vexp = kc0.clone(), vc0.clone()
    for b in range(2):
        for tk in range(4):
            pos = int(s["ctxs"][b]) + tk
            blk, slot = int(s["bt"][b][pos // PAGE]), pos % PAGE
            kexp[blk, slot] = s["nk"][b, tk]
            vexp[blk, slot] = s["nv"][b, tk]
    assert torch.equal(s["kc"].view(torch.int16), kexp.view(torch.int16))
    assert torch.equal(s["vc"].view(torch.int16), vexp.view(torch.int16))


@pytest.mark.parametrize("nsplit", [1, 2, 7, 40])
def test_decode_split_count_invariance(nsplit):
    case = CASES[0]
    s = _setup(case, "bf16", nsplit=nsplit)
    _launch(s, "bf16")
    assert O.rel_rms(to_np(s["o"]), s["ref"][0]) < TOL["bf16"]


def test_decode_bad_page_index_sets_flag():
    """A block-table entry past the cache is never dereferenced: the position is skipped and the
    caller's error flag is raised."""
    case = CASES[1]
    s = _setup(case, "bf16")
    s["keep"]["bt"][0, 2] = 1 << 30
    _launch(s, "bf16")
    assert int(s["err"].item()) == 1


@pytest.mark.parametrize("in_dt,out_dt", [("fp32", "bf16"), ("fp32", "fp16"), ("bf16", "bf16"), ("fp32", "fp32")])
def test_combine_kernel(in_dt, out_dt):
    rng = np.random.default_rng(17)
    ns, B, S, H, D = 5, 2, 3, 8, 128
    opn, op = randn(rng, (ns, B, S, H, D), in_dt)
    lpn = (rng.standard_normal((ns, B, H, S)) * 3).astype(np.float32)
    lpn[:, 1, 2, 0] = -np.inf
    lp = torch.from_numpy(lpn).cuda()
    out = torch.empty((B, S, H, D), device="cuda", dtype=TDT[out_dt])
    lse = torch.empty((B, H, S), device="cuda", dtype=torch.float32)
    p = A.FaCombineParams()
    p.struct_size = C.sizeof(A.FaCombineParams)
    p.out_partial, p.in_dtype, p.lse_partial = A.ptr(op), A.DT[in_dt], A.ptr(lp)
    p.out, p.out_dtype, p.lse_out = A.ptr(out), A.DT[out_dt], A.ptr(lse)
    p.nsplit, p.B, p.S, p.H, p.D = ns, B, S, H, D
    A.check(A.lib().fa_combine_launch(C.byref(p), stream()))
    torch.cuda.synchronize()
    ro, rl = O.combine(opn, lpn)
    assert O.rel_rms(to_np(out), ro) < TOL[out_dt]
    got_l = lse.cpu().numpy()
    assert np.array_equal(np.isfinite(got_l), np.isfinite(rl))
    assert np.abs(got_l[np.isfinite(rl)] - rl[np.isfinite(rl)]).max() < 1e-4


# The tensor-core decode (one new token, 16-bit cache, head_dim 128, gqa <= 16): page sizes from
# one swizzle atom (8 rows) to two tiles, several work items per sequence (long contexts), a
# sequence with an empty context, and query-head groups that fill 1..16 of its 16 MMA rows.
TC_CASES = [
    # (name, page, ctxs, NH, gqa, window, leftpad, append, rotary, softcap, alibi)
    ("p256_long", 256, [5000, 3100, 129], 32, 4, -1, 0, False, 0, 0.0, False),
    ("p8_gqa8", 8, [1500, 700], 32, 8, -1, 0, False, 0, 0.0, False),
    ("p64_gqa16", 64, [2300, 1100], 32, 16, -1, 0, True, 1, 0.0, False),
    ("p128_gqa2_window", 128, [4000, 260], 16, 2, 700, 0, False, 0, 0.0, False),
    ("p32_gqa3_leftpad", 32, [3000, 900], 12, 3, -1, 130, False, 0, 30.0, True),
    ("p256_empty_seq", 256, [2000, 0, 777], 16, 4, -1, 0, False, 0, 0.0, False),
]


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("tc", TC_CASES, ids=[c[0] for c in TC_CASES])
def test_decode_tensor_core_envelope(tc, dt):
    name, page, ctxs, NH, gqa, window, leftpad, append, rotary, sc, al = tc
    case = (name, 128, NH, gqa, max(ctxs), window, rotary, append, leftpad, 1, sc, al)
    s = _setup(case, dt, page=page, ctxs=ctxs)
    _launch(s, dt)
    ro, rl = s["ref"]
    e = O.rel_rms(to_np(s["o"]), ro)
    assert e < TOL[dt], f"O rel_rms {e:.3e}"
    lse = s["lse"].cpu().numpy()
    fin = np.isfinite(rl)
    assert np.array_equal(np.isfinite(lse), fin)   # empty contexts: LSE -inf, O 0
    assert O.rel_rms(lse[fin], rl[fin]) < TOL[dt]
    assert int(s["err"].item()) == 0


# Several new tokens per sequence on the tensor-core decode (query rows = tokens x heads of a kv
# group, up to 16 per launch, larger groups in token chunks): token tk sits at position ctx + tk and, with append, sees the cache and new
# tokens 0..tk (the reference's multi-token decode, kernels/fa_decode.hip:57-252, nq <= 8).
TC_MULTI = [
    # (name, page, ctxs, NH, gqa, nq, window, leftpad, append, rotary, softcap, alibi)
    ("p64_gqa4_nq4_append_rot", 64, [2300, 1100], 32, 4, 4, -1, 0, True, 1, 0.0, False),
    ("p8_gqa8_nq2", 8, [1500, 700], 32, 8, 2, -1, 0, False, 0, 0.0, False),
    ("p128_gqa2_nq8_window", 128, [4000, 260], 16, 2, 8, 700, 0, True, 0, 0.0, False),
    ("p32_gqa3_nq5_leftpad_cap_alibi", 32, [3000, 900], 12, 3, 5, -1, 130, True, 0, 30.0, True),
    ("p256_gqa1_nq7_empty_seq", 256, [2000, 0, 777], 8, 1, 7, 64, 0, False, 2, 0.0, False),
    # more than 16 query rows: tokens in chunks of 16 / gqa, one launch each
    ("p64_gqa4_nq8_append_rot", 64, [2300, 1100], 32, 4, 8, -1, 0, True, 1, 0.0, False),
    ("p16_gqa16_nq3", 16, [900, 1300], 32, 16, 3, -1, 0, True, 0, 0.0, False),
    ("p128_gqa3_nq7_window_alibi", 128, [3000, 500], 12, 3, 7, 300, 0, True, 0, 0.0, True),
]


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("tc", TC_MULTI, ids=[c[0] for c in TC_MULTI])
def test_decode_tensor_core_multi_token(tc, dt, monkeypatch):
    name, page, ctxs, NH, gqa, nq, window, leftpad, append, rotary, sc, al = tc
    case = (name, 128, NH, gqa, max(ctxs), window, rotary, append, leftpad, nq, sc, al)
    s = _setup(case, dt, page=page, ctxs=ctxs)
    _launch(s, dt)
    ro, rl = s["ref"]
    assert O.rel_rms(to_np(s["o"]), ro) < TOL[dt]
    lse = s["lse"].cpu().numpy()
    fin = np.isfinite(rl)
    assert np.array_equal(np.isfinite(lse), fin)   # tokens that see no key: LSE -inf, O 0
    assert O.rel_rms(lse[fin], rl[fin]) < TOL[dt]
    assert int(s["err"].item()) == 0
    # the CUDA-core decode gives the same answer by other arithmetic (so the two paths differ in
    # their last bits, which shows the tensor-core kernel ran)
    tc_o = s["o"].clone()
    monkeypatch.setenv("FABLE_ATTN_DECODE_NO_TC", "1")
    s2 = _setup(case, dt, page=page, ctxs=ctxs)
    _launch(s2, dt)
    assert O.rel_rms(to_np(s2["o"]), ro) < TOL[dt]
    assert not torch.equal(tc_o, s2["o"])


@pytest.mark.parametrize("nsplit", [1, 3, 64])
def test_decode_tensor_core_split_invariance(nsplit):
    tc = TC_CASES[0]
    case = (tc[0], 128, tc[3], tc[4], max(tc[2]), -1, 0, False, 0, 1, 0.0, False)
    s = _setup(case, "bf16", nsplit=nsplit, page=tc[1], ctxs=tc[2])
    _launch(s, "bf16")
    assert O.rel_rms(to_np(s["o"]), s["ref"][0]) < TOL["bf16"]


@pytest.mark.parametrize("paged", [True, False])
@pytest.mark.parametrize("rotary", [False, True])
def test_kvcache_varlen_queries_one_launch_no_host_sync(paged, rotary):
    """flash_attn_with_kvcache(q (total_q, H, D), cu_seqlens_q=, max_seqlen_q=): sequence i's tokens
    attend to cache row i at positions cache_seqlens[i] + t, computed in one decode launch with no
    host synchronisation (torch's sync debug mode raises on one) and equal to per-sequence calls."""
    import fable_attn as fa
    g = torch.Generator(device="cuda").manual_seed(4)
    B, H, Hk, D, page = 3, 8, 2, 128, 64
    nq = [3, 1, 5]
    ctx = torch.tensor([500, 64, 1000], dtype=torch.int32, device="cuda")
    nper = 20
    if paged:
        kc = torch.randn(B * nper, page, Hk, D, device="cuda", dtype=torch.bfloat16, generator=g)
        vc = torch.randn_like(kc)
        bt = torch.randperm(B * nper, generator=torch.Generator().manual_seed(1)).view(B, nper).int().cuda()
    else:
        kc = torch.randn(B, 1024 + 64, Hk, D, device="cuda", dtype=torch.bfloat16, generator=g)
        vc = torch.randn_like(kc)
        bt = None
    q = torch.randn(sum(nq), H, D, device="cuda", dtype=torch.bfloat16, generator=g)
    cu = torch.tensor([0, 3, 4, 9], dtype=torch.int32, device="cuda")
    kw = {}
    if rotary:
        ang = torch.arange(2048, device="cuda", dtype=torch.float32)[:, None] * 0.01 * torch.arange(
            1, 33, device="cuda", dtype=torch.float32)[None]
        kw = dict(rotary_cos=ang.cos(), rotary_sin=ang.sin(), rotary_interleaved=False)
    if not paged:   # a dense cache must be a power-of-two long per row
        kc, vc = kc[:, :1024].contiguous(), vc[:, :1024].contiguous()
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        out, lse = fa.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=ctx, block_table=bt, cu_seqlens_q=cu,
                                              max_seqlen_q=5, return_softmax_lse=True, **kw)
    finally:
        torch.cuda.set_sync_debug_mode(0)
    assert out.shape == q.shape and lse.shape == (H, sum(nq))
    for i in range(B):
        a, b = int(cu[i]), int(cu[i + 1])
        ref, rl = fa.flash_attn_with_kvcache(q[a:b][None], kc if paged else kc[i:i + 1], vc if paged else vc[i:i + 1],
                                             cache_seqlens=ctx[i:i + 1], block_table=bt[i:i + 1] if paged else None,
                                             return_softmax_lse=True, **kw)
        assert (out[a:b].float() - ref[0].float()).norm() <= 2e-3 * ref.float().norm()
        assert torch.allclose(lse[:, a:b], rl[0], rtol=1e-4, atol=1e-4)
