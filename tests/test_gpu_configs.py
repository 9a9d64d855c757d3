"""Parity at the BASELINE configs' own shapes, through the public API, against the oracle.

The gate tables (test_gpu_forward / _backward / _decode) cover every feature at small shapes, as
the reference's kernel gates do (kernels/fa_forward_gate.inc:33-80, kernels/backward.hip:610-631,
kernels/fa_decode_gate.inc:110-131).  These tests run the five benchmark configurations at full
size and compare with the float64 oracle:
  1  B1 S512 H8 D64 fp32 causal                 every row and head, O and LSE at 1e-5
  2  B1 S16384 H32 D128 bf16 non-causal          every row computed; 4 blocks of 64 rows in each of
                                                 3 heads checked (the oracle's cost is per row)
  3  B2 S4096 H32 D128 fp16 causal, dropout 0.1  O, LSE, dQ, dK, dV of 2 (batch, head) pairs in full
                                                 at 3e-4; keep-mask words of sampled rows bit-exact
  4  paged decode B16 Hq32 Hk8 D128 bf16, page 256, 2048 permuted pages, ctx ~ U[16K, 32K]:
                                                 every row, O and LSE; the append of one token per
                                                 sequence lands bit-exactly at its page slot
  5  varlen SWA prefill, 16 seqs ~ U[256, 8192], Hq64 Hk8 D128 bf16, window (512, 0), softcap 30,
     NeoX rotary rd 64 (fused in the kernel and rotate-then-attend): one query head of every kv
     group (8 of 64), every sequence and row, O and LSE
Inputs are N(0,1) in the tested dtype from generators seeded per config (numpy for configs 1-3,
torch's CUDA generator for the multi-GB tensors of configs 4 and 5); the oracle reads the same
rounded values, copied back to the host for the heads it checks.  Each test prints the rel_rms
it measured."""
import random

import numpy as np
import pytest
import torch

import fable_attn as fa
from fable_attn import _C
from gpu_util import TDT, TOL, to_np
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _rand(rng, shape, dt):
    x = O.round_to(rng.standard_normal(shape, dtype=np.float32), dt)
    return x, torch.from_numpy(x).to("cuda", TDT[dt])


def _dev_rand(gen, shape, dt):
    return torch.randn(shape, device="cuda", dtype=TDT[dt], generator=gen)


def _lse_rel(got, ref):
    fin = np.isfinite(ref)
    assert np.array_equal(fin, np.isfinite(got)), "empty-row pattern differs"
    return O.rel_rms(got[fin], ref[fin]) if fin.any() else 0.0


def test_config1_fp32_causal_full():
    rng = np.random.default_rng(1)
    B, S, H, D = 1, 512, 8, 64
    qn, q = _rand(rng, (B, S, H, D), "fp32")
    kn, k = _rand(rng, (B, S, H, D), "fp32")
    vn, v = _rand(rng, (B, S, H, D), "fp32")
    out, lse, _ = fa.flash_attn_func(q, k, v, softmax_scale=1 / 8, causal=True, return_attn_probs=True)
    ro, rl = O.forward(qn, kn, vn, 1 / 8, True)
    e, el = O.rel_rms(to_np(out), ro), _lse_rel(lse.cpu().numpy(), rl)
    print(f"config1 fp32: O {e:.2e} LSE {el:.2e}")
    assert e < TOL["fp32"] and el < TOL["fp32"]
    if O.ref_lib() is not None:   # and the reference's own ref_attention on the same inputs
        ro2, rl2 = O.ref_forward(qn[0], kn[0], vn[0], 1 / 8, True)
        assert O.rel_rms(to_np(out)[0], ro2) < TOL["fp32"]
        assert _lse_rel(lse.cpu().numpy()[0], rl2) < TOL["fp32"]


def test_config2_dense_bf16_s16384_sampled_rows():
    rng = np.random.default_rng(2)
    B, S, H, D = 1, 16384, 32, 128
    qn, q = _rand(rng, (B, S, H, D), "bf16")
    kn, k = _rand(rng, (B, S, H, D), "bf16")
    vn, v = _rand(rng, (B, S, H, D), "bf16")
    out = fa.flash_attn_func(q, k, v)
    out_c, lse = _C.fwd(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), D ** -0.5, False, -1, -1, 0.0, None,
                        0.0, 0)
    torch.cuda.synchronize()
    assert torch.equal(out, out_c.transpose(1, 2)), "public API and _C.fwd disagree"
    on, ln = to_np(out), lse.cpu().numpy()
    worst = 0.0
    for h in (0, 13, 31):
        for r0 in sorted(rng.choice(S // 64, 4, replace=False) * 64):
            ro, rl = O.forward(qn[:, :, h:h + 1], kn[:, :, h:h + 1], vn[:, :, h:h + 1], D ** -0.5,
                               rows=(int(r0), int(r0) + 64))
            e = O.rel_rms(on[0, r0:r0 + 64, h], ro[0, r0:r0 + 64, 0])
            el = _lse_rel(ln[0, h, r0:r0 + 64], rl[0, 0, r0:r0 + 64])
            worst = max(worst, e, el)
            assert e < TOL["bf16"] and el < TOL["bf16"], f"head {h} rows {r0}: O {e:.2e} LSE {el:.2e}"
    print(f"config2 bf16 S16384: worst rel_rms over 768 sampled rows {worst:.2e}")


def test_config3_causal_fwd_bwd_fp16_dropout():
    rng = np.random.default_rng(3)
    B, S, H, D, p = 2, 4096, 32, 128, 0.1
    qn, q = _rand(rng, (B, S, H, D), "fp16")
    kn, k = _rand(rng, (B, S, H, D), "fp16")
    vn, v = _rand(rng, (B, S, H, D), "fp16")
    don, do = _rand(rng, (B, S, H, D), "fp16")
    for t in (q, k, v):
        t.requires_grad_()
    # the reference draws the Philox seed with random.getrandbits(63); seeding `random` fixes it
    random.seed(3)
    seed = random.getrandbits(63)
    random.seed(3)
    out = fa.flash_attn_func(q, k, v, dropout_p=p, causal=True, deterministic=True)
    out.backward(do)
    qh, kh, vh = (t.detach().transpose(1, 2) for t in (q, k, v))
    bits = _C.dropout_mask(qh, seed, p, H, S, S, True, -1, 0)
    out_c, lse = _C.fwd(qh, kh, vh, D ** -0.5, True, -1, 0, 0.0, None, p, seed, 0, None, bits)
    torch.cuda.synchronize()
    assert torch.equal(out.detach(), out_c.transpose(1, 2)), "public API and _C.fwd (same seed) disagree"
    # keep-mask words of sampled rows, bit-exact against Philox in the oracle
    W = (S + 31) // 32
    words = bits.cpu().numpy().view(np.uint32).reshape(H, W, S)
    for h in (0, 9, 31):
        for r in rng.choice(S, 6, replace=False):
            ref = O.dropout_block(seed, h, S, S, p, int(r), int(r) + 1, 0, S)[0]
            vis = np.arange(S) <= r
            got = (words[h, np.arange(S) // 32, r] >> (np.arange(S) % 32).astype(np.uint32)) & 1
            assert np.array_equal(got[vis], ref[vis]), f"keep bits of head {h} row {r} differ"
    on, ln = to_np(out.detach()), lse.cpu().numpy()
    gq, gk, gv = to_np(q.grad), to_np(k.grad), to_np(v.grad)
    for b, h in ((0, 5), (1, 30)):
        r = O.attention_head(qn[b, :, h], kn[b, :, h], vn[b, :, h], D ** -0.5, causal=True, dropout_p=p, seed=seed,
                             h=h, do=don[b, :, h])
        errs = {"O": O.rel_rms(on[b, :, h], r["O"]), "LSE": _lse_rel(ln[b, h], r["LSE"]),
                "dQ": O.rel_rms(gq[b, :, h], r["dQ"]), "dK": O.rel_rms(gk[b, :, h], r["dK"]),
                "dV": O.rel_rms(gv[b, :, h], r["dV"])}
        print(f"config3 fp16 (b={b}, h={h}):", {n: f"{x:.2e}" for n, x in errs.items()})
        bad = {n: x for n, x in errs.items() if not x < TOL["fp16"]}
        assert not bad, f"(b={b}, h={h}) above the fp16 bar: {bad}"


def _config4(seed, append):
    B, Hq, Hk, D, page, maxctx = 16, 32, 8, 128, 256, 32768
    nper = maxctx // page
    rng = np.random.default_rng(seed)
    gen = torch.Generator(device="cuda").manual_seed(seed)
    kc, vc = _dev_rand(gen, (B * nper, page, Hk, D), "bf16"), _dev_rand(gen, (B * nper, page, Hk, D), "bf16")
    q = _dev_rand(gen, (B, 1, Hq, D), "bf16")
    bt = rng.permutation(B * nper).astype(np.int32).reshape(B, nper)
    lens = rng.integers(16384, 32768 if append else 32769, size=B).astype(np.int32)
    nk = nv = None
    if append:
        nk, nv = _dev_rand(gen, (B, 1, Hk, D), "bf16"), _dev_rand(gen, (B, 1, Hk, D), "bf16")
    host = lambda t: None if t is None else t.float().cpu().numpy()   # noqa: E731
    return dict(B=B, page=page, kc=kc, vc=vc, bt=bt, lens=lens, q=q, nk=nk, nv=nv, kcn=host(kc), vcn=host(vc),
                qn=host(q), nkn=host(nk), nvn=host(nv))


def test_config4_paged_decode_full():
    c = _config4(4, append=False)
    out, lse = fa.flash_attn_with_kvcache(c["q"], c["kc"], c["vc"], cache_seqlens=torch.from_numpy(c["lens"]).cuda(),
                                         block_table=torch.from_numpy(c["bt"]).cuda(), return_softmax_lse=True)
    ro, rl = O.decode(c["qn"], c["kcn"], c["vcn"], c["bt"], c["lens"])
    e = O.rel_rms(to_np(out), ro)
    el = _lse_rel(lse.cpu().numpy(), rl.transpose(0, 2, 1))
    print(f"config4 bf16 decode: O {e:.2e} LSE {el:.2e}")
    assert e < TOL["bf16"] and el < TOL["bf16"]


def test_config4_append_lands_bit_exact():
    c = _config4(44, append=True)
    kc0, vc0 = c["kc"].clone(), c["vc"].clone()
    out = fa.flash_attn_with_kvcache(c["q"], c["kc"], c["vc"], k=c["nk"], v=c["nv"],
                                     cache_seqlens=torch.from_numpy(c["lens"]).cuda(),
                                     block_table=torch.from_numpy(c["bt"]).cuda())
    torch.cuda.synchronize()
    kexp, vexp = kc0, vc0
    for b in range(c["B"]):
        pos = int(c["lens"][b])
        blk, slot = int(c["bt"][b][pos // c["page"]]), pos % c["page"]
        kexp[blk, slot] = c["nk"][b, 0]
        vexp[blk, slot] = c["nv"][b, 0]
    assert torch.equal(c["kc"].view(torch.int16), kexp.view(torch.int16)), "K cache bytes differ"
    assert torch.equal(c["vc"].view(torch.int16), vexp.view(torch.int16)), "V cache bytes differ"
    ro, _ = O.decode(c["qn"], c["kcn"], c["vcn"], c["bt"], c["lens"], c["nkn"], c["nvn"])
    e = O.rel_rms(to_np(out), ro)
    print(f"config4 bf16 decode with append: O {e:.2e}")
    assert e < TOL["bf16"]


@pytest.mark.parametrize("fused", [True, False], ids=["fused_rotary", "rotate_then_attend"])
def test_config5_varlen_swa_softcap_rotary(fused):
    from fable_attn.layers.rotary import apply_rotary_emb
    rng = np.random.default_rng(5)
    lens = rng.integers(256, 8193, size=16)
    cu_np = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    tot, Hq, Hk, D, rd = int(lens.sum()), 64, 8, 128, 64
    gen = torch.Generator(device="cuda").manual_seed(5)
    q, k, v = (_dev_rand(gen, (tot, hh, D), "bf16") for hh in (Hq, Hk, Hk))
    heads = [8 * g + (3 * g) % 8 for g in range(Hk)]   # one query head of every kv group
    qn = q[:, heads].float().cpu().numpy()
    kn, vn = k.float().cpu().numpy(), v.float().cpu().numpy()
    inv = 10000.0 ** (-np.arange(0, rd, 2, dtype=np.float32) / rd)
    ang = np.arange(int(lens.max()), dtype=np.float32)[:, None] * inv[None]
    cos, sin = torch.from_numpy(np.cos(ang)), torch.from_numpy(np.sin(ang))
    cu = torch.from_numpy(cu_np).cuda()
    mx, sc = int(lens.max()), D ** -0.5
    kw = dict(softmax_scale=sc, causal=True, window_size=(512, 0), softcap=30.0)
    if fused:
        out = fa.flash_attn_varlen_func(q, k, v, cu, cu, mx, mx, rotary_cos=cos.cuda(), rotary_sin=sin.cuda(), **kw)
    else:
        qr = apply_rotary_emb(q, cos.cuda(), sin.cuda(), cu_seqlens=cu, max_seqlen=mx)
        kr = apply_rotary_emb(k, cos.cuda(), sin.cuda(), cu_seqlens=cu, max_seqlen=mx)
        out = fa.flash_attn_varlen_func(qr, kr, v, cu, cu, mx, mx, **kw)
    # LSE of the same call through the extension (same kernel; the output must agree bitwise)
    out2, lse = _C.fwd_varlen(q, k, v, cu, cu, mx, mx, sc, True, 512, 0, 30.0, None, 0.0, 0, 0, None, None, True,
                              rotary_cos=cos.cuda(), rotary_sin=sin.cuda(), rotary_interleaved=False)
    torch.cuda.synchronize()
    if fused:
        assert torch.equal(out, out2)
    # the oracle rotates with the reference's torch arithmetic (host tensors, bf16 roundings)
    cu_cpu = torch.from_numpy(cu_np)
    qrn = apply_rotary_emb(torch.from_numpy(qn).bfloat16(), cos, sin, cu_seqlens=cu_cpu).float().numpy()
    krn = apply_rotary_emb(torch.from_numpy(kn).bfloat16(), cos, sin, cu_seqlens=cu_cpu).float().numpy()
    on, ln = to_np(out), lse.cpu().numpy()
    num = den = lnum = lden = 0.0
    for g, h in enumerate(heads):
        for i in range(16):
            a, b = int(cu_np[i]), int(cu_np[i + 1])
            r = O.attention_head(qrn[a:b, g], krn[a:b, g], vn[a:b, g], sc, causal=True, wl=512, wr=0, softcap=30.0)
            num += float(((on[a:b, h] - r["O"]) ** 2).sum())
            den += float((r["O"] ** 2).sum())
            lnum += float(((ln[h, a:b] - r["LSE"]) ** 2).sum())
            lden += float((r["LSE"] ** 2).sum())
    e, el = (num / den) ** 0.5, (lnum / lden) ** 0.5
    print(f"config5 bf16 ({'fused' if fused else 'unfused'} rotary): O {e:.2e} LSE {el:.2e}")
    assert e < TOL["bf16"] and el < TOL["bf16"]
