"""Public-API parity on the GPU: the semantics checked by the reference's lab/parity_test.py,
lab/parity_new_api.py and package/tests/test_fable_attn.py, against an exact torch fp32
reference of the same op (ref_attn below restates lab/parity_new_api.py:36-75)."""
import math
import random

import pytest
import torch

import fable_attn as fa

pytestmark = pytest.mark.gpu
DEV = "cuda"


def ref_attn(q, k, v, scale, causal=False, chunk=0, qv=None, wl=None, wr=None, softcap=0.0, alibi=None, qpos=None):
    """Exact fp32 attention, (B,S,H,D).  alibi adds slope*(key - query) with the query index
    taken as the bottom-right-aligned position in decode (qpos) and as the row index otherwise."""
    q_, k_, v_ = (x.transpose(1, 2).float() for x in (q, k, v))
    B, H, Sq, _ = q_.shape
    if H != k_.shape[1]:
        k_ = k_.repeat_interleave(H // k_.shape[1], dim=1)
        v_ = v_.repeat_interleave(H // v_.shape[1], dim=1)
    s = q_ @ k_.transpose(-1, -2)
    if qv is not None:
        s = s + qv.transpose(1, 2).float() @ v_.transpose(-1, -2)
    s = softcap * torch.tanh(s * scale / softcap) if softcap and softcap > 0 else s * scale
    Sk = k_.shape[2]
    qi = torch.arange(Sq, device=q.device).view(-1, 1)
    ki = torch.arange(Sk, device=q.device).view(1, -1)
    delta = Sk - Sq
    if alibi is not None:
        base = qi if qpos is None else torch.full_like(qi, qpos)
        s = s + alibi.view(1, H, 1, 1).float() * (ki - base).float()
    mask = torch.zeros(Sq, Sk, device=q.device, dtype=torch.bool)
    if causal:
        mask |= ki > qi + delta
    if wl is not None and wl >= 0:
        mask |= ki < qi + delta - wl
    if wr is not None and wr >= 0:
        mask |= ki > qi + delta + wr
    if chunk:
        cs = ((qi + delta).clamp_min(0) // chunk) * chunk
        mask |= (ki < cs) | (ki >= cs + chunk)
    p = torch.nan_to_num(s.masked_fill(mask, float("-inf")).softmax(-1), nan=0.0)
    return (p @ v_).transpose(1, 2)


def rnd(*shape, dt=torch.float16):
    return torch.randn(*shape, device=DEV, dtype=dt)


def close(got, ref, tol=3e-3):
    e = (got.float() - ref.float()).abs().max().item()
    return e < tol and bool(torch.isfinite(got.float()).all()), e


def relerr(a, b):
    a, b = a.float(), b.float()
    return (a - b).norm().item() / (b.norm().item() + 1e-12)


@pytest.mark.parametrize("D", [16, 32, 48, 64, 80, 96, 112, 128, 160, 192, 224, 256, 40, 100, 144, 200, 255])
def test_head_dims_native_and_padded(D):
    torch.manual_seed(D)
    q, k, v = rnd(1, 128, 4, D), rnd(1, 128, 4, D), rnd(1, 128, 4, D)
    ok, e = close(fa.flash_attn_func(q, k, v, causal=True), ref_attn(q, k, v, D ** -0.5, causal=True), 6e-3)
    assert ok, e


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("kw,refkw", [
    (dict(causal=True), dict(causal=True)), (dict(window_size=(63, 0)), dict(wl=63, wr=0)),
    (dict(softcap=30.0), dict(softcap=30.0)), (dict(window_size=(32, 32)), dict(wl=32, wr=32)),
    (dict(window_size=(-1, 0)), dict(wr=0)), (dict(window_size=(0, 0)), dict(wl=0, wr=0)),
    (dict(window_size=(0, -1)), dict(wl=0)), (dict(window_size=(16, 48)), dict(wl=16, wr=48)),
    (dict(causal=True, attention_chunk=64), dict(causal=True, chunk=64)),
    (dict(causal=True, attention_chunk=37), dict(causal=True, chunk=37)),
    (dict(attention_chunk=128), dict(chunk=128)),
    (dict(causal=True, attention_chunk=128, window_size=(31, 0)), dict(causal=True, chunk=128, wl=31))])
def test_masks_and_modifiers(dtype, kw, refkw):
    torch.manual_seed(0)
    q, k, v = rnd(1, 256, 8, 128, dt=dtype), rnd(1, 256, 8, 128, dt=dtype), rnd(1, 256, 8, 128, dt=dtype)
    tol = 3e-3 if dtype == torch.float16 else 2e-2
    ok, e = close(fa.flash_attn_func(q, k, v, **kw), ref_attn(q, k, v, 128 ** -0.5, **refkw), tol)
    assert ok, e


def test_alibi():
    torch.manual_seed(1)
    H = 8
    q, k, v = rnd(1, 256, H, 128), rnd(1, 256, H, 128), rnd(1, 256, H, 128)
    al = -(2.0 ** (-torch.arange(1, H + 1, device=DEV, dtype=torch.float32) * 8.0 / H))
    ok, e = close(fa.flash_attn_func(q, k, v, alibi_slopes=al), ref_attn(q, k, v, 128 ** -0.5, alibi=al))
    assert ok, e


@pytest.mark.parametrize("Hk", [8, 4, 2, 1])
def test_gqa_mqa(Hk):
    torch.manual_seed(2)
    q = rnd(1, 256, 8, 128)
    k, v = rnd(1, 256, Hk, 128), rnd(1, 256, Hk, 128)
    assert close(fa.flash_attn_func(q, k, v), ref_attn(q, k, v, 128 ** -0.5))[0]


def test_sq_ne_sk_and_empty_rows():
    torch.manual_seed(3)
    k, v = rnd(1, 256, 8, 128), rnd(1, 256, 8, 128)
    q2 = rnd(1, 64, 8, 128)
    assert close(fa.flash_attn_func(q2, k, v, causal=True), ref_attn(q2, k, v, 128 ** -0.5, causal=True))[0]
    qbig, ksm, vsm = rnd(1, 256, 8, 128), rnd(1, 64, 8, 128), rnd(1, 64, 8, 128)
    o = fa.flash_attn_func(qbig, ksm, vsm, causal=True)
    assert close(o, ref_attn(qbig, ksm, vsm, 128 ** -0.5, causal=True))[0]
    assert bool((o[:, :192] == 0).all())


def test_packed_variants():
    torch.manual_seed(4)
    q, k, v = rnd(2, 64, 4, 64), rnd(2, 64, 4, 64), rnd(2, 64, 4, 64)
    qkv = torch.stack([q, k, v], dim=2)
    assert close(fa.flash_attn_qkvpacked_func(qkv, causal=True), ref_attn(q, k, v, 0.125, causal=True))[0]
    kv = torch.stack([k, v], dim=2)
    assert close(fa.flash_attn_kvpacked_func(q, kv, causal=True), ref_attn(q, k, v, 0.125, causal=True))[0]


@pytest.mark.parametrize("causal", [False, True])
def test_varlen_and_packed_varlen(causal):
    torch.manual_seed(5)
    lens = [128, 64, 200, 32]
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), device=DEV, dtype=torch.int32)
    tot = sum(lens)
    q, k, v = rnd(tot, 8, 128), rnd(tot, 8, 128), rnd(tot, 8, 128)
    o = fa.flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), causal=causal)
    ref = torch.cat([ref_attn(q[a:b][None], k[a:b][None], v[a:b][None], 128 ** -0.5, causal=causal)[0]
                     for a, b in zip(cu[:-1].tolist(), cu[1:].tolist())])
    assert close(o, ref)[0]
    assert torch.equal(fa.flash_attn_varlen_qkvpacked_func(torch.stack([q, k, v], 1), cu, max(lens), causal=causal), o)
    assert torch.equal(fa.flash_attn_varlen_kvpacked_func(q, torch.stack([k, v], 1), cu, cu, max(lens), max(lens),
                                                          causal=causal), o)


def test_varlen_seqused():
    torch.manual_seed(7)
    lens, uq, uk = [128, 64, 200], [70, 64, 150], [90, 30, 180]
    cu = torch.tensor([0, 128, 192, 392], device=DEV, dtype=torch.int32)
    q, k, v = rnd(392, 8, 128), rnd(392, 8, 128), rnd(392, 8, 128)
    out = fa.flash_attn_varlen_func(q, k, v, cu, cu, 200, 200, causal=True,
                                    seqused_q=torch.tensor(uq, device=DEV, dtype=torch.int32),
                                    seqused_k=torch.tensor(uk, device=DEV, dtype=torch.int32))
    exp = torch.zeros_like(out)
    for i, a in enumerate([0, 128, 192]):
        exp[a:a + uq[i]] = ref_attn(q[a:a + uq[i]][None], k[a:a + uk[i]][None], v[a:a + uk[i]][None], 128 ** -0.5,
                                    causal=True)[0]
    assert close(out, exp)[0]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("causal", [False, True])
def test_backward_vs_torch_autograd(dtype, causal):
    torch.manual_seed(1)
    q, k, v = (rnd(2, 96, 4, 64, dt=dtype).requires_grad_() for _ in range(3))
    qr, kr, vr = (x.detach().float().requires_grad_() for x in (q, k, v))
    g = rnd(2, 96, 4, 64, dt=dtype)
    fa.flash_attn_func(q, k, v, causal=causal).backward(g)
    ref_attn(qr, kr, vr, 0.125, causal=causal).backward(g.float())
    tol = 1e-2 if dtype == torch.bfloat16 else 2e-3
    for a, b in ((q.grad, qr.grad), (k.grad, kr.grad), (v.grad, vr.grad)):
        assert relerr(a, b) < tol


def test_backward_gqa_varlen_and_big_dims():
    torch.manual_seed(2)
    lens = [70, 128, 33]
    cu = torch.tensor([0, 70, 198, 231], device=DEV, dtype=torch.int32)
    q = rnd(231, 8, 64).requires_grad_()
    k = rnd(231, 2, 64).requires_grad_()
    v = rnd(231, 2, 64).requires_grad_()
    fa.flash_attn_varlen_func(q, k, v, cu, cu, 128, 128, causal=True).sum().backward()
    qr, kr, vr = (x.detach().float().requires_grad_() for x in (q, k, v))
    outs = [ref_attn(qr[a:b][None], kr[a:b][None], vr[a:b][None], 0.125, causal=True)[0]
            for a, b in zip(cu[:-1].tolist(), cu[1:].tolist())]
    torch.cat(outs).sum().backward()
    for a, b in ((q.grad, qr.grad), (k.grad, kr.grad), (v.grad, vr.grad)):
        assert relerr(a, b) < 3e-3
    for D in (192, 256):
        x = rnd(1, 64, 2, D).requires_grad_()
        fa.flash_attn_func(x, x.detach(), x.detach(), causal=True).sum().backward()
        assert bool(torch.isfinite(x.grad).all())


def test_determinism_and_layout_independence():
    torch.manual_seed(12)
    q, k, v = (rnd(2, 256, 8, 128) for _ in range(3))
    o = fa.flash_attn_func(q, k, v, causal=True)
    assert o.is_contiguous()
    o.view(2, 256, 8 * 128)
    assert torch.equal(o, fa.flash_attn_func(q, k, v, causal=True))
    assert torch.equal(o, fa.flash_attn_func(q, k.contiguous(), v.contiguous(), causal=True))
    og = fa.flash_attn_func(q.clone().requires_grad_(), k, v, causal=True)
    assert og.is_contiguous() and torch.equal(og.detach(), o)
    base = fa.flash_attn_func(q, k, v, causal=True)
    for kw in (dict(num_splits=4), dict(pack_gqa=True), dict(sm_margin=8), dict(deterministic=True)):
        assert torch.equal(fa.flash_attn_func(q, k, v, causal=True, **kw), base)


def test_qv_and_headdim_v():
    torch.manual_seed(4)
    q, k, v, qv = rnd(1, 256, 8, 128), rnd(1, 256, 8, 128), rnd(1, 256, 8, 128), rnd(1, 256, 8, 128)
    for causal in (False, True):
        assert close(fa.flash_attn_func(q, k, v, causal=causal, qv=qv),
                     ref_attn(q, k, v, 256 ** -0.5, causal=causal, qv=qv), 6e-3)[0]
    q64, k64, v192 = rnd(1, 256, 8, 64), rnd(1, 256, 8, 64), rnd(1, 256, 8, 192)
    assert close(fa.flash_attn_func(q64, k64, v192, causal=True, softmax_scale=0.125),
                 ref_attn(q64, k64, v192, 0.125, causal=True), 6e-3)[0]
    v80, qv80 = rnd(1, 256, 8, 80), rnd(1, 256, 8, 80)
    assert close(fa.flash_attn_func(q, k, v80, causal=True, qv=qv80),
                 ref_attn(q, k, v80, 208 ** -0.5, causal=True, qv=qv80), 6e-3)[0]
    with pytest.raises(NotImplementedError, match="256"):
        fa.flash_attn_func(q, k, rnd(1, 256, 8, 160), qv=rnd(1, 256, 8, 160))


def test_return_attn_probs_and_combine():
    torch.manual_seed(6)
    q, k, v = rnd(1, 256, 8, 128), rnd(1, 256, 8, 128), rnd(1, 256, 8, 128)
    o, lse, p = fa.flash_attn_func(q, k, v, causal=True, return_attn_probs=True)
    assert tuple(lse.shape) == (1, 8, 256) and tuple(p.shape) == (1, 8, 256, 256)
    assert float((p.sum(-1) - 1).abs().max()) < 3e-3
    assert close((p @ v.transpose(1, 2).float()).transpose(1, 2), o.float())[0]
    o1, l1, _ = fa.flash_attn_func(q, k[:, :128], v[:, :128], return_attn_probs=True)
    o2, l2, _ = fa.flash_attn_func(q, k[:, 128:], v[:, 128:], return_attn_probs=True)
    got = fa.flash_attn_combine(torch.stack([o1, o2]).float(), torch.stack([l1, l2]), out_dtype=torch.float16)
    assert close(got, ref_attn(q, k, v, 128 ** -0.5), 6e-3)[0]


def test_kvcache_paged_and_extras():
    torch.manual_seed(9)
    H, Hk, D, page, ctx = 8, 2, 128, 32, 400
    nblk = (ctx + page - 1) // page
    qd = rnd(1, 1, H, D)
    kc, vc = rnd(nblk, page, Hk, D), rnd(nblk, page, Hk, D)
    bt = torch.arange(nblk, device=DEV, dtype=torch.int32).view(1, nblk)
    cs = torch.tensor([ctx], device=DEV, dtype=torch.int32)
    kd = kc.reshape(nblk * page, Hk, D)[:ctx][None]
    vd = vc.reshape(nblk * page, Hk, D)[:ctx][None]
    sc = D ** -0.5
    for lp in (0, 37, 100):
        o = fa.flash_attn_with_kvcache(qd, kc, vc, cache_seqlens=cs, block_table=bt,
                                       cache_leftpad=torch.tensor([lp], device=DEV, dtype=torch.int32))
        assert close(o, ref_attn(qd, kd[:, lp:], vd[:, lp:], sc))[0]
    assert torch.equal(fa.flash_attn_with_kvcache(qd, kc, vc, cache_seqlens=cs, page_table=bt),
                       fa.flash_attn_with_kvcache(qd, kc, vc, cache_seqlens=cs, block_table=bt))
    o, lse = fa.flash_attn_with_kvcache(qd, kc, vc, cache_seqlens=cs, block_table=bt, return_softmax_lse=True)
    s = (qd.transpose(1, 2).float() @ kd.transpose(1, 2).float().repeat_interleave(H // Hk, 1).transpose(-1, -2)) * sc
    assert close(lse, torch.logsumexp(s, -1), 1e-2)[0]
    Bd, Sd, L = 4, 256, 100
    qdd, kcd, vcd = rnd(Bd, 1, H, D), rnd(Bd, Sd, Hk, D), rnd(Bd, Sd, Hk, D)
    idx = torch.tensor([3, 1, 0, 2], device=DEV, dtype=torch.int32)
    o = fa.flash_attn_with_kvcache(qdd, kcd, vcd, cache_seqlens=L, cache_batch_idx=idx)
    exp = torch.cat([ref_attn(qdd[b:b + 1], kcd[idx[b]:idx[b] + 1, :L], vcd[idx[b]:idx[b] + 1, :L], sc)
                     for b in range(Bd)])
    assert close(o, exp)[0]


def test_kvcache_softcap_alibi_multitoken_append():
    torch.manual_seed(10)
    Hk2, D2, L2 = 2, 64, 100
    sc2 = D2 ** -0.5
    qd = rnd(2, 1, 8, D2)
    kcd, vcd = rnd(2, 256, Hk2, D2), rnd(2, 256, Hk2, D2)
    assert close(fa.flash_attn_with_kvcache(qd, kcd, vcd, cache_seqlens=L2, softcap=30.0),
                 ref_attn(qd, kcd[:, :L2], vcd[:, :L2], sc2, softcap=30.0), 6e-3)[0]
    al = (-0.1 * torch.arange(1, 9, device=DEV)).float()
    assert close(fa.flash_attn_with_kvcache(qd, kcd, vcd, cache_seqlens=L2, alibi_slopes=al),
                 ref_attn(qd, kcd[:, :L2], vcd[:, :L2], sc2, alibi=al, qpos=L2), 6e-3)[0]
    qm = rnd(2, 4, 8, D2)
    assert close(fa.flash_attn_with_kvcache(qm, kcd, vcd, cache_seqlens=L2),
                 ref_attn(qm, kcd[:, :L2], vcd[:, :L2], sc2), 6e-3)[0]
    kc2, vc2 = kcd.clone(), vcd.clone()
    kn, vn = rnd(2, 4, Hk2, D2), rnd(2, 4, Hk2, D2)
    oa = fa.flash_attn_with_kvcache(qm, kc2, vc2, k=kn, v=vn, cache_seqlens=L2)
    exp = torch.stack([ref_attn(qm[:, i:i + 1], torch.cat([kcd[:, :L2], kn[:, :i + 1]], 1),
                                torch.cat([vcd[:, :L2], vn[:, :i + 1]], 1), sc2)[:, 0] for i in range(4)], 1)
    assert close(oa, exp, 6e-3)[0]
    assert torch.equal(kc2[:, L2:L2 + 4], kn) and torch.equal(vc2[:, L2:L2 + 4], vn)


def test_paged_varlen_prefill_and_probs_list():
    torch.manual_seed(11)
    lens, page, H, D = [96, 64], 32, 8, 128
    cu = torch.tensor([0, 96, 160], device=DEV, dtype=torch.int32)
    q = rnd(160, H, D)
    kp, vp = rnd(5, page, H, D), rnd(5, page, H, D)
    bt = torch.tensor([[0, 1, 2], [3, 4, 0]], device=DEV, dtype=torch.int32)
    o = fa.flash_attn_varlen_func(q, kp, vp, cu, cu, 96, 96, causal=True, block_table=bt)
    exp = []
    for i, L in enumerate(lens):
        nb = (L + page - 1) // page
        kd = kp[bt[i, :nb].long()].reshape(-1, H, D)[:L]
        vd = vp[bt[i, :nb].long()].reshape(-1, H, D)[:L]
        a = int(cu[i])
        exp.append(ref_attn(q[a:a + L][None], kd[None], vd[None], D ** -0.5, causal=True)[0])
    assert close(o, torch.cat(exp))[0]
    r = fa.flash_attn_varlen_func(q, q, q, cu, cu, 96, 96, return_attn_probs=True)
    assert isinstance(r, tuple) and len(r) == 3 and tuple(r[2][0].shape) == (H, 96, 96)


def test_rejections():
    q = rnd(1, 32, 2, 64)
    with pytest.raises(NotImplementedError, match="FP8"):
        fa.flash_attn_func(q, q, q, q_descale=torch.ones(1, device=DEV))
    with pytest.raises(TypeError):
        fa.flash_attn_func(q, q, q, num_splits="many")
    qg = rnd(1, 128, 4, 64).requires_grad_()
    with pytest.raises(NotImplementedError):
        fa.flash_attn_func(qg, qg.detach(), qg.detach(), causal=True, attention_chunk=64).sum().backward()
    with pytest.raises(ValueError):
        fa.flash_attn_func(q, rnd(1, 32, 3, 64), rnd(1, 32, 3, 64))


def test_install_as_flash_attn_and_fa3_order():
    fa.install_as_flash_attn()
    import flash_attn
    import flash_attn_interface as fa3
    from flash_attn.bert_padding import pad_input, unpad_input  # noqa: F401
    assert flash_attn.__version__.startswith("2.")
    torch.manual_seed(8)
    q, k, v = (rnd(1, 64, 2, 64) for _ in range(3))
    assert close(fa3.flash_attn_func(q, k, v, 0.125, True), ref_attn(q, k, v, 0.125, causal=True))[0]
    o, lse = fa3.flash_attn_func(q, k, v, 0.125, True, return_attn_probs=True)
    assert o.shape == q.shape and tuple(lse.shape) == (1, 2, 64)
    assert fa3.get_scheduler_metadata() is None


def test_torch_op_contract():
    torch.manual_seed(13)
    q, k, v = (rnd(1, 4, 128, 64) for _ in range(3))   # [B, H, S, D]
    o = torch.ops.fable_attn.forward(q, k, v, 0.125, True)
    ref = ref_attn(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), 0.125, causal=True).transpose(1, 2)
    assert close(o, ref)[0]
    assert torch.ops.fable_attn.forward(q.float(), k.float(), v.float(), 0.125, True).numel() == 0


def test_vram_no_s_by_s():
    torch.manual_seed(13)
    q, k, v = (rnd(2, 4096, 16, 128) for _ in range(3))
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    o = fa.flash_attn_func(q, k, v, causal=True)
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated() - base
    del o
    assert peak < 2 * 4096 * 16 * 128 * 2 * 2   # out + LSE, far below the 4 GiB of an SxS fp32 matrix


@pytest.mark.parametrize("cap_mb", ["0", "4"])
def test_vram_no_s_by_s_with_dropout(monkeypatch, cap_mb):
    """Training with dropout keeps O(S) memory once the per-call keep-mask cap is exceeded (here
    16 heads x 4096^2 causal bits = 32 MiB > the cap): nothing S x S lives from the forward to the
    backward, and the gradients equal those computed with the mask (bitwise)."""
    torch.manual_seed(14)
    q, k, v, do = (rnd(2, 4096, 16, 128) for _ in range(4))
    # the same forward kernel in both runs (the keep bits come from the mask or from Philox in the
    # kernel: the same decisions, so the same bits everywhere)
    monkeypatch.setenv("FABLE_ATTN_FWD_TILES", "1")
    grads = {}
    for mode in ("mask", "philox"):
        if mode == "philox":
            monkeypatch.setenv("FABLE_ATTN_DROPOUT_MASK_MAX_MB", cap_mb)
        qa, ka, va = (t.clone().requires_grad_() for t in (q, k, v))
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats()
        base = torch.cuda.memory_allocated()
        random.seed(5)
        o = fa.flash_attn_func(qa, ka, va, dropout_p=0.1, causal=True)
        torch.cuda.synchronize()
        held = torch.cuda.memory_allocated() - base        # what autograd keeps until the backward
        o.backward(do)
        grads[mode] = (o.detach(), qa.grad, ka.grad, va.grad)
        if mode == "philox":
            assert held < 2 * (2 * 4096 * 16 * 128 * 2) + 2 * 16 * 4096 * 4 * 2, held   # out + LSE (+ slack)
    for a, b in zip(grads["mask"], grads["philox"]):
        assert torch.equal(a, b)
