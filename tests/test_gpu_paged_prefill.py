"""Paged varlen prefill (flash_attn_varlen_func with block_table) read in place by the forward
kernels: bitwise equal to the same call on K/V gathered into packed varlen form, for page sizes
from 16 to 256 (tensor-core kernel: fp16/bf16 D=128; CUDA-core kernel: fp32 and D=96), with
seqused_k, causal and sliding-window masks, and keys longer than queries."""
import pytest
import torch

import fable_attn as fa

pytestmark = pytest.mark.gpu


def _case(dt, D, page, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    lq = [300, 1, 129, 64]
    lk = [700, 17, 129, 300]
    H, Hk = 8, 2
    nper = max((L + page - 1) // page for L in lk)
    nblocks = len(lk) * nper + 5
    kc = torch.randn(nblocks, page, Hk, D, device="cuda", dtype=dt, generator=g)
    vc = torch.randn(nblocks, page, Hk, D, device="cuda", dtype=dt, generator=g)
    perm = torch.randperm(nblocks, generator=torch.Generator().manual_seed(seed))[: len(lk) * nper]
    bt = perm.view(len(lk), nper).to(torch.int32).cuda()
    q = torch.randn(sum(lq), H, D, device="cuda", dtype=dt, generator=g)
    cq = torch.tensor([0] + list(torch.tensor(lq).cumsum(0)), dtype=torch.int32, device="cuda")
    ck = torch.tensor([0] + list(torch.tensor(lk).cumsum(0)), dtype=torch.int32, device="cuda")
    # packed form of the same keys
    ks = [kc[bt[i, :(L + page - 1) // page].long()].reshape(-1, Hk, D)[:L] for i, L in enumerate(lk)]
    vs = [vc[bt[i, :(L + page - 1) // page].long()].reshape(-1, Hk, D)[:L] for i, L in enumerate(lk)]
    return q, kc, vc, bt, cq, ck, torch.cat(ks), torch.cat(vs), max(lq), max(lk)


@pytest.mark.parametrize("dt,D", [(torch.float16, 128), (torch.bfloat16, 128), (torch.float32, 128),
                                  (torch.bfloat16, 96)])
@pytest.mark.parametrize("page", [16, 64, 256])
@pytest.mark.parametrize("mask", ["causal", "window", "full"])
def test_paged_prefill_equals_packed(dt, D, page, mask):
    q, kc, vc, bt, cq, ck, kp, vp, mq, mk = _case(dt, D, page)
    kw = dict(causal=mask != "full", window_size=(100, 0) if mask == "window" else (-1, -1))
    with torch.no_grad():
        got = fa.flash_attn_varlen_func(q, kc, vc, cq, ck, mq, mk, block_table=bt, **kw)
        ref = fa.flash_attn_varlen_func(q, kp, vp, cq, ck, mq, mk, **kw)
    assert torch.equal(got, ref)


def test_paged_prefill_seqused_and_autograd_path():
    q, kc, vc, bt, cq, ck, kp, vp, mq, mk = _case(torch.bfloat16, 128, 64, seed=3)
    used = torch.tensor([650, 17, 100, 299], dtype=torch.int32, device="cuda")
    with torch.no_grad():
        got = fa.flash_attn_varlen_func(q, kc, vc, cq, ck, mq, mk, causal=True, block_table=bt, seqused_k=used)
    # reference: pack only the used keys
    lk = (ck[1:] - ck[:-1]).tolist()
    ks, vs, offs = [], [], [0]
    for i, L in enumerate(lk):
        a = int(ck[i])
        ks.append(kp[a:a + int(used[i])])
        vs.append(vp[a:a + int(used[i])])
        offs.append(offs[-1] + int(used[i]))
    cu = torch.tensor(offs, dtype=torch.int32, device="cuda")
    with torch.no_grad():
        ref = fa.flash_attn_varlen_func(q, torch.cat(ks), torch.cat(vs), cq, cu, mq, int(used.max()), causal=True)
    assert torch.equal(got, ref)
    # with gradients the pages are gathered first (the backward reads packed K/V)
    qg = q.clone().requires_grad_()
    out = fa.flash_attn_varlen_func(qg, kc, vc, cq, ck, mq, mk, causal=True, block_table=bt)
    out.float().sum().backward()
    assert qg.grad is not None and bool(torch.isfinite(qg.grad).all())


@pytest.mark.parametrize("seqused", [False, True])
def test_paged_prefill_gradients_reach_the_cache_without_host_sync(seqused):
    """Autograd through a paged cache: dQ and the gradients of k_cache / v_cache (page rows the
    block table does not name get 0) equal those of the same attention on packed K/V, and neither
    the forward nor the backward synchronises with the host (torch's sync debug mode raises)."""
    q, kc, vc, bt, cq, ck, kp, vp, mq, mk = _case(torch.bfloat16, 128, 64, seed=5)
    page = kc.shape[1]
    used = torch.tensor([650, 17, 100, 299], dtype=torch.int32, device="cuda") if seqused else None
    g = torch.Generator(device="cuda").manual_seed(9)
    dout = torch.randn(q.shape, device="cuda", dtype=q.dtype, generator=g)
    qa, kca, vca = (t.clone().requires_grad_() for t in (q, kc, vc))
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        out = fa.flash_attn_varlen_func(qa, kca, vca, cq, ck, mq, mk, causal=True, block_table=bt, seqused_k=used)
        out.backward(dout)
    finally:
        torch.cuda.set_sync_debug_mode(0)
    # reference: the same keys packed by hand, gradients scattered back to the pages
    lk = (ck[1:] - ck[:-1]).tolist()
    lu = used.tolist() if seqused else lk
    qb, kb, vb = q.clone().requires_grad_(), kp.clone().requires_grad_(), vp.clone().requires_grad_()
    ks = [kb[int(ck[i]):int(ck[i]) + lu[i]] for i in range(len(lk))]
    vs = [vb[int(ck[i]):int(ck[i]) + lu[i]] for i in range(len(lk))]
    cu = torch.tensor([0] + list(torch.tensor(lu).cumsum(0)), dtype=torch.int32, device="cuda")
    ref = fa.flash_attn_varlen_func(qb, torch.cat(ks), torch.cat(vs), cq, cu, mq, max(lu), causal=True)
    ref.backward(dout)
    assert torch.equal(out, ref)
    assert (qa.grad.float() - qb.grad.float()).norm() <= 1e-6 * qb.grad.float().norm() + 1e-6
    dkc, dvc = torch.zeros_like(kc, dtype=torch.float32), torch.zeros_like(vc, dtype=torch.float32)
    for i, L in enumerate(lk):
        for p in range((L + page - 1) // page):
            n = min(page, L - p * page)
            dkc[int(bt[i, p]), :n] += kb.grad[int(ck[i]) + p * page:int(ck[i]) + p * page + n].float()
            dvc[int(bt[i, p]), :n] += vb.grad[int(ck[i]) + p * page:int(ck[i]) + p * page + n].float()
    for nm, got, want in (("dk_cache", kca.grad, dkc), ("dv_cache", vca.grad, dvc)):
        # each cache row receives its one gathered row's gradient (plus exact zeros): same values
        e = (got.float() - want).norm() / want.norm()
        assert e < 1e-6, f"{nm} differs: rel {e:.3e}"
