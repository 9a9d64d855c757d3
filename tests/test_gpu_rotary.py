"""GPU parity of the rotary kernel (fa_rotary_launch via fable_attn.layers.rotary) against the
reference's torch arithmetic (package/fable_attn/layers/rotary.py:20-68, run here on the host):
bit-identical outputs for fp16 / bf16 / fp32, NeoX and interleaved pairs, partial rotary dims,
packed varlen positions, per-sequence and scalar offsets, in place and out of place."""
import pytest
import torch

from fable_attn.layers import rotary as R

pytestmark = pytest.mark.gpu


def _tables(rd, n=700):
    inv = 10000.0 ** (-torch.arange(0, rd, 2, dtype=torch.float32) / rd)
    ang = torch.arange(n, dtype=torch.float32)[:, None] * inv[None]
    return ang.cos(), ang.sin()


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("interleaved", [False, True])
@pytest.mark.parametrize("rd", [64, 128, 20])   # 20: rows not in 16-byte units (scalar kernel)
def test_rotary_varlen_bit_exact(dt, interleaved, rd):
    g = torch.Generator().manual_seed(3)
    cu = torch.tensor([0, 100, 357, 360, 611], dtype=torch.int32)
    x = torch.randn(611, 6, 128, generator=g).to(dt)
    cos, sin = _tables(rd)
    ref = R.apply_rotary_emb(x, cos, sin, interleaved=interleaved, cu_seqlens=cu, max_seqlen=257)
    got = R.apply_rotary_emb(x.cuda(), cos.cuda(), sin.cuda(), interleaved=interleaved, cu_seqlens=cu.cuda(),
                             max_seqlen=257)
    assert torch.equal(got.cpu(), ref)
    offs = torch.tensor([3, 0, 90, 1], dtype=torch.int32)
    ref = R.apply_rotary_emb(x, cos, sin, interleaved=interleaved, seqlen_offsets=offs, cu_seqlens=cu, max_seqlen=257)
    got = R.apply_rotary_emb(x.cuda(), cos.cuda(), sin.cuda(), interleaved=interleaved, seqlen_offsets=offs.cuda(),
                             cu_seqlens=cu.cuda(), max_seqlen=257)
    assert torch.equal(got.cpu(), ref)


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("interleaved", [False, True])
def test_rotary_dense_offsets_inplace(dt, interleaved):
    g = torch.Generator().manual_seed(4)
    x = torch.randn(3, 50, 4, 96, generator=g).to(dt)
    cos, sin = _tables(32)
    offs = torch.tensor([0, 7, 300], dtype=torch.int32)
    ref = R.apply_rotary_emb(x, cos, sin, interleaved=interleaved, seqlen_offsets=offs)
    got = R.apply_rotary_emb(x.cuda(), cos.cuda(), sin.cuda(), interleaved=interleaved, seqlen_offsets=offs.cuda())
    assert torch.equal(got.cpu(), ref)
    xi = x.cuda()
    out = R.apply_rotary_emb(xi, cos.cuda(), sin.cuda(), interleaved=interleaved, seqlen_offsets=5, inplace=True)
    assert out.data_ptr() == xi.data_ptr()
    assert torch.equal(xi.cpu(), R.apply_rotary_emb(x, cos, sin, interleaved=interleaved, seqlen_offsets=5))
    # a strided view (q of a packed qkv) is rotated in place through the same kernel
    qkv = torch.randn(2, 40, 3, 4, 64, generator=g).to(dt)
    ref = R.apply_rotary_emb(qkv[:, :, 0], cos, sin, interleaved=interleaved)
    dq = qkv.cuda()
    R.apply_rotary_emb(dq[:, :, 0], cos.cuda(), sin.cuda(), interleaved=interleaved, inplace=True)
    assert torch.equal(dq[:, :, 0].cpu(), ref)
    assert torch.equal(dq[:, :, 1:].cpu(), qkv[:, :, 1:])


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("interleaved", [False, True])
def test_rotary_autograd_matches_host_arithmetic(dt, interleaved):
    """Device rotary with requires_grad: the forward and the gradient are bitwise those of the
    reference's torch arithmetic differentiated by autograd on the host."""
    g = torch.Generator().manual_seed(8)
    cu = torch.tensor([0, 37, 200, 311], dtype=torch.int32)
    x = torch.randn(311, 3, 64, generator=g).to(dt)
    gout = torch.randn(311, 3, 64, generator=g).to(dt)
    cos, sin = _tables(48)
    xh = x.clone().requires_grad_(True)
    ref = R.apply_rotary_emb(xh, cos, sin, interleaved=interleaved, cu_seqlens=cu)
    ref.backward(gout)
    xd = x.cuda().requires_grad_(True)
    got = R.apply_rotary_emb(xd, cos.cuda(), sin.cuda(), interleaved=interleaved, cu_seqlens=cu.cuda())
    assert got.requires_grad
    got.backward(gout.cuda())
    assert torch.equal(got.detach().cpu(), ref.detach())
    assert torch.equal(xd.grad.cpu(), xh.grad)


def _attn_inputs(dt, varlen, D, seed=5):
    g = torch.Generator(device="cuda").manual_seed(seed)
    if varlen:
        lens = [129, 300, 64, 517]
        cu = torch.tensor([0] + list(__import__("itertools").accumulate(lens)), dtype=torch.int32, device="cuda")
        tot = int(cu[-1])
        q = torch.randn(tot, 8, D, device="cuda", generator=g).to(dt)
        k = torch.randn(tot, 2, D, device="cuda", generator=g).to(dt)
        v = torch.randn(tot, 2, D, device="cuda", generator=g).to(dt)
        return q, k, v, cu, max(lens)
    q = torch.randn(2, 300, 8, D, device="cuda", generator=g).to(dt)
    k = torch.randn(2, 300, 2, D, device="cuda", generator=g).to(dt)
    v = torch.randn(2, 300, 2, D, device="cuda", generator=g).to(dt)
    return q, k, v, None, 300


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("varlen", [False, True])
@pytest.mark.parametrize("D,rd,interleaved,softcap", [(128, 64, False, 30.0), (128, 128, True, 0.0),
                                                      (64, 32, False, 0.0), (64, 64, True, 50.0),
                                                      (128, 20, False, 0.0), (128, 36, True, 0.0)])
def test_attention_with_fused_rotary_equals_rotate_then_attend(dt, varlen, D, rd, interleaved, softcap, monkeypatch):
    """flash_attn_(varlen_)func with rotary_cos/sin (q rotated inside the forward kernel, k in one
    pass) gives bitwise the output of apply_rotary_emb on q and k followed by the plain call."""
    import fable_attn
    monkeypatch.setenv("FABLE_ATTN_FWD_TILES", "1")   # both calls on the same (one-tile) kernel
    q, k, v, cu, mx = _attn_inputs(dt, varlen, D)
    cos, sin = (t.cuda() for t in _tables(rd, n=1024))
    kw = dict(causal=True, softcap=softcap, window_size=(200, 0))
    with torch.no_grad():
        if varlen:
            fused = fable_attn.flash_attn_varlen_func(q, k, v, cu, cu, mx, mx, rotary_cos=cos, rotary_sin=sin,
                                                      rotary_interleaved=interleaved, **kw)
            qr = R.apply_rotary_emb(q, cos, sin, interleaved=interleaved, cu_seqlens=cu)
            kr = R.apply_rotary_emb(k, cos, sin, interleaved=interleaved, cu_seqlens=cu)
            plain = fable_attn.flash_attn_varlen_func(qr, kr, v, cu, cu, mx, mx, **kw)
        else:
            fused = fable_attn.flash_attn_func(q, k, v, rotary_cos=cos, rotary_sin=sin,
                                               rotary_interleaved=interleaved, **kw)
            qr = R.apply_rotary_emb(q, cos, sin, interleaved=interleaved)
            kr = R.apply_rotary_emb(k, cos, sin, interleaved=interleaved)
            plain = fable_attn.flash_attn_func(qr, kr, v, **kw)
    assert torch.equal(fused, plain)


def test_attention_rotary_with_grad_is_differentiable():
    """With gradients enabled the rotation runs before the attention (differentiably): grads of
    q and k equal those of rotating by hand and attending."""
    import fable_attn
    q, k, v, _, _ = _attn_inputs(torch.bfloat16, False, 128, seed=9)
    cos, sin = (t.cuda() for t in _tables(64, n=512))
    grads = []
    for fused in (True, False):
        qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
        if fused:
            out = fable_attn.flash_attn_func(qq, kk, vv, causal=True, rotary_cos=cos, rotary_sin=sin)
        else:
            out = fable_attn.flash_attn_func(R.apply_rotary_emb(qq, cos, sin), R.apply_rotary_emb(kk, cos, sin), vv,
                                             causal=True)
        out.float().square().sum().backward()
        grads.append((qq.grad, kk.grad, vv.grad))
    for a, b in zip(*grads):
        assert torch.equal(a, b)


def test_attention_rotary_table_too_short():
    import fable_attn
    q, k, v, cu, mx = _attn_inputs(torch.bfloat16, True, 128)
    cos, sin = (t.cuda() for t in _tables(64, n=mx - 1))
    with pytest.raises(ValueError, match="seqlen_ro"):
        fable_attn.flash_attn_varlen_func(q, k, v, cu, cu, mx, mx, causal=True, rotary_cos=cos, rotary_sin=sin)
