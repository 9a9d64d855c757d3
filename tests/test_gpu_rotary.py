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
