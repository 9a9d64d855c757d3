"""flash_attn.layers.rotary API (apply_rotary_emb, RotaryEmbedding) in plain torch.

Rotary embedding rotates coordinate pairs of the first rotary_dim = 2*cos.shape[-1] dims by the
angle table cos/sin (seqlen_ro, rotary_dim/2); the remaining dims pass through:
  interleaved=False (GPT-NeoX): pairs (i, i + rotary_dim/2)
  interleaved=True  (GPT-J)   : pairs (2i, 2i+1)
x' = x*cos - y*sin, y' = y*cos + x*sin.  Same surface as the reference's
package/fable_attn/layers/rotary.py:43-178; the varlen form computes every token's position
in one vectorised gather instead of a per-sequence loop.
"""
from typing import Optional, Union

import torch
from torch import nn

__all__ = ["apply_rotary_emb", "apply_rotary_emb_func", "apply_rotary_emb_qkv_", "apply_rotary_emb_kv_",
           "RotaryEmbedding"]


def _rotate(x, cos, sin, interleaved):
    """x (..., d); cos/sin broadcastable to (..., rd/2) with rd <= d."""
    rd = cos.shape[-1] * 2
    xr = x[..., :rd]
    if interleaved:
        a, b = xr[..., 0::2], xr[..., 1::2]
        rot = torch.stack((a * cos - b * sin, b * cos + a * sin), dim=-1).flatten(-2)
    else:
        a, b = xr[..., : rd // 2], xr[..., rd // 2:]
        rot = torch.cat((a * cos - b * sin, b * cos + a * sin), dim=-1)
    return rot if rd == x.shape[-1] else torch.cat((rot, x[..., rd:]), dim=-1)


def _positions_varlen(cu_seqlens, total, offsets, device):
    cu = cu_seqlens.to(device=device, dtype=torch.long)
    lens = cu[1:] - cu[:-1]
    seq_of = torch.repeat_interleave(torch.arange(lens.numel(), device=device), lens, output_size=total)
    pos = torch.arange(total, device=device) - cu[:-1][seq_of]
    if isinstance(offsets, int):
        return pos + offsets
    return pos + offsets.to(device=device, dtype=torch.long)[seq_of]


class _RotaryFn(torch.autograd.Function):
    """Rotary on device tensors with autograd.  The gradient of a rotation by theta is the rotation
    of the incoming gradient by -theta; with sin negated the native kernel performs exactly the
    roundings torch autograd applies to the elementwise ops of the host path (each product and the
    sum rounded to the dtype), so both paths give the same gradient bits."""

    @staticmethod
    def forward(ctx, x, cos, sin, interleaved, offs, cu_seqlens):
        from .. import _C
        ctx.save_for_backward(cos, sin)
        ctx.interleaved, ctx.offs, ctx.cu = interleaved, offs, cu_seqlens
        return _C.rotary(x, cos, sin, interleaved, False, offs, cu_seqlens)

    @staticmethod
    def backward(ctx, grad):
        from .. import _C
        cos, sin = ctx.saved_tensors
        dx = _C.rotary(grad.contiguous(), cos, -sin, ctx.interleaved, False, ctx.offs, ctx.cu)
        return dx, None, None, None, None, None


def apply_rotary_emb(x, cos, sin, interleaved=False, inplace=False, seqlen_offsets=0, cu_seqlens=None,
                     max_seqlen=None):
    """x: (batch, seqlen, nheads, headdim), or (total, nheads, headdim) with cu_seqlens.
    cos/sin: (seqlen_ro, rotary_dim/2).  seqlen_offsets: int or (batch,) tensor.
    Device tensors are rotated by one native kernel (fa_rotary_launch) with the roundings of the
    torch arithmetic below, which host tensors use."""
    if x.is_cuda:
        if cu_seqlens is None and x.dim() != 4:
            raise ValueError(f"apply_rotary_emb expects (batch, seqlen, nheads, headdim), got {tuple(x.shape)}")
        if cu_seqlens is not None and x.dim() != 3:
            raise ValueError("apply_rotary_emb with cu_seqlens expects (total, nheads, headdim)")
        offs = seqlen_offsets if isinstance(seqlen_offsets, int) else seqlen_offsets
        if torch.is_grad_enabled() and x.requires_grad:
            if inplace:
                raise RuntimeError("apply_rotary_emb: inplace rotation of a tensor that requires grad")
            return _RotaryFn.apply(x, cos, sin, bool(interleaved), offs, cu_seqlens)
        from .. import _C
        return _C.rotary(x, cos, sin, bool(interleaved), bool(inplace), offs, cu_seqlens)
    if cu_seqlens is None:
        if x.dim() != 4:
            raise ValueError(f"apply_rotary_emb expects (batch, seqlen, nheads, headdim), got {tuple(x.shape)}")
        b, s = x.shape[0], x.shape[1]
        pos = torch.arange(s, device=x.device)
        if isinstance(seqlen_offsets, int):
            c, sn = cos[pos + seqlen_offsets][None, :, None], sin[pos + seqlen_offsets][None, :, None]
        else:
            idx = pos[None, :] + seqlen_offsets.to(x.device).view(b, 1)
            c, sn = cos[idx][:, :, None], sin[idx][:, :, None]
    else:
        if x.dim() != 3:
            raise ValueError("apply_rotary_emb with cu_seqlens expects (total, nheads, headdim)")
        idx = _positions_varlen(cu_seqlens, x.shape[0], seqlen_offsets, x.device)
        c, sn = cos[idx][:, None], sin[idx][:, None]
    out = _rotate(x, c.to(x.dtype), sn.to(x.dtype), interleaved)
    if inplace:
        x.copy_(out)
        return x
    return out


apply_rotary_emb_func = apply_rotary_emb


def apply_rotary_emb_qkv_(qkv, cos, sin, cos_k=None, sin_k=None, interleaved=False, seqlen_offsets=0,
                          cu_seqlens=None, max_seqlen=None, num_heads_q=None):
    """qkv (batch, seqlen, 3, nheads, headdim): rotates q and k in place."""
    qkv[:, :, 0].copy_(apply_rotary_emb(qkv[:, :, 0], cos, sin, interleaved, False, seqlen_offsets))
    qkv[:, :, 1].copy_(apply_rotary_emb(qkv[:, :, 1], cos if cos_k is None else cos_k,
                                        sin if sin_k is None else sin_k, interleaved, False, seqlen_offsets))
    return qkv


def apply_rotary_emb_kv_(kv, cos, sin, interleaved=False, seqlen_offsets=0, cu_seqlens=None, max_seqlen=None):
    """kv (batch, seqlen, 2, nheads, headdim): rotates k in place."""
    kv[:, :, 0].copy_(apply_rotary_emb(kv[:, :, 0], cos, sin, interleaved, False, seqlen_offsets))
    return kv


class RotaryEmbedding(nn.Module):
    """Cached cos/sin tables (base**(-2i/dim) frequencies, optional XPos scale_base)."""

    def __init__(self, dim: int, base=10000.0, interleaved=False, scale_base=None, pos_idx_in_fp32=True,
                 device=None):
        super().__init__()
        self.dim, self.base, self.interleaved = dim, float(base), interleaved
        self.scale_base, self.pos_idx_in_fp32 = scale_base, pos_idx_in_fp32
        self.register_buffer("inv_freq", self._inv_freq(device), persistent=False)
        scale = None
        if scale_base is not None:
            scale = (torch.arange(0, dim, 2, device=device, dtype=torch.float32) + 0.4 * dim) / (1.4 * dim)
        self.register_buffer("scale", scale, persistent=False)
        self._len = 0
        self._cos = self._sin = self._cos_k = self._sin_k = None

    def _inv_freq(self, device=None):
        return 1.0 / (self.base ** (torch.arange(0, self.dim, 2, device=device, dtype=torch.float32) / self.dim))

    def _update(self, seqlen, device, dtype):
        if self._cos is not None and seqlen <= self._len and self._cos.device == device and self._cos.dtype == dtype:
            return
        self._len = seqlen
        t = torch.arange(seqlen, device=device, dtype=torch.float32 if self.pos_idx_in_fp32 else dtype)
        inv = self._inv_freq(device) if self.pos_idx_in_fp32 else self.inv_freq
        freqs = torch.outer(t, inv.to(device=device, dtype=t.dtype))
        if self.scale is None:
            self._cos, self._sin = torch.cos(freqs).to(dtype), torch.sin(freqs).to(dtype)
            self._cos_k = self._sin_k = None
        else:
            power = (torch.arange(seqlen, dtype=self.scale.dtype, device=device) - seqlen // 2) / self.scale_base
            sc = self.scale.to(device) ** power.unsqueeze(-1)
            self._cos, self._sin = (torch.cos(freqs) * sc).to(dtype), (torch.sin(freqs) * sc).to(dtype)
            self._cos_k, self._sin_k = (torch.cos(freqs) / sc).to(dtype), (torch.sin(freqs) / sc).to(dtype)

    def forward(self, qkv: torch.Tensor, kv: Optional[torch.Tensor] = None,
                seqlen_offset: Union[int, torch.Tensor] = 0, max_seqlen: Optional[int] = None):
        seqlen = qkv.shape[1]
        need = max_seqlen if max_seqlen is not None else seqlen + (seqlen_offset if isinstance(seqlen_offset, int) else 0)
        self._update(need, qkv.device, qkv.dtype)
        ck = self._cos if self._cos_k is None else self._cos_k
        sk = self._sin if self._sin_k is None else self._sin_k
        if kv is None:
            if qkv.dim() == 5:
                return apply_rotary_emb_qkv_(qkv, self._cos, self._sin, ck, sk, self.interleaved, seqlen_offset)
            return apply_rotary_emb(qkv, self._cos, self._sin, self.interleaved, False, seqlen_offset)
        q = apply_rotary_emb(qkv, self._cos, self._sin, self.interleaved, False, seqlen_offset)
        return q, apply_rotary_emb_kv_(kv, ck, sk, self.interleaved, seqlen_offset)
