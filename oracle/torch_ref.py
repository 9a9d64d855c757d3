"""Exact attention in torch float32 — TEST AND BENCH INFRASTRUCTURE ONLY.

The reference's own exact torch reference (lab/parity_new_api.py:36-75, `ref_attn`) restated:
scores q.k^T in fp32, softcap c*tanh(s*scale/c) or s*scale, alibi slope*(key - (q + delta)),
bottom-right aligned causal / window / chunk masks, softmax, fully masked rows -> 0.  bench.py
times it on the host cores as the second CPU baseline ("path B"); nothing in the product path
imports it.
"""
import torch


def ref_attn(q, k, v, scale, causal=False, wl=-1, wr=-1, softcap=0.0, alibi=None, chunk=0, qpos=None):
    """q (B, Sq, H, D), k / v (B, Sk, Hk, D) -> (B, Sq, H, D) float32.  qpos: query position for
    alibi when Sq = 1 (decode), as in the reference."""
    qf, kf, vf = (x.transpose(1, 2).float() for x in (q, k, v))
    H, Hk = qf.shape[1], kf.shape[1]
    if H != Hk:
        kf = kf.repeat_interleave(H // Hk, dim=1)
        vf = vf.repeat_interleave(H // Hk, dim=1)
    s = qf @ kf.transpose(-1, -2)
    s = softcap * torch.tanh(s * scale / softcap) if softcap and softcap > 0 else s * scale
    Sq, Sk = qf.shape[2], kf.shape[2]
    qi = torch.arange(Sq, device=q.device).view(-1, 1)
    ki = torch.arange(Sk, device=q.device).view(1, -1)
    delta = Sk - Sq
    if alibi is not None:
        base = qi + delta if qpos is None else torch.full_like(qi, qpos)
        s = s + alibi.view(1, H, 1, 1).float() * (ki - base).float()
    hidden = torch.zeros(Sq, Sk, device=q.device, dtype=torch.bool)
    if causal:
        hidden |= ki > qi + delta
    if wl is not None and wl >= 0:
        hidden |= ki < qi + delta - wl
    if wr is not None and wr >= 0:
        hidden |= ki > qi + delta + wr
    if chunk:
        cs = ((qi + delta).clamp_min(0) // chunk) * chunk
        hidden |= (ki < cs) | (ki >= cs + chunk)
    p = torch.nan_to_num(s.masked_fill(hidden, float("-inf")).softmax(-1), nan=0.0)
    return (p @ vf).transpose(1, 2)
