"""`torch.ops.fable_attn.forward` — the operator contract older integrations look up.

Contract (reference package/fable_attn/torch_op.py:12-17, :51-71):
    forward(Tensor q, Tensor k, Tensor v, float scale, bool causal) -> Tensor
with q, k, v in [B, H, S, D] (the layout of F.scaled_dot_product_attention) and the result in the
same layout.  A request the kernels cannot serve returns an EMPTY tensor instead of raising: the
caller checks `o.numel() == 0` and takes its own path.  Registration never raises either.
"""
import torch

LAST_ERROR = None
REGISTERED = False
_LIB = None


def _forward(q, k, v, scale, causal):
    from . import _C
    empty = q.new_empty(0)
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        return empty
    if q.dtype not in (torch.float16, torch.bfloat16) or not q.is_cuda:
        return empty
    if q.shape[-1] != k.shape[-1] or q.shape[-1] > 256 or q.shape[-1] % 16:
        return empty
    if q.shape[1] % k.shape[1]:
        return empty
    q, k, v = (t if t.stride(-1) == 1 else t.contiguous() for t in (q, k, v))
    try:
        out, _ = _C.fwd(q, k, v, float(scale), bool(causal), -1, 0 if causal else -1, 0.0, None, 0.0, 0, 0, None)
    except Exception:
        return empty
    return out


def register():
    """Idempotent; returns True when the operator is available."""
    global _LIB, REGISTERED, LAST_ERROR
    if REGISTERED:
        return True
    try:
        ns = getattr(torch.ops, "fable_attn", None)
        if ns is not None and "forward" in dir(ns):
            REGISTERED = True
            return True
    except Exception:
        pass
    try:
        _LIB = torch.library.Library("fable_attn", "FRAGMENT")
        _LIB.define("forward(Tensor q, Tensor k, Tensor v, float scale, bool causal) -> Tensor")
        _LIB.impl("forward", _forward, "CUDA")
        REGISTERED = True
        return True
    except Exception as e:  # pragma: no cover
        LAST_ERROR = f"{type(e).__name__}: {e}"
        return False
