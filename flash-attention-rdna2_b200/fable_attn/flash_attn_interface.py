"""FA-2 argument-order API of fable_attn, running on the sm_100a kernels of fable_attn._C.

Same public functions, signatures, return shapes and error behaviour as the reference's
package/fable_attn/flash_attn_interface.py:378-771 (itself a transcription of the flash-attn 2.8
API): flash_attn_func, the qkv/kv-packed variants, the varlen family, flash_attn_combine and
flash_attn_with_kvcache.  Inputs use the public (batch, seqlen, nheads, headdim) layout; the
kernels read them through strides, so no layout copies are made.  FA-3-only arguments (qv,
attention_chunk, num_splits, pack_gqa, sm_margin, *_descale) are keyword-only.

There is no CPU path and no silent fallback: unsupported requests raise, and importing this
module fails if the compiled extension is missing.
"""
import itertools
import math
import random

import torch
import torch.nn.functional as F

try:
    from fable_attn import _C
except Exception as _e:  # pragma: no cover - exercised only on a broken install
    raise ImportError(
        "fable_attn._C (the sm_100a kernel extension) failed to load: "
        f"{type(_e).__name__}: {_e}. Build it with `python flash-attention-rdna2_b200/build.py`."
    ) from _e

# head dims the kernels are instantiated for; others are zero-padded up to the next one
# (zero columns leave q.k unchanged and give zero output columns that are sliced off)
_VALID_D = (16, 32, 48, 64, 80, 96, 112, 128, 160, 192, 224, 256)
_MAX_D = _VALID_D[-1]


def _pad_dim(d):
    for x in _VALID_D:
        if x >= d:
            return x
    return None


def _pad_last(t, d):
    return t if t.shape[-1] == d else F.pad(t, (0, d - t.shape[-1]))


def _map_window(causal, window_size):
    """(causal_flag, win_left, win_right) with flash-attn semantics: key j is visible to query i
    when i+delta-left <= j <= i+delta+right; a negative bound is unbounded and causal forces
    right = 0.  A right bound of 0 is reported as causal (reference flash_attn_interface.py:76-95)."""
    left, right = window_size
    wl = int(left) if left is not None and left >= 0 else -1
    wr = int(right) if right is not None and right >= 0 else -1
    if causal:
        wr = 0
    return (1 if wr == 0 else 0), wl, wr


def _reject_fp8(q_descale, k_descale, v_descale):
    if q_descale is not None or k_descale is not None or v_descale is not None:
        raise NotImplementedError(
            "fable_attn: q_descale/k_descale/v_descale (FP8 attention) is not supported: this engine "
            "computes exact attention in fp16/bf16/fp32; pass unquantised tensors.")


def _accept_hints(num_splits=None, pack_gqa=None, sm_margin=None):
    """FA-3 scheduling hints: type-checked, then ignored in prefill (they change the schedule,
    not the result).  The decode path honours num_splits."""
    if num_splits is not None and not isinstance(num_splits, int):
        raise TypeError(f"fable_attn: num_splits must be an int, got {type(num_splits)}")
    if pack_gqa is not None and not isinstance(pack_gqa, bool):
        raise TypeError(f"fable_attn: pack_gqa must be a bool or None, got {type(pack_gqa)}")
    if sm_margin is not None and not isinstance(sm_margin, int):
        raise TypeError(f"fable_attn: sm_margin must be an int, got {type(sm_margin)}")


def _check_chunk(attention_chunk):
    if attention_chunk is None:
        return 0
    if not isinstance(attention_chunk, int) or attention_chunk < 0:
        raise ValueError(f"fable_attn: attention_chunk must be a non-negative int, got {attention_chunk!r}")
    return attention_chunk


def _check_supported(q, k, head_dim_limit=True):
    if not q.is_cuda:
        raise ValueError("fable_attn: tensors must be on a CUDA device (q.is_cuda is False)")
    if head_dim_limit and q.shape[-1] > _MAX_D:
        raise ValueError(f"fable_attn: head_dim={q.shape[-1]} exceeds the maximum {_MAX_D}")
    if q.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError(f"fable_attn: dtype {q.dtype} not supported (fp16, bf16, fp32)")
    if q.shape[-2] % k.shape[-2] != 0:
        raise ValueError(f"fable_attn: nheads_q={q.shape[-2]} is not a multiple of nheads_k={k.shape[-2]}")


def _qv_concat(q, k, v, qv):
    """FA-3 qv / headdim_v != headdim: the score gains qv.v^T, i.e.
    S = [q | qv] . [k | v]^T and O = softmax(S) . [v | 0] restricted to the first dv columns.
    Expressed by concatenation so the kernels stay untouched."""
    d, dv = q.shape[-1], v.shape[-1]
    if d + dv > _MAX_D:
        raise NotImplementedError(
            f"fable_attn: qv/headdim_v needs a score head_dim of headdim+headdim_v = {d}+{dv} = {d + dv}, "
            f"above the kernel limit {_MAX_D}")
    if qv is None:
        qv = q.new_zeros(q.shape[:-1] + (dv,))
    elif qv.shape[-1] != dv:
        raise ValueError(f"fable_attn: qv.shape[-1]={qv.shape[-1]} must equal v.shape[-1]={dv}")
    return (torch.cat([q, qv], dim=-1), torch.cat([k, v], dim=-1),
            torch.cat([v, v.new_zeros(v.shape[:-1] + (d,))], dim=-1), dv)


def _needs_qv(q, v, qv):
    return qv is not None or v.shape[-1] != q.shape[-1]


def _lastdim_contig(t):
    return t if t.stride(-1) == 1 else t.contiguous()


def _rotary_plan(q, k, v, rotary_cos, rotary_sin, rotary_interleaved, return_attn_probs, qv, cu_q=None, cu_k=None,
                 paged=False):
    """Rotary embedding of q and k requested with the attention call (keyword-only extension;
    equivalent to layers.rotary.apply_rotary_emb on q and k first, positions restarting per
    sequence).  Inference calls on fp16/bf16 with an instantiated head_dim rotate q inside the
    forward kernel and k in one pass (returns the cos/sin/interleaved triple to hand to _C); anything else
    rotates both here, differentiably, and returns (q, k, None)."""
    if rotary_cos is None and rotary_sin is None:
        return q, k, None
    if (rotary_cos is None) != (rotary_sin is None):
        raise ValueError("fable_attn: rotary_cos and rotary_sin go together")
    # every position must have a table row (the reference's apply_rotary_emb indexes cos[pos])
    if cu_q is not None:
        longest = max(int((cu_q[1:] - cu_q[:-1]).max()), int((cu_k[1:] - cu_k[:-1]).max()))
    else:
        longest = max(q.shape[1], k.shape[1])
    if rotary_cos.shape[0] < longest or rotary_sin.shape != rotary_cos.shape:
        raise ValueError(f"fable_attn: rotary_cos / rotary_sin {tuple(rotary_cos.shape)} must be (seqlen_ro, "
                         f"rotary_dim / 2) with seqlen_ro >= the longest sequence ({longest})")
    grad = torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad)
    if (not grad and not return_attn_probs and qv is None and not paged and q.is_cuda
            and q.dtype in (torch.float16, torch.bfloat16) and q.shape[-1] in _VALID_D):
        return q, k, (rotary_cos, rotary_sin, bool(rotary_interleaved))
    from .layers.rotary import apply_rotary_emb
    q = apply_rotary_emb(q, rotary_cos, rotary_sin, rotary_interleaved, cu_seqlens=cu_q)
    k = apply_rotary_emb(k, rotary_cos, rotary_sin, rotary_interleaved, cu_seqlens=cu_k)
    return q, k, None


class _AttnFn(torch.autograd.Function):
    """Dense attention with autograd; q/k/v are [B,H,S,D] views (any strides, last dim 1)."""

    @staticmethod
    def forward(ctx, q, k, v, scale, causal, wl, wr, softcap, alibi, dropout_p, chunk, out_buf):
        seed = random.getrandbits(63) if dropout_p > 0 else 0
        # the keep mask is generated once (bits, no batch term) and read by forward and backward
        bits = (_C.dropout_mask(q, int(seed), float(dropout_p), q.shape[1], q.shape[2], k.shape[2], bool(causal),
                                int(wl), int(wr)) if dropout_p > 0 else None)
        out, lse = _C.fwd(q, k, v, float(scale), bool(causal), int(wl), int(wr), float(softcap), alibi,
                          float(dropout_p), int(seed), int(chunk), out_buf, bits)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.mark_non_differentiable(lse)
        ctx.bits = bits
        ctx.alibi = alibi
        ctx.cfg = (scale, causal, wl, wr, softcap, dropout_p, seed, chunk)
        return out, lse

    @staticmethod
    def backward(ctx, dout, dlse):
        scale, causal, wl, wr, softcap, dropout_p, seed, chunk = ctx.cfg
        if chunk:
            raise NotImplementedError(
                "fable_attn: backward with attention_chunk is not supported (as in FA-3); "
                "run the chunked forward under torch.no_grad()")
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = _C.bwd(_lastdim_contig(dout), q, k, v, out, lse, float(scale), bool(causal), int(wl),
                            int(wr), float(softcap), ctx.alibi, float(dropout_p), int(seed), ctx.bits)
        return dq, dk, dv, None, None, None, None, None, None, None, None, None


class _VarlenAttnFn(torch.autograd.Function):
    """Varlen attention with autograd: native kernels both ways (one launch per pass, no
    per-sequence Python loop)."""

    @staticmethod
    def forward(ctx, q, k, v, cu_q, cu_k, max_q, max_k, scale, causal, wl, wr, softcap, alibi, dropout_p,
                chunk, su_q, su_k):
        seed = random.getrandbits(63) if dropout_p > 0 else 0
        out, lse = _C.fwd_varlen(q, k, v, cu_q, cu_k, int(max_q), int(max_k), float(scale), bool(causal),
                                 int(wl), int(wr), float(softcap), alibi, float(dropout_p), int(seed), int(chunk),
                                 su_q, su_k, True)
        ctx.save_for_backward(q, k, v, out, lse, cu_q, cu_k)
        ctx.mark_non_differentiable(lse)
        ctx.extra = (alibi, su_q, su_k)
        ctx.cfg = (max_q, max_k, scale, causal, wl, wr, softcap, dropout_p, seed, chunk)
        return out, lse

    @staticmethod
    def backward(ctx, dout, dlse):
        max_q, max_k, scale, causal, wl, wr, softcap, dropout_p, seed, chunk = ctx.cfg
        if chunk:
            raise NotImplementedError("fable_attn: backward with attention_chunk is not supported (as in FA-3)")
        q, k, v, out, lse, cu_q, cu_k = ctx.saved_tensors
        alibi, su_q, su_k = ctx.extra
        dq, dk, dv = _C.bwd_varlen(_lastdim_contig(dout), q, k, v, out, lse, cu_q, cu_k, int(max_q), int(max_k),
                                   float(scale), bool(causal), int(wl), int(wr), float(softcap), alibi,
                                   float(dropout_p), int(seed), su_q, su_k)
        return (dq, dk, dv) + (None,) * 14


def _attn_probs(q, k, lse, scale, causal, wl, wr, softcap, alibi, chunk):
    """Debug output S_dmask of return_attn_probs: the full [B,H,SQ,SK] probability matrix
    p = exp(s - lse) from the kernel's own LSE, before dropout (flash-attn documents these values
    as a debugging aid).  Materialises SQ x SK, so a free-memory check comes first.
    q, k: [B,H,S,D] views."""
    B, Hq, SQ, _ = q.shape
    Hk, SK = k.shape[1], k.shape[2]
    need = B * Hq * SQ * SK * 4
    free = torch.cuda.mem_get_info(q.device)[0]
    if need > free * 0.8:
        raise torch.cuda.OutOfMemoryError(
            f"fable_attn: return_attn_probs needs a {need / 2**30:.1f} GiB SxS matrix "
            f"({free / 2**30:.1f} GiB free); the kernels themselves never materialise it")
    kk = k if Hk == Hq else k.repeat_interleave(Hq // Hk, dim=1)
    s = torch.matmul(q.float(), kk.float().transpose(-1, -2))
    s = softcap * torch.tanh(s * scale / softcap) if softcap and softcap > 0 else s * scale
    delta = SK - SQ
    qi = torch.arange(SQ, device=q.device).view(-1, 1)
    ki = torch.arange(SK, device=q.device).view(1, -1)
    if alibi is not None:
        # the kernels add slope*(key - q); the reference's debug path matches its own
        # forward only up to the diagonal offset (flash_attn_interface.py:296), here it is exact
        s = s + alibi.view(1, Hq, 1, 1).float() * (ki - qi).float()
    hidden = torch.zeros(SQ, SK, device=q.device, dtype=torch.bool)
    if causal:
        hidden |= ki > qi + delta
    if wl >= 0:
        hidden |= ki < qi + delta - wl
    if wr >= 0:
        hidden |= ki > qi + delta + wr
    if chunk:
        start = ((qi + delta).clamp_min(0) // chunk) * chunk
        hidden |= (ki < start) | (ki >= start + chunk)
    return torch.exp(s - lse.unsqueeze(-1)).masked_fill(hidden, 0.0)


def _fwd_bshd(q, k, v, dropout_p, softmax_scale, causal, window_size, softcap, alibi_slopes, deterministic,
              return_attn_probs, qv, attention_chunk, q_descale, k_descale, v_descale, num_splits, pack_gqa,
              sm_margin, rotary_cos=None, rotary_sin=None, rotary_interleaved=False):
    """Shared body of flash_attn_func and the packed variants; inputs (B, S, H, D)."""
    _reject_fp8(q_descale, k_descale, v_descale)
    _accept_hints(num_splits, pack_gqa, sm_margin)
    chunk = _check_chunk(attention_chunk)
    q, k, rot = _rotary_plan(q, k, v, rotary_cos, rotary_sin, rotary_interleaved, return_attn_probs, qv)
    keep_cols = None
    if _needs_qv(q, v, qv):
        if softmax_scale is None:
            softmax_scale = (q.shape[-1] + v.shape[-1]) ** -0.5
        q, k, v, keep_cols = _qv_concat(q, k, v, qv)
    elif softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(q.shape[-1])
    _check_supported(q, k)
    cflag, wl, wr = _map_window(causal, window_size)
    d = q.shape[-1]
    dp = _pad_dim(d)
    if dp != d:
        q, k, v = _pad_last(q, dp), _pad_last(k, dp), _pad_last(v, dp)
        keep_cols = keep_cols or d
    q, k, v = _lastdim_contig(q), _lastdim_contig(k), _lastdim_contig(v)
    B, SQ, Hq, D = q.shape
    # dense (B, S, H, D) output, handed to the kernel as its [B,H,S,D] view
    out_buf = torch.empty((B, SQ, Hq, D), dtype=q.dtype, device=q.device).transpose(1, 2)
    al = alibi_slopes.float().contiguous() if alibi_slopes is not None else None
    qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    if rot is not None:   # inference with in-kernel rotary of q (k rotated once by the glue)
        seed = random.getrandbits(63) if dropout_p > 0 else 0
        bits = (_C.dropout_mask(qh, int(seed), float(dropout_p), Hq, SQ, kh.shape[2], bool(cflag), int(wl), int(wr))
                if dropout_p > 0 else None)
        out, lse = _C.fwd(qh, kh, vh, float(softmax_scale), bool(cflag), int(wl), int(wr), float(softcap), al,
                          float(dropout_p), int(seed), int(chunk), out_buf, bits, rotary_cos=rot[0],
                          rotary_sin=rot[1], rotary_interleaved=rot[2])
    else:
        out, lse = _AttnFn.apply(qh, kh, vh, softmax_scale, cflag, wl, wr, softcap, al, dropout_p, chunk, out_buf)
    res = out.transpose(1, 2)
    if keep_cols is not None:
        res = res[..., :keep_cols].contiguous()
    if return_attn_probs:
        probs = _attn_probs(qh, kh, lse, softmax_scale, bool(cflag), wl, wr, softcap, al, chunk)
        return res, lse, probs
    return res


def flash_attn_func(q, k, v, dropout_p=0.0, softmax_scale=None, causal=False, window_size=(-1, -1),
                    softcap=0.0, alibi_slopes=None, deterministic=False, return_attn_probs=False, *,
                    qv=None, attention_chunk=0, q_descale=None, k_descale=None, v_descale=None,
                    num_splits=1, pack_gqa=None, sm_margin=0, rotary_cos=None, rotary_sin=None,
                    rotary_interleaved=False):
    """q: (batch, seqlen_q, nheads, headdim); k, v: (batch, seqlen_k, nheads_k, headdim).
    Returns out (batch, seqlen_q, nheads, headdim), or (out, softmax_lse, S_dmask) when
    return_attn_probs.  deterministic is accepted; the backward is always deterministic.
    rotary_cos / rotary_sin (seqlen_ro, rotary_dim/2), keyword-only: rotate q and k first, as
    layers.rotary.apply_rotary_emb does (positions 0..seqlen-1), inside the kernel for inference."""
    return _fwd_bshd(q, k, v, dropout_p, softmax_scale, causal, window_size, softcap, alibi_slopes, deterministic,
                     return_attn_probs, qv, attention_chunk, q_descale, k_descale, v_descale, num_splits, pack_gqa,
                     sm_margin, rotary_cos, rotary_sin, rotary_interleaved)


def flash_attn_qkvpacked_func(qkv, dropout_p=0.0, softmax_scale=None, causal=False, window_size=(-1, -1),
                              softcap=0.0, alibi_slopes=None, deterministic=False, return_attn_probs=False, *,
                              qv=None, attention_chunk=0, q_descale=None, k_descale=None, v_descale=None,
                              num_splits=1, pack_gqa=None, sm_margin=0):
    """qkv: (batch, seqlen, 3, nheads, headdim)."""
    return _fwd_bshd(qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2], dropout_p, softmax_scale, causal, window_size,
                     softcap, alibi_slopes, deterministic, return_attn_probs, qv, attention_chunk, q_descale,
                     k_descale, v_descale, num_splits, pack_gqa, sm_margin)


def flash_attn_kvpacked_func(q, kv, dropout_p=0.0, softmax_scale=None, causal=False, window_size=(-1, -1),
                             softcap=0.0, alibi_slopes=None, deterministic=False, return_attn_probs=False, *,
                             qv=None, attention_chunk=0, q_descale=None, k_descale=None, v_descale=None,
                             num_splits=1, pack_gqa=None, sm_margin=0):
    """q: (batch, seqlen_q, nheads, d); kv: (batch, seqlen_k, 2, nheads_k, d)."""
    return _fwd_bshd(q, kv[:, :, 0], kv[:, :, 1], dropout_p, softmax_scale, causal, window_size, softcap,
                     alibi_slopes, deterministic, return_attn_probs, qv, attention_chunk, q_descale, k_descale,
                     v_descale, num_splits, pack_gqa, sm_margin)


def _check_paged(k, v, block_table, cu_seqlens_k):
    if k.dim() != 4 or v.dim() != 4:
        raise ValueError(
            "fable_attn: with block_table, k and v must be paged (num_blocks, page_block_size, nheads_k, "
            f"headdim); got k.shape={tuple(k.shape)}")
    bt = block_table.to(torch.int32)
    nseq = cu_seqlens_k.numel() - 1
    if bt.dim() != 2 or bt.shape[0] != nseq:
        raise ValueError(f"fable_attn: block_table must be (batch, max_blocks), got {tuple(bt.shape)} for "
                         f"batch={nseq}")
    return bt


def _unpage(k, v, block_table, cu_seqlens_k, seqused_k, max_seqlen_k):
    """Paged (num_blocks, page, nheads_k, d) K/V + block_table -> a padded varlen K/V, gathered on
    the device with no host synchronisation: sequence b's positions 0 .. max_seqlen_k-1 occupy rows
    b*max_seqlen_k + p (row of page block_table[b, p // page], slot p % page), its length is given
    as seqused_k, and cu_seqlens_k becomes b*max_seqlen_k.  The gather is differentiable (the
    gradient of each cache row is the sum of its gathered rows' gradients), so autograd carries
    dK / dV back into the caches.  Used where the kernels cannot read the pages in place
    (gradients, return_attn_probs, qv, padded head dims)."""
    bt = _check_paged(k, v, block_table, cu_seqlens_k)
    nb, page = k.shape[0], k.shape[1]
    B, mx = bt.shape[0], int(max_seqlen_k)
    dev = k.device
    pos = torch.arange(mx, device=dev)
    blk = bt[:, (pos // page).clamp_max(bt.shape[1] - 1)].long().clamp(0, nb - 1)   # positions past a table row or
    rows = (blk * page + (pos % page)).reshape(-1)                                    # invalid entries: masked below
    kd = k.reshape(-1, k.shape[2], k.shape[3])[rows]
    vd = v.reshape(-1, v.shape[2], v.shape[3])[rows]
    cu = torch.arange(B + 1, device=dev, dtype=torch.int32) * mx
    lens = (seqused_k if seqused_k is not None else cu_seqlens_k[1:] - cu_seqlens_k[:-1]).to(dev, torch.int32)
    return kd, vd, cu, lens.clamp(0, mx).contiguous()


def flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, dropout_p=0.0,
                           softmax_scale=None, causal=False, window_size=(-1, -1), softcap=0.0, alibi_slopes=None,
                           deterministic=False, return_attn_probs=False, *, seqused_q=None, seqused_k=None,
                           qv=None, attention_chunk=0, q_descale=None, k_descale=None, v_descale=None,
                           num_splits=1, pack_gqa=None, sm_margin=0, block_table=None, rotary_cos=None,
                           rotary_sin=None, rotary_interleaved=False):
    """Packed variable-length attention: q (total_q, nheads, d), k/v (total_k, nheads_k, d) with
    cu_seqlens_* int32 (batch+1).  seqused_q/seqused_k clip each sequence.  With block_table, k/v
    are paged (num_blocks, page, nheads_k, d).  Forward and backward are single native launches.
    rotary_cos / rotary_sin (seqlen_ro, rotary_dim/2), keyword-only: rotate q and k first, as
    layers.rotary.apply_rotary_emb(..., cu_seqlens=...) does (positions restart per sequence),
    inside the kernel for inference."""
    _reject_fp8(q_descale, k_descale, v_descale)
    _accept_hints(num_splits, pack_gqa, sm_margin)
    chunk = _check_chunk(attention_chunk)
    q, k, rot = _rotary_plan(q, k, v, rotary_cos, rotary_sin, rotary_interleaved, return_attn_probs, qv,
                             cu_q=cu_seqlens_q, cu_k=cu_seqlens_k, paged=block_table is not None)
    paged_bt = None
    if block_table is not None:
        grad = torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad)
        if (grad or return_attn_probs or qv is not None or _pad_dim(q.shape[-1]) != q.shape[-1]
                or not k.is_cuda or not k.is_contiguous() or not v.is_contiguous()):
            k, v, cu_seqlens_k, seqused_k = _unpage(k, v, block_table, cu_seqlens_k, seqused_k, max_seqlen_k)
        else:   # the forward kernel reads the pages in place (no gather, no host sync)
            paged_bt = _check_paged(k, v, block_table, cu_seqlens_k).contiguous()
    keep_cols = None
    if _needs_qv(q, v, qv):
        if softmax_scale is None:
            softmax_scale = (q.shape[-1] + v.shape[-1]) ** -0.5
        q, k, v, keep_cols = _qv_concat(q, k, v, qv)
    elif softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(q.shape[-1])
    if q.dim() != 3:
        raise ValueError(f"fable_attn: varlen expects (total, nheads, headdim), got {tuple(q.shape)}")
    _check_supported(q, k)
    d = q.shape[-1]
    dp = _pad_dim(d)
    if dp != d:
        q, k, v = _pad_last(q, dp), _pad_last(k, dp), _pad_last(v, dp)
        keep_cols = keep_cols or d
    cflag, wl, wr = _map_window(causal, window_size)
    al = alibi_slopes.float().contiguous() if alibi_slopes is not None else None
    cu_q = cu_seqlens_q.to(torch.int32).contiguous()
    cu_k = cu_seqlens_k.to(torch.int32).contiguous()
    su_q = seqused_q.to(torch.int32).contiguous() if seqused_q is not None else None
    su_k = seqused_k.to(torch.int32).contiguous() if seqused_k is not None else None
    q, k, v = _lastdim_contig(q), _lastdim_contig(k), _lastdim_contig(v)
    if paged_bt is not None:
        seed = random.getrandbits(63) if dropout_p > 0 else 0
        out, lse = _C.fwd_varlen(q, k, v, cu_q, cu_k, int(max_seqlen_q), int(max_seqlen_k), float(softmax_scale),
                                 bool(cflag), int(wl), int(wr), float(softcap), al, float(dropout_p), int(seed),
                                 int(chunk), su_q, su_k, True, block_table=paged_bt)
    elif rot is not None:   # inference with in-kernel rotary of q (k rotated once by the glue)
        seed = random.getrandbits(63) if dropout_p > 0 else 0
        out, lse = _C.fwd_varlen(q, k, v, cu_q, cu_k, int(max_seqlen_q), int(max_seqlen_k), float(softmax_scale),
                                 bool(cflag), int(wl), int(wr), float(softcap), al, float(dropout_p), int(seed),
                                 int(chunk), su_q, su_k, True, rotary_cos=rot[0], rotary_sin=rot[1],
                                 rotary_interleaved=rot[2])
    else:
        out, lse = _VarlenAttnFn.apply(q, k, v, cu_q, cu_k, max_seqlen_q, max_seqlen_k, softmax_scale, cflag, wl,
                                       wr, softcap, al, dropout_p, chunk, su_q, su_k)
    if keep_cols is not None:
        out = out[..., :keep_cols]
    if return_attn_probs:
        # ragged lengths have no single SxS shape: per-sequence lists, as in the reference
        lses, probs = [], []
        for i in range(cu_q.numel() - 1):
            a, b = int(cu_q[i]), int(cu_q[i + 1])
            c, e = int(cu_k[i]), int(cu_k[i + 1])
            if su_q is not None:
                b = a + int(su_q[i])
            if su_k is not None:
                e = c + int(su_k[i])
            qh = q[a:b].unsqueeze(0).transpose(1, 2)
            kh = k[c:e].unsqueeze(0).transpose(1, 2)
            lse_i = lse[:, a:b].unsqueeze(0)
            lses.append(lse_i.squeeze(0))
            probs.append(_attn_probs(qh, kh, lse_i, softmax_scale, bool(cflag), wl, wr, softcap, al, chunk).squeeze(0))
        return out, lses, probs
    return out


def flash_attn_varlen_qkvpacked_func(qkv, cu_seqlens, max_seqlen, dropout_p=0.0, softmax_scale=None, causal=False,
                                     window_size=(-1, -1), softcap=0.0, alibi_slopes=None, deterministic=False,
                                     return_attn_probs=False, **kw):
    """qkv: (total_tokens, 3, nheads, headdim)."""
    return flash_attn_varlen_func(qkv[:, 0], qkv[:, 1], qkv[:, 2], cu_seqlens, cu_seqlens, max_seqlen, max_seqlen,
                                  dropout_p, softmax_scale, causal, window_size, softcap, alibi_slopes,
                                  deterministic, return_attn_probs, **kw)


def flash_attn_varlen_kvpacked_func(q, kv, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, dropout_p=0.0,
                                    softmax_scale=None, causal=False, window_size=(-1, -1), softcap=0.0,
                                    alibi_slopes=None, deterministic=False, return_attn_probs=False, **kw):
    """q: (total_q, nheads, d); kv: (total_k, 2, nheads_k, d)."""
    return flash_attn_varlen_func(q, kv[:, 0], kv[:, 1], cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                                  dropout_p, softmax_scale, causal, window_size, softcap, alibi_slopes,
                                  deterministic, return_attn_probs, **kw)


def flash_attn_combine(out_partial, lse_partial, out=None, out_dtype=None):
    """Merge split-KV partial results: out_partial (nsplit, B, S, H, D), lse_partial (nsplit, B, H, S)
    natural-log LSE  ->  (B, S, H, D).  One GPU kernel (the reference does this in torch,
    flash_attn_interface.py:567-580)."""
    if not out_partial.is_cuda:
        raise ValueError("fable_attn: flash_attn_combine needs CUDA tensors")
    dt = out_dtype or out_partial.dtype
    res, _ = _C.combine(out_partial.contiguous(), lse_partial.float().contiguous(), dt, False)
    if out is not None:
        out.copy_(res)
        return out
    return res


@torch.no_grad()
def flash_attn_with_kvcache(q, k_cache, v_cache, k=None, v=None, qv=None, rotary_cos=None, rotary_sin=None,
                            cache_seqlens=None, cache_batch_idx=None, cache_leftpad=None, block_table=None,
                            softmax_scale=None, causal=False, window_size=(-1, -1), softcap=0.0,
                            rotary_interleaved=True, alibi_slopes=None, num_splits=0, return_softmax_lse=False, *,
                            page_table=None, attention_chunk=0, q_descale=None, k_descale=None, v_descale=None,
                            pack_gqa=None, sm_margin=0, scheduler_metadata=None, cu_seqlens_q=None,
                            cu_seqlens_k_new=None, max_seqlen_q=None, rotary_seqlens=None):
    """Decode / multi-token decode against a KV cache (split-K kernel + LSE merge kernel).

    q: (batch, seqlen_q, nheads, headdim); seqlen_q > 1 places the new tokens at
    cache_seqlens .. cache_seqlens+seqlen_q-1 with causality among them when k/v are appended.
    Paged cache: k_cache/v_cache (num_blocks, page_block_size, nheads_k, headdim) + block_table
    (batch, max_blocks); a dense cache (batch, seqlen, nheads_k, headdim) is one page per row.
    cache_seqlens is the cache length BEFORE appending k/v.  rotary_cos/sin are tables
    (seqlen_ro, rotary_dim/2).  page_table is the FA-3 name of block_table.  Returns out, or
    (out, softmax_lse (batch, nheads, seqlen_q)) with return_softmax_lse."""
    _reject_fp8(q_descale, k_descale, v_descale)
    _accept_hints(num_splits, pack_gqa, sm_margin)
    if softmax_scale is None:
        softmax_scale = (q.shape[-1] + (qv.shape[-1] if qv is not None else 0)) ** -0.5
    del scheduler_metadata  # precomputed FA-3 schedules are not needed: the launcher plans per call
    if cu_seqlens_k_new is not None:
        raise NotImplementedError("fable_attn: cu_seqlens_k_new (ragged append) is not supported; append the "
                                  "same number of tokens to every sequence")
    if not q.is_cuda:
        raise ValueError("fable_attn: tensors must be on a CUDA device (q.is_cuda is False)")
    if cu_seqlens_q is not None and k is None and v is None and qv is None:
        # Varlen queries (q (total_q, nheads, d), sequence i = tokens cu[i] .. cu[i+1]-1 attending to
        # cache row i) as ONE decode launch, with no host synchronisation: the tokens are scattered on
        # the device into a (batch, max_seqlen_q) query block, decoded as multi-token decode (token t
        # of sequence i sits at position cache_seqlens[i] + t), and gathered back.  Rows past a
        # sequence's length are computed on zeros and dropped.  max_seqlen_q bounds the block (when it
        # is not given it is read from cu_seqlens_q, the one synchronising step).
        q3 = q if q.dim() == 3 else q.reshape(-1, q.shape[-2], q.shape[-1])
        cu = cu_seqlens_q.to(device=q.device, dtype=torch.long)
        B = cu.numel() - 1
        mq = int(max_seqlen_q) if max_seqlen_q is not None else int((cu[1:] - cu[:-1]).max())
        tok = torch.arange(q3.shape[0], device=q.device)
        seq = torch.searchsorted(cu[1:], tok, right=True).clamp_max(max(B - 1, 0))
        slot = (seq * mq + (tok - cu[seq])).clamp(0, max(B * mq - 1, 0))
        qpad = q3.new_zeros((B * mq,) + tuple(q3.shape[1:])).index_copy_(0, slot, q3).view(B, mq, *q3.shape[1:])
        r = flash_attn_with_kvcache(qpad, k_cache, v_cache, rotary_cos=rotary_cos, rotary_sin=rotary_sin,
                                    cache_seqlens=cache_seqlens, cache_batch_idx=cache_batch_idx,
                                    cache_leftpad=cache_leftpad, block_table=block_table,
                                    softmax_scale=softmax_scale, causal=causal, window_size=window_size,
                                    softcap=softcap, rotary_interleaved=rotary_interleaved, alibi_slopes=alibi_slopes,
                                    num_splits=num_splits, return_softmax_lse=return_softmax_lse,
                                    page_table=page_table, attention_chunk=attention_chunk, pack_gqa=pack_gqa,
                                    sm_margin=sm_margin, rotary_seqlens=rotary_seqlens)
        o = r[0] if return_softmax_lse else r
        out = o.reshape(B * mq, *o.shape[2:]).index_select(0, slot)
        if q.dim() == 4:
            out = out.unsqueeze(0)
        if not return_softmax_lse:
            return out
        lse = r[1].transpose(0, 1).reshape(r[1].shape[1], B * mq).index_select(1, slot)   # (nheads, total_q)
        return out, lse
    if q.dim() != 4:
        raise ValueError(f"fable_attn: decode expects q as (batch, seqlen_q, nheads, headdim), got {tuple(q.shape)}")
    if cu_seqlens_q is not None:
        # with new k / v appended, each sequence's call gets the whole k / v (the reference's
        # per-sequence form, package/fable_attn/flash_attn_interface.py:636-658)
        cu = cu_seqlens_q.to(torch.int32).cpu()
        outs, lses = [], []
        for i in range(cu.numel() - 1):
            a, b = int(cu[i]), int(cu[i + 1])
            qi = q[a:b].unsqueeze(0) if q.dim() == 3 else q[:, a:b]
            csi = cache_seqlens[i:i + 1] if torch.is_tensor(cache_seqlens) else cache_seqlens
            r = flash_attn_with_kvcache(qi, k_cache, v_cache, k=k, v=v, qv=qv, rotary_cos=rotary_cos,
                                        rotary_sin=rotary_sin, cache_seqlens=csi, cache_batch_idx=cache_batch_idx,
                                        cache_leftpad=cache_leftpad, block_table=block_table,
                                        softmax_scale=softmax_scale, causal=causal, window_size=window_size,
                                        softcap=softcap, rotary_interleaved=rotary_interleaved,
                                        alibi_slopes=alibi_slopes, num_splits=num_splits,
                                        return_softmax_lse=return_softmax_lse, page_table=page_table,
                                        attention_chunk=attention_chunk, pack_gqa=pack_gqa, sm_margin=sm_margin,
                                        rotary_seqlens=rotary_seqlens)
            if return_softmax_lse:
                outs.append(r[0].squeeze(0))
                lses.append(r[1])
            else:
                outs.append(r.squeeze(0))
        out = torch.cat(outs, dim=0)
        return (out, torch.cat(lses, dim=0)) if return_softmax_lse else out
    if page_table is not None:
        if block_table is not None:
            raise ValueError("fable_attn: block_table and page_table are the same argument; give one")
        block_table = page_table

    B, NQ = q.shape[0], q.shape[1]
    dev = q.device
    d_real = q.shape[-1]
    if qv is not None:
        # score += qv.v^T over the whole cache: correct but doubles cache traffic (compat path)
        if qv.shape[-1] != v_cache.shape[-1]:
            raise ValueError("fable_attn: qv.shape[-1] must equal the value head_dim")
        if d_real + qv.shape[-1] > _MAX_D:
            raise NotImplementedError(f"fable_attn: qv in decode needs headdim+headdim_v <= {_MAX_D}")
        q = torch.cat([q, qv], dim=-1)
        k_cache = torch.cat([k_cache, v_cache], dim=-1)
        v_cache = torch.cat([v_cache, torch.zeros_like(v_cache[..., :d_real])], dim=-1)
        if k is not None:
            k = torch.cat([k, v], dim=-1)
            v = torch.cat([v, torch.zeros_like(v[..., :d_real])], dim=-1)

    if cache_seqlens is None:
        seqlens = torch.full((B,), k_cache.shape[1], dtype=torch.int32, device=dev)
    elif isinstance(cache_seqlens, int):
        seqlens = torch.full((B,), cache_seqlens, dtype=torch.int32, device=dev)
    else:
        seqlens = cache_seqlens.to(device=dev, dtype=torch.int32).contiguous()

    if block_table is None:
        page = k_cache.shape[1]
        if page & (page - 1):
            raise NotImplementedError(f"fable_attn: dense cache length {page} must be a power of two "
                                      "(or pass block_table)")
        rows = (torch.arange(B, dtype=torch.int32, device=dev) if cache_batch_idx is None
                else cache_batch_idx.to(device=dev, dtype=torch.int32))
        bt = rows.contiguous().view(B, 1)
    else:
        if cache_batch_idx is not None:
            raise ValueError("fable_attn: cache_batch_idx applies to a dense cache only; with a paged cache "
                             "block_table selects the rows")
        bt = block_table.to(device=dev, dtype=torch.int32).contiguous()

    _, wl, _ = _map_window(True, window_size)
    win = (wl + 1) if wl >= 0 else -1          # keys visible behind the query, itself included
    lp = cache_leftpad.to(device=dev, dtype=torch.int32).contiguous() if cache_leftpad is not None else None
    chunk = _check_chunk(attention_chunk)
    if chunk:
        if NQ > 1:
            raise NotImplementedError("fable_attn: attention_chunk in decode is supported for one new token "
                                      "per sequence (the chunk start differs per token)")
        start = ((seqlens.to(torch.int64) // chunk) * chunk).to(torch.int32)
        lp = start if lp is None else torch.maximum(lp, start)
    al = alibi_slopes.float().contiguous() if alibi_slopes is not None else None
    cos = rotary_cos.float().contiguous() if rotary_cos is not None else None
    sin = rotary_sin.float().contiguous() if rotary_sin is not None else None
    rdim = int(cos.shape[-1] * 2) if cos is not None else 0
    rpos = rotary_seqlens.to(device=dev, dtype=torch.int32).contiguous() if rotary_seqlens is not None else None
    if (k is None) != (v is None):
        raise ValueError("fable_attn: k and v are appended to the cache together")
    nk = k.contiguous() if k is not None else None
    nv = v.contiguous() if v is not None else None

    cut = None
    kc, vc = k_cache, v_cache
    dq = q.shape[-1]
    dp = _pad_dim(dq)
    if dp is None:
        raise ValueError(f"fable_attn: head_dim={dq} exceeds the maximum {_MAX_D}")
    if dp != dq:
        q, kc, vc = _pad_last(q, dp), _pad_last(kc, dp), _pad_last(vc, dp)
        if nk is not None:
            nk, nv = _pad_last(nk, dp), _pad_last(nv, dp)
        cut = dq
    if qv is not None:
        cut = v_cache.shape[-1] - d_real if cut is None else cut
    out, lse = _C.dec(q.contiguous(), kc.contiguous(), vc.contiguous(), bt, seqlens, nk, nv, cos, sin,
                      bool(rotary_interleaved), float(softmax_scale), int(win), int(num_splits or 0), lp,
                      bool(return_softmax_lse), float(softcap or 0.0), al, int(rdim), rpos)
    if qv is not None:
        out = out[..., :qv.shape[-1]].contiguous()
    elif cut is not None:
        out = out[..., :cut].contiguous()
    if return_softmax_lse:
        return out, lse.transpose(1, 2).contiguous()
    return out
