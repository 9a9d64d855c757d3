"""FA-3 argument order (the `flash_attn_interface` module of flash-attn's hopper/ build).

FA-2 and FA-3 disagree on positional order: FA-2's 4th positional argument is dropout_p, FA-3's
is softmax_scale.  Guessing from the value would silently compute the wrong thing, so each order
has its own module: `import flash_attn` gives the FA-2 order (fable_attn.flash_attn_interface) and
`import flash_attn_interface` this one (registered by fable_attn.install_as_flash_attn()).  Both
call the same kernels; with return_attn_probs FA-3 returns the pair (out, softmax_lse).
Mirrors package/fable_attn/fa3_interface.py:26-102 of the reference.
"""
from . import flash_attn_interface as _fa2

__all__ = ["flash_attn_func", "flash_attn_qkvpacked_func", "flash_attn_varlen_func", "flash_attn_with_kvcache",
           "flash_attn_combine", "get_scheduler_metadata"]


def _pair(r, return_attn_probs):
    return (r[0], r[1]) if return_attn_probs else r


def flash_attn_func(q, k, v, softmax_scale=None, causal=False, qv=None, q_descale=None, k_descale=None,
                    v_descale=None, window_size=(-1, -1), attention_chunk=0, softcap=0.0, num_splits=1,
                    pack_gqa=None, deterministic=False, sm_margin=0, return_attn_probs=False):
    r = _fa2.flash_attn_func(q, k, v, 0.0, softmax_scale, causal, window_size, softcap, None, deterministic,
                             return_attn_probs, qv=qv, attention_chunk=attention_chunk, q_descale=q_descale,
                             k_descale=k_descale, v_descale=v_descale, num_splits=num_splits, pack_gqa=pack_gqa,
                             sm_margin=sm_margin)
    return _pair(r, return_attn_probs)


def flash_attn_qkvpacked_func(qkv, softmax_scale=None, causal=False, q_descale=None, k_descale=None,
                              v_descale=None, window_size=(-1, -1), attention_chunk=0, softcap=0.0, num_splits=1,
                              pack_gqa=None, deterministic=False, sm_margin=0, return_attn_probs=False):
    r = _fa2.flash_attn_qkvpacked_func(qkv, 0.0, softmax_scale, causal, window_size, softcap, None, deterministic,
                                       return_attn_probs, attention_chunk=attention_chunk, q_descale=q_descale,
                                       k_descale=k_descale, v_descale=v_descale, num_splits=num_splits,
                                       pack_gqa=pack_gqa, sm_margin=sm_margin)
    return _pair(r, return_attn_probs)


def flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, seqused_q=None,
                           seqused_k=None, softmax_scale=None, causal=False, qv=None, q_descale=None,
                           k_descale=None, v_descale=None, window_size=(-1, -1), attention_chunk=0, softcap=0.0,
                           num_splits=1, pack_gqa=None, deterministic=False, sm_margin=0, return_attn_probs=False):
    r = _fa2.flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, 0.0,
                                    softmax_scale, causal, window_size, softcap, None, deterministic,
                                    return_attn_probs, seqused_q=seqused_q, seqused_k=seqused_k, qv=qv,
                                    attention_chunk=attention_chunk, q_descale=q_descale, k_descale=k_descale,
                                    v_descale=v_descale, num_splits=num_splits, pack_gqa=pack_gqa,
                                    sm_margin=sm_margin)
    return _pair(r, return_attn_probs)


def flash_attn_with_kvcache(q, k_cache, v_cache, k=None, v=None, qv=None, rotary_cos=None, rotary_sin=None,
                            cache_seqlens=None, cache_batch_idx=None, cache_leftpad=None, page_table=None,
                            cu_seqlens_q=None, cu_seqlens_k_new=None, max_seqlen_q=None, rotary_seqlens=None,
                            q_descale=None, k_descale=None, v_descale=None, softmax_scale=None, causal=False,
                            window_size=(-1, -1), attention_chunk=0, softcap=0.0, rotary_interleaved=True,
                            scheduler_metadata=None, num_splits=0, pack_gqa=None, sm_margin=0,
                            return_softmax_lse=False):
    return _fa2.flash_attn_with_kvcache(
        q, k_cache, v_cache, k=k, v=v, qv=qv, rotary_cos=rotary_cos, rotary_sin=rotary_sin,
        cache_seqlens=cache_seqlens, cache_batch_idx=cache_batch_idx, cache_leftpad=cache_leftpad,
        block_table=None, softmax_scale=softmax_scale, causal=causal, window_size=window_size, softcap=softcap,
        rotary_interleaved=rotary_interleaved, alibi_slopes=None, num_splits=num_splits,
        return_softmax_lse=return_softmax_lse, page_table=page_table, attention_chunk=attention_chunk,
        q_descale=q_descale, k_descale=k_descale, v_descale=v_descale, pack_gqa=pack_gqa, sm_margin=sm_margin,
        scheduler_metadata=scheduler_metadata, cu_seqlens_q=cu_seqlens_q, cu_seqlens_k_new=cu_seqlens_k_new,
        max_seqlen_q=max_seqlen_q, rotary_seqlens=rotary_seqlens)


flash_attn_combine = _fa2.flash_attn_combine


def get_scheduler_metadata(*args, **kw):
    """FA-3 precomputes a schedule and takes it back as scheduler_metadata.  The launcher here
    plans every call itself in microseconds, so there is nothing to cache: None, which FA-3
    callers treat as 'plan it yourself'."""
    return None
