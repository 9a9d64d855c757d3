"""flash_attn.bert_padding API in plain torch: pack a padded batch into the varlen layout and back.

transformers imports pad_input/unpad_input from here when attn_implementation is
"flash_attention_2", so the module must exist for the drop-in to import.  Gather/scatter with
autograd, same surface as the reference's package/fable_attn/bert_padding.py:18-126.
"""
import torch
import torch.nn.functional as F

__all__ = ["index_first_axis", "index_put_first_axis", "index_first_axis_residual", "pad_input", "unpad_input",
           "unpad_input_for_concatenated_sequences", "IndexFirstAxis", "IndexPutFirstAxis",
           "IndexFirstAxisResidual"]


class IndexFirstAxis(torch.autograd.Function):
    """out = input[indices] along dim 0; backward scatters into zeros."""

    @staticmethod
    def forward(ctx, input, indices):
        ctx.save_for_backward(indices)
        ctx.n = input.shape[0]
        return input[indices]

    @staticmethod
    def backward(ctx, grad_output):
        (indices,) = ctx.saved_tensors
        g = grad_output.new_zeros((ctx.n,) + tuple(grad_output.shape[1:]))
        g.index_copy_(0, indices, grad_output)
        return g, None


index_first_axis = IndexFirstAxis.apply


class IndexPutFirstAxis(torch.autograd.Function):
    """out = zeros(first_axis_dim, ...) with out[indices] = values."""

    @staticmethod
    def forward(ctx, values, indices, first_axis_dim):
        ctx.save_for_backward(indices)
        out = values.new_zeros((first_axis_dim,) + tuple(values.shape[1:]))
        out[indices] = values
        return out

    @staticmethod
    def backward(ctx, grad_output):
        (indices,) = ctx.saved_tensors
        return grad_output[indices], None, None


index_put_first_axis = IndexPutFirstAxis.apply


class IndexFirstAxisResidual(torch.autograd.Function):
    """Returns (input[indices], input) so the caller can add a residual to the full tensor."""

    @staticmethod
    def forward(ctx, input, indices):
        ctx.save_for_backward(indices)
        return input[indices], input.detach()

    @staticmethod
    def backward(ctx, grad_output, grad_residual):
        (indices,) = ctx.saved_tensors
        g = grad_residual.clone()
        g.index_add_(0, indices, grad_output)
        return g, None


index_first_axis_residual = IndexFirstAxisResidual.apply


def unpad_input(hidden_states, attention_mask, unused_mask=None):
    """hidden_states (batch, seqlen, ...), attention_mask (batch, seqlen) with 1 on real tokens.
    Returns (hidden_states_unpad, indices, cu_seqlens, max_seqlen_in_batch, used_seqlens_in_batch)."""
    mask = attention_mask + unused_mask if unused_mask is not None else attention_mask
    seqlens = mask.sum(dim=-1, dtype=torch.int32)
    used = attention_mask.sum(dim=-1, dtype=torch.int32)
    indices = torch.nonzero(mask.flatten(), as_tuple=False).flatten()
    max_len = int(seqlens.max().item())
    cu = F.pad(torch.cumsum(seqlens, dim=0, dtype=torch.int32), (1, 0))
    flat = hidden_states.reshape(-1, *hidden_states.shape[2:])
    return index_first_axis(flat, indices), indices, cu, max_len, used


def unpad_input_for_concatenated_sequences(hidden_states, attention_mask_in_length):
    """attention_mask_in_length (batch, seqlen) holds the lengths of the sequences packed in each
    row (zeros = padding).  Returns (hidden_states_unpad, indices, cu_seqlens, max_seqlen)."""
    length = attention_mask_in_length.sum(dim=-1)
    seqlen = attention_mask_in_length.size(-1)
    mask_2d = torch.arange(seqlen, device=length.device).unsqueeze(0) < length.unsqueeze(-1)
    nz = torch.nonzero(attention_mask_in_length.flatten(), as_tuple=False).flatten()
    seqlens = attention_mask_in_length.flatten()[nz]
    indices = torch.nonzero(mask_2d.flatten(), as_tuple=False).flatten()
    max_len = int(seqlens.max().item())
    cu = F.pad(torch.cumsum(seqlens, dim=0, dtype=torch.int32), (1, 0))
    flat = hidden_states.reshape(-1, *hidden_states.shape[2:])
    return index_first_axis(flat, indices), indices, cu, max_len


def pad_input(hidden_states, indices, batch, seqlen):
    """Inverse of unpad_input: (total, ...) -> (batch, seqlen, ...), zeros at padding."""
    out = index_put_first_axis(hidden_states, indices, batch * seqlen)
    return out.reshape(batch, seqlen, *out.shape[1:])
