"""CPU tests of the host-side Python layer: error behaviour, name registration, window mapping,
padding helpers, bert_padding and rotary (plain torch), and the torch-op fallback contract.
No kernel launches."""
import numpy as np
import pytest
import torch

import fable_attn as fa
from fable_attn import flash_attn_interface as fi
from fable_attn.layers import rotary


def test_cpu_tensors_are_rejected_not_computed():
    q = torch.randn(1, 16, 2, 64)
    with pytest.raises(ValueError, match="CUDA"):
        fa.flash_attn_func(q, q, q)
    with pytest.raises(ValueError, match="CUDA"):
        fa.flash_attn_with_kvcache(q[:, :1], q, q)


def test_fp8_and_hint_errors_precede_everything():
    q = torch.randn(1, 16, 2, 64)
    with pytest.raises(NotImplementedError, match="FP8"):
        fa.flash_attn_func(q, q, q, q_descale=torch.ones(1))
    with pytest.raises(TypeError):
        fa.flash_attn_func(q, q, q, num_splits="many")
    with pytest.raises(TypeError):
        fa.flash_attn_func(q, q, q, pack_gqa=1)
    with pytest.raises(ValueError):
        fa.flash_attn_func(q, q, q, attention_chunk=-1)
    with pytest.raises(NotImplementedError):
        fa.flash_attn_with_kvcache(q[:, :1], q, q, cu_seqlens_k_new=torch.zeros(2, dtype=torch.int32))


@pytest.mark.parametrize("causal,ws,exp", [
    (False, (-1, -1), (0, -1, -1)), (True, (-1, -1), (1, -1, 0)), (False, (-1, 0), (1, -1, 0)),
    (False, (32, 32), (0, 32, 32)), (True, (63, 5), (1, 63, 0)), (False, (0, -1), (0, 0, -1))])
def test_window_mapping(causal, ws, exp):
    assert fi._map_window(causal, ws) == exp


def test_head_dim_padding_table():
    assert [fi._pad_dim(d) for d in (1, 16, 17, 40, 100, 144, 200, 255, 256)] == [16, 16, 32, 48, 112, 160, 224,
                                                                                    256, 256]
    assert fi._pad_dim(257) is None


def test_install_as_flash_attn_registers_names():
    fa.install_as_flash_attn()
    import flash_attn
    import flash_attn_interface
    from flash_attn.bert_padding import pad_input, unpad_input  # noqa: F401
    from flash_attn.layers.rotary import apply_rotary_emb  # noqa: F401
    assert flash_attn.__version__.startswith("2.8.3")
    assert flash_attn_interface.flash_attn_func.__module__.endswith("fa3_interface")
    assert flash_attn.flash_attn_func is fa.flash_attn_func


def test_compat_distribution_metadata():
    import tomllib
    import os
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    meta = tomllib.load(open(os.path.join(root, "flash-attention-rdna2_b200", "compat", "pyproject.toml"), "rb"))
    assert meta["project"]["name"] == "flash_attn"
    major, minor, patch = (int(x) for x in meta["project"]["version"].split("+")[0].split("."))
    assert (major, minor, patch) >= (2, 3, 3)    # transformers' flash_attention_2 gate


def test_bert_padding_round_trip():
    torch.manual_seed(0)
    hs = torch.randn(3, 16, 8, requires_grad=True)
    am = torch.zeros(3, 16, dtype=torch.long)
    am[0, :10] = 1
    am[1, :] = 1
    am[2, :4] = 1
    unp, idx, cu, mx, used = fa.bert_padding.unpad_input(hs, am)
    assert unp.shape == (30, 8) and mx == 16 and cu.tolist() == [0, 10, 26, 30] and used.tolist() == [10, 16, 4]
    back = fa.bert_padding.pad_input(unp, idx, 3, 16)
    assert torch.equal(back * am[..., None], hs * am[..., None])
    back.sum().backward()
    assert torch.equal(hs.grad, am[..., None].float().expand(3, 16, 8))


@pytest.mark.parametrize("interleaved", [False, True])
def test_rotary_matches_pairwise_formula(interleaved):
    torch.manual_seed(1)
    B, S, H, D, rd = 2, 12, 3, 16, 8
    x = torch.randn(B, S, H, D, dtype=torch.float64)
    ang = torch.arange(40, dtype=torch.float64)[:, None] * 10000.0 ** (-2 * torch.arange(rd // 2) / rd)
    cos, sin = ang.cos(), ang.sin()
    y = rotary.apply_rotary_emb(x, cos, sin, interleaved=interleaved, seqlen_offsets=3)
    ref = x.clone().numpy()
    xn = x.numpy()
    for s in range(S):
        c, sn = cos[s + 3].numpy(), sin[s + 3].numpy()
        for i in range(rd // 2):
            a, b = (2 * i, 2 * i + 1) if interleaved else (i, i + rd // 2)
            ref[:, s, :, a] = xn[:, s, :, a] * c[i] - xn[:, s, :, b] * sn[i]
            ref[:, s, :, b] = xn[:, s, :, b] * c[i] + xn[:, s, :, a] * sn[i]
    assert np.allclose(y.numpy(), ref)
    # varlen form: positions restart per sequence
    cu = torch.tensor([0, 5, 12])
    xv = x[0].clone()
    yv = rotary.apply_rotary_emb(xv, cos, sin, interleaved=interleaved, cu_seqlens=cu)
    y0 = rotary.apply_rotary_emb(xv[None, :5], cos, sin, interleaved=interleaved)[0]
    y1 = rotary.apply_rotary_emb(xv[None, 5:], cos, sin, interleaved=interleaved)[0]
    assert torch.allclose(yv, torch.cat([y0, y1]))


def test_torch_op_returns_empty_on_unsupported():
    q = torch.randn(1, 2, 8, 64)
    assert fa.torch_op._forward(q, q, q, 0.125, True).numel() == 0          # CPU tensor
    assert fa.torch_op.REGISTERED


def test_rotary_arguments_validated_before_any_device_work():
    """rotary_cos / rotary_sin (keyword-only extension) must come together and cover every position
    (the reference's apply_rotary_emb indexes cos[pos]); both errors are raised on the host."""
    import torch
    import fable_attn
    q = torch.zeros(2, 50, 4, 64, dtype=torch.bfloat16)
    k = torch.zeros(2, 50, 2, 64, dtype=torch.bfloat16)
    cos = torch.zeros(49, 16)
    with pytest.raises(ValueError, match="seqlen_ro"):
        fable_attn.flash_attn_func(q, k, k, rotary_cos=cos, rotary_sin=cos)
    with pytest.raises(ValueError, match="go together"):
        fable_attn.flash_attn_func(q, k, k, rotary_cos=cos)
