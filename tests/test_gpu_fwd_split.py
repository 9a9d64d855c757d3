"""Wave-tail split of the two-query-tile forward: units past the last full wave are cut into key
ranges run by separate CTAs and merged with flash_attn_combine's rule
(package/fable_attn/flash_attn_interface.py:567-580).  Checked against the oracle (small cases)
and against the unsplit kernel (the shard shape of the dense config at 8 GPUs)."""
import numpy as np
import pytest
import torch

from fable_attn import _C
from gpu_util import TOL, lse_close, randn, to_np
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _run(q, k, v):
    """The extension's forward on (B, S, H, D) tensors: (out (B, S, H, D), LSE (B, H, S))."""
    B, SQ, H, D = q.shape
    buf = torch.empty((B, SQ, H, D), dtype=q.dtype, device=q.device).transpose(1, 2)
    out, lse = _C.fwd(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), D ** -0.5, False, -1, -1, 0.0, None,
                      0.0, 0, 0, buf, None)
    torch.cuda.synchronize()
    return out.transpose(1, 2), lse


def _fwd(q, k, v, split, monkeypatch):
    monkeypatch.setenv("FABLE_ATTN_FWD_TILES", "2")
    monkeypatch.setenv("FABLE_ATTN_REQUIRE_TC", "1")
    if split is None:
        monkeypatch.delenv("FABLE_ATTN_FWD_SPLIT", raising=False)
    else:
        monkeypatch.setenv("FABLE_ATTN_FWD_SPLIT", str(split))
    return _run(q, k, v)


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("split", [2, 4, 8])
@pytest.mark.parametrize("SQ,SK", [(1024, 1024), (1000, 1160), (600, 2048)])
def test_split_matches_oracle(SQ, SK, split, dt, monkeypatch):
    """Every unit is a tail unit here (fewer units than SMs); ragged query and key lengths."""
    rng = np.random.default_rng(SQ * 7 + SK + split)
    B, NH, D = 1, 4, 128
    qn, q = randn(rng, (B, SQ, NH, D), dt)
    kn, k = randn(rng, (B, SK, NH, D), dt)
    vn, v = randn(rng, (B, SK, NH, D), dt)
    out, lse = _fwd(q, k, v, split, monkeypatch)
    ro, rl = O.forward(qn, kn, vn, D ** -0.5, False, -1, -1, 0.0, None, 0, 0.0, 0)
    e = O.rel_rms(to_np(out), ro)
    assert e < TOL[dt], f"O rel_rms {e:.3e}"
    ok, el = lse_close(lse.cpu().numpy(), rl, TOL[dt])
    assert ok, f"LSE {el:.3e}"


@pytest.mark.parametrize("dt", ["bf16"])
def test_split_equals_unsplit_at_the_8_gpu_shard_shape(dt, monkeypatch):
    """B1 S16384, 4 heads (32 heads over 8 GPUs): 256 units on the SMs, the tail split by the
    heuristic and by every forced range count, against the unsplit kernel."""
    rng = np.random.default_rng(8)
    _, q = randn(rng, (1, 16384, 4, 128), dt)
    _, k = randn(rng, (1, 16384, 4, 128), dt)
    _, v = randn(rng, (1, 16384, 4, 128), dt)
    ref_o, ref_l = _fwd(q, k, v, 1, monkeypatch)   # 1: no split
    for split in (None, 2, 4, 8):   # None: the heuristic's choice
        out, lse = _fwd(q, k, v, split, monkeypatch)
        e = ((out.float() - ref_o.float()).norm() / ref_o.float().norm()).item()
        assert e < 2e-3, f"split {split}: rel_rms vs unsplit {e:.3e}"
        assert (lse - ref_l).abs().max().item() < 1e-4
        assert torch.isfinite(out).all()
