"""Failure detection on the GPU without a GPU fault: the bounded mbarrier wait the tensor-core
pipelines use gives up after its limit, records a bit in fa_device_error and lets the kernel
return; the context stays usable afterwards (a forward right after is checked against the
oracle).  The wait that runs out is one that nothing can satisfy (no copy or MMA in flight)."""
import numpy as np
import pytest
import torch

import fable_attn
from fable_attn import _C
from gpu_util import TOL, randn, to_np
from oracle import oracle as O

pytestmark = pytest.mark.gpu

FA_DEVERR_WAIT_SELFTEST = 65536


@pytest.mark.parametrize("limit_ns", [200_000, 2_000_000])
def test_bounded_wait_gives_up_and_reports(limit_ns):
    fable_attn.device_error(clear=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    _C.wait_selftest(limit_ns)
    e1.record()
    torch.cuda.synchronize()
    flags = fable_attn.device_error(clear=True)
    assert flags & FA_DEVERR_WAIT_SELFTEST, f"flags 0x{flags:x}"
    assert flags == FA_DEVERR_WAIT_SELFTEST, f"unexpected bits 0x{flags:x}"
    # the kernel gave up after (about) its limit, not at once and not much later
    ms = e0.elapsed_time(e1)
    assert limit_ns / 1e6 * 0.9 <= ms < limit_ns / 1e6 + 50.0, f"{ms:.3f} ms for a {limit_ns} ns limit"
    assert fable_attn.device_error() == 0
    # the context is still usable: a forward right after matches the oracle
    rng = np.random.default_rng(3)
    qn, q = randn(rng, (1, 256, 2, 128), "bf16")
    kn, k = randn(rng, (1, 256, 2, 128), "bf16")
    vn, v = randn(rng, (1, 256, 2, 128), "bf16")
    out = fable_attn.flash_attn_func(q, k, v, causal=True)
    ro, _ = O.forward(qn, kn, vn, 128 ** -0.5, True)
    assert O.rel_rms(to_np(out), ro) < TOL["bf16"]


def test_wait_selftest_rejects_bad_limits():
    with pytest.raises(ValueError, match="limit_ns"):
        _C.wait_selftest(0)
    with pytest.raises(ValueError, match="limit_ns"):
        _C.wait_selftest(20_000_000_000)
