"""fa_decode_launch_noalloc: decode for callers that cannot allocate device memory at call time
(a host binding only the C ABI with no CUDA allocator of its own, a process whose HBM is reserved
up front by a pool, a decode step that cannot afford cudaMalloc/cudaFree).  Its split-K scratch
comes from a fixed array inside the library instead of the caller.

Checked through the C ABI against the allocating entry point (fa_decode_launch) on the same
inputs, for two calls in a row (the array keeps the previous call's contents), within the decode
tests' rel_rms bar; plus the size refusal.  Collected last so a failure here comes after every
other test has run."""
import ctypes as C

import numpy as np
import pytest
import torch

import fa_abi as A
from gpu_util import TOL, randn, stream, to_np

pytestmark = pytest.mark.gpu


# (nq, page, ctx): nq = 2 runs the CUDA-core split-K partial; nq = 1 with head_dim 128 and a page
# of at least 8 runs the tensor-core partial (stream-K work split; the 5-position context leaves
# most of its split slots empty, which the merge must see as empty in the reused array)
SHAPES = {"cuda_core": (2, 16, (700, 333, 1021)), "tensor_core": (1, 256, (700, 5, 3000))}


def _decode_case(dt, nsplit, shape="cuda_core"):
    rng = np.random.default_rng(2024)
    nq, page, ctx = SHAPES[shape]
    B, NH, gqa, HD = 3, 16, 4, 128
    NKV = NH // gqa
    ctx = np.array(ctx, np.int32)
    max_blocks = int((ctx.max() + nq + page - 1) // page)
    nblocks = B * max_blocks
    bt = rng.permutation(nblocks).astype(np.int32).reshape(B, max_blocks)
    _, kc = randn(rng, (nblocks, page, NKV, HD), dt)
    _, vc = randn(rng, (nblocks, page, NKV, HD), dt)
    _, q = randn(rng, (B, nq, NH, HD), dt)
    keep = dict(bt=torch.from_numpy(bt).cuda(), ctx=torch.from_numpy(ctx).cuda(), q=q, kc=kc, vc=vc)

    def params(o, lse, scratch):
        p = A.FaDecParams()
        p.struct_size = C.sizeof(A.FaDecParams)
        p.q, p.Kc, p.Vc, p.block_table, p.o = A.ptr(q), A.ptr(kc), A.ptr(vc), A.ptr(keep["bt"]), A.ptr(o)
        p.scratch, p.ctx_len, p.lse_out = A.ptr(scratch), A.ptr(keep["ctx"]), A.ptr(lse)
        p.batch, p.NH, p.gqa, p.HD, p.page, p.max_blocks, p.nsplit, p.window = B, NH, gqa, HD, page, max_blocks, nsplit, -1
        p.scale, p.nq, p.num_blocks = HD ** -0.5, nq, nblocks
        return p

    return keep, params, (B, nq, NH, HD)


@pytest.mark.parametrize("shape", ["cuda_core", "tensor_core"])
@pytest.mark.parametrize("dt", ["bf16", "fp16"])
def test_noalloc_matches_allocating_decode_twice(dt, shape):
    L = A.lib()
    L.fa_decode_launch_noalloc.argtypes = [C.POINTER(A.FaDecParams), C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
    nsplit = 6
    keep, params, (B, nq, NH, HD) = _decode_case(dt, nsplit, shape)
    o_ref = torch.empty((B, nq, NH, HD), device="cuda", dtype=keep["q"].dtype)
    l_ref = torch.empty((B, nq, NH), device="cuda", dtype=torch.float32)
    scratch = torch.empty(L.fa_decode_scratch_floats(B, nq, NH, HD, nsplit), device="cuda")
    A.check(L.fa_decode_launch(C.byref(params(o_ref, l_ref, scratch)), A.DT[dt], stream(), None, None))
    torch.cuda.synchronize()
    for call in range(2):
        o = torch.full_like(o_ref, float("nan"))
        lse = torch.full_like(l_ref, float("nan"))
        torch.cuda.synchronize()
        before = torch.cuda.memory_allocated()
        p = params(o, lse, None)            # no scratch from the caller
        A.check(L.fa_decode_launch_noalloc(C.byref(p), A.DT[dt], stream(), None, None))
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated() == before
        e = float(np.sqrt(((to_np(o) - to_np(o_ref)) ** 2).sum() / (to_np(o_ref) ** 2).sum()))
        assert e < TOL[dt], f"call {call}: O rel_rms {e:.3e}"
        el = float(np.sqrt(((lse.cpu().numpy() - l_ref.cpu().numpy()) ** 2).sum() / (l_ref.cpu().numpy() ** 2).sum()))
        assert el < TOL[dt], f"call {call}: LSE rel_rms {el:.3e}"


def test_noalloc_refuses_oversized_requests():
    L = A.lib()
    L.fa_decode_launch_noalloc.argtypes = [C.POINTER(A.FaDecParams), C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
    keep, params, (B, nq, NH, HD) = _decode_case("bf16", 512)
    o = torch.empty((B, nq, NH, HD), device="cuda", dtype=torch.bfloat16)
    p = params(o, None, None)
    assert L.fa_decode_scratch_floats(B, nq, NH, HD, 512) > (4 << 20)
    assert L.fa_decode_launch_noalloc(C.byref(p), A.DT["bf16"], stream(), None, None) == A.FA_ERR_SIZE
    assert b"maximum" in L.fa_last_error()
