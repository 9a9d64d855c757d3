"""CPU tests of the C-ABI shared library: it loads without a GPU, exports every entry point the
header declares, its structs have the layout the header gives (checked with the C compiler), and
malformed requests are refused with a status code before any device work."""
import ctypes as C
import os
import subprocess
import tempfile

import pytest

import fa_abi as A

STRUCTS = {
    "FaStrides": A.FaStrides, "FaFwdParams": A.FaFwdParams, "FaBwdParams": A.FaBwdParams,
    "FaDecParams": A.FaDecParams, "FaCombineParams": A.FaCombineParams,
    "FaPeerMergeParams": A.FaPeerMergeParams,
}


def test_library_loads_and_exports_declared_symbols():
    L = A.lib()
    names = A.declared_symbols()
    assert {"fa_forward_launch", "fable_attn_backward_launch", "fa_decode_launch", "fa_combine_launch"} <= set(names)
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/fable_attn.h but not exported"
    assert L.fa_abi_version() == 1


def test_ctypes_mirror_matches_header_layout():
    """Compile a probe against include/fable_attn.h and compare sizeof/offsetof with the mirror."""
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "fable_attn.h"', "int main(void){"]
    for sname, cls in STRUCTS.items():
        lines.append(f'printf("{sname} size %zu\\n", sizeof({sname}));')
        for fname, _ in cls._fields_:
            lines.append(f'printf("{sname} {fname} %zu\\n", offsetof({sname}, {fname}));')
    lines.append("return 0;}")
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "probe.c"), os.path.join(d, "probe")
        open(src, "w").write("\n".join(lines))
        subprocess.run(["gcc", "-I", os.path.dirname(A.HEADER), src, "-o", exe], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {}
    for ln in out:
        if ln:
            s, f, v = ln.split()
            got[(s, f)] = int(v)
    for sname, cls in STRUCTS.items():
        assert got[(sname, "size")] == C.sizeof(cls), sname
        for fname, _ in cls._fields_:
            assert got[(sname, fname)] == getattr(cls, fname).offset, f"{sname}.{fname}"


def test_struct_size_mismatch_is_refused():
    L = A.lib()
    p = A.FaFwdParams()
    p.struct_size = C.sizeof(A.FaFwdParams) - 8
    assert L.fa_forward_launch(C.byref(p), 0, None) == A.FA_ERR_ABI
    assert b"struct_size" in L.fa_last_error()
    assert L.fa_forward_launch(None, 0, None) == A.FA_ERR_INVALID


def _fwd_params(**kw):
    p = A.FaFwdParams()
    p.struct_size = C.sizeof(A.FaFwdParams)
    # non-null placeholders: validation rejects before any pointer is dereferenced
    p.Q = p.K = p.V = p.O = 16
    p.batch, p.SQ, p.SK, p.HD, p.NH, p.gqa = 1, 8, 8, 64, 2, 1
    p.scale = 0.125
    p.win_left = p.win_right = -1
    for k, v in kw.items():
        setattr(p, k, v)
    return p


@pytest.mark.parametrize("kw,code", [
    (dict(HD=72), A.FA_ERR_UNSUPPORTED), (dict(NH=3, gqa=2), A.FA_ERR_INVALID),
    (dict(dropout_p=1.0), A.FA_ERR_INVALID), (dict(Q=None), A.FA_ERR_INVALID),
    (dict(attn_chunk=-4), A.FA_ERR_INVALID), (dict(cu_q=16), A.FA_ERR_INVALID)])
def test_forward_rejects_bad_requests(kw, code):
    L = A.lib()
    p = _fwd_params(**kw)
    assert L.fa_forward_launch(C.byref(p), 1, None) == code
    assert L.fa_forward_launch(C.byref(_fwd_params()), 7, None) == A.FA_ERR_INVALID   # dtype code


def test_decode_rejects_bad_requests():
    L = A.lib()
    p = A.FaDecParams()
    p.struct_size = C.sizeof(A.FaDecParams)
    p.q = p.Kc = p.Vc = p.block_table = p.o = p.scratch = p.ctx_len = 16
    p.batch, p.NH, p.gqa, p.HD, p.page, p.max_blocks, p.nsplit, p.window = 1, 8, 4, 128, 24, 4, 1, -1
    assert L.fa_decode_launch(C.byref(p), 1, None, None, None) == A.FA_ERR_INVALID   # page not a power of 2
    p.page = 16
    p.nsplit = 0
    assert L.fa_decode_launch(C.byref(p), 1, None, None, None) == A.FA_ERR_INVALID
    p.nsplit = 1
    assert L.fa_decode_launch(C.byref(p), 1, None, C.c_void_p(16), None) == A.FA_ERR_INVALID  # new_k without new_v


def test_peer_merge_rejects_bad_requests():
    """Argument checks of the peer-memory merge run before any launch (no GPU needed)."""
    L = A.lib()
    p = A.FaPeerMergeParams()
    p.struct_size = C.sizeof(A.FaPeerMergeParams) - 8
    assert L.fa_peer_merge_launch(C.byref(p), None) == A.FA_ERR_ABI
    p.struct_size = C.sizeof(A.FaPeerMergeParams)
    p.peer_bufs = p.peer_signals = p.out = p.step = 16
    p.rank, p.world, p.B, p.S, p.H, p.D, p.out_dtype = 0, 9, 1, 1, 8, 128, 1
    assert L.fa_peer_merge_launch(C.byref(p), None) == A.FA_ERR_INVALID     # more than 8 ranks
    p.world, p.rank = 2, 2
    assert L.fa_peer_merge_launch(C.byref(p), None) == A.FA_ERR_INVALID     # rank outside the world
    p.rank, p.D = 1, 126
    assert L.fa_peer_merge_launch(C.byref(p), None) == A.FA_ERR_INVALID     # D not a multiple of 4
    p.D, p.slot_floats = 128, 8 * 129
    assert L.fa_peer_merge_launch(C.byref(p), None) == A.FA_ERR_INVALID     # two slots without done_ctas
    p.done_ctas, p.slot_floats = 16, 8 * 128
    assert L.fa_peer_merge_launch(C.byref(p), None) == A.FA_ERR_INVALID     # slot smaller than a partial
    p.world = 0
    assert L.fa_peer_step_end_launch(C.byref(p), None) == A.FA_ERR_INVALID


def test_split_heuristic_bounds():
    L = A.lib()
    assert L.fa_decode_num_splits(16, 1, 8, 32768, 0) >= 1
    assert L.fa_decode_num_splits(1, 1, 1, 100, 0) == 1            # short context: one split
    assert L.fa_decode_num_splits(1, 1, 1, 1 << 30, 0) <= 512
    assert L.fa_decode_num_splits(4, 1, 8, 32768, 7) == 7            # caller's num_splits honoured
    assert L.fa_decode_num_splits(4, 1, 8, 32768, 9999) == 512
    assert L.fa_decode_scratch_floats(2, 3, 4, 64, 5) == 2 * 3 * 4 * 5 * 66
