"""ctypes mirror of include/fable_attn.h for the tests (the binding a ctypes host would write).

The struct definitions follow the header field by field; tests/test_abi.py checks that every
FA_API symbol the header declares is exported and that struct_size mismatches are refused.
"""
import ctypes as C
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(ROOT, "flash-attention-rdna2_b200", "fable_attn", "libfable_attn.so")
HEADER = os.path.join(ROOT, "include", "fable_attn.h")

FA_OK, FA_ERR_ABI, FA_ERR_INVALID, FA_ERR_UNSUPPORTED, FA_ERR_CUDA, FA_ERR_SIZE = range(6)
DT = {"fp16": 0, "bf16": 1, "fp32": 2}


class FaStrides(C.Structure):
    _fields_ = [("b", C.c_longlong), ("h", C.c_longlong), ("s", C.c_longlong)]


class FaFwdParams(C.Structure):
    _fields_ = [("struct_size", C.c_uint), ("Q", C.c_void_p), ("K", C.c_void_p), ("V", C.c_void_p),
                ("O", C.c_void_p), ("LSE", C.c_void_p), ("sQ", FaStrides), ("sK", FaStrides), ("sV", FaStrides),
                ("sO", FaStrides), ("batch", C.c_int), ("SQ", C.c_int), ("SK", C.c_int), ("HD", C.c_int),
                ("NH", C.c_int), ("gqa", C.c_int), ("scale", C.c_float), ("softcap", C.c_float),
                ("causal", C.c_int), ("win_left", C.c_int), ("win_right", C.c_int), ("attn_chunk", C.c_int),
                ("alibi_slopes", C.c_void_p), ("dropout_p", C.c_float), ("philox_seed", C.c_ulonglong),
                ("cu_q", C.c_void_p), ("cu_k", C.c_void_p), ("seqused_q", C.c_void_p), ("seqused_k", C.c_void_p),
                ("lse_total_q", C.c_longlong), ("dropout_bits", C.c_void_p), ("total_k", C.c_longlong),
                ("block_table", C.c_void_p), ("page", C.c_int), ("max_blocks", C.c_int), ("num_blocks", C.c_longlong),
                ("rot_cos", C.c_void_p), ("rot_sin", C.c_void_p), ("rot_dim", C.c_int), ("rot_seqlen_ro", C.c_int),
                ("rot_interleaved", C.c_int)]


class FaBwdParams(C.Structure):
    _fields_ = [("struct_size", C.c_uint)] + [(n, C.c_void_p) for n in
                                               ("Q", "K", "V", "O", "dO", "dQ", "dK", "dV", "lse", "dsum")] + [
        (n, FaStrides) for n in ("qs", "ks", "vs", "os", "dos", "dqs", "dks", "dvs")] + [
        (n, C.c_int) for n in ("B", "Hq", "Hk", "SQ", "SK", "D", "gqa")] + [
        ("scale", C.c_float), ("softcap", C.c_float), ("alibi", C.c_void_p), ("causal", C.c_int),
        ("win_left", C.c_int), ("win_right", C.c_int), ("dropout", C.c_int), ("drop_seed", C.c_ulonglong),
        ("dropout_p", C.c_float), ("keep_scale", C.c_float), ("cu_q", C.c_void_p), ("cu_k", C.c_void_p),
        ("seqused_q", C.c_void_p), ("seqused_k", C.c_void_p), ("lse_total_q", C.c_longlong),
        ("dropout_bits", C.c_void_p), ("total_k", C.c_longlong), ("dropout_bits_t", C.c_void_p)]


class FaDecParams(C.Structure):
    _fields_ = [("struct_size", C.c_uint), ("q", C.c_void_p), ("Kc", C.c_void_p), ("Vc", C.c_void_p),
                ("block_table", C.c_void_p), ("o", C.c_void_p), ("scratch", C.c_void_p), ("ctx_len", C.c_void_p),
                ("cos", C.c_void_p), ("sin", C.c_void_p)] + [
        (n, C.c_int) for n in ("batch", "NH", "gqa", "HD", "page", "max_blocks", "nsplit", "window", "rotary")] + [
        ("scale", C.c_float), ("leftpad", C.c_void_p), ("lse_out", C.c_void_p), ("softcap", C.c_float),
        ("alibi", C.c_void_p), ("nq", C.c_int), ("append", C.c_int), ("rotary_dim", C.c_int),
        ("rotary_pos", C.c_void_p), ("num_blocks", C.c_longlong), ("err_flag", C.c_void_p), ("o_f32", C.c_int)]


class FaCombineParams(C.Structure):
    _fields_ = [("struct_size", C.c_uint), ("out_partial", C.c_void_p), ("in_dtype", C.c_int),
                ("lse_partial", C.c_void_p), ("out", C.c_void_p), ("out_dtype", C.c_int), ("lse_out", C.c_void_p),
                ("nsplit", C.c_int), ("B", C.c_int), ("S", C.c_int), ("H", C.c_int), ("D", C.c_int),
                ("out_split_stride", C.c_longlong), ("lse_split_stride", C.c_longlong), ("lse_bsh", C.c_int)]


class FaPeerMergeParams(C.Structure):
    _fields_ = [("struct_size", C.c_uint), ("peer_bufs", C.c_void_p), ("peer_signals", C.c_void_p),
                ("rank", C.c_int), ("world", C.c_int), ("B", C.c_int), ("S", C.c_int), ("H", C.c_int),
                ("D", C.c_int), ("out", C.c_void_p), ("out_dtype", C.c_int), ("lse_out", C.c_void_p),
                ("step", C.c_void_p), ("err_flag", C.c_void_p), ("wait_ns", C.c_ulonglong),
                ("slot_floats", C.c_longlong), ("done_ctas", C.c_void_p)]


_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        L = C.CDLL(LIB_PATH)
        L.fa_forward_launch.argtypes = [C.POINTER(FaFwdParams), C.c_int, C.c_void_p]
        L.fable_attn_backward_launch.argtypes = [C.POINTER(FaBwdParams), C.c_int, C.c_void_p]
        L.fa_decode_launch.argtypes = [C.POINTER(FaDecParams), C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
        L.fa_decode_num_splits.argtypes = [C.c_int, C.c_int, C.c_int, C.c_longlong, C.c_int]
        L.fa_decode_scratch_floats.restype = C.c_longlong
        L.fa_decode_scratch_floats.argtypes = [C.c_int] * 5
        L.fa_combine_launch.argtypes = [C.POINTER(FaCombineParams), C.c_void_p]
        L.fa_peer_merge_launch.argtypes = [C.POINTER(FaPeerMergeParams), C.c_void_p]
        L.fa_peer_step_end_launch.argtypes = [C.POINTER(FaPeerMergeParams), C.c_void_p]
        L.fa_dropout_mask_words.restype = C.c_longlong
        L.fa_dropout_mask_words.argtypes = [C.c_int] * 3
        L.fa_dropout_mask_launch.argtypes = [C.c_ulonglong, C.c_float] + [C.c_int] * 6 + [C.c_void_p, C.c_void_p]
        L.fa_last_error.restype = C.c_char_p
        L.fa_kernel_launch_count.restype = C.c_ulonglong
        _LIB = L
    return _LIB


def declared_symbols():
    """Function names the header exports (FA_API declarations)."""
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"^FA_API\s+[\w\s\*]*?\b(\w+)\s*\(", txt, re.M)))


def check(rc):
    if rc != FA_OK:
        raise RuntimeError(f"fable_attn C ABI returned {rc}: {lib().fa_last_error().decode()}")


def ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def strides4(t):
    """[B,H,S,D] view strides."""
    return FaStrides(t.stride(0), t.stride(1), t.stride(2))


def strides_bshd(t):
    """(B,S,H,D) tensor seen as [B,H,S,D]."""
    return FaStrides(t.stride(0), t.stride(2), t.stride(1))
