"""Generate tests/golden/*.npz from the REFERENCE's own CPU oracle.

The reference (MatafakaRespect/flash-attention-rdna2) ships no golden files: its gates draw
seeded inputs and compare against `ref_attention` (kernels/fa_common.hpp:102-134) at run time.
This script runs that same function — compiled from the reference sources by oracle/Makefile
into oracle/_ref/libfa_ref.so — on small seeded inputs and stores inputs and outputs, so the
restated oracle (oracle/fa_oracle.c) and the GPU kernels can be checked against the reference's
numbers on machines where the reference is absent.  Also stores Philox known answers from the
reference's `philox` (kernels/fa_common.hpp:71-82).

Run from the repo root:  make -C oracle REF_DIR=<reference checkout> && python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import oracle as O  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))

# (name, SQ, SK, D, NH, gqa, causal, alibi, wl, wr, softcap, chunk) — shapes of the reference's
# forward gate table (kernels/fa_forward_gate.inc:170-205) scaled down to fixture size
FWD_CASES = [
    ("causal_gqa2", 48, 48, 64, 4, 2, True, False, -1, -1, 0.0, 0),
    ("full", 40, 40, 64, 2, 1, False, False, -1, -1, 0.0, 0),
    ("sq_lt_sk_bottom_right", 24, 56, 64, 2, 1, True, False, -1, -1, 0.0, 0),
    ("sq_gt_sk_empty_rows", 56, 16, 64, 2, 1, True, False, -1, -1, 0.0, 0),
    ("window_15_0", 48, 48, 64, 2, 1, True, False, 15, 0, 0.0, 0),
    ("window_8_8", 48, 48, 64, 2, 1, False, False, 8, 8, 0.0, 0),
    ("window_0_0", 32, 32, 32, 2, 1, False, False, 0, 0, 0.0, 0),
    ("window_0_open", 32, 32, 32, 2, 1, False, False, 0, -1, 0.0, 0),
    ("softcap30", 40, 40, 64, 2, 1, True, False, -1, -1, 30.0, 0),
    ("alibi", 40, 40, 64, 4, 1, True, True, -1, -1, 0.0, 0),
    ("chunk16_causal", 48, 48, 32, 2, 1, True, False, -1, -1, 0.0, 16),
    ("chunk20_full", 48, 48, 32, 2, 1, False, False, -1, -1, 0.0, 20),
    ("d128", 32, 32, 128, 2, 2, True, False, -1, -1, 0.0, 0),
    ("d16", 32, 32, 16, 2, 1, True, False, -1, -1, 0.0, 0),
]


def main():
    if O.ref_lib() is None:
        raise SystemExit("oracle/_ref/libfa_ref.so is missing: run `make -C oracle REF_DIR=<reference checkout>`")
    arrays = {}
    for i, (name, SQ, SK, D, NH, g, causal, al, wl, wr, sc, ch) in enumerate(FWD_CASES):
        rng = np.random.default_rng(1000 + i)
        q = O.round_to(rng.standard_normal((SQ, NH, D)), "fp16")
        k = O.round_to(rng.standard_normal((SK, NH // g, D)), "fp16")
        v = O.round_to(rng.standard_normal((SK, NH // g, D)), "fp16")
        slopes = (-(2.0 ** (-(8.0 * (np.arange(NH) + 1) / NH)))).astype(np.float32) if al else None
        o, lse = O.ref_forward(q, k, v, D ** -0.5, causal, wl, wr, sc, slopes, ch)
        p = f"fwd/{name}/"
        arrays[p + "q"] = q.astype(np.float16)
        arrays[p + "k"] = k.astype(np.float16)
        arrays[p + "v"] = v.astype(np.float16)
        arrays[p + "o"] = o
        arrays[p + "lse"] = lse
        arrays[p + "cfg"] = np.array([SQ, SK, D, NH, g, int(causal), int(al), wl, wr, sc, ch], dtype=np.float64)
        if slopes is not None:
            arrays[p + "slopes"] = slopes
    # Philox known answers from the reference's generator
    seeds = [0, 1, 777, 0x123456789ABCDEF, (1 << 63) - 25]
    idxs = [0, 1, 12345, 1 << 32, (1 << 40) + 7, 4096 * 4096 * 64 - 1]
    kat = np.array([[s, i, *O.ref_philox(s, i)] for s in seeds for i in idxs], dtype=np.uint64)
    arrays["philox/kat"] = kat
    # a keep mask: query head 3 of a 24x40 score block, p = 0.2, seed 777 (the reference gate's seed)
    R = O.ref_lib()
    mask = np.array([[R.ref_dropout_mul_c(777, (3 * 24 + qq) * 40 + kk, 0.2) != 0.0 for kk in range(40)]
                     for qq in range(24)], dtype=np.uint8)
    arrays["philox/mask_h3_24x40_p0.2_seed777"] = mask
    path = os.path.join(OUT, "reference_oracle.npz")
    np.savez_compressed(path, **arrays)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
