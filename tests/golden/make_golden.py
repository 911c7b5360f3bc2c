"""Writes the golden fixtures of tests/test_oracle_golden.py.

cpu_ref_decode_layer.npz: outputs of the reference's own f64 single-layer
decode check `cpu_ref` (tool/decode_eager_baseline.cu:160-198), compiled
from the reference source into oracle/_ref/libcpu_ref.so by oracle/Makefile,
on the inputs its main() draws (:209-219) at cache lengths 1, 17 and 256.

Run from the repository root where the reference tree is mounted:
    make -C oracle && python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import oracle as O  # noqa: E402

KEYS = ("x", "g1", "g2", "Wq", "Wk", "Wv", "Wo", "Wg", "Wu", "Wd", "Kc", "Vc")


def main():
    R = O.ref_lib()
    if R is None:
        sys.exit("oracle/_ref/libcpu_ref.so missing: run `make -C oracle ref` with the reference tree mounted")
    out = {}
    for L in (1, 17, 256):
        inp = O.ref_inputs(L)
        bufs = [np.empty_like(inp[k]) for k in KEYS]
        R.ref_make_inputs(L, *[b.ctypes.data for b in bufs])
        for k, b in zip(KEYS, bufs):  # the restated generator draws the same inputs
            assert np.array_equal(inp[k], b), k
        y = np.empty(O.REF_D, np.float64)
        R.ref_cpu_ref(*[b.ctypes.data for b in bufs], L, y.ctypes.data)
        out[f"L{L}"] = y
    np.savez(os.path.join(HERE, "cpu_ref_decode_layer.npz"), **out)
    print("wrote", sorted(out))


if __name__ == "__main__":
    main()
