"""Writes tests/golden/ref_vectors.npz: outputs of the reference's OWN code (phone-attn/pa-tool.cpp helpers and
phone-attn/phone-attn.h merge_partial, compiled from the reference sources into oracle/_ref/libparef.so by
oracle/Makefile) on fixed inputs. The oracle tests compare the oracle restatement against these bit for bit, so the
pin holds on machines without the reference tree.

    make -C oracle ref && python tests/golden/make_golden.py
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import oracle as orc  # noqa: E402

F = ctypes.POINTER(ctypes.c_float)
U8 = ctypes.POINTER(ctypes.c_uint8)


def main():
    R = orc.ref()
    out = {}
    seed = 0x9E3779B97F4A7C15          # pa-tool.cpp:16 initial LCG state
    n = 257
    fr = np.empty(n, np.float32)
    R.ref_frand_seq(seed, fr.ctypes.data_as(F), n)
    out["lcg_seed"] = np.array([seed], np.uint64)
    out["lcg_seq"] = fr
    # pa-tool test rows: K amp 1.5, V amp 1.0 (pa-tool.cpp:118-121), nkv 4 (pa-tool.cpp:100)
    for q4 in (0, 1):
        rs = 4 * (144 if q4 else 272)
        rows = np.zeros((6, rs), np.uint8)
        R.ref_make_rows(12345, q4, 6, 4, 1.5, rows.ctypes.data_as(U8))
        out[f"rows_q{4 if q4 else 8}"] = rows
        deq = np.array([[R.ref_deq(rows[j].ctypes.data_as(U8), q4, h, d) for h in range(4) for d in range(256)]
                        for j in range(6)], np.float32)
        out[f"deq_q{4 if q4 else 8}"] = deq
    # f16 conversions on a spread of floats (normals, subnormals, ties, overflow)
    rng = np.random.default_rng(7)
    xs = np.concatenate([
        rng.standard_normal(4000).astype(np.float32) * np.float32(10.0) ** rng.integers(-9, 6, 4000).astype(np.float32),
        np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e9, -1e9, 2.0 ** -24, 2.0 ** -25, 2.0 ** -26, 3 * 2.0 ** -26,
                  5.9604645e-08, 6.1035156e-05, 1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11], np.float32)])
    out["f2h_in"] = xs
    out["f2h_out"] = np.array([R.ref_f2h(float(x)) for x in xs], np.uint16)
    hs = np.arange(0, 65536, dtype=np.uint32)
    h2f = np.array([R.ref_h2f(int(h)) for h in hs], np.float32)
    out["h2f_out"] = h2f
    # merge_partial (rows of HD 256), with empty partials on either side
    rows = 6
    O = rng.standard_normal((rows, 256)).astype(np.float32)
    m = rng.standard_normal(rows).astype(np.float32) * 3
    l = np.abs(rng.standard_normal(rows)).astype(np.float32) + 0.5
    O2 = rng.standard_normal((rows, 256)).astype(np.float32)
    m2 = rng.standard_normal(rows).astype(np.float32) * 3
    l2 = np.abs(rng.standard_normal(rows)).astype(np.float32) + 0.5
    l[1] = 0.0
    l2[2] = 0.0
    out["merge_in"] = np.concatenate([O.ravel(), m, l, O2.ravel(), m2, l2])
    Oc, mc, lc = O.copy(), m.copy(), l.copy()
    R.ref_merge_partial(Oc.ctypes.data_as(F), mc.ctypes.data_as(F), lc.ctypes.data_as(F), O2.ctypes.data_as(F),
                        m2.ctypes.data_as(F), l2.ctypes.data_as(F), rows)
    out["merge_out"] = np.concatenate([Oc.ravel(), mc, lc])
    np.savez_compressed(os.path.join(HERE, "ref_vectors.npz"), **out)
    print("wrote", os.path.join(HERE, "ref_vectors.npz"), {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
