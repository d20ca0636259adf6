"""The F(4x4,3x3) kernel's transform tables (csrc/winograd_f43.cuh) are the
oracle's Toom-Cook matrices: B^T and A^T exactly, G after rounding to fp32.
CPU only: the tables are read from the kernel source."""
import os
import re

import numpy as np

from oracle import winograd as owg

SRC = os.path.join(os.path.dirname(__file__), "..", "rdv_project_b200", "csrc", "winograd_f43.cuh")


def _table(src: str, decl: str, rows: int, cols: int) -> np.ndarray:
    body = src[src.index(decl):]
    body = body[body.index("=") + 1:body.index("};")]
    vals = []
    for num, den in re.findall(r"(-?[0-9.]+)f(?:\s*/\s*(-?[0-9.]+)f)?", body):
        v = np.float32(num)
        if den:
            v = np.float32(v / np.float32(den))  # the fp32 division the compiler folds
        vals.append(v)
    return np.array(vals, dtype=np.float32).reshape(rows, cols)


def test_tables_match_toom_cook():
    src = open(SRC).read()
    BT = _table(src, "kBT[kA][kA]", 6, 6)
    AT = _table(src, "kAT[kM][kA]", 4, 6)
    G = _table(src, "kG[kA][3]", 6, 3)
    np.testing.assert_array_equal(BT.astype(np.float64), owg.BT_F43)
    np.testing.assert_array_equal(AT.astype(np.float64), owg.AT_F43)
    np.testing.assert_array_equal(G, owg.G_F43.astype(np.float32))


def test_points_of_the_tables():
    # A^T's second row lists the finite evaluation points of the construction
    AT, _, _ = owg.toom_cook_matrices(owg.F43_POINTS, 4)
    np.testing.assert_array_equal(AT[1, :5], np.array(owg.F43_POINTS))
