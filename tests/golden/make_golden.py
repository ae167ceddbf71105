"""Regenerate the golden dequantization vectors in this directory.

The expected values come from ``gguf`` 0.19.0's ``gguf.quants.dequantize``
(the Python reference implementation of the GGUF block formats that the
reference's candle QMatMul consumes).  The raw blocks are made by this
project's quantizers plus hand-built edge blocks (all-zero, extreme codes,
maximal 6-bit scales, negative Q6_K scales, subnormal f16 d).

Run from the repository root:  python tests/golden/make_golden.py
"""

import importlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))


def main() -> None:
    import gguf
    from gguf import quants

    gs = importlib.import_module("abyo-speculate_b200.gguf_synth")
    rng = np.random.default_rng(20261201)
    out = {}
    for qt in (gs.Q4_K, gs.Q5_K, gs.Q6_K, gs.Q8_0):
        name = gs.TYPE_NAMES[qt]
        bb, be = gs.BLOCK_BYTES[qt], gs.BLOCK_ELEMS[qt]
        w = rng.standard_normal((4, 1024), dtype=np.float32) * np.float32(0.02)
        w[1] *= 50.0  # wide dynamic range row
        w[2, :256] = 0.0  # an all-zero superblock
        raw = gs.quantize(w, qt).reshape(-1, bb).copy()
        # Hand-built edge blocks: every code maximal / random bytes with small d.
        edge = rng.integers(0, 256, size=(3, bb), dtype=np.uint8)
        if qt in (gs.Q4_K, gs.Q5_K):
            edge[0, 0:2] = np.array([0x3C00], np.uint16).view(np.uint8)  # d = 1.0
            edge[0, 2:4] = np.array([0x3800], np.uint16).view(np.uint8)  # dmin = 0.5
            edge[0, 4:16] = 0xFF  # all scales / mins = 63
            edge[1, 0:2] = np.array([0x0001], np.uint16).view(np.uint8)  # subnormal d
            edge[2, 0:4] = np.array([0x1400, 0x1000], np.uint16).view(np.uint8)
        elif qt == gs.Q6_K:
            edge[0, 208:210] = np.array([0x3C00], np.uint16).view(np.uint8)
            edge[0, 192:208] = np.array([-128, 127] * 8, np.int8).view(np.uint8)
            edge[1, 208:210] = np.array([0x0001], np.uint16).view(np.uint8)
            edge[2, 208:210] = np.array([0x2000], np.uint16).view(np.uint8)
        else:
            edge[0, 0:2] = np.array([0x3C00], np.uint16).view(np.uint8)
            edge[0, 2:] = np.array([-128, 127] * 16, np.int8).view(np.uint8)
            edge[1, 0:2] = np.array([0x0001], np.uint16).view(np.uint8)
            edge[2, 0:2] = np.array([0xBC00], np.uint16).view(np.uint8)  # d = -1.0
        blocks = np.concatenate([raw, edge], axis=0)
        expect = quants.dequantize(blocks.reshape(1, -1), gguf.GGMLQuantizationType(qt))
        expect = np.asarray(expect, dtype=np.float32).reshape(-1)
        assert expect.size == blocks.shape[0] * be
        out[f"{name}_blocks"] = blocks
        out[f"{name}_expect"] = expect
    np.savez_compressed(os.path.join(HERE, "dequant_gguf019.npz"), **out)
    print("wrote", os.path.join(HERE, "dequant_gguf019.npz"))


if __name__ == "__main__":
    main()
