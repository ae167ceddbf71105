"""The EAGLE-2 round tree (CPU): the oracle's restatement of the reference's
Cartesian tree and its pruning, on the reference's own unit cases
(eagle.rs:894-949), and spec_eagle_build_tree (the library's version, host
code) against the oracle on seeded cases up to depth 6 x top-10 (1,111,111
candidate nodes)."""

import ctypes
import importlib

import numpy as np
import pytest


def _eo():
    return importlib.import_module("oracle.eagle")


def test_prune_keeps_root_and_top_paths():
    """eagle.rs:894-928: k=2 depth=2 (7 nodes) pruned to 4."""
    eo = _eo()
    cart = eo.build_cartesian_tree(42, [[10, 20], [30, 40]])
    assert len(cart) == 7
    pruned = eo.prune_cartesian_tree(cart, [[-0.1, -2.0], [-0.2, -3.0]], 4)
    assert 0 < len(pruned) <= 4
    assert pruned[0][1] == 42
    toks = [t for _, t in pruned]
    assert 10 in toks and 30 in toks


def test_prune_returns_full_tree_when_under_limit():
    """eagle.rs:930-949."""
    eo = _eo()
    cart = eo.build_cartesian_tree(1, [[2], [3]])
    assert len(cart) == 3
    assert len(eo.prune_cartesian_tree(cart, [[-0.1], [-0.2]], 100)) == 3


def _lib_tree(pkg, root, ids, lps, max_nodes, cap=64):
    L = importlib.import_module("abyo-speculate_b200._lib")
    depth, k = ids.shape
    toks = np.zeros(cap, dtype=np.uint32)
    par = np.zeros(cap, dtype=np.int32)
    n = ctypes.c_int()
    rc = L.load().spec_eagle_build_tree(root, ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                        lps.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), depth, k, max_nodes,
                                        toks.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)),
                                        par.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), cap, ctypes.byref(n))
    return rc, [(int(par[i]) if i else 0, int(toks[i])) for i in range(n.value)]


@pytest.mark.parametrize("depth,k,max_nodes,ties", [(2, 2, 4, False), (4, 2, 20, False), (3, 3, 0, False),
                                                     (6, 10, 60, False), (6, 10, 60, True), (5, 4, 32, True)])
def test_library_tree_equals_oracle(pkg, depth, k, max_nodes, ties):
    eo = _eo()
    rng = np.random.default_rng(depth * 100 + k)
    ids = rng.integers(0, 50000, size=(depth, k)).astype(np.int32)
    # log-probs: <= 0, each step's in descending order (as top-k returns them)
    lps = np.sort(-np.abs(rng.standard_normal((depth, k)).astype(np.float32) * np.float32(2.0)))[:, ::-1]
    if ties:  # equal log-probs: the stable order decides
        lps = np.round(lps * 4) / 4
    lps = np.ascontiguousarray(lps.astype(np.float32))
    rc, got = _lib_tree(pkg, 7, ids, lps, max_nodes)
    cart = eo.build_cartesian_tree(7, ids.tolist())
    want = eo.prune_cartesian_tree(cart, lps.tolist(), max_nodes) if max_nodes else cart
    assert rc == 0
    assert got == want
