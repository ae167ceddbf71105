"""Host DraftTree: ports of the reference's tree.rs unit tests (CPU)."""

import numpy as np
import pytest


def test_linear_tree_is_a_chain(pkg):
    t = pkg.DraftTree.linear(10, [20, 30, 40])
    assert len(t) == 4 and t.tokens() == [10, 20, 30, 40]
    assert [t.parent_of(i) for i in range(4)] == [0, 0, 1, 2]
    assert t.depth_of(3) == 3
    assert t.paths() == [[0, 1, 2, 3]]


def test_branching_tree_paths(pkg):
    t = pkg.DraftTree.from_parent_table([(0, 100), (0, 11), (0, 12), (1, 23), (1, 24), (2, 35)])
    assert len(t) == 6 and t.depth_of(3) == 2 and t.depth_of(5) == 2
    assert sorted(t.paths(), key=lambda p: (len(p), p)) == [[0, 1, 3], [0, 1, 4], [0, 2, 5]]


def test_linear_mask_is_lower_triangular(pkg):
    m = pkg.DraftTree.linear(10, [20, 30, 40]).attention_mask_bool()
    for i in range(4):
        for j in range(4):
            assert m[i][j] == (j <= i)


def test_branching_mask_blocks_siblings(pkg):
    t = pkg.DraftTree.from_parent_table([(0, 100), (0, 11), (0, 12), (1, 23), (1, 24), (2, 35)])
    m = t.attention_mask_bool()
    assert m[3][0] and m[3][1] and m[3][3]
    assert not m[3][2] and not m[3][4] and not m[3][5]
    assert m[5][0] and m[5][2] and m[5][5]
    assert not m[5][1] and not m[5][3] and not m[5][4]


def test_position_ids_offset_by_prefix(pkg):
    assert pkg.DraftTree.linear(0, [1, 2, 3]).position_ids(7) == [7, 8, 9, 10]


def test_rejects_forward_parent_reference(pkg):
    with pytest.raises(pkg.SamplingError):
        pkg.DraftTree.from_parent_table([(0, 0), (5, 1)])


def test_rejects_empty_tree(pkg):
    with pytest.raises(pkg.SamplingError):
        pkg.DraftTree.from_parent_table([])


def test_path_to_walks_root_first(pkg):
    t = pkg.DraftTree.from_parent_table([(0, 0), (0, 1), (1, 2), (2, 3)])
    assert t.path_to(3) == [0, 1, 2, 3]


def test_full_attention_bias_keeps_prefix_unmasked(pkg):
    b = pkg.DraftTree.linear(0, [1, 2]).full_attention_bias(5)
    assert b.shape == (3, 8)
    assert np.all(b[:, :5] == 0)
    for i in range(3):
        for j in range(3):
            assert (b[i, 5 + j] == 0) == (j <= i)
            if j > i:
                assert np.isneginf(b[i, 5 + j])


def test_ancestor_bits_match_mask(pkg):
    t = pkg.DraftTree.from_parent_table([(0, 9), (0, 1), (0, 2), (1, 3), (1, 4), (2, 5), (3, 6)])
    m = t.attention_mask_bool()
    for i, bits in enumerate(t.ancestor_bits()):
        for j in range(len(t)):
            assert bool((bits >> j) & 1) == m[i][j]
