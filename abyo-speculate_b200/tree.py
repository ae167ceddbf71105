"""Draft trees: the host-side data structure a tree verify consumes.

Mirrors ``DraftTree`` of crates/speculate/src/tree.rs (parent-pointer BFS
representation, :38-74; ancestors / depth / paths, :110-176; attention masks
and biases, :149-264) so callers build trees exactly as the reference's SD
methods do.  The device never sees the bias matrix: the verify kernels take
one ancestor bitmask per node instead (see attention.cu).
"""

from __future__ import annotations

from typing import List, Sequence, Tuple

import numpy as np

from ._lib import SamplingError, SPEC_ERR_INVALID


class DraftTree:
    """A draft tree rooted at the last committed token, nodes in BFS order."""

    def __init__(self, tokens: Sequence[int], parents: Sequence[int]):
        self._tokens = [int(t) for t in tokens]
        self._parents = [int(p) for p in parents]

    @classmethod
    def from_parent_table(cls, nodes: Sequence[Tuple[int, int]]) -> "DraftTree":
        """`(parent_index, token)` pairs; entry 0 is the root (tree.rs:51-74)."""
        if len(nodes) == 0:
            raise SamplingError(SPEC_ERR_INVALID, "DraftTree must have at least a root")
        tokens = [int(nodes[0][1])]
        parents = [0]
        for i, (p, tok) in enumerate(nodes):
            if i == 0:
                continue
            if p >= i:
                raise SamplingError(SPEC_ERR_INVALID,
                                    f"node {i} has parent index {p}, which is not strictly smaller")
            tokens.append(int(tok))
            parents.append(int(p))
        return cls(tokens, parents)

    @classmethod
    def linear(cls, root: int, tail: Sequence[int]) -> "DraftTree":
        """root -> tail[0] -> tail[1] ... (tree.rs:77-88)."""
        return cls([root, *tail], [0] + list(range(len(tail))))

    def __len__(self) -> int:
        return len(self._tokens)

    def is_empty(self) -> bool:
        return len(self._tokens) <= 1

    def token_at(self, i: int) -> int:
        return self._tokens[i]

    def tokens(self) -> List[int]:
        return list(self._tokens)

    def parent_of(self, i: int) -> int:
        return self._parents[i]

    def parents(self) -> List[int]:
        return list(self._parents)

    def ancestors(self, i: int) -> List[int]:
        out = [i]
        while i != 0:
            i = self._parents[i]
            out.append(i)
        return out

    def depth_of(self, i: int) -> int:
        d = 0
        while i != 0:
            i = self._parents[i]
            d += 1
        return d

    def position_ids(self, prefix_len: int) -> List[int]:
        return [prefix_len + self.depth_of(i) for i in range(len(self))]

    def attention_mask_bool(self) -> List[List[bool]]:
        n = len(self)
        m = [[False] * n for _ in range(n)]
        for i in range(n):
            for j in self.ancestors(i):
                m[i][j] = True
        return m

    def paths(self) -> List[List[int]]:
        """All root-to-leaf chains, leaves in index order (tree.rs:162-176)."""
        is_leaf = [True] * len(self)
        for p in self._parents[1:]:
            is_leaf[p] = False
        out = []
        for i, leaf in enumerate(is_leaf):
            if leaf:
                out.append(list(reversed(self.ancestors(i))))
        return out

    def path_to(self, target: int) -> List[int]:
        return list(reversed(self.ancestors(target)))

    def is_ancestor_of(self, ancestor_idx: int, node_idx: int) -> bool:
        cur = node_idx
        if cur == ancestor_idx:
            return True
        while cur != 0:
            cur = self._parents[cur]
            if cur == ancestor_idx:
                return True
        return ancestor_idx == 0

    def full_attention_bias(self, prefix_len: int) -> np.ndarray:
        """[n, prefix_len + n] additive bias: 0 visible, -inf masked (tree.rs:220-240)."""
        n = len(self)
        out = np.zeros((n, prefix_len + n), dtype=np.float32)
        for i in range(n):
            for j in range(n):
                if not self.is_ancestor_of(j, i):
                    out[i, prefix_len + j] = -np.inf
        return out

    def ancestor_bits(self) -> List[int]:
        """Per-node bitmask of ancestors-or-self: the device form of the mask."""
        out = []
        for i in range(len(self)):
            b = 0
            for j in self.ancestors(i):
                b |= 1 << j
            out.append(b | 1)
        return out
