"""oracle/eagle.py -- CPU restatement of the reference's EAGLE draft loop.

TEST INFRASTRUCTURE ONLY: imported by tests/ as the checker of
spec_eagle_draft; the shipped library never uses it.

Restates crates/speculate/src/methods/eagle.rs:
* DraftAttention::load (:117-160): RoPE tables from f32 inv_freq, then
  positions, inv_freq, their product and cos/sin in the checkpoint dtype
  (BF16 here);
* DraftAttention::forward (:163-263): q/k/v projections, rotate-half RoPE
  (candle_nn::rotary_emb::rope), per-round KV cache, GQA, softmax(q k^T /
  sqrt(d) + causal bias) v, o_proj;
* EagleDraftCandle::forward (:390-427): concat(target hidden, token
  embedding) -> fc -> attention (no input norm) + residual ->
  post_attention_layernorm -> SiLU MLP (:271-296) + residual;
* run_eagle's draft loop (:531-575): reset, then per step the draft
  forward at position history_len + step, the target's lm_head,
  top_k_indices (medusa.rs:477-487), log-softmax (logit - lse), and the top-1
  token as the next input.

Math in float64 over BF16 weights.  Activations are rounded to BF16 where the
device's GEMV operands and KV cache are (the reference computes the whole
draft in BF16), so the comparison tolerance only covers accumulation order.
"""

from __future__ import annotations

from typing import Dict, List, Sequence, Tuple

import numpy as np

from .accept import top_k_indices


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> BF16 bits, round to nearest even."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_round(x: np.ndarray) -> np.ndarray:
    return (bf16_bits(x).astype(np.uint32) << 16).view(np.float32)


def bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


class EagleOracle:
    """The draft block over an OracleModel target (its embedding and lm_head)."""

    def __init__(self, target, weights: Dict[str, np.ndarray], theta: float = 0.0, max_pos: int = 4096):
        self.t = target
        self.w = {k: bits_to_f32(v).astype(np.float64) for k, v in weights.items() if k != "post_norm"}
        self.post_norm = np.asarray(weights["post_norm"], dtype=np.float64)
        self.nq, self.nkv, self.hd = target.n_heads, target.n_kv, target.head_dim
        theta = theta if theta > 0 else target.theta
        half = self.hd // 2
        inv = bf16_round(np.float32(1.0) / np.power(np.float32(theta),
                                                    np.arange(0, self.hd, 2, dtype=np.float32) / np.float32(self.hd)))
        pos = bf16_round(np.arange(max_pos, dtype=np.float32))
        ang = bf16_round(pos[:, None] * inv[None, :])
        self.cos = bf16_round(np.cos(ang)).astype(np.float64)
        self.sin = bf16_round(np.sin(ang)).astype(np.float64)
        assert self.cos.shape[1] == half
        self.reset()

    def reset(self) -> None:
        self.k: List[np.ndarray] = []
        self.v: List[np.ndarray] = []

    def _rope(self, x: np.ndarray, pos: int) -> np.ndarray:
        h = self.hd // 2
        c, s = self.cos[pos], self.sin[pos]
        a, b = x[..., :h], x[..., h:]
        return np.concatenate([a * c - b * s, a * s + b * c], axis=-1)

    @staticmethod
    def _op(x: np.ndarray) -> np.ndarray:
        """A GEMV operand: the device feeds BF16 values."""
        return bf16_round(x.astype(np.float32)).astype(np.float64)

    def forward(self, hidden: np.ndarray, token: int, pos: int) -> np.ndarray:
        """eagle.rs:390-427 for one row."""
        emb = self.t.embed([token])[0]
        x2 = self._op(np.concatenate([np.asarray(hidden, dtype=np.float64), emb]))
        h = self.w["fc"] @ x2
        xo = self._op(h)
        q = (self.w["q"] @ xo).reshape(self.nq, self.hd)
        k = (self.w["k"] @ xo).reshape(self.nkv, self.hd)
        v = (self.w["v"] @ xo).reshape(self.nkv, self.hd)
        q = self._op(self._rope(q, pos))
        k = self._op(self._rope(k, pos))
        v = self._op(v)
        self.k.append(k)
        self.v.append(v)
        K = np.stack(self.k, axis=1)  # [nkv, T, hd]
        Vv = np.stack(self.v, axis=1)
        G = self.nq // self.nkv
        att = np.empty((self.nq, self.hd))
        for hq in range(self.nq):
            kv = hq // G
            sc = K[kv] @ q[hq] / np.sqrt(self.hd)
            p = np.exp(sc - sc.max())
            att[hq] = (p / p.sum()) @ Vv[kv]
        t = self.w["o"] @ self._op(att.reshape(-1))
        h2 = t + h
        xn = h2 / np.sqrt(np.mean(h2 * h2) + self.t.eps) * self.post_norm
        xn = self._op(xn)
        g = self.w["gate"] @ xn
        u = self.w["up"] @ xn
        a = self._op(g / (1.0 + np.exp(-g)) * u)
        return self.w["down"] @ a + h2

    def draft(self, hidden: np.ndarray, root: int, position: int, depth: int, k: int,
              follow: Sequence[int] = ()) -> Tuple[List[List[int]], np.ndarray, List[np.ndarray]]:
        """eagle.rs:531-575.  `follow` overrides the top-1 fed to the next step
        (a test replays the device's choices through near-ties).  Returns the
        top-k ids per step, their log-probs, and the logits rows."""
        self.reset()
        ids, lps, rows = [], [], []
        cur_h, cur_t = np.asarray(hidden, dtype=np.float64), int(root)
        for step in range(depth):
            dh = self.forward(cur_h, cur_t, position + step)
            lhs = dh.astype(np.float32) if not self.t.bf16 else dh
            logits = self.t.lm_head(self._op_lm(lhs)[None])[0]
            top = top_k_indices(logits, k)
            mx = np.max(logits)
            lse = np.log(np.sum(np.exp(logits - mx))) + mx
            ids.append(top)
            lps.append(np.array([logits[i] - lse for i in top]))
            rows.append(logits)
            cur_t = int(follow[step]) if step < len(follow) else top[0]
            cur_h = dh
        return ids, np.array(lps), rows

    def _op_lm(self, x: np.ndarray) -> np.ndarray:
        """The LM head's operand: f16 for quantized targets, BF16 for BF16 ones."""
        if self.t.bf16:
            return self._op(x)
        return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float64)


# ---------------------------------------------------------------------------
# EAGLE-2 round tree: Cartesian product of the draft steps' top-k, pruned by
# path log-prob (test infrastructure: the checker of spec_eagle_build_tree).
# ---------------------------------------------------------------------------
def build_cartesian_tree(root: int, step_top_k: Sequence[Sequence[int]]) -> List[Tuple[int, int]]:
    """medusa.rs:172-189 (build_cartesian_tree): BFS parent table; layer h+1 =
    every candidate of step h under every node of layer h, parents in layer
    order, candidates in their order.  Entries are (parent, token); entry 0
    is (0, root)."""
    nodes = [(0, int(root))]
    prev = [0]
    for cands in step_top_k:
        nxt = []
        for p in prev:
            for c in cands:
                nodes.append((p, int(c)))
                nxt.append(len(nodes) - 1)
        prev = nxt
    return nodes


def prune_cartesian_tree(nodes: List[Tuple[int, int]], step_log_probs: Sequence[Sequence[float]],
                         max_total_nodes: int) -> List[Tuple[int, int]]:
    """eagle.rs:763-843 (prune_cartesian_tree): a tree of at most
    max_total_nodes entries returned as is; otherwise every non-root node is
    scored by the f32 sum of the per-step log-probs of its candidates,
    deepest step first (:800-812), nodes are stably sorted by descending
    score (:815), the root and the first max_total_nodes - 1 are kept, every
    kept node's ancestors are added (:822-827), and the kept nodes are
    re-emitted ordered by depth, index order within a depth (:829-842)."""
    n = len(nodes)
    if n <= max_total_nodes:
        return list(nodes)
    parent = np.array([p for p, _ in nodes], dtype=np.int64)
    depth = np.zeros(n, dtype=np.int64)
    for i in range(1, n):  # parents precede their children
        depth[i] = depth[parent[i]] + 1
    # Candidate index = rank among the parent's children in index order.
    cand = np.zeros(n, dtype=np.int64)
    seen: Dict[int, int] = {}
    for i in range(1, n):
        p = int(parent[i])
        cand[i] = seen.get(p, 0)
        seen[p] = cand[i] + 1
    width = max(len(v) for v in step_log_probs)
    lp = np.full((len(step_log_probs), width), np.nan, dtype=np.float32)
    for d, v in enumerate(step_log_probs):
        lp[d, :len(v)] = np.asarray(v, dtype=np.float32)
    # s = ((0 + lp[D-1][c_i]) + lp[D-2][c_parent]) + ...: one f32 add per
    # level, every node at once.
    idx = np.arange(1, n)
    cur = idx.copy()
    dep = depth[idx]
    s = np.zeros(n - 1, dtype=np.float32)
    for t in range(int(dep.max())):
        live = dep > t
        s[live] = (s[live] + lp[dep[live] - 1 - t, cand[cur[live]]]).astype(np.float32)
        cur[live] = parent[cur[live]]
    order_by_score = np.argsort(-s, kind="stable")  # stable: equal scores keep index order
    want = min(max_total_nodes - 1, n - 1)
    keep = np.zeros(n, dtype=bool)
    keep[0] = True
    keep[idx[order_by_score[:want]]] = True
    for i in range(n - 1, 0, -1):
        if keep[i]:
            keep[parent[i]] = True
    depth = depth.tolist()
    parent = parent.tolist()
    order = sorted((i for i in range(n) if keep[i]), key=lambda i: depth[i])
    new_index = {old: new for new, old in enumerate(order)}
    return [(new_index[parent[old] if old else 0], nodes[old][1]) for old in order]
