"""oracle/accept.py -- CPU restatement of the reference's acceptance rules.

TEST INFRASTRUCTURE ONLY (checker for tests/ and smoke()).

Restates, with float32 arithmetic in the reference's sequential order:
* crates/speculate/src/sampling/tokens.rs:15-55 softmax_with_temperature
  (temperature 0 -> one-hot first-max argmax; else exp((l - max) / t) / sum),
  :99-120 sample_from_distribution (u = gen::<f32>() * sum, linear cumulative
  scan, fallback to the last index);
* crates/speculate/src/methods/vanilla.rs:59-73 modified_rejection_step,
  :83-106 adjusted_distribution, :120-229 run_vanilla_sd (draw order: k draft
  samples, then per verified position one uniform, then one resample on
  reject or one bonus sample when all k were accepted);
* crates/speculate/src/methods/eagle.rs:618-661 greedy tree acceptance
  (walk every root-to-leaf path in leaf-index order, count leading
  argmax matches, first longest wins; bonus = argmax of the deepest node);
* crates/speculate/src/methods/medusa.rs:424-445 typical acceptance
  (p(x) >= max(epsilon, delta * exp(-H(p)))) and the same tree walk with it
  (:290-326, :391-411);
* crates/speculate/src/model/mock.rs:164-180 fixed_distribution.

Uniforms are explicit inputs so decisions can be compared bit-exactly with
the device path given identical logits and identical uniforms.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np


class SamplingError(ValueError):
    pass


def argmax_first(row: np.ndarray) -> int:
    """tokens.rs:26-36 fold: strict '>' from (0, -inf)."""
    bi, bv = 0, np.float32(-np.inf)
    for i, v in enumerate(np.asarray(row, dtype=np.float32).tolist()):
        if v > bv:
            bi, bv = i, v
    return bi


def top_k_indices(logits, k: int):
    """methods/medusa.rs:477-487: indices sorted by value descending, ties by
    ascending index (a stable sort on the value), the first k.  NaN entries
    rank last here (the reference's comparator calls them equal to
    everything; the backend documents them as lowest)."""
    r = np.asarray(logits, dtype=np.float32)
    v = np.where(np.isnan(r), -np.inf, r).astype(np.float64)
    v = np.where(v == 0.0, 0.0, v)  # -0.0 equals +0.0
    nan_last = np.isnan(r).astype(np.int8)
    order = np.lexsort((np.arange(r.size), -v, nan_last))
    return [int(i) for i in order[:min(k, r.size)]]


def argmax_first_fast(row: np.ndarray) -> int:
    r = np.asarray(row, dtype=np.float32)
    finite = ~np.isnan(r)
    if not finite.any():
        return 0
    mx = np.max(r[finite])
    if mx == -np.inf:
        return 0
    return int(np.flatnonzero(r == mx)[0])


def seq_sum_f32(a: np.ndarray) -> np.float32:
    """Sequential float32 sum (Rust `iter().sum::<f32>()`)."""
    a = np.asarray(a, dtype=np.float32)
    if a.size == 0:
        return np.float32(0.0)
    return np.cumsum(a, dtype=np.float32)[-1]


def exp_f32(x: np.ndarray) -> np.ndarray:
    """f32::exp as modelled here: the correctly rounded exp of the f32
    argument (exp in double, one rounding to f32).  Rust calls the platform
    libm's expf, which is within 0.502 ulp of that; tests/test_exp_model.py
    measures how often the two differ and whether the decisions do."""
    return np.exp(np.asarray(x, dtype=np.float32).astype(np.float64)).astype(np.float32)


def softmax_with_temperature(logits: np.ndarray, temperature: float) -> np.ndarray:
    logits = np.asarray(logits, dtype=np.float32)
    if logits.size == 0:
        raise SamplingError("empty logits")
    if not np.isfinite(temperature) or temperature < 0:
        raise SamplingError(f"invalid temperature: {temperature}")
    if temperature == 0.0:
        out = np.zeros_like(logits)
        out[argmax_first_fast(logits)] = 1.0
        return out
    inv_t = np.float32(1.0) / np.float32(temperature)
    finite = logits[~np.isnan(logits)]  # fold(NEG_INFINITY, f32::max) skips NaN
    mx = np.float32(np.max(finite)) if finite.size else np.float32(-np.inf)
    out = exp_f32((logits - mx) * inv_t)
    s = seq_sum_f32(out)
    if not (s > 0) or not np.isfinite(s):
        raise SamplingError(f"softmax produced non-positive sum: {s}")
    return (out / s).astype(np.float32)


def sample_from_distribution(u01: float, probs: np.ndarray) -> int:
    """tokens.rs:99-120 with the uniform `u01` = gen::<f32>() given explicitly."""
    probs = np.asarray(probs, dtype=np.float32)
    if probs.size == 0:
        raise SamplingError("empty distribution")
    s = seq_sum_f32(probs)
    if not np.isfinite(s) or s <= 0:
        raise SamplingError(f"invalid distribution sum: {s}")
    if np.any(~np.isfinite(probs)) or np.any(probs < 0):
        raise SamplingError("invalid probability")
    u = np.float32(u01) * s
    acc = np.cumsum(probs, dtype=np.float32)
    idx = np.flatnonzero(u < acc)
    return int(idx[0]) if idx.size else probs.size - 1


def modified_rejection_step(q_draft: float, p_target: float, u: float) -> bool:
    """vanilla.rs:59-73: True = accepted."""
    if q_draft <= 0.0:
        return True
    ratio = min(np.float32(p_target) / np.float32(q_draft), np.float32(1.0))
    return bool(np.float32(u) <= ratio)


def adjusted_distribution(p: np.ndarray, q: np.ndarray) -> np.ndarray:
    p = np.asarray(p, dtype=np.float32)
    q = np.asarray(q, dtype=np.float32)
    if p.size != q.size:
        raise SamplingError(f"vocab size mismatch: target={p.size}, draft={q.size}")
    adj = np.maximum(p - q, np.float32(0.0)).astype(np.float32)
    s = seq_sum_f32(adj)
    if s <= 0 or not np.isfinite(s):
        raise SamplingError(f"adjusted distribution has non-positive mass: sum={s}")
    return (adj / s).astype(np.float32)


def vanilla_round(target_rows: np.ndarray, draft_tokens: Sequence[int], draft_dists: Sequence[np.ndarray],
                  temperature: float, uniforms: Sequence[float], generated: int,
                  max_new: int) -> Tuple[List[int], int]:
    """Steps 3-4 of vanilla.rs:172-210: returns (commits, uniforms consumed)."""
    k = len(draft_tokens)
    commits: List[int] = []
    used = 0
    rejected = False
    for i in range(k):
        p_probs = softmax_with_temperature(target_rows[i], temperature)
        q_probs = draft_dists[i]
        tok = int(draft_tokens[i])
        u = uniforms[used]
        used += 1
        if modified_rejection_step(float(q_probs[tok]), float(p_probs[tok]), u):
            commits.append(tok)
            if generated + len(commits) >= max_new:
                break
        else:
            adj = adjusted_distribution(p_probs, q_probs)
            commits.append(sample_from_distribution(uniforms[used], adj))
            used += 1
            rejected = True
            break
    if not rejected and len(commits) == k and generated + len(commits) < max_new:
        p_probs = softmax_with_temperature(target_rows[k], temperature)
        commits.append(sample_from_distribution(uniforms[used], p_probs))
        used += 1
    return commits, used


def greedy_linear_accept(target_rows: np.ndarray, drafts: Sequence[int]) -> Tuple[int, int]:
    """Temperature-0 vanilla round: (n_accepted, token after them)."""
    acc = 0
    while acc < len(drafts) and argmax_first_fast(target_rows[acc]) == int(drafts[acc]):
        acc += 1
    return acc, argmax_first_fast(target_rows[acc])


def tree_paths(parents: Sequence[int]) -> List[List[int]]:
    n = len(parents)
    is_leaf = [True] * n
    for p in parents[1:]:
        is_leaf[p] = False
    out = []
    for i in range(n):
        if is_leaf[i]:
            chain = [i]
            cur = i
            while cur != 0:
                cur = parents[cur]
                chain.append(cur)
            out.append(list(reversed(chain)))
    return out


def greedy_tree_accept(tokens: Sequence[int], parents: Sequence[int], rows: np.ndarray) -> Tuple[List[int], int]:
    """eagle.rs:618-661 over per-node logits rows: (best_path, bonus)."""
    am = [argmax_first_fast(r) for r in rows]
    best = [0]
    for path in tree_paths(parents):
        accepted = 0
        for parent, child in zip(path[:-1], path[1:]):
            if am[parent] == int(tokens[child]):
                accepted += 1
            else:
                break
        if accepted + 1 > len(best):
            best = path[: accepted + 1]
    return best, am[best[-1]]


def ln_f32(x: np.ndarray) -> np.ndarray:
    """f32::ln as modelled here: the correctly rounded natural log of the f32
    argument (log in double, one rounding to f32).  Rust calls the platform
    libm's logf; tests/test_exp_model.py measures how often glibc's differs
    from this model and whether a typical-acceptance decision does."""
    return np.log(np.asarray(x, dtype=np.float32).astype(np.float64)).astype(np.float32)


def typical_threshold(logits: np.ndarray, epsilon: float, delta: float):
    """medusa.rs:424-443 up to the comparison: (probs, threshold), or None
    where the reference returns false for a non-positive / non-finite softmax
    mass.  softmax: max by the NaN-skipping f32::max fold, exp(l - max),
    sequential f32 sum, p = e / sum; entropy = sequential f32 sum of
    (-p) * ln(p) over p > 0; threshold = epsilon.max(delta * exp(-entropy))."""
    lg = np.asarray(logits, dtype=np.float32)
    finite = lg[~np.isnan(lg)]
    mx = np.float32(np.max(finite)) if finite.size else np.float32(-np.inf)
    with np.errstate(invalid="ignore", over="ignore"):
        e = exp_f32(lg - mx)
        s = seq_sum_f32(e)
        if not (s > 0) or not np.isfinite(s):
            return None
        p = (e / s).astype(np.float32)
        pos = p[p > 0]
        ent = seq_sum_f32(((-pos) * ln_f32(pos)).astype(np.float32))
        t = np.float32(np.float32(delta) * exp_f32(np.float32(-ent)))
    return p, np.float32(np.fmax(np.float32(epsilon), t))  # f32::max: a NaN side yields the other


def typical_accept_one(logits: np.ndarray, candidate: int, epsilon: float, delta: float) -> bool:
    """medusa.rs:424-445 (Acceptance::Typical): p(candidate) >= threshold."""
    r = typical_threshold(logits, epsilon, delta)
    if r is None:
        return False
    p, thr = r
    return bool(p[int(candidate)] >= thr)


def typical_tree_accept(tokens: Sequence[int], parents: Sequence[int], rows: np.ndarray, epsilon: float,
                        delta: float) -> Tuple[List[int], int]:
    """medusa.rs:290-326 with Acceptance::Typical: every root-to-leaf path
    (leaves in index order) accepts while typical_accept_one holds against the
    parent's row (:391-411); the first longest accepted prefix wins (:296-301)
    and the bonus is the argmax of its deepest node (:311-316, :451-470)."""
    thr = [typical_threshold(r, epsilon, delta) for r in rows]

    def ok(parent: int, child: int) -> bool:
        t = thr[parent]
        return t is not None and bool(t[0][int(tokens[child])] >= t[1])

    best = [0]
    for path in tree_paths(parents):
        accepted = 0
        for parent, child in zip(path[:-1], path[1:]):
            if ok(parent, child):
                accepted += 1
            else:
                break
        if accepted + 1 > len(best):
            best = path[: accepted + 1]
    return best, argmax_first_fast(rows[best[-1]])


def top2_margin(row: np.ndarray) -> float:
    s = np.sort(np.asarray(row, dtype=np.float64))
    return float(s[-1] - s[-2])


# ---- mock decoders (mock.rs) and the reference vanilla loop (vanilla.rs) ----
class MockDecoder:
    def __init__(self, vocab: int, logits_fn: Callable[[List[int], int], np.ndarray]):
        self.vocab = vocab
        self.hist: List[int] = []
        self.fn = logits_fn

    def vocab_size(self) -> int:
        return self.vocab

    def history_len(self) -> int:
        return len(self.hist)

    def reset(self) -> None:
        self.hist = []

    def observe(self, ids) -> None:
        self.hist.extend(int(t) for t in ids)

    def next_logits(self) -> np.ndarray:
        return self.fn(self.hist, len(self.hist))

    def batched_logits(self, drafts) -> np.ndarray:
        out = [self.fn(list(self.hist), len(self.hist))]
        pre = list(self.hist)
        for d in drafts:
            pre.append(int(d))
            out.append(self.fn(list(pre), len(pre)))
        self.hist.extend(int(d) for d in drafts)
        return np.stack(out)

    def rollback_to(self, n: int) -> None:
        if n > len(self.hist):
            raise SamplingError("CacheRollback")
        self.hist = self.hist[:n]


def fixed_distribution(probs: Sequence[float]) -> MockDecoder:
    logits = np.log(np.maximum(np.asarray(probs, dtype=np.float32), np.float32(1e-30))).astype(np.float32)
    return MockDecoder(len(logits), lambda h, pos: logits.copy())


def run_vanilla_sd(target, draft, prompt, max_new: int, k: int, temperature: float,
                   next_u: Callable[[], float]) -> List[int]:
    """vanilla.rs:120-229 with `next_u()` standing in for rng.gen::<f32>()."""
    if target.vocab_size() != draft.vocab_size():
        raise SamplingError("vocab mismatch")
    target.reset()
    draft.reset()
    target.observe(prompt)
    draft.observe(prompt)
    gen: List[int] = []
    while len(gen) < max_new:
        kk = min(k, max_new - len(gen))
        if kk == 0:
            break
        pre_t, pre_d = target.history_len(), draft.history_len()
        toks, dists = [], []
        for _ in range(kk):
            probs = softmax_with_temperature(draft.next_logits(), temperature)
            tok = sample_from_distribution(next_u(), probs)
            toks.append(tok)
            dists.append(probs)
            draft.observe([tok])
        rows = target.batched_logits(toks)
        # draw uniforms lazily in the reference order
        pool: List[float] = []

        class _U(list):
            def __getitem__(self, i):
                while len(pool) <= i:
                    pool.append(next_u())
                return pool[i]

        commits, _ = vanilla_round(rows, toks, dists, temperature, _U(), len(gen), max_new)
        acc = min(len(commits), kk)
        target.rollback_to(pre_t + acc)
        target.observe(commits[acc:])
        draft.rollback_to(pre_d + acc)
        draft.observe(commits[acc:])
        gen.extend(commits)
    return gen
