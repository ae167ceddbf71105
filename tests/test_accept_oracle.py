"""Acceptance rules (oracle): ports of vanilla.rs / tokens.rs tests (CPU)."""

import numpy as np
import pytest


def test_always_accept_when_target_geq_draft(accept):
    for u in range(101):
        assert accept.modified_rejection_step(0.4, 0.8, u / 100.0)


def test_reject_when_u_above_ratio(accept):
    assert not accept.modified_rejection_step(0.8, 0.4, 0.6)
    assert accept.modified_rejection_step(0.8, 0.4, 0.4)


def test_adjusted_distribution(accept):
    adj = accept.adjusted_distribution([0.5, 0.3, 0.2], [0.1, 0.4, 0.5])
    assert np.allclose(adj, [1.0, 0.0, 0.0], atol=1e-6)
    with pytest.raises(accept.SamplingError):
        accept.adjusted_distribution([0.5, 0.5], [0.5, 0.5])
    with pytest.raises(accept.SamplingError):
        accept.adjusted_distribution([0.5, 0.5], [1.0])


def test_softmax_and_greedy(accept):
    p = accept.softmax_with_temperature([1.0, 2.0, 3.0], 1.0)
    assert abs(float(p.sum()) - 1.0) < 1e-5
    assert list(accept.softmax_with_temperature([0.1, 5.0, 0.1, 4.99], 0.0)) == [0, 1, 0, 0]
    assert accept.argmax_first([1.0, 3.0, 3.0, 2.0]) == 1
    assert accept.argmax_first_fast(np.array([1.0, 3.0, 3.0, 2.0])) == 1


def test_sample_respects_mass(accept):
    rng = np.random.default_rng(7)
    for _ in range(200):
        assert accept.sample_from_distribution(rng.random(), [0.0, 0.0, 1.0, 0.0]) == 2


def _empirical(accept, target, draft, trials, seed):
    rng = np.random.default_rng(seed)
    counts = np.zeros(len(target))
    for _ in range(trials):
        t = accept.fixed_distribution(target)
        d = accept.fixed_distribution(draft)
        out = accept.run_vanilla_sd(t, d, [0], 1, 4, 1.0, lambda: float(np.float32(rng.random())))
        counts[out[0]] += 1
    return counts / trials


@pytest.mark.parametrize("target,draft,tol", [
    ([0.5, 0.3, 0.15, 0.05], [0.25] * 4, 0.025),
    ([0.7, 0.15, 0.1, 0.05], [0.05, 0.1, 0.15, 0.7], 0.03),
    ([0.4, 0.3, 0.2, 0.1], [0.4, 0.3, 0.2, 0.1], 0.025),
])
def test_sd_matches_target_distribution(accept, target, draft, tol):
    emp = _empirical(accept, target, draft, 6000, 11)
    tv = 0.5 * np.abs(emp - np.asarray(target)).sum()
    assert tv < tol


def test_sd_emits_only_supported_tokens(accept):
    rng = np.random.default_rng(99)
    t = accept.fixed_distribution([0.6, 0.4, 0.0, 0.0])
    d = accept.fixed_distribution([0.25] * 4)
    for _ in range(500):
        out = accept.run_vanilla_sd(t, d, [0], 1, 4, 1.0, lambda: float(np.float32(rng.random())))
        assert out[0] < 2


def test_sd_produces_max_new_tokens(accept):
    rng = np.random.default_rng(1)
    t = accept.fixed_distribution([0.4, 0.3, 0.2, 0.1])
    d = accept.fixed_distribution([0.25] * 4)
    for n in (1, 5, 16, 32):
        out = accept.run_vanilla_sd(t, d, [0], n, 3, 1.0, lambda: float(np.float32(rng.random())))
        assert len(out) == n


def test_greedy_tree_accept_first_longest(accept):
    # tree: 0 -> {1 (tok 5), 2 (tok 6)}; 1 -> 3 (tok 7); 2 -> 4 (tok 8)
    tokens = [9, 5, 6, 7, 8]
    parents = [0, 0, 0, 1, 2]
    rows = np.full((5, 10), -1.0, dtype=np.float32)
    rows[0, 6] = 1.0   # root predicts 6 -> path via node 2
    rows[2, 8] = 1.0   # node 2 predicts 8 -> node 4 accepted
    rows[4, 3] = 1.0   # bonus 3
    best, bonus = accept.greedy_tree_accept(tokens, parents, rows)
    assert best == [0, 2, 4] and bonus == 3
    rows2 = np.zeros((5, 10), dtype=np.float32)  # all ties -> argmax 0, nothing accepted
    best, bonus = accept.greedy_tree_accept(tokens, parents, rows2)
    assert best == [0] and bonus == 0


def test_top_k_indices_order(accept):
    """medusa.rs:477-487: value descending, ties by ascending index."""
    row = np.array([0.5, 2.0, 2.0, -1.0, 2.0, 0.5, -0.0, 0.0, np.nan], dtype=np.float32)
    assert accept.top_k_indices(row, 5) == [1, 2, 4, 0, 5]
    assert accept.top_k_indices(row, 9) == [1, 2, 4, 0, 5, 6, 7, 3, 8]
    assert accept.top_k_indices(row, 20) == [1, 2, 4, 0, 5, 6, 7, 3, 8]


def test_typical_threshold_blocks_low_mass_token(accept):
    """medusa.rs:1060-1090: mass spread thinly over 50 tokens with a peak at 0;
    under epsilon = 0.5, delta = 1.0 the low-mass candidate 25 is rejected on
    every path, so each round commits only the bonus (the argmax, 0)."""
    vocab = 50
    probs = np.full(vocab, 0.01, dtype=np.float32)
    probs[0] = np.float32(1.0) - np.float32(0.01) * np.float32(vocab - 1)
    row = accept.fixed_distribution(probs).next_logits()
    assert not accept.typical_accept_one(row, 25, 0.5, 1.0)
    assert accept.typical_accept_one(row, 0, 0.5, 1.0)
    # Greedy topology with top-1 per head: the chain root -> 25 -> 25.
    rows = np.stack([row, row, row])
    best, bonus = accept.typical_tree_accept([1, 25, 25], [0, 0, 1], rows, 0.5, 1.0)
    assert best == [0] and bonus == 0


def test_typical_threshold_against_float64(accept):
    """The f32 entropy threshold agrees with a float64 evaluation to f32
    rounding, and the epsilon floor / delta scale act as the reference
    states (threshold = max(epsilon, delta * exp(-H)))."""
    rng = np.random.default_rng(3)
    for scale in (0.1, 1.0, 4.0, 20.0):
        row = (rng.standard_normal(5000) * scale).astype(np.float32)
        p, thr = accept.typical_threshold(row, 0.0, 1.0)
        x = row.astype(np.float64)
        q = np.exp(x - x.max())
        q /= q.sum()
        h = -(q[q > 0] * np.log(q[q > 0])).sum()
        assert abs(float(thr) - np.exp(-h)) <= 1e-4 * np.exp(-h) + 1e-7
        assert accept.typical_threshold(row, 0.9, 1.0)[1] == np.float32(max(0.9, float(thr)))
    # One-hot rows: H = 0, threshold = max(epsilon, delta).
    row = np.full(8, -np.inf, dtype=np.float32)
    row[3] = 0.0
    _, thr = accept.typical_threshold(row, 0.2, 0.7)
    assert thr == np.float32(0.7)
    assert accept.typical_accept_one(row, 3, 0.2, 0.7) and not accept.typical_accept_one(row, 2, 0.2, 0.7)
    # An all -inf row has no finite mass: the reference returns false.
    assert accept.typical_threshold(np.full(4, -np.inf, dtype=np.float32), 0.0, 0.0) is None
    assert not accept.typical_accept_one(np.full(4, -np.inf, dtype=np.float32), 0, 0.0, 0.0)


def test_typical_tree_accept_first_longest(accept):
    # tree: 0 -> {1 (tok 5), 2 (tok 6)}; 1 -> 3 (tok 7); 2 -> 4 (tok 8)
    tokens = [9, 5, 6, 7, 8]
    parents = [0, 0, 0, 1, 2]
    rows = np.full((5, 10), -4.0, dtype=np.float32)
    rows[0, 5] = rows[0, 6] = 3.0   # both children pass at the root
    rows[1, 7] = -4.0               # node 1's row flat: 7 fails at epsilon 0.3
    rows[2, 8] = 6.0                # node 2 strongly predicts 8
    rows[4, 1] = 2.0                # bonus 1
    best, bonus = accept.typical_tree_accept(tokens, parents, rows, 0.3, 0.5)
    assert best == [0, 2, 4] and bonus == 1
