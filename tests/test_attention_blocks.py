"""The online-softmax update of one attention split, restated in numpy with
the kernel's roundings (f32 state, P rounded to f16 for the P.V product), to
check on the CPU the two exactness claims the split kernel relies on:

* a key block whose keys are all masked leaves (m, l, o) bit-identical, so
  blocks past the last key may be skipped;
* a row's split result does not depend on how many keys after its own last
  visible key the call holds (M-invariance: a row computed alone or together
  with later rows of the same step gives the same bits).
"""

import numpy as np

BLOCK = 32


def split_state(scores, v, visible, n_keys):
    """Processes keys [0, n_keys) of one split in BLOCK-key steps; keys past
    the scores' length count as masked.  Returns (m, l, o) of one row."""
    f32 = np.float32
    m, l = f32(-np.inf), f32(0.0)
    o = np.zeros(v.shape[1], dtype=np.float32)
    for b0 in range(0, n_keys, BLOCK):
        idx = np.arange(b0, b0 + BLOCK)
        inside = idx < len(scores)
        s = np.full(BLOCK, -np.inf, dtype=np.float32)
        s[inside] = np.where(visible[idx[inside]], scores[idx[inside]], -np.inf).astype(np.float32)
        bmax = s.max()
        mnew = max(m, bmax)
        muse = f32(0.0) if mnew == -np.inf else mnew
        alpha = np.exp2(f32(m - muse)).astype(np.float32)
        m = mnew
        p = np.exp2((s - muse).astype(np.float32)).astype(np.float16)
        l = f32(l * alpha + p.astype(np.float32).sum(dtype=np.float32))
        vb = np.zeros((BLOCK, v.shape[1]), dtype=np.float16)
        vb[inside] = v[idx[inside]]
        o = (o * alpha).astype(np.float32) + p.astype(np.float32) @ vb.astype(np.float32)
    return m, l, o


def _case(seed, n, hd=64):
    rng = np.random.default_rng(seed)
    scores = (rng.standard_normal(n) * 3).astype(np.float32)
    v = rng.standard_normal((n, hd)).astype(np.float16)
    return scores, v


def _same(a, b):
    return all(np.array_equal(np.asarray(x).view(np.uint32), np.asarray(y).view(np.uint32)) for x, y in zip(a, b))


def test_masked_tail_blocks_change_nothing():
    for seed in range(20):
        n = 40 + seed * 3  # the split's last key is inside its second or third block
        scores, v = _case(seed, n)
        visible = np.ones(n, dtype=bool)
        trimmed = split_state(scores, v, visible, (n + BLOCK - 1) // BLOCK * BLOCK)
        full = split_state(scores, v, visible, 128)  # the whole 128-key split, tail masked
        assert _same(trimmed, full), seed


def test_row_result_independent_of_later_keys():
    # Row i of a step sees the prefix and new keys up to its own; the call
    # holds the keys of every row.  Its result must match the call that holds
    # only the keys up to row i's.
    for seed in range(20):
        prefix, rows = 50 + seed, 8
        n_all = prefix + rows
        scores, v = _case(100 + seed, n_all)
        for i in range(rows):
            visible = np.arange(n_all) < prefix + i + 1
            alone = split_state(scores[: prefix + i + 1], v[: prefix + i + 1], visible, 128)
            together = split_state(scores, v, visible, 128)
            assert _same(alone, together), (seed, i)


def test_fully_masked_split_is_empty():
    scores, v = _case(7, 64)
    m, l, o = split_state(scores, v, np.zeros(64, dtype=bool), 64)
    assert m == -np.inf and l == 0.0 and not o.any()
