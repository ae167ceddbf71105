"""Medusa heads on the device (spec_medusa_topk) against the restated
medusa.rs heads (oracle/medusa.py) on the same BF16 weights.

Every head maps the target's hidden row through its residual blocks and its
output projection; a device top-k and log-softmax follow.  The check: the
device's k ids are a top-k of the oracle's logits row within the tolerance,
and their log-probs match within it.  The tolerance is 2 % of the row's
scale (BF16 operands into each linear, as in the reference's BF16 heads)."""

import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL = 2e-2


def _bf(rng, shape, s):
    eo = importlib.import_module("oracle.eagle")
    return eo.bf16_bits(rng.standard_normal(shape).astype(np.float32) * np.float32(s))


@pytest.mark.parametrize("name,heads,layers", [("llama_q4km", 4, 1), ("qwen_q4km", 3, 2), ("llama_bf16", 2, 0)])
def test_medusa_topk_matches_oracle(pkg, tiny_gguf, name, heads, layers):
    mo = importlib.import_module("oracle.medusa")
    dec = pkg.B200Decoder.from_gguf(tiny_gguf(name), max_ctx=128)
    H, V = dec.hidden_size(), dec.vocab_size()
    rng = np.random.default_rng(11)
    res_w = [[_bf(rng, (H, H), 0.05) for _ in range(layers)] for _ in range(heads)]
    res_b = [[(0.1 * rng.standard_normal(H)).astype(np.float32) for _ in range(layers)] for _ in range(heads)]
    out_w = [_bf(rng, (V, H), 0.05) for _ in range(heads)]
    dec.medusa_attach(res_w, res_b, out_w)
    assert dec.medusa_num_heads() == heads
    hidden = rng.standard_normal(H).astype(np.float32)
    k = 10
    ids, lp = dec.medusa_topk(hidden, k)
    assert ids.shape == (heads, k) and lp.shape == (heads, k)
    _, rows = mo.MedusaOracle(res_w, res_b, out_w).top_k_per_head(hidden, k)
    for h in range(heads):
        row = rows[h]
        tol = REL * max(1.0, float(np.max(np.abs(row))))
        mx = np.max(row)
        lse = np.log(np.sum(np.exp(row - mx))) + mx
        kth = np.sort(row)[::-1][k - 1]
        assert np.all(row[ids[h]] >= kth - 2 * tol), h
        err = float(np.abs(lp[h] - (row[ids[h]] - lse)).max())
        assert err <= tol, (h, err, tol)
        assert np.all(np.diff(lp[h]) <= 0)
    # the same call again gives the same bits
    ids2, lp2 = dec.medusa_topk(hidden, k)
    assert np.array_equal(ids, ids2) and np.array_equal(lp, lp2)


def test_medusa_errors_and_synthetic(pkg, tiny_gguf):
    dec = pkg.B200Decoder.from_gguf(tiny_gguf("llama_q4km"), max_ctx=128)
    h = np.zeros(dec.hidden_size(), np.float32)
    with pytest.raises(pkg.SamplingError):
        dec.medusa_topk(h, 4)  # nothing attached
    with pytest.raises(pkg.SamplingError):
        dec.medusa_attach_synthetic(9, 1, 0)  # more than 8 heads
    dec.medusa_attach_synthetic(4, 1, 5)
    ids, lp = dec.medusa_topk(h + 0.5, 8)
    assert ids.shape == (4, 8) and np.isfinite(lp).all() and (ids >= 0).all() and (ids < dec.vocab_size()).all()
    with pytest.raises(pkg.SamplingError):
        dec.medusa_topk(h, 65)


def _grown_tree(pkg, dec, root, rng, depth, V):
    """A tree whose children are, per node, its row's top two tokens and one
    random token (rows from tree forwards of the tree grown so far), so that
    the typical rule both passes and fails along its paths."""
    tokens, parents = [int(root)], [0]
    frontier = [0]
    for _ in range(depth):
        rows, _ = dec.tree_logits_keep_kv(pkg.DraftTree(tokens, parents))
        nxt = []
        for f in frontier:
            top = np.argsort(-rows[f], kind="stable")[:2].tolist()
            for t in top + [int(rng.integers(0, V))]:
                if len(tokens) < 40:
                    tokens.append(int(t))
                    parents.append(f)
                    nxt.append(len(tokens) - 1)
        frontier = nxt
    return pkg.DraftTree(tokens, parents)


@pytest.mark.parametrize("name", ["llama_q4km", "qwen_q4km", "llama_bf16"])
def test_verify_tree_typical_matches_oracle(pkg, tiny_gguf, accept, name):
    """spec_verify_tree_typical (device softmax/entropy per node row, host
    walk) against medusa.rs typical acceptance restated on the same node rows
    (oracle.accept.typical_tree_accept): identical accepted paths and bonus
    tokens, bit for bit, for several (epsilon, delta), and the KV/history
    state of spec_verify_tree_greedy."""
    dec = pkg.B200Decoder.from_gguf(tiny_gguf(name), max_ctx=256)
    V = dec.vocab_size()
    rng = np.random.default_rng(21)
    prompt = rng.integers(0, V, size=17).tolist()
    dec.observe(prompt)
    tree = _grown_tree(pkg, dec, prompt[-1], rng, 3, V)
    rows, _ = dec.tree_logits_keep_kv(tree)
    lengths = set()
    for eps, delta in [(0.0, 1.0), (0.001, 0.5), (0.01, 0.3), (0.05, 2.0), (0.3, 0.3), (1.0, 0.0)]:
        want_best, want_bonus = accept.typical_tree_accept(tree.tokens(), tree.parents(), rows, eps, delta)
        best, bonus = dec.verify_tree_typical(tree, eps, delta)
        assert best == want_best and bonus == want_bonus, (eps, delta)
        assert dec.kv_len() == len(prompt) - 1 + len(tree) and dec.history() == prompt
        lengths.add(len(best))
    assert 1 in lengths and max(lengths) >= 3, lengths
    # Greedy and typical share the forward and the walk: with epsilon above
    # every probability nothing passes, as a greedy walk on a root whose
    # argmax is not a child.
    best, bonus = dec.verify_tree_typical(tree, 2.0, 0.0)
    assert best == [0] and bonus == int(accept.argmax_first_fast(rows[0]))
    with pytest.raises(pkg.SamplingError):
        dec.verify_tree_typical(pkg.DraftTree([prompt[-1] + 1 if prompt[-1] + 1 < V else 0], [0]), 0.1, 0.1)
    dec.close()


def _medusa_tree(pkg, root, ids, topology):
    """medusa.rs:167-189: the greedy chain of each head's top-1, or the
    Cartesian product in BFS layers."""
    if topology == "greedy":
        return pkg.DraftTree.linear(int(root), [int(c[0]) for c in ids])
    tokens, parents, prev = [int(root)], [0], [0]
    for cands in ids:
        nxt = []
        for p in prev:
            for c in cands:
                tokens.append(int(c))
                parents.append(p)
                nxt.append(len(tokens) - 1)
        prev = nxt
    return pkg.DraftTree(tokens, parents)


def _medusa_round_by_trait_calls(pkg, dec, hidden, k, topology, acceptance, eps, delta, budget):
    """run_medusa_real's loop body (medusa.rs:761-810) from the trait calls:
    heads' top-k, tree, tree forward + walk, commit of the path, bonus."""
    root = dec.history()[-1]
    ids, _ = dec.medusa_topk(hidden, k)
    tree = _medusa_tree(pkg, root, ids, topology)
    if acceptance == "greedy":
        best, bonus = dec.verify_tree_greedy(tree)
    else:
        best, bonus = dec.verify_tree_typical(tree, eps, delta)
    committed = [tree.token_at(i) for i in best[1:]]
    dec.commit_tree_path(tree, best)
    if len(committed) < budget:
        committed.append(int(bonus))
        return committed, dec.observe_returning_last_hidden([int(bonus)])
    return committed, None


@pytest.mark.parametrize("name,heads,k,topology,acceptance", [
    ("llama_q4km", 4, 2, "cartesian", "greedy"),
    ("qwen_q4km", 3, 3, "cartesian", "typical"),
    ("llama_bf16", 4, 2, "greedy", "typical"),
    ("llama_q4km", 4, 3, "cartesian", "greedy"),   # 121 nodes: ancestor-closed chunks
    ("qwen_q4km", 4, 3, "cartesian", "typical"),
])
def test_native_medusa_round_equals_trait_calls(pkg, tiny_gguf, name, heads, k, topology, acceptance):
    """spec_medusa_round against the same rounds made of trait calls: equal
    commits, histories, KV lengths and next hidden rows (bit for bit) over
    several rounds, the last one cut by the token budget."""
    path = tiny_gguf(name)
    a = pkg.B200Decoder.from_gguf(path, max_ctx=256)
    b = pkg.B200Decoder.from_gguf(path, max_ctx=256)
    for d in (a, b):
        d.medusa_attach_synthetic(heads, 1, 17)
    rng = np.random.default_rng(9)
    prompt = rng.integers(0, a.vocab_size(), size=19).tolist()
    ha = a.observe_returning_last_hidden(prompt)
    hb = b.observe_returning_last_hidden(prompt)
    assert np.array_equal(ha.view(np.uint32), hb.view(np.uint32))
    eps, delta = 0.002, 0.3
    total, max_new = 0, 14
    while total < max_new:
        budget = max_new - total
        ca, ha = a.medusa_round(ha, k, topology, acceptance, eps, delta, budget)
        cb, hb = _medusa_round_by_trait_calls(pkg, b, hb, k, topology, acceptance, eps, delta, budget)
        assert ca == cb
        assert a.history() == b.history() and a.kv_len() == b.kv_len()
        if hb is not None:
            assert np.array_equal(ha.view(np.uint32), hb.view(np.uint32))
        total += len(ca)
        if hb is None:
            break
    # The accepted path is committed whole; the budget only withholds the bonus (:786-800).
    assert total >= max_new and len(a.history()) == len(prompt) + total
    # A Cartesian tree over 16384 nodes is refused with the state unchanged.
    if topology == "cartesian":
        hist, kv = a.history(), a.kv_len()
        with pytest.raises(pkg.SpecError):
            a.medusa_round(ha, 64, "cartesian")
        assert a.history() == hist and a.kv_len() == kv
    a.close()
    b.close()


@pytest.mark.parametrize("name", ["llama_q4km", "qwen_q4km"])
def test_verify_tree_typical_over_max_rows(pkg, tiny_gguf, accept, name):
    """Typical acceptance over a 121-node tree (chunks of at most 64 rows):
    the same decisions as the restated rule on the chunked forward's rows."""
    dec = pkg.B200Decoder.from_gguf(tiny_gguf(name), max_ctx=256)
    V = dec.vocab_size()
    rng = np.random.default_rng(43)
    prompt = rng.integers(0, V, size=15).tolist()
    dec.observe(prompt)
    tokens, parents, frontier = [prompt[-1]], [0], [0]
    for _ in range(4):  # every node: its row's top two tokens and a random one
        rows, _ = dec.tree_logits_keep_kv(pkg.DraftTree(tokens, parents))
        nxt = []
        for f in frontier:
            for t in np.argsort(-rows[f], kind="stable")[:2].tolist() + [int(rng.integers(0, V))]:
                tokens.append(int(t))
                parents.append(f)
                nxt.append(len(tokens) - 1)
        frontier = nxt
    tree = pkg.DraftTree(tokens, parents)
    assert len(tree) > 64
    rows, _ = dec.tree_logits_keep_kv(tree)
    lengths = set()
    for eps, delta in [(0.0, 1.0), (0.001, 0.5), (0.01, 0.3), (0.3, 0.3)]:
        want = accept.typical_tree_accept(tokens, parents, rows, eps, delta)
        assert dec.verify_tree_typical(tree, eps, delta) == want, (eps, delta)
        lengths.add(len(want[0]))
    assert max(lengths) >= 3, lengths
    dec.close()
