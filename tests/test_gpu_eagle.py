"""EAGLE draft loop on the device (spec_eagle_draft) against the restated
eagle.rs loop (oracle/eagle.py) on the same BF16 weights.

Per step: the draft block, the target's LM head, a device top-k and the
log-softmax; the next step takes the top-1 on the device.  The oracle replays
the device's top-1 choices (so a near-tie cannot make the two walks diverge)
and the check is: the device's k ids are a top-k of the oracle's logits row
within the tolerance, and their log-probs match within it.  The tolerance is
2 % of the row's scale: each step's hidden row feeds the next through five
BF16-rounded operands, so single BF16 rounding differences compound over the
depth (a wrong position, mask or weight moves logits by O(1))."""

import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL = 2e-2


def _weights(rng, H, nq, nkv, hd, F):
    eo = importlib.import_module("oracle.eagle")

    def bf(shape, s=0.05):
        return eo.bf16_bits(rng.standard_normal(shape).astype(np.float32) * np.float32(s))
    return {"fc": bf((H, 2 * H)), "q": bf((nq * hd, H)), "k": bf((nkv * hd, H)), "v": bf((nkv * hd, H)),
            "o": bf((H, nq * hd)), "gate": bf((F, H)), "up": bf((F, H)), "down": bf((H, F)),
            "post_norm": (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)}


@pytest.mark.parametrize("name", ["llama_q4km", "qwen_q4km"])
def test_eagle_draft_matches_oracle(pkg, oracle, tiny_gguf, name):
    eo = importlib.import_module("oracle.eagle")
    path = tiny_gguf(name)
    dec = pkg.B200Decoder.from_gguf(path, max_ctx=256)
    om = oracle.OracleModel(path, max_ctx=256)
    H, nq, nkv = om.hidden, om.n_heads, om.n_kv
    hd, F = om.head_dim, om.tensors["blk.0.ffn_gate.weight"].shape[0]
    rng = np.random.default_rng(7)
    w = _weights(rng, H, nq, nkv, hd, F)
    dec.eagle_attach(w)
    hidden = rng.standard_normal(H).astype(np.float32)
    depth, k, pos, root = 6, 10, 37, 123
    ids, lp = dec.eagle_draft(hidden, root, pos, depth, k)
    assert ids.shape == (depth, k) and lp.shape == (depth, k)
    ref = eo.EagleOracle(om, w)
    oids, olp, rows = ref.draft(hidden, root, pos, depth, k, follow=ids[:, 0].tolist())
    for s in range(depth):
        row = rows[s]
        tol = REL * max(1.0, float(np.max(np.abs(row))))
        mx = np.max(row)
        lse = np.log(np.sum(np.exp(row - mx))) + mx
        kth = np.sort(row)[::-1][k - 1]
        assert np.all(row[ids[s]] >= kth - 2 * tol), s
        err = float(np.abs(lp[s] - (row[ids[s]] - lse)).max())
        assert err <= tol, (s, err, tol)
        # descending order, as top_k_indices returns them
        assert np.all(np.diff(lp[s]) <= 0)
    # a second call starts a new round (the draft cache is per round)
    ids2, lp2 = dec.eagle_draft(hidden, root, pos, depth, k)
    assert np.array_equal(ids, ids2) and np.array_equal(lp, lp2)


def test_eagle_errors_and_synthetic(pkg, tiny_gguf):
    dec = pkg.B200Decoder.from_gguf(tiny_gguf("llama_q4km"), max_ctx=128)
    h = np.zeros(dec.hidden_size(), np.float32)
    with pytest.raises(pkg.SamplingError):
        dec.eagle_draft(h, 1, 0, 2, 4)  # nothing attached
    dec.eagle_attach_synthetic(3)
    ids, lp = dec.eagle_draft(h, 1, 0, 4, 8)
    assert ids.shape == (4, 8) and np.isfinite(lp).all() and (ids >= 0).all()
    with pytest.raises(pkg.UnsupportedMethodError):
        dec.eagle_draft(h, 1, 0, 65, 8)
    with pytest.raises(pkg.SamplingError):
        dec.eagle_draft(h, 10 ** 6, 0, 2, 8)


def _py_eagle_round(pkg, dec, hidden, depth, k, max_nodes, strict, eos):
    """run_eagle's loop body (eagle.rs:531-731, greedy) written over the
    trait calls, with the tree of oracle/eagle.py: the counterpart of
    spec_eagle_round."""
    eo = importlib.import_module("oracle.eagle")
    root, pos = dec.history()[-1], dec.history_len()
    ids, lp = dec.eagle_draft(hidden, root, pos, depth, k)
    nodes = eo.build_cartesian_tree(root, ids.tolist())
    if max_nodes:
        nodes = eo.prune_cartesian_tree(nodes, lp.tolist(), max_nodes)
    tree = pkg.DraftTree.from_parent_table(nodes)
    _, hid = dec.tree_logits_keep_kv(tree)
    best, bonus = dec.verify_tree_greedy(tree)  # the same tree forward again, then the walk
    committed = [tree.token_at(i) for i in best[1:]] + [int(bonus)]
    eos_at = next((i for i, t in enumerate(committed) if t in eos), None)
    if eos_at is not None:
        committed = committed[:eos_at + 1]
    if eos_at is not None and eos_at < len(best) - 1:
        dec.commit_tree_path(tree, best[:eos_at + 2])
        return committed, None, True, False
    bn = None
    if not strict:
        bn = next((i for i in range(1, len(tree)) if tree.parent_of(i) == best[-1] and tree.token_at(i) == bonus),
                  None)
    if bn is not None:
        dec.commit_tree_path(tree, list(best) + [bn])
        return committed, hid[bn].copy(), eos_at is not None, True
    dec.commit_tree_path(tree, best)
    return committed, dec.observe_returning_last_hidden([int(bonus)]), eos_at is not None, False


@pytest.mark.parametrize("depth,k,max_nodes,strict", [(2, 4, 0, False), (4, 4, 40, False), (3, 8, 60, True),
                                                      (3, 6, 0, True)])  # 259 nodes: ancestor-closed chunks
def test_native_eagle_round_equals_trait_calls(pkg, tiny_gguf, depth, k, max_nodes, strict):
    """spec_eagle_round (draft loop, tree, tree forward, walk, KV commit in
    one call) against the same round made of the trait calls in the
    reference's order: identical commits, next hidden rows (bit for bit),
    histories and KV lengths over several rounds, with an EOS id taken from
    a dry run so one round stops on it."""
    path = tiny_gguf("llama_q4km")
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, 1024, size=21).tolist()
    dec_probe = pkg.B200Decoder.from_gguf(path, max_ctx=256)
    dec_probe.eagle_attach_synthetic(99)
    hid = dec_probe.observe_returning_last_hidden(prompt)
    dry = []
    for _ in range(6):
        c, hid, _ = dec_probe.eagle_round(hid, depth, k, max_nodes, strict)
        dry.append(c)
    eos = {dry[3][-1]}
    runs = []
    for native in (True, False):
        dec = pkg.B200Decoder.from_gguf(path, max_ctx=256)
        dec.eagle_attach_synthetic(99)
        hid = dec.observe_returning_last_hidden(prompt)
        rec = []
        for _ in range(6):
            if native:
                c, nh, stop = dec.eagle_round(hid, depth, k, max_nodes, strict, eos)
            else:
                c, nh, stop, _ = _py_eagle_round(pkg, dec, hid, depth, k, max_nodes, strict, eos)
            rec.append((c, stop, dec.history(), dec.kv_len()))
            if stop:
                break
            assert nh is not None
            rec.append(nh.view(np.uint32).tolist())
            hid = nh
        runs.append(rec)
    assert runs[0] == runs[1]
    assert any(r[1] for r in runs[0] if isinstance(r, tuple)), "the EOS round stops"
