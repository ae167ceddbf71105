"""Decoder / TreeDecoder parity through the C ABI against the oracle (GPU).

Bars (north star): logits max-abs <= 2e-2 vs the oracle; decisions, history,
KV lengths bit-exact; batched rows bit-identical to sequential rows
(M-invariance) and tree row 0 bit-identical to next_logits.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-2
MODELS = ["llama_q4km", "llama_hd128", "qwen_q4km", "qwen_q5k", "qwen_q80", "llama_bf16"]


def _pair(pkg, oracle, path, max_ctx=512):
    dec = pkg.B200Decoder.from_gguf(path, max_ctx=max_ctx)
    om = oracle.OracleModel(path, max_ctx=max_ctx)
    return dec, oracle.OracleDecoder(om)


def _prompt(vocab, n, seed):
    return np.random.default_rng(seed).integers(0, vocab, size=n).tolist()


@pytest.mark.parametrize("name", MODELS)
def test_observe_next_and_batched_logits(pkg, oracle, tiny_gguf, name):
    dec, ref = _pair(pkg, oracle, tiny_gguf(name))
    prompt = _prompt(dec.vocab_size(), 37, 1)
    dec.observe(prompt)
    ref.observe(prompt)
    assert np.abs(dec.next_logits() - ref.next_logits()).max() <= TOL
    drafts = _prompt(dec.vocab_size(), 4, 2)
    a = dec.batched_logits(drafts)
    b = ref.batched_logits(drafts)
    assert a.shape == (5, dec.vocab_size())
    assert np.abs(a - b).max() <= TOL
    assert dec.history() == ref.history and dec.kv_len() == ref.cache_len
    # rollback + re-observe, as the vanilla loop does (vanilla.rs:358-362)
    dec.rollback_to(len(prompt) + 2)
    ref.rollback_to(len(prompt) + 2)
    dec.observe([5])
    ref.observe([5])
    assert np.abs(dec.next_logits() - ref.next_logits()).max() <= TOL
    assert dec.history() == ref.history and dec.kv_len() == ref.cache_len


@pytest.mark.parametrize("name", ["llama_q4km", "qwen_q5k", "qwen_q80"])
def test_logits_against_q8_1_activation_oracle(pkg, oracle, tiny_gguf, name):
    """The reference's CUDA matmul is expected to quantize activations to Q8_1
    (restated by OracleModel(act_quant="q8_1")); that alone moves logits by 0.015-0.023
    from the f32 restatement on these models (tests/test_oracle_act_quant.py).
    The device logits must sit within the same distance of it: 3e-2, and the
    device's distance to the f32 oracle stays within 2e-2."""
    path = tiny_gguf(name)
    dec = pkg.B200Decoder.from_gguf(path, max_ctx=512)
    q8 = oracle.OracleDecoder(oracle.OracleModel(path, max_ctx=512, act_quant="q8_1"))
    f32 = oracle.OracleDecoder(oracle.OracleModel(path, max_ctx=512))
    prompt = _prompt(dec.vocab_size(), 60, 11)
    drafts = _prompt(dec.vocab_size(), 4, 3)
    rows = []
    for d in (dec, q8, f32):
        d.observe(prompt)
        rows.append(np.concatenate([d.next_logits()[None], d.batched_logits(drafts)]))
    got, ref_q8, ref_f32 = rows
    print(f"{name}: device vs Q8_1 oracle {np.abs(got - ref_q8).max():.4f}, "
          f"vs f32 oracle {np.abs(got - ref_f32).max():.4f}")
    assert np.abs(got - ref_q8).max() <= 3e-2
    assert np.abs(got - ref_f32).max() <= TOL


@pytest.mark.parametrize("name", ["llama_q4km", "qwen_q4km", "llama_bf16"])
def test_long_observe_chunks(pkg, oracle, tiny_gguf, name):
    dec, ref = _pair(pkg, oracle, tiny_gguf(name))
    prompt = _prompt(dec.vocab_size(), 150, 3)  # > 64 rows: chunked forwards
    dec.observe(prompt)
    ref.observe(prompt)
    assert np.abs(dec.next_logits() - ref.next_logits()).max() <= TOL


@pytest.mark.parametrize("name", MODELS)
def test_batched_equals_sequential_bitwise(pkg, tiny_gguf, name):
    path = tiny_gguf(name)
    a = pkg.B200Decoder.from_gguf(path, max_ctx=512)
    b = pkg.B200Decoder.from_gguf(path, max_ctx=512)
    prompt = _prompt(a.vocab_size(), 20, 4)
    drafts = _prompt(a.vocab_size(), 8, 5)
    a.observe(prompt)
    rows = a.batched_logits(drafts)
    b.observe(prompt)
    seq = [b.next_logits()]
    for d in drafts:
        b.observe([d])
        seq.append(b.next_logits())
    for i in range(len(seq)):
        assert np.array_equal(rows[i].view(np.uint32), seq[i].view(np.uint32)), f"row {i}"


def _tree(pkg, root, vocab, seed):
    rng = np.random.default_rng(seed)
    nodes = [(0, root)]
    for i in range(1, 12):
        nodes.append((int(rng.integers(0, i)), int(rng.integers(0, vocab))))
    return pkg.DraftTree.from_parent_table(nodes)


@pytest.mark.parametrize("name", MODELS)
def test_tree_logits_and_restore(pkg, oracle, tiny_gguf, name):
    dec, ref = _pair(pkg, oracle, tiny_gguf(name))
    prompt = _prompt(dec.vocab_size(), 30, 6)
    dec.observe(prompt)
    ref.observe(prompt)
    nxt = dec.next_logits()
    tree = _tree(pkg, prompt[-1], dec.vocab_size(), 7)
    a = dec.tree_logits(tree)
    b = ref.tree_logits(tree.tokens(), tree.parents())
    assert np.abs(a - b).max() <= TOL
    assert np.array_equal(a[0].view(np.uint32), nxt.view(np.uint32))
    assert dec.history() == ref.history and dec.kv_len() == ref.cache_len
    assert np.array_equal(dec.next_logits().view(np.uint32), nxt.view(np.uint32))


@pytest.mark.parametrize("name", ["llama_q4km", "qwen_q4km", "llama_bf16"])
def test_tree_logits_over_max_rows(pkg, oracle, tiny_gguf, name):
    """Trees over SPEC_MAX_ROWS nodes (the reference's DraftTree has no cap):
    a 121-node Cartesian tree (4 levels of 3, Medusa's 4 heads x top-3) and a
    deep 70-node chain with side branches run as ancestor-closed chunks of at
    most 64 rows.  Every node's row matches the oracle's single tree forward,
    each node's row equals its own ancestor chain's tree forward, and the
    state is restored as for a small tree."""
    dec, ref = _pair(pkg, oracle, tiny_gguf(name))
    V = dec.vocab_size()
    rng = np.random.default_rng(31)
    prompt = _prompt(V, 23, 12)
    dec.observe(prompt)
    ref.observe(prompt)
    nxt = dec.next_logits()
    tokens, parents, prev = [prompt[-1]], [0], [0]
    for _ in range(4):
        layer = []
        cands = rng.integers(0, V, size=3).tolist()
        for p in prev:
            for c in cands:
                tokens.append(int(c))
                parents.append(p)
                layer.append(len(tokens) - 1)
        prev = layer
    chain_t, chain_p = [prompt[-1]], [0]
    for i in range(1, 70):
        chain_t.append(int(rng.integers(0, V)))
        chain_p.append(i - 1 if i % 5 else max(0, i - 3))
    for tt, pp in ((tokens, parents), (chain_t, chain_p)):
        tree = pkg.DraftTree(tt, pp)
        a = dec.tree_logits(tree)
        b = ref.tree_logits(tt, pp)
        assert a.shape == (len(tt), V)
        assert np.abs(a - b).max() <= TOL
        assert np.array_equal(a[0].view(np.uint32), nxt.view(np.uint32))
        assert dec.history() == ref.history and dec.kv_len() == ref.cache_len
        assert np.array_equal(dec.next_logits().view(np.uint32), nxt.view(np.uint32))
        for i in (len(tt) - 1, len(tt) // 2, 40):
            anc = tree.path_to(i)
            if len(anc) > 64:
                continue
            row = dec.tree_logits(pkg.DraftTree([tt[j] for j in anc], [0] + list(range(len(anc) - 1))))[-1]
            assert np.abs(row - a[i]).max() <= TOL
    # A chain deeper than 64 nodes cannot be cut into ancestor-closed chunks.
    deep = pkg.DraftTree([prompt[-1]] + [5] * 64, [0] + list(range(64)))
    with pytest.raises(pkg.SpecError):
        dec.tree_logits(deep)
    assert np.array_equal(dec.next_logits().view(np.uint32), nxt.view(np.uint32))


def _cartesian(root, V, rng, levels=4, width=3):
    tokens, parents, prev = [int(root)], [0], [0]
    for _ in range(levels):
        layer = []
        cands = rng.integers(0, V, size=width).tolist()
        for p in prev:
            for c in cands:
                tokens.append(int(c))
                parents.append(p)
                layer.append(len(tokens) - 1)
        prev = layer
    return tokens, parents


@pytest.mark.parametrize("name", ["llama_q4km", "qwen_q4km"])
def test_tree_over_max_rows_keep_kv_verify_commit(pkg, oracle, accept, tiny_gguf, name):
    """A 121-node tree with the KV kept: logits and hidden rows against the
    oracle; committing a path whose nodes are not in the last chunk's KV
    rows (the chunk is brought back) and then the greedy verify's own best
    path leave the KV the oracle's commit leaves (next logits after a
    further token)."""
    dec, ref = _pair(pkg, oracle, tiny_gguf(name))
    V = dec.vocab_size()
    rng = np.random.default_rng(41)
    prompt = _prompt(V, 21, 14)
    dec.observe(prompt)
    ref.observe(prompt)
    tt, pp = _cartesian(prompt[-1], V, rng)
    tree = pkg.DraftTree(tt, pp)
    lo, hi = dec.tree_logits_keep_kv(tree)
    rlo, rhi = ref.tree_logits_keep_kv(tt, pp)
    assert np.abs(lo - rlo).max() <= TOL and np.abs(hi - rhi).max() <= TOL
    path = tree.path_to(5)  # nodes 0 -> 1 -> 5, all in the first chunk
    dec.commit_tree_path(tree, path)
    ref.commit_tree_path(tt, pp, path)
    assert dec.history() == ref.history and dec.kv_len() == ref.cache_len
    dec.observe([7])
    ref.observe([7])
    assert np.abs(dec.next_logits() - ref.next_logits()).max() <= TOL
    # Greedy verify over the big tree: decisions from the device's own rows.
    tt, pp = _cartesian(dec.history()[-1], V, rng)
    tree = pkg.DraftTree(tt, pp)
    rows, _ = dec.tree_logits_keep_kv(tree)
    best, bonus = dec.verify_tree_greedy(tree)
    assert (best, bonus) == accept.greedy_tree_accept(tt, pp, rows)
    # A non-path commit is refused over 64 nodes; a path commit works.
    with pytest.raises(pkg.SpecError):
        dec.commit_tree_path(tree, [0, 1, 2])
    deep = max(tree.paths(), key=len)
    ref.tree_logits_keep_kv(tt, pp)
    dec.commit_tree_path(tree, deep)
    ref.commit_tree_path(tt, pp, deep)
    assert dec.history() == ref.history and dec.kv_len() == ref.cache_len
    dec.observe([int(bonus)])
    ref.observe([int(bonus)])
    assert np.abs(dec.next_logits() - ref.next_logits()).max() <= TOL


@pytest.mark.parametrize("name", MODELS)
def test_tree_keep_kv_commit_path(pkg, oracle, tiny_gguf, name):
    dec, ref = _pair(pkg, oracle, tiny_gguf(name))
    prompt = _prompt(dec.vocab_size(), 25, 8)
    dec.observe(prompt)
    ref.observe(prompt)
    tree = _tree(pkg, prompt[-1], dec.vocab_size(), 9)
    lo, hi = dec.tree_logits_keep_kv(tree)
    rlo, rhi = ref.tree_logits_keep_kv(tree.tokens(), tree.parents())
    assert np.abs(lo - rlo).max() <= TOL
    assert np.abs(hi - rhi).max() <= TOL
    assert dec.kv_len() == ref.cache_len
    path = max(tree.paths(), key=len)
    dec.commit_tree_path(tree, path)
    ref.commit_tree_path(tree.tokens(), tree.parents(), path)
    assert dec.history() == ref.history and dec.kv_len() == ref.cache_len
    dec.observe([3])
    ref.observe([3])
    assert np.abs(dec.next_logits() - ref.next_logits()).max() <= TOL


def test_commit_equals_linear_replay_bitwise(pkg, tiny_gguf):
    """Committing a tree path leaves exactly the KV a plain replay would."""
    path = tiny_gguf("llama_q4km")
    a = pkg.B200Decoder.from_gguf(path, max_ctx=512)
    b = pkg.B200Decoder.from_gguf(path, max_ctx=512)
    prompt = _prompt(a.vocab_size(), 25, 10)
    a.observe(prompt)
    b.observe(prompt)
    tree = _tree(pkg, prompt[-1], a.vocab_size(), 11)
    a.tree_logits_keep_kv(tree)
    chain = max(tree.paths(), key=len)
    a.commit_tree_path(tree, chain)
    b.observe([tree.token_at(i) for i in chain[1:]])
    a.observe([7])
    b.observe([7])
    assert a.history() == b.history()
    assert np.array_equal(a.next_logits().view(np.uint32), b.next_logits().view(np.uint32))


@pytest.mark.parametrize("name", ["llama_q4km", "qwen_q80", "llama_bf16"])
def test_hidden_embed_lm_head(pkg, oracle, tiny_gguf, name):
    dec, ref = _pair(pkg, oracle, tiny_gguf(name))
    ids = _prompt(dec.vocab_size(), 9, 12)
    emb = dec.embed_tokens(ids)
    assert np.array_equal(emb, ref.m.embed(ids).astype(np.float32))
    dec.observe(ids)
    ref.observe(ids)
    h = dec.last_hidden_state()
    rh, _ = ref.m.forward([ids[-1]], [len(ids) - 1], [len(ids) - 1], len(ids) - 1, [1])
    assert np.abs(h - rh[0]).max() <= TOL
    lo = dec.apply_lm_head(h[None])
    assert np.abs(lo[0] - ref.m.lm_head(h[None].astype(np.float64))[0]).max() <= TOL
    fin, mids = dec.last_hidden_states_multi([0, 1])
    assert np.abs(fin - h).max() <= 1e-5 and len(mids) == 2
    hid = dec.observe_returning_last_hidden([4, 5])
    rh2, _ = ref.m.forward([4, 5], [len(ids), len(ids) + 1], [len(ids), len(ids) + 1], len(ids), [1, 3])
    assert np.abs(hid - rh2[-1]).max() <= TOL


@pytest.mark.parametrize("name", ["llama_q4km", "qwen_q4km"])
def test_verify_greedy_decisions(pkg, accept, tiny_gguf, name):
    path = tiny_gguf(name)
    a = pkg.B200Decoder.from_gguf(path, max_ctx=512)
    b = pkg.B200Decoder.from_gguf(path, max_ctx=512)
    prompt = _prompt(a.vocab_size(), 16, 13)
    a.observe(prompt)
    b.observe(prompt)
    # drafts = the model's own greedy continuation, one token corrupted
    cont = []
    for _ in range(4):
        t = accept.argmax_first(b.next_logits())
        cont.append(t)
        b.observe([t])
    b.rollback_to(len(prompt))
    drafts = cont[:2] + [(cont[2] + 1) % a.vocab_size()] + cont[3:]
    n_acc, nxt, am = a.verify_greedy(drafts)
    rows = b.batched_logits(drafts)
    exp_acc, exp_next = accept.greedy_linear_accept(rows, drafts)
    assert (n_acc, nxt) == (exp_acc, exp_next) and n_acc == 2
    assert list(am) == [accept.argmax_first(r) for r in rows]
    assert a.history() == b.history() and a.kv_len() == b.kv_len()


def test_verify_tree_greedy(pkg, accept, tiny_gguf):
    path = tiny_gguf("llama_q4km")
    a = pkg.B200Decoder.from_gguf(path, max_ctx=512)
    b = pkg.B200Decoder.from_gguf(path, max_ctx=512)
    prompt = _prompt(a.vocab_size(), 16, 14)
    a.observe(prompt)
    b.observe(prompt)
    g1 = accept.argmax_first(b.next_logits())
    b.observe([g1])
    g2 = accept.argmax_first(b.next_logits())
    b.rollback_to(len(prompt))
    tree = pkg.DraftTree.from_parent_table([(0, prompt[-1]), (0, (g1 + 1) % 1024), (0, g1), (2, g2), (2, 5)])
    best, bonus = a.verify_tree_greedy(tree)
    rows, _ = b.tree_logits_keep_kv(tree)
    eb, ebonus = accept.greedy_tree_accept(tree.tokens(), tree.parents(), rows)
    assert (best, bonus) == (eb, ebonus) and best[:3] == [0, 2, 3]
    assert a.kv_len() == b.kv_len()


def test_error_behaviour(pkg, tiny_gguf):
    dec = pkg.B200Decoder.from_gguf(tiny_gguf("llama_q4km"), max_ctx=128)
    with pytest.raises(pkg.SamplingError):
        dec.next_logits()  # empty history
    dec.observe([1, 2, 3])
    with pytest.raises(pkg.CacheRollbackError):
        dec.rollback_to(4)
    with pytest.raises(pkg.SamplingError):
        dec.observe([10 ** 6])  # token out of range; state unchanged
    assert dec.history() == [1, 2, 3] and dec.kv_len() == 3
    with pytest.raises(pkg.SamplingError):
        dec.tree_logits(pkg.DraftTree.linear(9, [1]))  # root != last committed
    with pytest.raises(pkg.SamplingError):
        dec.observe(list(range(200)))  # exceeds KV capacity
    assert dec.kv_len() == 3
    with pytest.raises(pkg.IoError):
        pkg.B200Decoder.from_gguf("/nonexistent/model.gguf")
    dec.reset()
    assert dec.history() == [] and dec.kv_len() == 0


def test_large_residual_stays_finite(pkg, oracle, tiny_gguf):
    """Weights N(0, 2): the residual stream passes the f16 range by layer 1.

    The operands of the GEMVs after each residual update are emitted
    pre-scaled by the previous residual's RMS, so they stay O(1); logits must be
    finite and match the float64 oracle within 1 % of their range (the f16
    operand rounding is relative, and these logits are large)."""
    dec, ref = _pair(pkg, oracle, tiny_gguf("llama_hot"))
    prompt = _prompt(dec.vocab_size(), 21, 4)
    dec.observe(prompt)
    ref.observe(prompt)
    h = dec.last_hidden_states_multi([0, 1, 2])[1]
    assert np.abs(np.asarray(h)).max() > 65504.0  # the stress actually happened
    drafts = _prompt(dec.vocab_size(), 4, 5)
    a = dec.batched_logits(drafts)
    b = ref.batched_logits(drafts)
    assert np.isfinite(a).all()
    assert np.abs(a - b).max() <= 1e-2 * np.abs(b).max()


def test_lazy_observe_matches_eager(pkg, oracle, tiny_gguf):
    """observe leaves its last token pending; every observable result is the
    eager decoder's: KV length, rollback bounds, logits of the vanilla round
    protocol (batched verify, rollback, observe of the commits), hidden
    states after a pending token."""
    dec, ref = _pair(pkg, oracle, tiny_gguf("llama_q4km"))
    prompt = _prompt(dec.vocab_size(), 20, 21)
    dec.observe(prompt)
    ref.observe(prompt)
    assert dec.kv_len() == ref.cache_len == 20
    dec.rollback_to(20)  # no-op at the logical length
    ref.rollback_to(20)
    for rnd in range(3):  # vanilla.rs:285-369 round shape, k = 3
        drafts = _prompt(dec.vocab_size(), 3, 30 + rnd)
        pre = len(dec.history())
        a = dec.batched_logits(drafts)
        b = ref.batched_logits(drafts)
        assert np.abs(a - b).max() <= TOL
        acc = rnd % 3
        commits = drafts[:acc] + [int(np.argmax(a[acc]))]
        dec.rollback_to(pre + acc)
        ref.rollback_to(pre + acc)
        dec.observe(commits[acc:])
        ref.observe(commits[acc:])
        assert dec.history() == ref.history and dec.kv_len() == ref.cache_len
    assert np.abs(dec.next_logits() - ref.next_logits()).max() <= TOL
    # a pending token ahead of observe_returning_last_hidden
    dec.observe([7, 8])
    ref.observe([7, 8])
    h = dec.observe_returning_last_hidden([9])
    n = len(ref.history)
    rh, _ = ref.m.forward([9], [n], [n], n, [1])
    ref.observe([9])
    assert np.abs(h - rh[-1]).max() <= TOL
    assert dec.history() == ref.history and dec.kv_len() == ref.cache_len
    assert np.abs(dec.next_logits() - ref.next_logits()).max() <= TOL


def test_apply_lm_head_topk(pkg, accept, tiny_gguf):
    """Device top-k after the LM head == medusa.rs top_k_indices over the
    same logits rows (ids and values), > 64 rows (chunked), all-tie rows."""
    dec = pkg.B200Decoder.from_gguf(tiny_gguf("llama_q4km"), max_ctx=128)
    rng = np.random.default_rng(31)
    hid = rng.standard_normal((70, dec.hidden_size())).astype(np.float32)
    hid[3] = 0.0  # every logit equal: ties resolve by ascending index
    full = dec.apply_lm_head(hid)
    for k in (1, 10, 64):
        ids, vals = dec.apply_lm_head_topk(hid, k)
        assert ids.shape == (70, k)
        for r in range(70):
            want = accept.top_k_indices(full[r], k)
            assert ids[r].tolist() == want, (k, r)
            assert np.array_equal(vals[r], full[r][want])
    assert dec.apply_lm_head_topk(hid[3:4], 5)[0].tolist() == [[0, 1, 2, 3, 4]]
    with pytest.raises(pkg.SamplingError):
        dec.apply_lm_head_topk(hid[:1], 65)


@pytest.mark.parametrize("name", MODELS)
def test_fused_attention_matches_attention_kernels(pkg, tiny_gguf, name, monkeypatch):
    """Attention as its own kernels (the default) and as ops of the forward
    kernel (SPEC_B200_FUSED_ATTN, read at load) run the same arithmetic
    (attn_core.cuh): logits must agree bit for bit, at M = 5 / 13 / 40 rows
    (three forward-kernel instantiations) over a multi-split KV."""
    path = tiny_gguf(name)
    sep = pkg.B200Decoder.from_gguf(path, max_ctx=512)
    monkeypatch.setenv("SPEC_B200_FUSED_ATTN", "1")
    fused = pkg.B200Decoder.from_gguf(path, max_ctx=512)
    monkeypatch.delenv("SPEC_B200_FUSED_ATTN")
    v = fused.vocab_size()
    prompt = _prompt(v, 300, 11)  # several 128-key splits; chunked observes
    for d in (fused, sep):
        d.observe(prompt)
    assert np.array_equal(fused.next_logits(), sep.next_logits())
    for k in (4, 12):
        drafts = _prompt(v, k, 12 + k)
        a, b = fused.batched_logits(drafts), sep.batched_logits(drafts)
        assert np.array_equal(a, b), (k, float(np.abs(a - b).max()))
        fused.rollback_to(len(prompt))
        sep.rollback_to(len(prompt))
    rng = np.random.default_rng(5)
    edges = [(0, prompt[-1])] + [(int(rng.integers(0, i)), int(rng.integers(0, v))) for i in range(1, 40)]
    tree = pkg.DraftTree.from_parent_table(edges)
    a, b = fused.tree_logits(tree), sep.tree_logits(tree)
    assert np.array_equal(a, b), float(np.abs(a - b).max())
    assert fused.kernels_per_forward(5) < sep.kernels_per_forward(5)
    fused.close()
    sep.close()


def test_batched_logits_into_pinned_buffer(pkg, tiny_gguf):
    """Logits rows DMA'd into a page-locked caller array equal the rows copied
    through the library's staging buffer, bit for bit; a wrongly shaped
    array is refused before the call."""
    torch = pytest.importorskip("torch")
    dec = pkg.B200Decoder.from_gguf(tiny_gguf("llama_q4km"), max_ctx=256)
    V = dec.vocab_size()
    prompt = _prompt(V, 20, 3)
    dec.observe(prompt)
    drafts = [5, 6, 7, 8]
    a = dec.batched_logits(drafts)
    dec.rollback_to(len(prompt))
    buf = torch.empty((5, V), dtype=torch.float32, pin_memory=True).numpy()
    b = dec.batched_logits(drafts, out=buf)
    assert b is buf and np.array_equal(a.view(np.uint32), buf.view(np.uint32))
    dec.rollback_to(len(prompt))
    with pytest.raises(ValueError):
        dec.batched_logits(drafts, out=np.empty((4, V), dtype=np.float32))
    assert dec.history() == prompt
    tree = pkg.DraftTree([prompt[-1], 5, 6, 7, 8, 9], [0, 0, 0, 1, 1, 2])
    t0 = dec.tree_logits(tree)
    tbuf = torch.empty((6, V), dtype=torch.float32, pin_memory=True).numpy()
    t1 = dec.tree_logits(tree, out=tbuf)
    assert t1 is tbuf and np.array_equal(t0.view(np.uint32), tbuf.view(np.uint32))
    dec.close()
