"""Parity at the benchmarked shapes (GPU): the code paths that produce bench.py's numbers.

* Dequant-matmul at the Llama-3-8B matrix shapes (14336 x 4096 gate/up,
  4096 x 14336 down, 128256 x 4096 LM head) in Q4_K and Q6_K at
  M in {1, 5, 8, 16, 64}, on weights from the device generator the benchmark
  uses (spec_synthetic_tensor), against the oracle's block-direct C matmul
  (oracle/quants.c, double accumulation).  These shapes run the default
  stream-K cut (one chunk per resident CTA) with split-K groups.
  Bounds: |dy| <= 2e-4 * max|y| against activations rounded to f16 (the
  kernel's operand type); <= 2e-2 absolute against raw f32 activations (the
  north-star bound); rows bit-identical for every M (M-invariance).
* A 2-layer model with exactly the Llama-3-8B layer shapes (hidden 4096,
  32 / 8 heads of 128, FFN 14336, vocabulary 128256, Q4_K_M), created on the
  device by spec_create_synthetic exactly as the benchmark creates its
  32-layer target, exported to GGUF with the same generator
  (write_device_synthetic_gguf) and loaded by the oracle.  A 2048-token
  prefill, then a k=4 verify (5 rows over 2053 keys: 128-key attention
  splits): logits max-abs <= 2e-2, history and KV length exact, device greedy
  decisions equal the oracle's argmax wherever its top-2 margin is >= 2e-2.
  The same GGUF loaded through spec_load_gguf gives bit-identical logits.
* A 1-layer model with the Qwen2.5-7B layer shapes (hidden 3584, 28 / 4 heads,
  FFN 18944; vocabulary cut to 4096) in Q5_K with a 9300-token cache, so the
  attention runs 256-key splits (caches above 8192 tokens), after a
  9000-token prefill: k=8 verify logits within 2e-2 of the oracle.
"""

import importlib
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-2
STRICT = 2e-4


def _device_blocks(synth, fmt, n, k, seed):
    lib = importlib.import_module("abyo-speculate_b200._lib")
    L = lib.load()
    nbytes = n * (k // synth.BLOCK_ELEMS[fmt]) * synth.BLOCK_BYTES[fmt]
    buf = np.empty(nbytes, dtype=np.uint8)
    lib.check(L.spec_synthetic_tensor(0, fmt, n, k, seed, 0.02, buf.ctypes.data, nbytes))
    return buf.reshape(n, -1)


@pytest.mark.parametrize("fmt", [12, 14], ids=["Q4_K", "Q6_K"])
@pytest.mark.parametrize("n,k", [(14336, 4096), (4096, 14336), (128256, 4096)])
def test_qmatmul_bench_shapes(pkg, synth, oracle, fmt, n, k):
    import torch
    raw = _device_blocks(synth, fmt, n, k, seed=int(fmt) * 1000 + n + k)
    # The device generator's blocks are valid GGUF blocks of N(0, 0.02) values.
    sample = oracle.dequant(fmt, raw[:256], 256 * k)
    assert np.isfinite(sample).all()
    assert abs(float(sample.mean())) < 1e-3 and 0.018 < float(sample.std()) < 0.022
    qw = pkg.QWeight(fmt, raw, n, k)
    rng = np.random.default_rng(n + k + fmt)
    x64 = rng.standard_normal((64, k), dtype=np.float32)
    rows = {}
    for m in (1, 5, 8, 16, 64):
        x = torch.from_numpy(np.ascontiguousarray(x64[:m])).cuda()
        y = torch.empty((m, n), dtype=torch.float32, device="cuda")
        qw.matmul(x.data_ptr(), m, y.data_ptr())
        torch.cuda.synchronize()
        rows[m] = y.cpu().numpy()
    want16 = oracle.qmatmul(fmt, raw, n, k, x64.astype(np.float16).astype(np.float32), acc_double=True)
    want32 = oracle.qmatmul(fmt, raw, n, k, x64, acc_double=True)
    scale = float(np.abs(want16).max())
    for m, y in rows.items():
        assert np.abs(y - want16[:m]).max() <= STRICT * scale, f"M={m} vs oracle (f16 operand)"
        assert np.abs(y - want32[:m]).max() <= TOL, f"M={m} vs oracle (f32 activations)"
        # M-invariance: row r is the same bits whatever the row count.
        assert np.array_equal(y.view(np.uint32), rows[64][:m].view(np.uint32)), f"M={m} rows differ from M=64"
    qw.close()


LLAMA8B = dict(arch="llama", n_layers=2, hidden=4096, n_heads=32, n_kv_heads=8, ffn=14336, vocab=128256,
               rope_theta=5e5, eps=1e-5)
SEED = 1234


@pytest.fixture(scope="module")
def llama8b(pkg, synth, oracle, tmp_path_factory):
    path = os.path.join(str(tmp_path_factory.mktemp("bench_shapes")), "llama8b_2l.gguf")
    spec = synth.ModelSpec(ctx_len=8192, quant_mix="Q4_K_M", **LLAMA8B)
    synth.write_device_synthetic_gguf(path, spec, SEED)
    dec = pkg.B200Decoder.synthetic(**LLAMA8B, quant_mix="Q4_K_M", seed=SEED, max_ctx=4096)
    ref = oracle.OracleDecoder(oracle.OracleModel(path, max_ctx=2112))
    yield dec, ref, path
    dec.close()


def test_llama8b_shapes_prefill_and_verify(pkg, oracle, llama8b):
    dec, ref, path = llama8b
    rng = np.random.default_rng(7)
    V = LLAMA8B["vocab"]
    prompt = rng.integers(0, V, size=2048).tolist()
    dec.observe(prompt)
    ref.observe(prompt)
    assert np.abs(dec.next_logits() - ref.next_logits()).max() <= TOL
    drafts = rng.integers(0, V, size=4).tolist()
    got = dec.batched_logits(drafts)
    want = ref.batched_logits(drafts)
    assert got.shape == (5, V)
    assert np.abs(got - want).max() <= TOL
    assert dec.history() == ref.history and dec.kv_len() == ref.cache_len
    # Device greedy verify (device argmax over the same 5 rows): decisions
    # equal the oracle's wherever the oracle's top-2 margin is clear.
    dec.rollback_to(2048)
    ref.rollback_to(2048)
    n_acc, nxt, am = dec.verify_greedy(drafts)
    top2 = np.sort(want, axis=1)[:, -2:]
    for r in range(5):
        if top2[r, 1] - top2[r, 0] >= TOL:
            assert int(am[r]) == int(np.argmax(want[r])), f"row {r}"
    assert int(am[0]) == int(np.argmax(got[0]))
    # The exported GGUF through the file loader runs bit-identically.
    dec.rollback_to(2048)
    other = pkg.B200Decoder.from_gguf(path, max_ctx=4096)
    other.observe(prompt)
    again = other.batched_logits(drafts)
    dec.rollback_to(2048)
    mine = dec.batched_logits(drafts)
    assert np.array_equal(again.view(np.uint32), mine.view(np.uint32))
    other.close()


def test_llama8b_vocab_typical_tree(pkg, accept, llama8b):
    """Medusa typical acceptance (spec_verify_tree_typical) over 128256-wide
    node rows of the Llama-3-8B-shaped model: the device's softmax and
    entropy (33 sequential chunks per row) decide every node as the
    restated rule does on the same rows."""
    dec, _, _ = llama8b
    V = LLAMA8B["vocab"]
    rng = np.random.default_rng(13)
    dec.reset()
    prompt = rng.integers(0, V, size=64).tolist()
    dec.observe(prompt)
    tokens, parents = [prompt[-1]], [0]
    rows, _ = dec.tree_logits_keep_kv(pkg.DraftTree(tokens, parents))
    for t in np.argsort(-rows[0], kind="stable")[:3].tolist() + [int(rng.integers(0, V))]:
        tokens.append(int(t))
        parents.append(0)
    rows, _ = dec.tree_logits_keep_kv(pkg.DraftTree(tokens, parents))
    for f in range(1, 5):
        for t in np.argsort(-rows[f], kind="stable")[:2].tolist():
            tokens.append(int(t))
            parents.append(f)
    tree = pkg.DraftTree(tokens, parents)
    rows, _ = dec.tree_logits_keep_kv(tree)
    for eps, delta in [(0.0, 1.0), (1e-5, 0.5), (1e-3, 3.0), (0.5, 0.5)]:
        want = accept.typical_tree_accept(tokens, parents, rows, eps, delta)
        assert dec.verify_tree_typical(tree, eps, delta) == want, (eps, delta)
    dec.reset()


def test_llama8b_shapes_tree_over_max_rows(pkg, oracle, llama8b):
    """A 121-node tree (4 levels of 3: Medusa's 4 heads x top-3) over the
    Llama-3-8B-shaped model, 128256-wide rows: ancestor-closed chunks of at
    most 64 rows against the oracle's single tree forward, then a kept-KV
    forward, the greedy verify and the commit of its path (next logits after
    the bonus against the oracle)."""
    dec, ref, _ = llama8b
    V = LLAMA8B["vocab"]
    rng = np.random.default_rng(17)
    dec.reset()
    ref.reset()
    prompt = rng.integers(0, V, size=96).tolist()
    dec.observe(prompt)
    ref.observe(prompt)
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
    tree = pkg.DraftTree(tokens, parents)
    a = dec.tree_logits(tree)
    b = ref.tree_logits(tokens, parents)
    assert np.abs(a - b).max() <= TOL
    assert dec.history() == ref.history and dec.kv_len() == ref.cache_len
    best, bonus = dec.verify_tree_greedy(tree)
    ref.tree_logits_keep_kv(tokens, parents)
    dec.commit_tree_path(tree, best)
    ref.commit_tree_path(tokens, parents, best)
    assert dec.history() == ref.history and dec.kv_len() == ref.cache_len
    dec.observe([int(bonus)])
    ref.observe([int(bonus)])
    assert np.abs(dec.next_logits() - ref.next_logits()).max() <= TOL
    dec.reset()
    ref.reset()


QWEN7B_1L = dict(arch="qwen2", n_layers=1, hidden=3584, n_heads=28, n_kv_heads=4, ffn=18944, vocab=4096,
                 rope_theta=1e6, eps=1e-6)


def test_qwen7b_shapes_long_context_256_key_splits(pkg, synth, oracle, tmp_path):
    path = os.path.join(str(tmp_path), "qwen7b_1l.gguf")
    spec = synth.ModelSpec(ctx_len=32768, quant_mix="Q5_K", **QWEN7B_1L)
    synth.write_device_synthetic_gguf(path, spec, 99)
    dec = pkg.B200Decoder.synthetic(**QWEN7B_1L, quant_mix="Q5_K", seed=99, max_ctx=9300)
    assert dec.max_ctx() > 8192  # attention uses 256-key splits above 8192 tokens
    ref = oracle.OracleDecoder(oracle.OracleModel(path, max_ctx=9300))
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, QWEN7B_1L["vocab"], size=9000).tolist()
    for i in range(0, 9000, 1000):
        dec.observe(prompt[i:i + 1000])
        ref.observe(prompt[i:i + 1000])
    drafts = rng.integers(0, QWEN7B_1L["vocab"], size=8).tolist()
    got = dec.batched_logits(drafts)
    want = ref.batched_logits(drafts)
    assert np.abs(got - want).max() <= TOL
    assert dec.history() == ref.history and dec.kv_len() == ref.cache_len
    dec.close()


def test_shallow_same_seed_model_shares_tensors(synth):
    """spec_create_synthetic numbers the output norm, embedding and head first,
    so a 2-layer model with the target's seed shares them and layers 0-1
    exactly (the bench's shared-prefix draft); damped layers draw o / down at
    sigma 0.02 x damp."""
    spec4 = synth.ModelSpec("llama", 4, 256, 4, 2, 512, 1024, 5e5, 2048, 1e-5, "Q4_K_M")
    spec2 = synth.ModelSpec("llama", 2, 256, 4, 2, 512, 1024, 5e5, 2048, 1e-5, "Q4_K_M")
    t4 = synth.device_synthetic_tensors(spec4, 77, damp_from_layer=2, damp=0.05)
    t2 = synth.device_synthetic_tensors(spec2, 77)
    assert set(t2) <= set(t4)
    for name, (data, qt) in t2.items():
        assert qt == t4[name][1] and np.array_equal(np.asarray(data), np.asarray(t4[name][0])), name
    import importlib
    om = importlib.import_module("oracle.model")
    for layer, want in ((1, 0.02), (2, 0.001), (3, 0.001)):
        raw, qt = t4[f"blk.{layer}.attn_output.weight"]
        w = om.dequant(qt, raw, 256 * 256)
        assert abs(float(w.std()) - want) < 0.15 * want, (layer, float(w.std()))
