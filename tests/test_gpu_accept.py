"""Device rejection-sampling round (spec_verify_rejection) against the oracle (GPU).

Parity contract: given the same target logits rows (the device's own batched
rows, which are deterministic), the same draft distributions and the same
uniforms, the committed tokens and the number of uniforms consumed must equal
oracle.accept.vanilla_round exactly (vanilla.rs:172-210 with tokens.rs:14-120).
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _softmax32(x):
    x = np.asarray(x, dtype=np.float32)
    e = np.exp((x - x.max()).astype(np.float64)).astype(np.float32)
    return (e / np.cumsum(e, dtype=np.float32)[-1]).astype(np.float32)


def _round_case(dec, accept, rng, prompt, k, temperature, budget, greedy_frac):
    V = dec.vocab_size()
    dec.rollback_to(len(prompt))
    probe = rng.integers(0, V, size=k).astype(np.uint32)
    rows = np.asarray(dec.batched_logits(probe.tolist()), dtype=np.float32)
    dec.rollback_to(len(prompt))
    # Drafts: a mix of the target's own argmax chain (to get accepts) and
    # random tokens; draft distributions put extra mass on the drafted token.
    drafts = []
    for i in range(k):
        drafts.append(int(probe[i]) if rng.random() > greedy_frac else int(np.argmax(rows[i])))
    # Rows for the chosen drafts: recompute with the final draft list.
    rows = np.asarray(dec.batched_logits(drafts), dtype=np.float32)
    dec.rollback_to(len(prompt))
    q = np.stack([_softmax32(rng.standard_normal(V).astype(np.float32) * 2) for _ in range(k)]) if k else \
        np.zeros((0, V), np.float32)
    for i, t in enumerate(drafts):
        q[i, t] += np.float32(rng.random() * 0.5)
        q[i] = (q[i] / np.cumsum(q[i], dtype=np.float32)[-1]).astype(np.float32)
    u = rng.random(k + 1).astype(np.float32)
    got, used = dec.verify_rejection(drafts, q, temperature, u, budget=budget)
    want, want_used = accept.vanilla_round(rows, drafts, list(q), temperature, [float(x) for x in u], 0, budget)
    assert got == [int(x) for x in want], (temperature, budget, drafts)
    assert used == want_used
    assert dec.history()[-k:] == drafts if k else True
    return got


@pytest.mark.parametrize("name", ["llama_q4km", "qwen_q4km"])
def test_rejection_round_matches_oracle(pkg, accept, tiny_gguf, name):
    dec = pkg.B200Decoder.from_gguf(tiny_gguf(name), max_ctx=256)
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, dec.vocab_size(), size=12).tolist()
    dec.observe(prompt)
    outcomes = set()
    for trial in range(24):
        k = [1, 2, 4, 7][trial % 4]
        t = [0.0, 0.6, 1.0, 1.7][(trial // 4) % 4]
        budget = k + 1 if trial % 3 else max(1, k - 1)
        got = _round_case(dec, accept, rng, prompt, k, t, budget, greedy_frac=0.6)
        outcomes.add(len(got))
    assert len(outcomes) > 1  # both early rejections and longer accepts were exercised


def test_rejection_bonus_only_and_errors(pkg, accept, tiny_gguf):
    dec = pkg.B200Decoder.from_gguf(tiny_gguf("llama_q4km"), max_ctx=256)
    rng = np.random.default_rng(9)
    prompt = rng.integers(0, dec.vocab_size(), size=8).tolist()
    dec.observe(prompt)
    _round_case(dec, accept, rng, prompt, 0, 1.0, 1, greedy_frac=0.0)  # k = 0: one bonus sample
    hist = dec.history()
    with pytest.raises(pkg.SamplingError):
        dec.verify_rejection([1, 2], np.full((2, dec.vocab_size()), 1.0 / dec.vocab_size(), np.float32), -1.0,
                             [0.5, 0.5, 0.5])
    with pytest.raises(pkg.SamplingError):  # 2 drafts need up to 3 uniforms; give 1 and force a reject path
        dec.verify_rejection([1, 2], np.full((2, dec.vocab_size()), 1.0 / dec.vocab_size(), np.float32), 1.0,
                             [0.999])
    assert dec.history() == hist
