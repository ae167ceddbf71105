"""Greedy vanilla SD rounds through the backend (GPU).

Greedy speculative decoding is lossless: whatever the draft proposes, the
committed stream must equal the target's own greedy decoding token for token
(methods/vanilla.rs:312-343 at temperature 0).  With the target as its own
draft every round accepts all k drafts.  Both checks run the reference's round
protocol (verify, rollback, observe) over lazy observes."""

import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _greedy_plain(pkg, accept, path, prompt, n):
    dec = pkg.B200Decoder.from_gguf(path, max_ctx=512)
    dec.observe(prompt)
    out = []
    for _ in range(n):
        t = accept.argmax_first(dec.next_logits())
        out.append(t)
        dec.observe([t])
    return out


@pytest.mark.parametrize("k,native", [(1, True), (4, True), (4, False)])
def test_sd_stream_equals_target_greedy(pkg, accept, tiny_gguf, k, native):
    sd = importlib.import_module("abyo-speculate_b200.sd_loop")
    tpath, dpath = tiny_gguf("llama_q4km"), tiny_gguf("llama_hd128")
    prompt = np.random.default_rng(41).integers(0, 1024, size=24).tolist()
    target = pkg.B200Decoder.from_gguf(tpath, max_ctx=512)
    draft = pkg.B200Decoder.from_gguf(dpath, max_ctx=512)
    toks, acc = sd.vanilla_greedy_generate(target, draft, prompt, 40, k, native=native)
    ref = _greedy_plain(pkg, accept, tpath, prompt, len(toks))
    assert toks == ref
    assert target.history() == prompt + toks and draft.history() == prompt + toks
    assert target.kv_len() == len(prompt) + len(toks)


def test_self_draft_accepts_everything(pkg, accept, tiny_gguf):
    sd = importlib.import_module("abyo-speculate_b200.sd_loop")
    path = tiny_gguf("qwen_q4km")
    prompt = np.random.default_rng(42).integers(0, 1024, size=16).tolist()
    target = pkg.B200Decoder.from_gguf(path, max_ctx=512)
    draft = pkg.B200Decoder.from_gguf(path, max_ctx=512)
    toks, acc = sd.vanilla_greedy_generate(target, draft, prompt, 30, 4)
    assert all(a == 4 for a in acc)
    assert toks == _greedy_plain(pkg, accept, path, prompt, len(toks))


def test_sampled_stream_replays_with_stdrng(pkg, accept, tiny_gguf):
    """Temperature-1.0 vanilla SD seeded like StdRng::seed_from_u64(7)
    (engine.rs:320-326): the device rounds (spec_verify_rejection fed from the
    restated ChaCha12 stream in the reference's draw order) produce the same
    token stream and acceptance counts as a host replay of vanilla.rs:285-369
    with the oracle's acceptance functions on the same decoders' logits rows
    and the same stream."""
    sd = importlib.import_module("abyo-speculate_b200.sd_loop")
    rng_mod = importlib.import_module("abyo-speculate_b200.rng")
    tpath, dpath = tiny_gguf("llama_q4km"), tiny_gguf("llama_hd128")
    prompt = np.random.default_rng(43).integers(0, 1024, size=20).tolist()
    T, k, n_new = 1.0, 4, 40
    target = pkg.B200Decoder.from_gguf(tpath, max_ctx=512)
    draft = pkg.B200Decoder.from_gguf(dpath, max_ctx=512)
    toks, accs = sd.vanilla_sampled_generate(target, draft, prompt, n_new, k, T, seed=7)
    assert len(toks) == n_new and sum(accs) > 0

    # Host replay: the same calls and draws, acceptance by the oracle.
    tr = pkg.B200Decoder.from_gguf(tpath, max_ctx=512)
    dr = pkg.B200Decoder.from_gguf(dpath, max_ctx=512)
    tr.observe(prompt)
    dr.observe(prompt)
    rng = rng_mod.StdRng(7)
    out, racc = [], []
    while len(out) < n_new:
        kk = min(k, n_new - len(out))
        pre_t, pre_d = tr.history_len(), dr.history_len()
        drafts, dists = [], []
        for _ in range(kk):
            probs = accept.softmax_with_temperature(dr.next_logits(), T)
            tok = accept.sample_from_distribution(rng.gen_f32(), probs)
            drafts.append(tok)
            dists.append(probs)
            dr.observe([tok])
        rows = tr.batched_logits(drafts)
        commits, used = accept.vanilla_round(rows, drafts, dists, T, list(rng.peek_f32(kk + 1)), len(out), n_new)
        rng.advance(used)
        racc.append(len(commits) if (used == len(commits) and len(commits) <= kk) else len(commits) - 1)
        a = min(len(commits), kk)
        tr.rollback_to(pre_t + a)
        tr.observe(commits[a:])
        dr.rollback_to(pre_d + a)
        dr.observe(commits[a:])
        out.extend(commits)
    assert toks == out
    assert accs == racc


@pytest.mark.parametrize("T", [1.0, 0.7])
def test_native_sampled_round_equals_host_orchestrated(pkg, tiny_gguf, T):
    """spec_sd_sampled_round (draft sampling and both distributions on the
    device, the stream in the library) commits the same tokens and accepts
    the same drafts as the same rounds orchestrated from Python (host
    softmax and sampling of the draft rows, spec_verify_rejection fed host
    distributions), seeded like StdRng::seed_from_u64(11)."""
    sd = importlib.import_module("abyo-speculate_b200.sd_loop")
    tpath, dpath = tiny_gguf("llama_q4km"), tiny_gguf("llama_hd128")
    prompt = np.random.default_rng(44).integers(0, 1024, size=18).tolist()
    k, n_new = 4, 40
    runs = []
    for native in (False, True):
        target = pkg.B200Decoder.from_gguf(tpath, max_ctx=512)
        draft = pkg.B200Decoder.from_gguf(dpath, max_ctx=512)
        toks, accs = sd.vanilla_sampled_generate(target, draft, prompt, n_new, k, T, seed=11, native=native)
        runs.append((toks, accs, target.history(), draft.history(), target.kv_len()))
    assert len(runs[0][0]) == n_new and sum(runs[0][1]) > 0
    assert runs[0] == runs[1]
