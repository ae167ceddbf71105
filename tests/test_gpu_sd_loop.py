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
