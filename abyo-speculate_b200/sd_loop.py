"""Greedy vanilla speculative-decoding rounds over two B200Decoder handles.

A measurement and test harness, not an engine: it issues the trait calls of
one vanilla SD round in the reference's order (methods/vanilla.rs:285-369 at
temperature 0), with the device-side greedy calls in place of host softmax
and argmax:

  draft:  k x (greedy next token, observe it)           vanilla.rs:297-305
  target: verify [last] + drafts, accept walk           vanilla.rs:308-343
  both:   rollback to the accepted prefix, observe the
          token that follows it                         vanilla.rs:358-362

With lazy observe the post-round observes cost no forward; the next round's
draft step and verify compute the pending token's KV row.  The same round is
also one native call (spec_sd_greedy_round), the default in
vanilla_greedy_generate.
"""

from __future__ import annotations

from typing import List, Sequence, Tuple


def greedy_next(dec) -> int:
    """The argmax of the next-token row, computed on the device (a verify of
    zero drafts: one forward of the pending token plus a device argmax)."""
    _, nxt, _ = dec.verify_greedy([])
    return int(nxt)


def vanilla_greedy_round_native(target, draft, k: int) -> List[int]:
    """The same round as one C call (spec_sd_greedy_round)."""
    import ctypes
    out = (ctypes.c_uint32 * (k + 1))()
    n = ctypes.c_int()
    target._check(target._lib.spec_sd_greedy_round(target._h, draft._h, k, out, ctypes.byref(n)))
    return [int(out[i]) for i in range(n.value)]


def vanilla_greedy_round(target, draft, k: int) -> List[int]:
    """One round; returns the committed tokens (accepted drafts + the next one)."""
    pre = target.history_len()
    drafts = []
    for _ in range(k):
        t = greedy_next(draft)
        drafts.append(t)
        draft.observe([t])
    n_acc, bonus, _ = target.verify_greedy(drafts)
    commits = drafts[:n_acc] + [int(bonus)]
    target.rollback_to(pre + n_acc)
    target.observe([int(bonus)])
    draft.rollback_to(pre + n_acc)
    draft.observe([int(bonus)])
    return commits


def vanilla_greedy_generate(target, draft, prompt: Sequence[int], n_new: int, k: int,
                            observe_prompt: bool = True, native: bool = True) -> Tuple[List[int], List[int]]:
    """Generates at least n_new tokens; returns (tokens, accepted drafts per round)."""
    if observe_prompt:
        target.reset()
        draft.reset()
        target.observe(list(prompt))
        draft.observe(list(prompt))
    out: List[int] = []
    accepted: List[int] = []
    while len(out) < n_new:
        c = (vanilla_greedy_round_native if native else vanilla_greedy_round)(target, draft, k)
        out.extend(c)
        accepted.append(len(c) - 1)
    return out, accepted


# ---------------------------------------------------------------------------
# Sampled rounds (temperature > 0) with the reference's seeded RNG stream.
# ---------------------------------------------------------------------------
def softmax_with_temperature(logits, temperature: float):
    """sampling/tokens.rs:15-55 for temperature > 0: exp((l - max) / t), summed
    sequentially in f32 (f32::exp taken as the correctly rounded exp, as the
    device round does)."""
    import numpy as np
    logits = np.asarray(logits, dtype=np.float32)
    inv_t = np.float32(1.0) / np.float32(temperature)
    finite = logits[~np.isnan(logits)]
    mx = np.float32(np.max(finite))
    out = np.exp(((logits - mx) * inv_t).astype(np.float64)).astype(np.float32)
    s = np.cumsum(out, dtype=np.float32)[-1]
    if not (s > 0) or not np.isfinite(s):
        raise ValueError(f"softmax produced non-positive sum: {s}")
    return (out / s).astype(np.float32)


def sample_from_distribution(u01: float, probs) -> int:
    """sampling/tokens.rs:99-120 with u01 = gen::<f32>(): u = u01 * sum, the
    first index whose running f32 sum exceeds u (the last index otherwise)."""
    import numpy as np
    acc = np.cumsum(np.asarray(probs, dtype=np.float32), dtype=np.float32)
    u = np.float32(u01) * acc[-1]
    idx = np.flatnonzero(u < acc)
    return int(idx[0]) if idx.size else int(acc.size - 1)


def vanilla_sampled_round(target, draft, k: int, temperature: float, rng, budget: int) -> Tuple[List[int], int]:
    """One vanilla SD round at temperature > 0 in the reference's order and
    RNG draw order (methods/vanilla.rs:285-369): k draft samples (one
    gen::<f32>() each, on the host from the draft's logits), then the
    target's batched verify and the rejection walk on the device
    (spec_verify_rejection: one draw per verified position, then one for the
    resample or the bonus), then both decoders re-anchored to the commits.
    `rng` is an abyo-speculate_b200.rng.StdRng; `budget` = tokens still
    allowed (max_new_tokens - generated).

    Re-anchoring follows the reference exactly: both decoders are rolled back
    to pre + min(len(commits), k) and observe commits[min(len(commits), k):]
    (vanilla.rs:352-362).  After a rejection at position j that keeps the
    rejected draft j in both histories (the resampled token is emitted but not
    observed), which is what the reference does; the seeded token stream is
    only comparable with it that way.

    Returns (committed tokens, drafts accepted)."""
    import numpy as np
    k = min(k, budget)
    pre_t, pre_d = target.history_len(), draft.history_len()
    drafts, dists = [], []
    for _ in range(k):
        probs = softmax_with_temperature(draft.next_logits(), temperature)
        tok = sample_from_distribution(rng.gen_f32(), probs)
        drafts.append(tok)
        dists.append(probs)
        draft.observe([tok])
    q = np.stack(dists) if dists else np.zeros((0, target.vocab_size()), dtype=np.float32)
    commits, used = target.verify_rejection(drafts, q, temperature, rng.peek_f32(k + 1), budget)
    rng.advance(used)
    # Drafts accepted: a rejection or the bonus adds one commit beyond them;
    # a budget cut-off does not (then every draw was an accept test).
    n_acc = len(commits) if (used == len(commits) and len(commits) <= k) else len(commits) - 1
    acc = min(len(commits), k)
    target.rollback_to(pre_t + acc)
    target.observe(commits[acc:])
    draft.rollback_to(pre_d + acc)
    draft.observe(commits[acc:])
    return commits, n_acc


class NativeRng:
    """The same seeded stream held by the library (spec_rng): what
    spec_sd_sampled_round draws from."""

    def __init__(self, seed: int):
        import ctypes
        from . import _lib
        self._lib = _lib.load()
        h = ctypes.c_void_p()
        _lib.check(self._lib.spec_rng_create(ctypes.c_uint64(seed & 0xFFFFFFFFFFFFFFFF), ctypes.byref(h)), None)
        self.h = h

    def next_f32(self, n: int):
        import numpy as np
        out = np.zeros(n, dtype=np.float32)
        from . import _lib
        _lib.check(self._lib.spec_rng_next_f32(self.h, out.ctypes.data_as(_lib.c_f32_p), n), None)
        return out

    def close(self) -> None:
        if self.h:
            self._lib.spec_rng_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def vanilla_sampled_round_native(target, draft, k: int, temperature: float, rng: NativeRng,
                                 budget: int) -> Tuple[List[int], int]:
    """The same round as one C call (spec_sd_sampled_round): draft sampling
    and both distributions stay on the device."""
    import ctypes
    out = (ctypes.c_uint32 * (k + 1))()
    n, n_acc = ctypes.c_int(), ctypes.c_int()
    target._check(target._lib.spec_sd_sampled_round(target._h, draft._h, k, ctypes.c_float(temperature), rng.h,
                                                     budget, out, ctypes.byref(n), ctypes.byref(n_acc)))
    return [int(out[i]) for i in range(n.value)], int(n_acc.value)


def vanilla_sampled_generate(target, draft, prompt: Sequence[int], n_new: int, k: int, temperature: float,
                             seed: int, native: bool = False) -> Tuple[List[int], List[int]]:
    """run_vanilla_sd at temperature > 0 with StdRng::seed_from_u64(seed)
    (engine.rs:320-326); returns (tokens, accepted drafts per round).
    native: each round is one spec_sd_sampled_round call."""
    from .rng import StdRng
    rng = NativeRng(seed) if native else StdRng(seed)
    target.reset()
    draft.reset()
    target.observe(list(prompt))
    draft.observe(list(prompt))
    out: List[int] = []
    accepted: List[int] = []
    while len(out) < n_new:
        budget = n_new - len(out)
        kk = min(k, budget)
        rnd = vanilla_sampled_round_native if native else vanilla_sampled_round
        c, n_acc = rnd(target, draft, kk, temperature, rng, budget)
        out.extend(c)
        accepted.append(n_acc)
    return out, accepted
