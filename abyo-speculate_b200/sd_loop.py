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
