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
