"""How far the modelled f32::exp is from the one the reference actually calls.

The device rejection round and the oracle model Rust's ``f32::exp`` as the
correctly rounded exp of the f32 argument.  Rust on Linux calls the platform
libm's ``expf``; glibc's is documented within 0.502 ulp, so it differs from
the correctly rounded value on a small fraction of arguments.  These tests
measure that fraction on the softmax's argument range, and then whether it
changes any decision of the temperature > 0 vanilla round
(methods/vanilla.rs:59-106, sampling/tokens.rs:15-55, :99-120) when the
host libm's expf replaces the model everywhere (target softmax, draft
distributions, adjusted distribution, sampling).
"""

import ctypes
import ctypes.util

import numpy as np
import pytest


def _libm_expf():
    name = ctypes.util.find_library("m") or "libm.so.6"
    try:
        lib = ctypes.CDLL(name)
    except OSError:
        pytest.skip("no C math library to call")
    f = lib.expf
    f.restype = ctypes.c_float
    f.argtypes = [ctypes.c_float]
    return f


def _vec(expf):
    def run(x):
        x = np.asarray(x, dtype=np.float32)
        return np.fromiter((expf(float(v)) for v in x.ravel()), dtype=np.float32, count=x.size).reshape(x.shape)
    return run


def test_libm_expf_against_the_correctly_rounded_model(accept):
    expf = _libm_expf()
    rng = np.random.default_rng(1)
    # (l - max) / t for logits within ~30 of the row maximum.
    x = (-rng.random(300_000) * 30.0).astype(np.float32)
    got = _vec(expf)(x)
    model = accept.exp_f32(x)
    exact = np.exp(x.astype(np.longdouble)).astype(np.float32)  # independent check of the model
    assert np.array_equal(model, exact)
    diff = got != model
    rate = float(diff.mean())
    ulps = np.abs(got.view(np.int32).astype(np.int64) - model.view(np.int32).astype(np.int64))
    print(f"libm expf differs from the correctly rounded exp on {int(diff.sum())} of {x.size} arguments "
          f"({rate:.3%}), by at most {int(ulps.max())} ulp")
    assert int(ulps.max()) <= 1
    assert rate < 2e-3


def test_vanilla_round_decisions_with_libm_expf(accept, monkeypatch):
    """300 seeded temperature > 0 rounds (V = 4096, k = 4) run twice: with the
    model exp and with the host libm's expf.  The committed tokens and the
    uniforms consumed are compared round by round."""
    expf = _vec(_libm_expf())
    rng = np.random.default_rng(7)
    V, k = 4096, 4
    rounds = []
    for i in range(300):
        t = float(rng.choice([0.7, 1.0, 1.3]))
        tgt = (rng.standard_normal((k + 1, V)) * 3.0).astype(np.float32)
        drf = (tgt[:k] + rng.standard_normal((k, V)).astype(np.float32) * 1.5).astype(np.float32)
        u = rng.random(2 * k + 2).astype(np.float32)
        rounds.append((t, tgt, drf, u))

    def play(exp_fn):
        monkeypatch.setattr(accept, "exp_f32", exp_fn)
        out = []
        for t, tgt, drf, u in rounds:
            q = [accept.softmax_with_temperature(r, t) for r in drf]
            # Draft samples from q with the first k uniforms (vanilla.rs:297-305).
            toks = [accept.sample_from_distribution(float(u[j]), q[j]) for j in range(k)]
            out.append(accept.vanilla_round(tgt, toks, q, t, [float(v) for v in u[k:]], 0, 1 << 30))
        return out

    model = play(accept.exp_f32)
    libm = play(expf)
    differ = sum(a != b for a, b in zip(model, libm))
    accepted = sum(len(c) - 1 for c, _ in model)
    print(f"{differ} of {len(rounds)} rounds differ between the exp model and libm expf "
          f"({accepted} drafts accepted in total)")
    assert differ == 0


def _libm_logf():
    name = ctypes.util.find_library("m") or "libm.so.6"
    try:
        lib = ctypes.CDLL(name)
    except OSError:
        pytest.skip("no C math library to call")
    f = lib.logf
    f.restype = ctypes.c_float
    f.argtypes = [ctypes.c_float]
    return f


def test_libm_logf_against_the_correctly_rounded_model(accept):
    """Typical acceptance (medusa.rs:424-445) takes ln of every probability;
    the oracle and the device model f32::ln as the correctly rounded log."""
    logf = _libm_logf()
    rng = np.random.default_rng(2)
    x = np.exp(-rng.random(300_000) * 25.0).astype(np.float32)  # probabilities in (e^-25, 1]
    got = _vec(logf)(x)
    model = accept.ln_f32(x)
    exact = np.log(x.astype(np.longdouble)).astype(np.float32)
    assert np.array_equal(model, exact)
    diff = got != model
    ulps = np.abs(got.view(np.int32).astype(np.int64) - model.view(np.int32).astype(np.int64))
    print(f"libm logf differs from the correctly rounded log on {int(diff.sum())} of {x.size} arguments "
          f"({float(diff.mean()):.3%}), by at most {int(ulps.max())} ulp")
    assert int(ulps.max()) <= 1
    assert float(diff.mean()) < 2e-3


def test_typical_decisions_with_libm(accept, monkeypatch):
    """200 seeded typical-acceptance trees (V = 4096, 15 nodes) decided with
    the exp/ln models and again with the host libm's expf and logf: the
    accepted paths and bonus tokens are compared tree by tree."""
    expf, logf = _vec(_libm_expf()), _vec(_libm_logf())
    rng = np.random.default_rng(11)
    V, n = 4096, 15
    parents = [0] + [(i - 1) // 2 for i in range(1, n)]
    cases = []
    for _ in range(200):
        rows = (rng.standard_normal((n, V)) * rng.choice([1.0, 3.0, 6.0])).astype(np.float32)
        toks = [0] + [int(np.argsort(rows[parents[i]])[-1 - int(rng.integers(0, 3))]) for i in range(1, n)]
        eps, delta = float(rng.choice([0.01, 0.05, 0.1])), float(rng.choice([0.1, 0.3, 0.6]))
        cases.append((toks, rows, eps, delta))

    def play(exp_fn, ln_fn):
        monkeypatch.setattr(accept, "exp_f32", exp_fn)
        monkeypatch.setattr(accept, "ln_f32", ln_fn)
        return [accept.typical_tree_accept(t, parents, r, e, d) for t, r, e, d in cases]

    model = play(accept.exp_f32, accept.ln_f32)
    libm = play(expf, logf)
    differ = sum(a != b for a, b in zip(model, libm))
    accepted = sum(len(b) - 1 for b, _ in model)
    print(f"{differ} of {len(cases)} typical trees differ between the models and libm "
          f"({accepted} nodes accepted in total)")
    assert accepted > 0
    assert differ == 0
