"""The oracle's GGUF decode against gguf 0.19.0 golden vectors (CPU)."""

import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
TYPES = {"Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "Q8_0": 8}


@pytest.mark.parametrize("name", list(TYPES))
def test_dequant_matches_gguf_golden(oracle, name):
    d = np.load(os.path.join(HERE, "golden", "dequant_gguf019.npz"))
    blocks, expect = d[f"{name}_blocks"], d[f"{name}_expect"]
    got = oracle.dequant(TYPES[name], blocks, expect.size)
    assert np.array_equal(got.view(np.uint32), expect.view(np.uint32))


@pytest.mark.parametrize("name", list(TYPES))
def test_quantizer_roundtrip_error(synth, oracle, name):
    rng = np.random.default_rng(5)
    w = rng.standard_normal((8, 1024), dtype=np.float32) * np.float32(0.02)
    raw = synth.quantize(w, TYPES[name])
    back = oracle.dequant(TYPES[name], raw, w.size).reshape(w.shape)
    rel = np.sqrt(np.mean((back - w) ** 2)) / 0.02
    assert rel < {"Q4_K": 0.12, "Q5_K": 0.06, "Q6_K": 0.03, "Q8_0": 0.01}[name]


def test_quantizer_matches_gguf_py_decode(synth):
    gguf = pytest.importorskip("gguf")
    from gguf import quants
    rng = np.random.default_rng(9)
    w = rng.standard_normal((4, 512), dtype=np.float32)
    for name, t in TYPES.items():
        raw = synth.quantize(w, t)
        ref = quants.dequantize(raw, gguf.GGMLQuantizationType(t))
        assert np.abs(np.asarray(ref) - w).max() < 0.5, name


@pytest.mark.parametrize("name", list(TYPES))
def test_oracle_qmatmul_matches_dense(oracle, synth, name):
    rng = np.random.default_rng(3)
    w = rng.standard_normal((64, 512), dtype=np.float32) * np.float32(0.02)
    raw = synth.quantize(w, TYPES[name])
    x = rng.standard_normal((5, 512), dtype=np.float32)
    deq = oracle.dequant(TYPES[name], raw, w.size).reshape(w.shape).astype(np.float64)
    y = oracle.qmatmul(TYPES[name], raw, 64, 512, x)
    assert np.allclose(y, x.astype(np.float64) @ deq.T, atol=1e-5, rtol=1e-5)


def test_oracle_c_attention_matches_float64_model(oracle):
    """oq_attention (the C attention the CPU baseline times) against the
    float64 attention of oracle/model.py's forward: causal bias over the new
    rows, prefix keys visible, GQA head sharing."""
    rng = np.random.default_rng(9)
    nh, nkv, M, T, hd = 8, 2, 5, 70, 64
    q = rng.standard_normal((nh, M, hd)).astype(np.float32)
    k = rng.standard_normal((nkv, T, hd)).astype(np.float32)
    v = rng.standard_normal((nkv, T, hd)).astype(np.float32)
    got = oracle.attention(q, k, v, threads=2)
    G = nh // nkv
    vis = np.zeros((M, T), dtype=bool)
    vis[:, :T - M] = True
    vis[:, T - M:] = np.tril(np.ones((M, M), dtype=bool))
    want = np.empty((M, nh, hd))
    for h in range(nh):
        sc = q[h].astype(np.float64) @ k[h // G].astype(np.float64).T / np.sqrt(hd)
        sc = np.where(vis, sc, -np.inf)
        p = np.exp(sc - sc.max(axis=-1, keepdims=True))
        p /= p.sum(axis=-1, keepdims=True)
        want[:, h] = p @ v[h // G]
    assert np.abs(got - want.reshape(M, -1)).max() <= 1e-5
