"""The Medusa head restatement (oracle/medusa.py) on the CPU: a residual block
with zero weights and bias is the identity (x + SiLU(0) = x), so the head
reduces to its output projection; top-k follows top_k_indices' order."""

import importlib

import numpy as np


def test_zero_residual_block_is_identity():
    mo = importlib.import_module("oracle.medusa")
    eo = importlib.import_module("oracle.eagle")
    rng = np.random.default_rng(3)
    H, V = 8, 16
    wo = eo.bf16_bits(rng.standard_normal((V, H)).astype(np.float32))
    zero = eo.bf16_bits(np.zeros((H, H), np.float32))
    hidden = eo.bf16_round(rng.standard_normal(H).astype(np.float32))
    ref = mo.MedusaOracle([[zero, zero]], [[np.zeros(H, np.float32)] * 2], [wo])
    rows = ref.forward(hidden)
    expect = eo.bits_to_f32(wo).astype(np.float64) @ hidden.astype(np.float64)
    assert np.allclose(rows[0], expect, rtol=0, atol=1e-12)
    ids, _ = ref.top_k_per_head(hidden, 4)
    assert ids[0] == list(np.argsort(-expect, kind="stable")[:4])


def test_residual_block_adds_silu():
    mo = importlib.import_module("oracle.medusa")
    eo = importlib.import_module("oracle.eagle")
    H = 4
    eye = eo.bf16_bits(np.eye(H, dtype=np.float32))
    b = np.array([0.5, -1.0, 2.0, 0.0], np.float32)
    x = np.array([1.0, 2.0, -3.0, 0.25], np.float32)
    ref = mo.MedusaOracle([[eye]], [[b]], [eye])
    y = x.astype(np.float64) + b
    # the output projection's input is rounded to BF16, as the device's is
    out = eo.bf16_round((x + y / (1 + np.exp(-y))).astype(np.float32))
    assert np.allclose(ref.forward(x)[0], out, rtol=0, atol=1e-12)
