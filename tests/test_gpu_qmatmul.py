"""Dequant-matmul kernel parity (spec_qmatmul) against the oracle (GPU).

Tolerances: with the activations pre-rounded to the operand dtype (f16 for
GGUF formats, bf16 for BF16) the kernel and the oracle differ only in f32
summation order: |dy| <= 2e-4 * max|y|.  With raw f32 activations the
north-star bound applies: max-abs <= 2e-2.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FMTS = {"Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "Q8_0": 8, "BF16": 30}


def _run(pkg, fmt, raw, n, k, x_np):
    import torch
    w = pkg.QWeight(fmt, raw, n, k)
    x = torch.from_numpy(np.ascontiguousarray(x_np)).cuda()
    y = torch.empty((x_np.shape[0], n), dtype=torch.float32, device="cuda")
    w.matmul(x.data_ptr(), x_np.shape[0], y.data_ptr())
    torch.cuda.synchronize()
    return y.cpu().numpy(), w


def _round_operand(x, fmt):
    if fmt == 30:
        import importlib
        om = importlib.import_module("oracle.model")
        return om.bf16_round(x)
    return x.astype(np.float16).astype(np.float32)


@pytest.mark.parametrize("name", list(FMTS))
@pytest.mark.parametrize("m", [1, 5, 8, 9, 16, 33, 64])
def test_qmatmul_parity(pkg, synth, oracle, name, m):
    fmt = FMTS[name]
    rng = np.random.default_rng(100 + m)
    n, k = 256, 512
    w = rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
    raw = synth.quantize(w, fmt)
    raw_bytes = raw.view(np.uint8).reshape(n, -1)
    x = rng.standard_normal((m, k), dtype=np.float32)
    y, _ = _run(pkg, fmt, raw_bytes, n, k, x)
    deq = w.astype(np.float64) if fmt == 30 else oracle.dequant(fmt, raw_bytes, n * k).reshape(n, k).astype(np.float64)
    if fmt == 30:
        deq = oracle.bf16_round(w).astype(np.float64)
    ref_strict = _round_operand(x, fmt).astype(np.float64) @ deq.T
    ref = x.astype(np.float64) @ deq.T
    scale = np.abs(ref).max()
    assert np.abs(y - ref_strict).max() <= 2e-4 * scale + 1e-6
    assert np.abs(y - ref).max() <= 2e-2


@pytest.mark.parametrize("name", ["Q4_K", "Q6_K", "Q8_0"])
def test_qmatmul_split_k_and_m_invariance(pkg, synth, oracle, name):
    fmt = FMTS[name]
    rng = np.random.default_rng(7)
    n, k = 1024, 4096
    w = rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
    raw = synth.quantize(w, fmt).view(np.uint8).reshape(n, -1)
    x = rng.standard_normal((9, k), dtype=np.float32)
    y9, _ = _run(pkg, fmt, raw, n, k, x)
    deq = oracle.dequant(fmt, raw, n * k).reshape(n, k).astype(np.float64)
    ref = x.astype(np.float16).astype(np.float64) @ deq.T
    assert np.abs(y9 - ref).max() <= 2e-4 * np.abs(ref).max()
    # Row r's result does not depend on how many rows share the call.
    for m in (1, 5):
        ym, _ = _run(pkg, fmt, raw, n, k, x[:m])
        assert np.array_equal(ym.view(np.uint32), y9[:m].view(np.uint32))


def test_bf16_tcgen05_split_k_and_m_invariance(pkg, synth, oracle):
    """BF16 weights run on tcgen05 with a TMEM accumulator at every M (MMA N =
    16, 16, 32, 64 for 1-8, 9-16, 17-32 and 33-64 rows).  A split-K shape at
    M = 64 against the oracle, and rows bit-identical for every smaller M, so
    the accumulator's arithmetic does not depend on the MMA's N."""
    fmt = FMTS["BF16"]
    rng = np.random.default_rng(8)
    n, k = 1024, 4096
    w = rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
    raw = synth.quantize(w, fmt).view(np.uint8).reshape(n, -1)
    x = rng.standard_normal((64, k), dtype=np.float32)
    y64, _ = _run(pkg, fmt, raw, n, k, x)
    deq = oracle.bf16_round(w).astype(np.float64)
    ref = _round_operand(x, fmt).astype(np.float64) @ deq.T
    assert np.abs(y64 - ref).max() <= 2e-4 * np.abs(ref).max()
    for m in (1, 5, 9, 16, 33):
        ym, _ = _run(pkg, fmt, raw, n, k, x[:m])
        assert np.array_equal(ym.view(np.uint32), y64[:m].view(np.uint32)), f"M={m} rows differ from M=64"


def test_qmatmul_lm_head_shape(pkg, synth, oracle):
    """A vocabulary-sized Q6_K head (many 128-row groups, no split)."""
    rng = np.random.default_rng(11)
    n, k = 8192, 1024
    w = rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
    raw = synth.quantize(w, 14).view(np.uint8).reshape(n, -1)
    x = rng.standard_normal((5, k), dtype=np.float32)
    y, qw = _run(pkg, 14, raw, n, k, x)
    assert qw.nbytes() == raw.nbytes
    deq = oracle.dequant(14, raw, n * k).reshape(n, k).astype(np.float64)
    ref = x.astype(np.float16).astype(np.float64) @ deq.T
    assert np.abs(y - ref).max() <= 2e-4 * np.abs(ref).max()
