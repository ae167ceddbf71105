"""spec_qmatmul_noalloc (the allocation-free matmul entry point) against spec_qmatmul and the oracle (GPU).

The no-allocation entry point is for callers that cannot allocate device
memory at call time (a runtime that has reserved nearly all HBM up front, a
loop that must not meet cudaFree's device-wide synchronisation, code inside
an allocator callback).  It runs the same kernel as spec_qmatmul with its
scratch in a static device array, so on the same inputs its output must agree
with spec_qmatmul's within |dy| <= 1e-5 * max|y| (in practice bit-identical),
and with the oracle (oracle/quants.c, double accumulation over the GGUF
blocks, activations rounded to the kernel's operand type) within
|dy| <= 2e-4 * max|y|, the bound of tests/test_gpu_qmatmul.py.
Each case makes two no-allocation calls in a row: the second one runs on
scratch the first one left behind (its split-K counters, partials, operand).
This file is named to be collected last, and must also pass on its own in a
fresh process.
"""

import ctypes
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-5          # against spec_qmatmul (same kernel)
ORACLE_TOL = 2e-4   # against the oracle, relative to max|y|


def _lib():
    return importlib.import_module("abyo-speculate_b200._lib")


def _raw(synth, fmt, n, k, seed):
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
    return synth.quantize(w, fmt).view(np.uint8).reshape(n, -1)


def _weight(pkg, synth, fmt, n, k, seed):
    return pkg.QWeight(fmt, _raw(synth, fmt, n, k, seed), n, k)


def _oracle_y(fmt, raw, n, k, x_np):
    """y = x . W^T by the oracle, with x rounded to the kernel's operand type."""
    om = importlib.import_module("oracle.model")
    xr = om.bf16_round(x_np) if fmt == 30 else x_np.astype(np.float16).astype(np.float32)
    return om.qmatmul(fmt, raw, n, k, xr, acc_double=True)


def _noalloc(qw, x, m, y, stream=None):
    L = _lib()
    rc = L.load().spec_qmatmul_noalloc(qw._h, ctypes.c_void_p(x.data_ptr()), m, ctypes.c_void_p(y.data_ptr()),
                                       ctypes.c_void_p(stream) if stream else None)
    L.check(rc, None)


@pytest.mark.parametrize("fmt,n,k", [(12, 1024, 4096), (14, 1024, 4096), (13, 1024, 4096), (30, 512, 1024),
                                     (8, 256, 512), (12, 4096, 4096)])
@pytest.mark.parametrize("m", [1, 5, 9, 33])
def test_noalloc_matches_qmatmul(pkg, synth, fmt, n, k, m):
    import torch
    raw = _raw(synth, fmt, n, k, seed=1000 + fmt + m)
    qw = pkg.QWeight(fmt, raw, n, k)
    rng = np.random.default_rng(m)
    x_np = rng.standard_normal((m, k), dtype=np.float32)
    x = torch.from_numpy(x_np).cuda()
    y_ref = torch.empty((m, n), dtype=torch.float32, device="cuda")
    qw.matmul(x.data_ptr(), m, y_ref.data_ptr())
    torch.cuda.synchronize()
    ref = y_ref.cpu().numpy()
    bound = TOL * float(np.abs(ref).max())
    want = _oracle_y(fmt, raw, n, k, x_np)
    obound = ORACLE_TOL * float(np.abs(want).max()) + 1e-6
    for call in range(2):
        y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        _noalloc(qw, x, m, y)
        got = y.cpu().numpy()
        assert np.isfinite(got).all(), f"call {call}"
        assert np.abs(got - ref).max() <= bound, f"call {call}"
        assert np.abs(got - want).max() <= obound, f"call {call} vs oracle"
    qw.close()


def test_noalloc_alternating_weights(pkg, synth):
    """Two weights take turns on one stream: a 4096 x 4096 Q4_K matmul cut into
    many split-K chunks at M=33 and a small Q8_0 one at M=1.  Each call runs on
    the counters, partials and descriptor the other shape left in the shared
    array; every output must still match spec_qmatmul and the oracle."""
    import torch
    cases = [(12, 4096, 4096, 33, 31), (8, 256, 512, 1, 32)]
    ws, xs, refs, wants = [], [], [], []
    for fmt, n, k, m, seed in cases:
        raw = _raw(synth, fmt, n, k, seed)
        qw = pkg.QWeight(fmt, raw, n, k)
        x_np = np.random.default_rng(seed).standard_normal((m, k), dtype=np.float32)
        x = torch.from_numpy(x_np).cuda()
        y = torch.empty((m, n), dtype=torch.float32, device="cuda")
        qw.matmul(x.data_ptr(), m, y.data_ptr())
        torch.cuda.synchronize()
        ws.append(qw)
        xs.append(x)
        refs.append(y.cpu().numpy())
        wants.append(_oracle_y(fmt, raw, n, k, x_np))
    for it in range(6):
        i = it % 2
        fmt, n, k, m, _ = cases[i]
        y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        _noalloc(ws[i], xs[i], m, y)
        got = y.cpu().numpy()
        assert np.isfinite(got).all(), f"call {it}"
        assert np.abs(got - refs[i]).max() <= TOL * float(np.abs(refs[i]).max()), f"call {it}"
        assert np.abs(got - wants[i]).max() <= ORACLE_TOL * float(np.abs(wants[i]).max()) + 1e-6, f"call {it}"
    for qw in ws:
        qw.close()


def test_noalloc_on_caller_stream(pkg, synth):
    import torch
    n, k, m = 1024, 4096, 5
    qw = _weight(pkg, synth, 12, n, k, seed=77)
    x = torch.from_numpy(np.random.default_rng(3).standard_normal((m, k), dtype=np.float32)).cuda()
    y_ref = torch.empty((m, n), dtype=torch.float32, device="cuda")
    qw.matmul(x.data_ptr(), m, y_ref.data_ptr())
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    outs = []
    with torch.cuda.stream(s):
        for _ in range(2):
            y = torch.empty((m, n), dtype=torch.float32, device="cuda")
            _noalloc(qw, x, m, y, stream=s.cuda_stream)
            outs.append(y)
    s.synchronize()
    ref = y_ref.cpu().numpy()
    for y in outs:
        assert np.abs(y.cpu().numpy() - ref).max() <= TOL * float(np.abs(ref).max())
    qw.close()


def test_noalloc_rejects_oversized_shape(pkg, synth):
    """A shape whose scratch exceeds SPEC_NOALLOC_SCRATCH_BYTES fails with a
    clear error before anything is launched."""
    import torch
    n, k, m = 128, 131072, 64  # operand alone: ~2.4 * k * 64 bytes > 16 MiB
    qw = _weight(pkg, synth, 8, n, k, seed=5)
    x = torch.zeros((m, k), dtype=torch.float32, device="cuda")
    y = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    L = _lib()
    with pytest.raises(L.SamplingError, match="SPEC_NOALLOC_SCRATCH_BYTES"):
        _noalloc(qw, x, m, y)
    assert float(y.abs().max()) == 0.0
    qw.close()
