"""Shared fixtures: the package under test, the oracle, and small seeded GGUF models.

`-m gpu` tests need a B200 and the built libspecb200.so; everything else runs
on the CPU (oracle vs golden vectors, host logic, ABI exports).
"""

import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


@pytest.fixture(scope="session")
def pkg():
    return importlib.import_module("abyo-speculate_b200")


@pytest.fixture(scope="session")
def synth():
    return importlib.import_module("abyo-speculate_b200.gguf_synth")


@pytest.fixture(scope="session")
def oracle():
    return importlib.import_module("oracle.model")


@pytest.fixture(scope="session")
def accept():
    return importlib.import_module("oracle.accept")


# Small shapes that exercise every code path: head_dim 64 and 128, GQA,
# Q4_K_M (Q4_K + Q6_K segments), the Q8_0 fallback for K % 256 != 0, Q5_K,
# pure Q8_0, BF16 with Llama-3 rope scaling.
TINY_SPECS = {
    "llama_q4km": dict(arch="llama", n_layers=2, hidden=256, n_heads=4, n_kv_heads=2, ffn=512, vocab=1024,
                       rope_theta=5e5, eps=1e-5, quant_mix="Q4_K_M"),
    "llama_hd128": dict(arch="llama", n_layers=2, hidden=512, n_heads=4, n_kv_heads=2, ffn=768, vocab=1024,
                        rope_theta=5e5, eps=1e-5, quant_mix="Q4_K_M"),
    "qwen_q4km": dict(arch="qwen2", n_layers=2, hidden=384, n_heads=6, n_kv_heads=2, ffn=768, vocab=1024,
                      rope_theta=1e6, eps=1e-6, quant_mix="Q4_K_M"),
    "qwen_q5k": dict(arch="qwen2", n_layers=2, hidden=512, n_heads=4, n_kv_heads=2, ffn=1024, vocab=1024,
                     rope_theta=1e6, eps=1e-6, quant_mix="Q5_K"),
    "qwen_q80": dict(arch="qwen2", n_layers=2, hidden=256, n_heads=4, n_kv_heads=1, ffn=512, vocab=1024,
                     rope_theta=1e6, eps=1e-6, quant_mix="Q8_0"),
    "llama_bf16": dict(arch="llama", n_layers=2, hidden=256, n_heads=2, n_kv_heads=1, ffn=512, vocab=1024,
                       rope_theta=5e5, eps=1e-5, quant_mix="BF16"),
    # Large weights: the residual stream passes the f16 range by layer 1.
    "llama_hot": dict(arch="llama", n_layers=3, hidden=256, n_heads=4, n_kv_heads=2, ffn=512, vocab=1024,
                      rope_theta=5e5, eps=1e-5, quant_mix="Q4_K_M"),
}
TINY_SIGMA = {"llama_hot": 2.0}


def make_tiny_gguf(synth_mod, name: str, out_dir: str, seed: int = 1234) -> str:
    spec = synth_mod.ModelSpec(ctx_len=2048, **TINY_SPECS[name])
    path = os.path.join(out_dir, f"{name}.gguf")
    if not os.path.exists(path):
        extra = {}
        if spec.quant_mix == "BF16":
            extra = {"rope_style": "half", "llama3_scaling": True}
        if name in TINY_SIGMA:
            extra["sigma"] = TINY_SIGMA[name]
        synth_mod.write_gguf(path, spec, seed, **extra)
    return path


@pytest.fixture(scope="session")
def tiny_dir(tmp_path_factory):
    return str(tmp_path_factory.mktemp("tiny_models"))


@pytest.fixture(scope="session")
def tiny_gguf(synth, tiny_dir):
    def get(name: str) -> str:
        return make_tiny_gguf(synth, name, tiny_dir)
    return get
