"""The C-ABI library loads and exports every symbol include/spec_b200.h declares (CPU)."""

import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(os.path.join(ROOT, "include", "spec_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(spec_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_trait_surface():
    names = declared_functions()
    for must in ["spec_load_gguf", "spec_observe", "spec_next_logits", "spec_batched_logits", "spec_rollback_to",
                 "spec_tree_logits", "spec_tree_logits_keep_kv", "spec_commit_tree_path", "spec_apply_lm_head",
                 "spec_verify_greedy", "spec_qmatmul"]:
        assert must in names


def test_library_exports_every_declared_symbol(pkg):
    lib = ctypes.CDLL(pkg.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header(pkg):
    from importlib import import_module
    _lib = import_module("abyo-speculate_b200._lib")
    bound = {s[0] for s in _lib.SIGNATURES}
    assert set(declared_functions()) <= bound


def test_load_without_gpu_fails_cleanly(pkg):
    import torch
    if torch.cuda.is_available():
        return
    try:
        pkg.B200Decoder.from_gguf("/nonexistent.gguf")
    except pkg.SpecError as e:
        assert e.code in (4, 5)
    else:
        raise AssertionError("expected an error")


def test_qweight_rejects_short_host_buffer(pkg):
    """The C entry point reads n_rows x K/256 blocks from the host pointer;
    the Python wrapper refuses a buffer that does not hold them (no device
    call is made)."""
    import numpy as np
    import pytest
    with pytest.raises(pkg.SamplingError):
        pkg.QWeight(12, np.zeros((10, 144 * 16), np.uint8), 11, 4096)
