"""Tensor-parallel verify forward (2 and 4 GPUs) against the oracle.

Each rank holds its heads' q/k/v rows, its FFN slice of gate/up, and the
matching columns of o and down; the row-parallel outputs are summed across
ranks inside the GEMV epilogue over NVLink.  A rank's share of the k/v rows must fill whole 128-row groups (head_dim 128
here, as in Llama-3-8B and Qwen2-7B).  Every rank must see the same
logits bit for bit (ranks are summed in rank order on every rank), within the
single-GPU tolerance of the float64 oracle, with the same history, KV length
and greedy decisions.  Skipped with fewer GPUs than ranks."""

import os

import numpy as np
import pytest

from test_tp_host import run_ranks

pytestmark = pytest.mark.gpu

TOL = 2e-2

TP_SPECS = {
    "llama_tp": dict(arch="llama", n_layers=2, hidden=512, n_heads=4, n_kv_heads=2, ffn=1024, vocab=1024,
                     rope_theta=5e5, eps=1e-5, quant_mix="Q4_K_M"),
    "qwen_tp_q80": dict(arch="qwen2", n_layers=2, hidden=512, n_heads=4, n_kv_heads=2, ffn=1024, vocab=1024,
                        rope_theta=1e6, eps=1e-6, quant_mix="Q8_0"),
    "llama_tp4": dict(arch="llama", n_layers=2, hidden=2048, n_heads=16, n_kv_heads=4, ffn=4096, vocab=1024,
                      rope_theta=5e5, eps=1e-5, quant_mix="Q4_K_M"),
    # Llama-3-8B's head layout (32 q / 8 kv heads of 128): 8 ranks hold one kv head each.
    "llama_tp8": dict(arch="llama", n_layers=2, hidden=4096, n_heads=32, n_kv_heads=8, ffn=4096, vocab=1024,
                      rope_theta=5e5, eps=1e-5, quant_mix="Q4_K_M"),
    # Slices that start inside a 256-column superblock (Qwen2.5-7B's case: 28
    # heads and FFN 18944 give 896 q columns and 4736 FFN columns per rank at
    # 4 ranks).  Here 3 heads (384 columns) and 384 FFN columns per rank: each
    # rank streams whole superblocks around its slice, zeros elsewhere.
    "qwen_tp2_uneven": dict(arch="qwen2", n_layers=2, hidden=768, n_heads=6, n_kv_heads=2, ffn=768, vocab=1024,
                            rope_theta=1e6, eps=1e-6, quant_mix="Q4_K_M"),
    "qwen_tp4_uneven": dict(arch="qwen2", n_layers=2, hidden=1536, n_heads=12, n_kv_heads=4, ffn=1536, vocab=1024,
                            rope_theta=1e6, eps=1e-6, quant_mix="Q4_K_M"),
}
CASES = [("llama_tp", 2), ("qwen_tp_q80", 2), ("llama_tp4", 2), ("llama_tp4", 4), ("llama_tp8", 8),
         ("qwen_tp2_uneven", 2), ("qwen_tp4_uneven", 4)]


def _prompt(vocab, n, seed):
    return np.random.default_rng(seed).integers(0, vocab, size=n).tolist()


def _oracle_script(oracle, path):
    od = oracle.OracleDecoder(oracle.OracleModel(path, max_ctx=512))
    v = od.m.vocab
    res = {}
    prompt = _prompt(v, 37, 1)
    od.observe(prompt)
    res["next"] = od.next_logits()
    drafts = _prompt(v, 4, 2)
    res["batched"] = od.batched_logits(drafts)
    od.rollback_to(len(prompt) + 2)
    od.observe([5])
    res["after_rollback"] = od.next_logits()
    od.rollback_to(len(prompt))
    long = _prompt(v, 90, 3)
    od.observe(long)
    res["long"] = od.next_logits()
    res["tree"] = od.tree_logits([long[-1], 7, 9, 11, 13], [-1, 0, 0, 2, 2])
    return res


@pytest.mark.parametrize("name,world", CASES)
def test_tp_matches_oracle(pkg, oracle, accept, synth, tmp_path, name, world):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    spec = synth.ModelSpec(ctx_len=2048, **TP_SPECS[name])
    path = str(tmp_path / f"{name}.gguf")
    synth.write_gguf(path, spec, 4321)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    run_ranks("decode", tmp_path, world, extra=(path,), timeout=600, env=env)
    got = [dict(np.load(tmp_path / f"decode_{r}.npz")) for r in range(world)]
    for r in range(1, world):
        for k in got[0]:
            assert np.array_equal(got[0][k], got[r][k]), (k, r)
    g = got[0]
    ref = _oracle_script(oracle, path)
    for k in ["next", "batched", "after_rollback", "long", "tree"]:
        assert g[k].shape == np.asarray(ref[k]).shape, k
        assert np.abs(g[k] - ref[k]).max() <= TOL, (k, float(np.abs(g[k] - ref[k]).max()))
    rows = g["verify_rows"]
    drafts = _prompt(1024, 4, 2)
    exp_acc, exp_next = accept.greedy_linear_accept(rows, drafts)
    assert list(g["greedy"][:2]) == [exp_acc, exp_next]
    assert list(g["greedy"][2:]) == [accept.argmax_first(r) for r in rows]
    assert int(g["kv_len"][0]) == len(g["history"])
