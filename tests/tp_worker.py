"""One rank of a tensor-parallel test, run as a child process by test_tp_*.py.

usage: python tp_worker.py MODE OUT_DIR RANK WORLD PORT [GGUF]

  exchange  handle exchange over gloo only (no GPU): each rank offers a
            rank-specific 64-byte handle and checks it receives all of them in
            rank order.
  decode    (GPU) loads rank RANK's shard of GGUF on cuda:RANK, connects the
            ranks' receive buffers and runs the Decoder / TreeDecoder calls the
            single-GPU tests run; every rank saves what it saw to OUT_DIR.
"""

import datetime
import importlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def _prompt(vocab, n, seed):
    return np.random.default_rng(seed).integers(0, vocab, size=n).tolist()


def run_exchange(pkg, out_dir, rank, world):
    dec_mod = importlib.import_module("abyo-speculate_b200.decoder")
    mine = bytes([rank + 1]) * 64
    got = dec_mod.exchange_tp_handles(mine)
    ok = got == [bytes([r + 1]) * 64 for r in range(world)]
    with open(os.path.join(out_dir, f"exchange_{rank}.json"), "w") as f:
        json.dump({"ok": ok, "n": len(got)}, f)


def run_decode(pkg, out_dir, rank, world, path):
    dec = pkg.B200Decoder.from_gguf(path, device=rank, max_ctx=512, tp_rank=rank, tp_size=world)
    dec.tp_connect_group()
    assert dec.tp_size() == world
    v = dec.vocab_size()
    res = {}
    prompt = _prompt(v, 37, 1)
    dec.observe(prompt)
    res["next"] = dec.next_logits()
    drafts = _prompt(v, 4, 2)
    res["batched"] = dec.batched_logits(drafts)
    dec.rollback_to(len(prompt) + 2)
    dec.observe([5])
    res["after_rollback"] = dec.next_logits()
    dec.rollback_to(len(prompt))
    long = _prompt(v, 90, 3)  # > 64 rows: chunked forwards
    dec.observe(long)
    res["long"] = dec.next_logits()
    tree = pkg.DraftTree.from_parent_table([(0, long[-1]), (0, 7), (0, 9), (2, 11), (2, 13)])
    res["tree"] = dec.tree_logits(tree)
    h = dec.history_len()
    res["verify_rows"] = dec.batched_logits(drafts)
    dec.rollback_to(h)
    n_acc, nxt, am = dec.verify_greedy(drafts)
    res["greedy"] = np.array([n_acc, nxt] + list(am), dtype=np.int64)
    res["history"] = np.array(dec.history(), dtype=np.int64)
    res["kv_len"] = np.array([dec.kv_len()], dtype=np.int64)
    np.savez(os.path.join(out_dir, f"decode_{rank}.npz"), **res)
    dec.close()


def main():
    mode, out_dir, rank, world, port = sys.argv[1], sys.argv[2], int(sys.argv[3]), int(sys.argv[4]), int(sys.argv[5])
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    pkg = importlib.import_module("abyo-speculate_b200")
    try:
        if mode == "exchange":
            run_exchange(pkg, out_dir, rank, world)
        else:
            run_decode(pkg, out_dir, rank, world, sys.argv[6])
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
