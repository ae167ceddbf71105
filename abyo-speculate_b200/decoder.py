"""``B200Decoder``: the reference's Decoder / TreeDecoder surface over the C ABI.

Method names, argument meaning, return shapes and error classes follow the
traits in crates/speculate/src/model/mod.rs:39-236 as implemented by
``LlamaQuantDecoder`` (crates/speculate/src/model/quantized_llama.rs),
``Qwen2QuantDecoder`` (quantized_qwen2.rs) and the BF16 ``LlamaDecoder``
(llama.rs).  Where the trait returns ``Vec<f32>`` this returns a 1-D float32
numpy array; ``Vec<Vec<f32>>`` becomes a 2-D array (rows x vocab); candle
tensors (hidden states) become float32 arrays.
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence, Tuple

import numpy as np

from . import _lib
from .tree import DraftTree


def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint32).reshape(-1))


def _ptr(a: np.ndarray, ct):
    return a.ctypes.data_as(ctypes.POINTER(ct))


def exchange_tp_handles(mine: bytes, group=None) -> List[bytes]:
    """All ranks' tensor-parallel handles in rank order (torch.distributed
    all_gather_object over `group`; works with the gloo and nccl backends)."""
    import torch.distributed as dist
    out: List[Optional[bytes]] = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(mine), group=group)
    if any(h is None or len(h) != len(mine) for h in out):
        raise _lib.SpecError(_lib.SPEC_ERR_INVALID, "tensor-parallel handle exchange returned a malformed handle")
    return [bytes(h) for h in out]


class B200Decoder:
    """One model resident on one B200; stateful like the reference decoders."""

    def __init__(self, handle: ctypes.c_void_p, eos_token_ids: Sequence[int] = ()):
        self._lib = _lib.load()
        self._h = handle
        self._eos = [int(t) for t in eos_token_ids]
        self._vocab = self._lib.spec_vocab_size(self._h)
        self._hidden = self._lib.spec_hidden_size(self._h)

    # ---- construction ----------------------------------------------------
    @classmethod
    def from_gguf(cls, path: str, device: int = 0, max_ctx: int = 0, use_graphs: bool = True,
                  eos_token_ids: Sequence[int] = (), tp_rank: int = 0, tp_size: int = 1) -> "B200Decoder":
        """LlamaQuantDecoder::from_gguf / Qwen2QuantDecoder::from_gguf (quantized_llama.rs:57-97).

        With tp_size > 1 the handle holds rank tp_rank's tensor-parallel shard;
        call tp_connect() on every rank before the first forward."""
        lib = _lib.load()
        opts = _lib.LoadOpts(device, max_ctx, 1 if use_graphs else 0, tp_rank, tp_size)
        h = ctypes.c_void_p()
        _lib.check(lib.spec_load_gguf(path.encode(), ctypes.byref(opts), ctypes.byref(h)), None)
        return cls(h, eos_token_ids)

    @classmethod
    def synthetic(cls, arch: str, n_layers: int, hidden: int, n_heads: int, n_kv_heads: int, ffn: int,
                  vocab: int, rope_theta: float, eps: float, quant_mix: str = "Q4_K_M", seed: int = 0,
                  device: int = 0, max_ctx: int = 0, use_graphs: bool = True, rope_half: bool = False,
                  eos_token_ids: Sequence[int] = (), tp_rank: int = 0, tp_size: int = 1,
                  damp_from_layer: int = 0, damp: float = 1.0) -> "B200Decoder":
        """A seeded synthetic model whose weights are generated on the device
        (the same weights for every tp_size; a tensor-parallel rank keeps its shard).
        Layers from damp_from_layer on (0 = none) draw attn_output / ffn_down
        with sigma 0.02 * damp: a model with the same seed and only the first
        damp_from_layer layers then predicts like this one (see spec_model_desc)."""
        lib = _lib.load()
        mixes = {"Q4_K_M": 0, "Q5_K": 1, "Q8_0": 2, "BF16": 3}
        d = _lib.ModelDesc(0 if arch == "llama" else 1, n_layers, hidden, n_heads, n_kv_heads, ffn, vocab,
                           rope_theta, eps, mixes[quant_mix], 1 if rope_half else 0, int(damp_from_layer),
                           int(round(damp * 10000)))
        opts = _lib.LoadOpts(device, max_ctx, 1 if use_graphs else 0, tp_rank, tp_size)
        h = ctypes.c_void_p()
        _lib.check(lib.spec_create_synthetic(ctypes.byref(d), seed, ctypes.byref(opts), ctypes.byref(h)), None)
        return cls(h, eos_token_ids)

    # ---- tensor parallelism ------------------------------------------------
    def tp_size(self) -> int:
        return int(self._lib.spec_tp_size(self._h))

    def tp_handle(self) -> bytes:
        """This rank's receive-buffer handle (CUDA IPC), to be shared with every rank."""
        buf = ctypes.create_string_buffer(256)
        n = self._lib.spec_tp_handle(self._h, buf, 256)
        if n < 0:
            self._check(-n)
        return buf.raw[:n]

    def tp_connect(self, handles: Sequence[bytes]) -> None:
        """Maps every rank's receive buffer (handles in rank order)."""
        blob = b"".join(handles)
        self._check(self._lib.spec_tp_connect(self._h, blob, len(handles)))

    def tp_connect_group(self, group=None) -> None:
        """Exchanges handles over a torch.distributed process group, then connects."""
        handles = exchange_tp_handles(self.tp_handle(), group)
        self.tp_connect(handles)

    def close(self) -> None:
        if self._h:
            self._lib.spec_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int) -> None:
        _lib.check(rc, self._h)

    # ---- Decoder -------------------------------------------------------------
    def vocab_size(self) -> int:
        return self._vocab

    def hidden_size(self) -> int:
        return self._hidden

    def history(self) -> List[int]:
        n = self._lib.spec_history_len(self._h)
        buf = np.zeros(max(n, 1), dtype=np.uint32)
        self._lib.spec_history(self._h, _ptr(buf, ctypes.c_uint32), n)
        return [int(x) for x in buf[:n]]

    def history_len(self) -> int:
        return self._lib.spec_history_len(self._h)

    def kv_len(self) -> int:
        """The reference decoder's `cache_len`."""
        return self._lib.spec_kv_len(self._h)

    def max_ctx(self) -> int:
        """KV capacity in tokens (the load's max_ctx)."""
        return self._lib.spec_max_ctx(self._h)

    def eos_token_ids(self) -> List[int]:
        return list(self._eos)

    def reset(self) -> None:
        self._check(self._lib.spec_reset(self._h))

    def observe(self, ids: Sequence[int]) -> None:
        a = _u32(ids)
        self._check(self._lib.spec_observe(self._h, _ptr(a, ctypes.c_uint32), a.size))

    def next_logits(self) -> np.ndarray:
        out = np.empty(self._vocab, dtype=np.float32)
        self._check(self._lib.spec_next_logits(self._h, _ptr(out, ctypes.c_float)))
        return out

    def batched_logits(self, drafts: Sequence[int], out: Optional[np.ndarray] = None) -> np.ndarray:
        """Decoder::batched_logits.  `out` (optional): a C-contiguous float32
        (k+1, V) array to fill; when it is page-locked (e.g. a pinned torch
        tensor's .numpy()), the rows are copied into it by DMA directly."""
        a = _u32(drafts)
        shape = (a.size + 1, self._vocab)
        if out is None:
            out = np.empty(shape, dtype=np.float32)
        elif out.shape != shape or out.dtype != np.float32 or not out.flags["C_CONTIGUOUS"]:
            raise ValueError(f"out must be a C-contiguous float32 array of shape {shape}")
        self._check(self._lib.spec_batched_logits(self._h, _ptr(a, ctypes.c_uint32), a.size,
                                                  _ptr(out, ctypes.c_float)))
        return out

    def rollback_to(self, length: int) -> None:
        self._check(self._lib.spec_rollback_to(self._h, int(length)))

    # ---- TreeDecoder -----------------------------------------------------------
    @staticmethod
    def _tree_arrays(tree: DraftTree) -> Tuple[np.ndarray, np.ndarray]:
        return _u32(tree.tokens()), np.ascontiguousarray(np.asarray(tree.parents(), dtype=np.int32))

    def tree_logits(self, tree: DraftTree, out: Optional[np.ndarray] = None) -> np.ndarray:
        """TreeDecoder::tree_logits; `out` as for batched_logits ((n, V) float32,
        filled by DMA when page-locked and the tree fits one forward)."""
        t, p = self._tree_arrays(tree)
        shape = (t.size, self._vocab)
        if out is None:
            out = np.empty(shape, dtype=np.float32)
        elif out.shape != shape or out.dtype != np.float32 or not out.flags["C_CONTIGUOUS"]:
            raise ValueError(f"out must be a C-contiguous float32 array of shape {shape}")
        self._check(self._lib.spec_tree_logits(self._h, _ptr(t, ctypes.c_uint32), _ptr(p, ctypes.c_int32), t.size,
                                               _ptr(out, ctypes.c_float)))
        return out

    def tree_logits_keep_kv(self, tree: DraftTree) -> Tuple[np.ndarray, np.ndarray]:
        t, p = self._tree_arrays(tree)
        lo = np.empty((t.size, self._vocab), dtype=np.float32)
        hi = np.empty((t.size, self._hidden), dtype=np.float32)
        self._check(self._lib.spec_tree_logits_keep_kv(self._h, _ptr(t, ctypes.c_uint32), _ptr(p, ctypes.c_int32),
                                                       t.size, _ptr(lo, ctypes.c_float), _ptr(hi, ctypes.c_float)))
        return lo, hi

    def commit_tree_path(self, tree: DraftTree, accepted: Sequence[int]) -> None:
        t, p = self._tree_arrays(tree)
        a = np.ascontiguousarray(np.asarray(accepted, dtype=np.int32))
        self._check(self._lib.spec_commit_tree_path(self._h, _ptr(t, ctypes.c_uint32), _ptr(p, ctypes.c_int32),
                                                    t.size, _ptr(a, ctypes.c_int32), a.size))

    def last_hidden_state(self) -> np.ndarray:
        out = np.empty(self._hidden, dtype=np.float32)
        self._check(self._lib.spec_last_hidden_state(self._h, _ptr(out, ctypes.c_float)))
        return out

    def observe_returning_last_hidden(self, ids: Sequence[int]) -> np.ndarray:
        a = _u32(ids)
        out = np.empty(self._hidden, dtype=np.float32)
        self._check(self._lib.spec_observe_returning_last_hidden(self._h, _ptr(a, ctypes.c_uint32), a.size,
                                                                 _ptr(out, ctypes.c_float)))
        return out

    def apply_lm_head(self, hidden: np.ndarray) -> np.ndarray:
        h = np.ascontiguousarray(np.asarray(hidden, dtype=np.float32))
        lead = h.shape[:-1]
        h2 = h.reshape(-1, self._hidden)
        out = np.empty((h2.shape[0], self._vocab), dtype=np.float32)
        self._check(self._lib.spec_apply_lm_head(self._h, _ptr(h2, ctypes.c_float), h2.shape[0],
                                                 _ptr(out, ctypes.c_float)))
        return out.reshape(*lead, self._vocab)

    def apply_lm_head_topk(self, hidden: np.ndarray, k: int) -> Tuple[np.ndarray, np.ndarray]:
        """apply_lm_head then medusa.rs:477-487 top_k_indices, the top-k on
        the device.  Returns (ids [..., k] int32, logits [..., k] f32)."""
        h = np.ascontiguousarray(np.asarray(hidden, dtype=np.float32))
        lead = h.shape[:-1]
        h2 = h.reshape(-1, self._hidden)
        ids = np.empty((h2.shape[0], k), dtype=np.int32)
        vals = np.empty((h2.shape[0], k), dtype=np.float32)
        self._check(self._lib.spec_apply_lm_head_topk(self._h, _ptr(h2, ctypes.c_float), h2.shape[0], k,
                                                      _ptr(ids, ctypes.c_int32), _ptr(vals, ctypes.c_float)))
        return ids.reshape(*lead, k), vals.reshape(*lead, k)

    # ---- EAGLE draft on the device (methods/eagle.rs) ----------------------
    def eagle_attach(self, weights: dict, rope_theta: float = 0.0) -> None:
        """weights: 'fc', 'q', 'k', 'v', 'o', 'gate', 'up', 'down' as uint16 BF16
        bit arrays [out, in]; 'post_norm' f32 [H]."""
        keep = {}
        ws = _lib.EagleWeights()
        for name in ("fc", "q", "k", "v", "o", "gate", "up", "down"):
            a = np.ascontiguousarray(weights[name], dtype=np.uint16)
            keep[name] = a
            setattr(ws, name, a.ctypes.data)
        pn = np.ascontiguousarray(weights["post_norm"], dtype=np.float32)
        keep["post_norm"] = pn
        ws.post_norm = pn.ctypes.data
        ws.rope_theta = float(rope_theta)
        self._check(self._lib.spec_eagle_attach(self._h, ctypes.byref(ws)))

    def eagle_attach_synthetic(self, seed: int = 0) -> None:
        self._check(self._lib.spec_eagle_attach_synthetic(self._h, int(seed)))

    def eagle_draft(self, hidden: np.ndarray, root: int, position: int, depth: int,
                    k: int) -> Tuple[np.ndarray, np.ndarray]:
        """eagle.rs:531-575 on the device: (ids [depth, k], log-probs [depth, k])."""
        h = np.ascontiguousarray(np.asarray(hidden, dtype=np.float32).reshape(-1))
        ids = np.empty((depth, k), dtype=np.int32)
        lp = np.empty((depth, k), dtype=np.float32)
        self._check(self._lib.spec_eagle_draft(self._h, _ptr(h, ctypes.c_float), int(root), int(position), depth, k,
                                               _ptr(ids, ctypes.c_int32), _ptr(lp, ctypes.c_float)))
        return ids, lp

    def eagle_round(self, hidden: np.ndarray, depth: int, top_k: int, max_tree_nodes: int = 0,
                    strict_root: bool = False, eos: Sequence[int] = ()) -> Tuple[List[int], np.ndarray, bool]:
        """One greedy EAGLE-2 round (eagle.rs:531-731) in one call:
        (committed tokens, the next round's hidden row, stop)."""
        h = np.ascontiguousarray(np.asarray(hidden, dtype=np.float32).reshape(-1))
        e = np.ascontiguousarray(np.asarray(list(eos), dtype=np.uint32))
        out = np.zeros(depth + 1, dtype=np.uint32)
        nxt = np.zeros(self.hidden_size(), dtype=np.float32)
        n, stop = ctypes.c_int(), ctypes.c_int()
        self._check(self._lib.spec_eagle_round(self._h, _ptr(h, ctypes.c_float), depth, top_k, max_tree_nodes,
                                               1 if strict_root else 0, _ptr(e, ctypes.c_uint32), int(e.size),
                                               _ptr(out, ctypes.c_uint32), ctypes.byref(n), _ptr(nxt, ctypes.c_float),
                                               ctypes.byref(stop)))
        return [int(t) for t in out[:n.value]], nxt, bool(stop.value)

    def medusa_attach(self, res_w: Sequence[Sequence[np.ndarray]], res_b: Sequence[Sequence[np.ndarray]],
                      out_w: Sequence[np.ndarray]) -> None:
        """Medusa heads (medusa.rs:509-584): res_w[head][layer] uint16 BF16 bits
        [H, H], res_b[head][layer] f32 [H], out_w[head] uint16 BF16 bits [V, H]."""
        n = len(out_w)
        layers = len(res_w[0]) if n and len(res_w) else 0
        if len(res_w) != n or len(res_b) != n or any(len(r) != layers for r in res_w) or \
                any(len(b) != layers for b in res_b):
            raise _lib.SamplingError(_lib.SPEC_ERR_INVALID, "res_w / res_b must be [n_heads][residual_layers]")
        keep = []

        def arr(a, dt):
            a = np.ascontiguousarray(a, dtype=dt)
            keep.append(a)
            return a.ctypes.data
        rw = (ctypes.c_void_p * max(n * layers, 1))(*[arr(w, np.uint16) for r in res_w for w in r])
        rb = (ctypes.c_void_p * max(n * layers, 1))(*[arr(b, np.float32) for r in res_b for b in r])
        ow = (ctypes.c_void_p * max(n, 1))(*[arr(w, np.uint16) for w in out_w])
        ws = _lib.MedusaWeights(n, layers, ctypes.cast(rw, ctypes.c_void_p), ctypes.cast(rb, ctypes.c_void_p),
                                ctypes.cast(ow, ctypes.c_void_p))
        self._check(self._lib.spec_medusa_attach(self._h, ctypes.byref(ws)))

    def medusa_attach_synthetic(self, n_heads: int, residual_layers: int = 1, seed: int = 0) -> None:
        self._check(self._lib.spec_medusa_attach_synthetic(self._h, int(n_heads), int(residual_layers), int(seed)))

    def medusa_num_heads(self) -> int:
        return self._lib.spec_medusa_num_heads(self._h)

    def medusa_topk(self, hidden: np.ndarray, k: int) -> Tuple[np.ndarray, np.ndarray]:
        """MedusaHeadsCandle::top_k_per_head (medusa.rs:713-734) on the device:
        (ids [n_heads, k], log-probs [n_heads, k])."""
        n = self.medusa_num_heads()
        h = np.ascontiguousarray(np.asarray(hidden, dtype=np.float32).reshape(-1))
        ids = np.empty((max(n, 1), k), dtype=np.int32)
        lp = np.empty((max(n, 1), k), dtype=np.float32)
        self._check(self._lib.spec_medusa_topk(self._h, _ptr(h, ctypes.c_float), int(k), _ptr(ids, ctypes.c_int32),
                                               _ptr(lp, ctypes.c_float)))
        return ids[:n], lp[:n]

    def medusa_round(self, hidden: np.ndarray, top_k: int, topology: str = "cartesian", acceptance: str = "greedy",
                     epsilon: float = 0.0, delta: float = 0.0, budget: int = 1 << 30) -> Tuple[List[int], np.ndarray]:
        """One Medusa round (medusa.rs:761-810) in one call: (committed tokens,
        the hidden row of the last one).  topology: "greedy" | "cartesian";
        acceptance: "greedy" | "typical" (with epsilon, delta)."""
        topo = {"greedy": 0, "cartesian": 1}[topology]
        acc = {"greedy": 0, "typical": 1}[acceptance]
        h = np.ascontiguousarray(np.asarray(hidden, dtype=np.float32).reshape(-1))
        out = np.zeros(self.medusa_num_heads() + 1, dtype=np.uint32)
        nxt = np.zeros(self.hidden_size(), dtype=np.float32)
        n = ctypes.c_int()
        self._check(self._lib.spec_medusa_round(self._h, _ptr(h, ctypes.c_float), int(top_k), topo, acc,
                                                float(epsilon), float(delta), int(budget), _ptr(out, ctypes.c_uint32),
                                                ctypes.byref(n), _ptr(nxt, ctypes.c_float)))
        return [int(t) for t in out[:n.value]], nxt

    def embed_tokens(self, ids: Sequence[int]) -> np.ndarray:
        a = _u32(ids)
        out = np.empty((a.size, self._hidden), dtype=np.float32)
        self._check(self._lib.spec_embed_tokens(self._h, _ptr(a, ctypes.c_uint32), a.size, _ptr(out, ctypes.c_float)))
        return out

    def last_hidden_states_multi(self, layers: Sequence[int]) -> Tuple[np.ndarray, List[np.ndarray]]:
        sel = np.ascontiguousarray(np.asarray(layers, dtype=np.int32))
        fin = np.empty(self._hidden, dtype=np.float32)
        outs = np.empty((max(sel.size, 1), self._hidden), dtype=np.float32)
        self._check(self._lib.spec_last_hidden_states_multi(self._h, _ptr(sel, ctypes.c_int32), sel.size,
                                                            _ptr(fin, ctypes.c_float), _ptr(outs, ctypes.c_float)))
        return fin, [outs[i].copy() for i in range(sel.size)]

    def num_hidden_layers(self) -> int:
        return self._lib.spec_num_layers(self._h)

    # ---- device-side acceptance ----------------------------------------------------
    def verify_greedy(self, drafts: Sequence[int]) -> Tuple[int, int, np.ndarray]:
        """Batched verify + device argmax + temperature-0 accept walk.

        Returns (n_accepted, next_token, row_argmax)."""
        a = _u32(drafts)
        n_acc = ctypes.c_int()
        nxt = ctypes.c_uint32()
        am = np.empty(a.size + 1, dtype=np.int32)
        self._check(self._lib.spec_verify_greedy(self._h, _ptr(a, ctypes.c_uint32), a.size, ctypes.byref(n_acc),
                                                 ctypes.byref(nxt), _ptr(am, ctypes.c_int32)))
        return n_acc.value, nxt.value, am

    def verify_rejection(self, drafts: Sequence[int], draft_probs: np.ndarray, temperature: float,
                         uniforms: Sequence[float], budget: Optional[int] = None) -> Tuple[List[int], int]:
        """Batched verify + the rejection-sampling round of vanilla.rs:172-210
        on the device.  draft_probs: k x V float32 draft distributions;
        uniforms: the round's gen::<f32>() draws in the reference order.

        Returns (committed tokens, uniforms used)."""
        a = _u32(drafts)
        q = np.ascontiguousarray(draft_probs, dtype=np.float32).reshape(a.size, -1) if a.size else \
            np.zeros((0, self.vocab_size()), dtype=np.float32)
        u = np.ascontiguousarray(uniforms, dtype=np.float32)
        commits = np.empty(a.size + 1, dtype=np.uint32)
        n = ctypes.c_int()
        used = ctypes.c_int()
        b = a.size + 1 if budget is None else int(budget)
        self._check(self._lib.spec_verify_rejection(self._h, _ptr(a, ctypes.c_uint32), a.size,
                                                    _ptr(q, ctypes.c_float), float(temperature),
                                                    _ptr(u, ctypes.c_float), u.size, b,
                                                    _ptr(commits, ctypes.c_uint32), ctypes.byref(n),
                                                    ctypes.byref(used)))
        return [int(x) for x in commits[: n.value]], used.value

    def verify_tree_greedy(self, tree: DraftTree) -> Tuple[List[int], int]:
        """Tree verify (KV kept) + device argmax + eagle.rs:618-661 path walk."""
        t, p = self._tree_arrays(tree)
        best = np.empty(t.size, dtype=np.int32)
        plen = ctypes.c_int()
        bonus = ctypes.c_uint32()
        self._check(self._lib.spec_verify_tree_greedy(self._h, _ptr(t, ctypes.c_uint32), _ptr(p, ctypes.c_int32),
                                                      t.size, _ptr(best, ctypes.c_int32), ctypes.byref(plen),
                                                      ctypes.byref(bonus)))
        return [int(x) for x in best[:plen.value]], bonus.value

    def verify_tree_typical(self, tree: DraftTree, epsilon: float, delta: float) -> Tuple[List[int], int]:
        """Tree verify (KV kept) + Medusa typical acceptance (medusa.rs:290-326,
        :424-445: p(x) >= max(epsilon, delta * exp(-H(p))) against the parent's
        row, first longest accepted path) + the argmax bonus of its deepest node."""
        t, p = self._tree_arrays(tree)
        best = np.empty(t.size, dtype=np.int32)
        plen = ctypes.c_int()
        bonus = ctypes.c_uint32()
        self._check(self._lib.spec_verify_tree_typical(self._h, _ptr(t, ctypes.c_uint32), _ptr(p, ctypes.c_int32),
                                                       t.size, float(epsilon), float(delta), _ptr(best, ctypes.c_int32),
                                                       ctypes.byref(plen), ctypes.byref(bonus)))
        return [int(x) for x in best[:plen.value]], bonus.value

    # ---- diagnostics -----------------------------------------------------------------
    def last_forward_ms(self) -> float:
        return float(self._lib.spec_last_forward_ms(self._h))

    def cuda_stream(self) -> int:
        """cudaStream_t (as an int) the library runs this model's forwards on."""
        return int(self._lib.spec_cuda_stream(self._h) or 0)

    def profile_forward(self, drafts: Sequence[int]):
        """Per-kernel (kind, ms, bytes) of one eager verify forward."""
        a = _u32(drafts)
        cap = 4096
        ms = np.zeros(cap, dtype=np.float32)
        kind = np.zeros(cap, dtype=np.int32)
        nb = np.zeros(cap, dtype=np.int64)
        n = self._lib.spec_profile_forward(self._h, _ptr(a, ctypes.c_uint32), a.size, _ptr(ms, ctypes.c_float),
                                           _ptr(kind, ctypes.c_int), nb.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                                           cap)
        if n < 0:
            self._check(-n)
        return kind[:n].copy(), ms[:n].copy(), nb[:n].copy()

    def kernels_per_forward(self, rows: int) -> int:
        return int(self._lib.spec_kernels_per_forward(self._h, rows))

    def weight_bytes(self) -> int:
        return int(self._lib.spec_weight_bytes(self._h))


class QWeight:
    """Standalone dequant-matmul (candle ``QMatMul::forward``) over device buffers."""

    def __init__(self, ggml_type: int, blocks: np.ndarray, n_rows: int, k_cols: int, device: int = 0):
        from .gguf_synth import BLOCK_BYTES, BLOCK_ELEMS
        self._lib = _lib.load()
        b = np.ascontiguousarray(blocks)
        # The C entry point reads n_rows x (k_cols / block) blocks from the
        # host pointer; check the buffer holds them before handing it over.
        if int(ggml_type) in BLOCK_ELEMS and k_cols % BLOCK_ELEMS[int(ggml_type)] == 0:
            need = n_rows * (k_cols // BLOCK_ELEMS[int(ggml_type)]) * BLOCK_BYTES[int(ggml_type)]
            if b.nbytes < need:
                raise _lib.SamplingError(_lib.SPEC_ERR_INVALID,
                                         f"blocks hold {b.nbytes} bytes, {n_rows} x {k_cols} needs {need}")
        h = ctypes.c_void_p()
        _lib.check(self._lib.spec_qweight_upload(int(ggml_type), b.ctypes.data, n_rows, k_cols, device,
                                                 ctypes.byref(h)), None)
        self._h = h
        self.n_rows, self.k_cols = n_rows, k_cols

    def matmul(self, x_dev_ptr: int, m: int, y_dev_ptr: int, stream: Optional[int] = None) -> None:
        _lib.check(self._lib.spec_qmatmul(self._h, ctypes.c_void_p(x_dev_ptr), m, ctypes.c_void_p(y_dev_ptr),
                                          ctypes.c_void_p(stream) if stream else None), None)

    def time_ms(self, m: int, iters: int, flush_l2: bool = True) -> float:
        out = ctypes.c_float()
        _lib.check(self._lib.spec_qmatmul_time(self._h, m, iters, 1 if flush_l2 else 0, ctypes.byref(out)), None)
        return out.value

    def nbytes(self) -> int:
        return int(self._lib.spec_qweight_bytes(self._h))

    def close(self) -> None:
        if self._h:
            self._lib.spec_qweight_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
