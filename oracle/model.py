"""oracle/model.py -- CPU restatement of the reference's verify-step model math.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py as the checker; the shipped library never uses it.

Restates, in float64 numpy over dequantized weights (dequantization by the C
restatement in oracle/quants.c, itself pinned against gguf 0.19.0):

* crates/speculate/src/model/quantized_llama_local.rs
    - Mlp::forward (:45-51): w2(silu(w1 x) * w3 x)
    - project_qkv (:71-92), rope_i interleaved pairs (:94-105)
    - run_attn (:107-136): cat KV, repeat_kv, softmax(q k^T / sqrt(d) + bias) v, wo
    - precomput_freqs_cis (:189-205): f32 theta_i = 1/base^(2i/d), f32 pos*theta
    - causal_bias (:332-350), forward_hidden_with_layers (:363-409),
      forward_with_positions (:413-432), truncate (:162-175), keep (:177-186, :451-463)
* crates/speculate/src/model/quantized_qwen2_local.rs: q/k/v biases (:74-82),
  rotate-half rope (:98-109)
* crates/speculate/src/model/llama_local.rs: Llama-3 frequency scaling (:47-75),
  bf16 cos/sin tables (:95-96), rotate-half rope (:231-233)
* the decoder protocol of crates/speculate/src/model/quantized_llama.rs:
  forward_advance_logits (:137-158), tree_logits (:262-325),
  tree_logits_keep_kv (:341-394), commit_tree_path (:409-440),
  next_logits (:528-551), batched_logits (:553-583), rollback_to (:585-599).

RMSNorm is candle's x / sqrt(mean(x^2) + eps) * w.  SiLU is x / (1 + exp(-x)).

Activation quantization (OracleModel(act_quant="q8_1")): the reference's
headline runs candle on CUDA, whose quantized matmuls follow ggml's CUDA
design (candle's source is not vendored here, so this is expected, not
verified): for small batches the activations are first quantized to ggml's
Q8_1 blocks (32 values, scale d = max|x| / 127 kept as f16, codes
round(x / d)) and dotted with the weight codes in integers.  That equals the dot product of the
dequantized weights with the Q8_1 round trip of the activations, up to the
float summation order, so this mode applies q8_1_roundtrip to the input of
every quantized matmul (not to BF16 weights, which candle multiplies
directly).  The default ("none") keeps f32 activations.
"""

from __future__ import annotations

import ctypes
import os
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def oracle_lib() -> ctypes.CDLL:
    """Load (building if needed) oracle/liboracle.so."""
    global _LIB
    if _LIB is None:
        so = os.path.join(HERE, "liboracle.so")
        src = os.path.join(HERE, "quants.c")
        if not os.path.exists(so) or os.path.getmtime(so) < os.path.getmtime(src):
            import subprocess
            subprocess.run(["make", "-s", "-C", HERE], check=True)
        lib = ctypes.CDLL(so)
        lib.oq_dequant.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        lib.oq_dequant.restype = ctypes.c_int
        lib.oq_qmatmul.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                                   ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        lib.oq_qmatmul.restype = ctypes.c_int
        _LIB = lib
    return _LIB


def dequant(qtype: int, raw: np.ndarray, n_elems: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw)
    out = np.empty(n_elems, dtype=np.float32)
    rc = oracle_lib().oq_dequant(int(qtype), raw.ctypes.data, n_elems, out.ctypes.data)
    if rc != 0:
        raise ValueError(f"oracle dequant failed for type {qtype}")
    return out


def qmatmul(qtype: int, raw: np.ndarray, n: int, k: int, x: np.ndarray, threads: int = 0,
            acc_double: bool = True) -> np.ndarray:
    """y = x . W^T straight from GGUF blocks (oracle/quants.c oq_qmatmul)."""
    raw = np.ascontiguousarray(raw)
    x = np.ascontiguousarray(x, dtype=np.float32)
    m = x.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    rc = oracle_lib().oq_qmatmul(int(qtype), raw.ctypes.data, n, k, x.ctypes.data, m, y.ctypes.data, threads,
                                 1 if acc_double else 0)
    if rc != 0:
        raise ValueError("oracle qmatmul failed")
    return y


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, threads: int = 0) -> np.ndarray:
    """Causal attention of M new rows (oracle/quants.c oq_attention, f32):
    q [n_heads, M, hd], k/v [n_kv, T, hd] with the M new keys last -> [M, n_heads * hd]."""
    lib = oracle_lib()
    if not getattr(lib, "_attn_bound", False):
        lib.oq_attention.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 5 + [ctypes.c_void_p, ctypes.c_int]
        lib.oq_attention.restype = ctypes.c_int
        lib._attn_bound = True
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    nh, M, hd = q.shape
    nkv, T, _ = k.shape
    out = np.empty((M, nh * hd), dtype=np.float32)
    if lib.oq_attention(q.ctypes.data, k.ctypes.data, v.ctypes.data, nh, nkv, M, T, hd, out.ctypes.data, threads):
        raise ValueError("oracle attention: bad shape")
    return out


def q8_1_roundtrip(x: np.ndarray) -> np.ndarray:
    """Rows of x through ggml's Q8_1 block format and back (the last axis in
    blocks of 32): d = max|x| / 127 rounded to f16, q = round-half-away(x / d)
    with the f32 scale, value = f16(d) * q."""
    a = np.asarray(x, dtype=np.float32)
    shp = a.shape
    b = a.reshape(-1, 32)
    amax = np.max(np.abs(b), axis=1, keepdims=True)
    d = (amax / np.float32(127.0)).astype(np.float32)
    safe = np.where(d > 0, d, np.float32(1.0))
    r = b / safe
    q = np.where(d > 0, np.sign(r) * np.floor(np.abs(r) + np.float32(0.5)), np.float32(0.0)).astype(np.float32)
    d16 = d.astype(np.float16).astype(np.float32)
    return (d16 * q).reshape(shp).astype(np.float64)


def bf16_round(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


class OracleModel:
    """Quantized Llama / Qwen2 (or BF16 Llama) from a GGUF file, float64 math."""

    def __init__(self, path: str, max_ctx: int = 512, act_quant: str = "none"):
        import gguf

        if act_quant not in ("none", "q8_1"):
            raise ValueError("act_quant must be 'none' or 'q8_1'")
        self.act_quant = act_quant

        r = gguf.GGUFReader(path)
        kv = {f.name: f for f in r.fields.values()}

        def scalar(key, default=None):
            f = kv.get(key)
            if f is None:
                return default
            return f.parts[f.data[0]][0].item()

        def string(key, default=None):
            f = kv.get(key)
            if f is None:
                return default
            return bytes(f.parts[f.data[0]]).decode()

        arch = string("general.architecture")
        self.arch = arch
        self.n_heads = int(scalar(f"{arch}.attention.head_count"))
        self.n_kv = int(scalar(f"{arch}.attention.head_count_kv"))
        self.hidden = int(scalar(f"{arch}.embedding_length"))
        self.n_layers = int(scalar(f"{arch}.block_count"))
        self.eps = float(scalar(f"{arch}.attention.layer_norm_rms_epsilon"))
        self.theta = float(scalar(f"{arch}.rope.freq_base", 10000.0))
        self.head_dim = self.hidden // self.n_heads
        toks = kv.get("tokenizer.ggml.tokens")
        self.rope_half = arch == "qwen2" or string("speculate_b200.rope_style", "") == "half"
        self.rope_scaling = string(f"{arch}.rope.scaling.type", "") == "llama3"
        self.rs = (float(scalar(f"{arch}.rope.scaling.factor", 8.0)),
                   float(scalar(f"{arch}.rope.scaling.low_freq_factor", 1.0)),
                   float(scalar(f"{arch}.rope.scaling.high_freq_factor", 4.0)),
                   int(scalar(f"{arch}.rope.scaling.original_context_length", 8192)))
        self.tensors: Dict[str, np.ndarray] = {}
        self.types: Dict[str, int] = {}
        for t in r.tensors:
            shape = [int(d) for d in reversed(t.shape.tolist())] if hasattr(t.shape, "tolist") else list(t.shape)
            n_el = int(np.prod(t.shape))
            qt = int(t.tensor_type)
            if qt == 0:
                w = np.asarray(t.data, dtype=np.float32).reshape(-1)
            elif qt == 30:
                raw = np.asarray(t.data).view(np.uint16).reshape(-1)
                w = (raw.astype(np.uint32) << 16).view(np.float32)
            else:
                w = dequant(qt, np.asarray(t.data), n_el)
            rows = n_el // int(t.shape[0])
            self.tensors[t.name] = w.reshape(rows, int(t.shape[0])) if rows > 1 else w.reshape(-1)
            self.types[t.name] = qt
        self.vocab = len(toks.data) if toks is not None else self.tensors["token_embd.weight"].shape[0]
        self.bf16 = self.types.get("blk.0.ffn_gate.weight") == 30
        self.max_ctx = max_ctx
        self._build_rope()
        self.clear()

    # -- tables ---------------------------------------------------------------
    def _build_rope(self) -> None:
        hd = self.head_dim
        i = np.arange(0, hd, 2, dtype=np.float32)
        inv = (np.float32(1.0) / np.power(np.float32(self.theta), i / np.float32(hd))).astype(np.float32)
        if self.rope_scaling:
            factor, low, high, orig = self.rs
            out = []
            for f in inv.tolist():
                f = np.float32(f)
                wavelen = np.float32(2.0) * np.float32(np.pi) / f
                lw, hw = np.float32(orig) / np.float32(low), np.float32(orig) / np.float32(high)
                if wavelen < hw:
                    out.append(f)
                elif wavelen > lw:
                    out.append(f / np.float32(factor))
                else:
                    smooth = (np.float32(orig) / wavelen - np.float32(low)) / (np.float32(high) - np.float32(low))
                    out.append((np.float32(1) - smooth) * f / np.float32(factor) + smooth * f)
            inv = np.asarray(out, dtype=np.float32)
        pos = np.arange(self.max_ctx, dtype=np.float32)[:, None]
        ang = (pos * inv[None, :]).astype(np.float32)
        cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
        if self.bf16 and self.arch == "llama":
            cos, sin = bf16_round(cos), bf16_round(sin)
        self.cos, self.sin = cos.astype(np.float64), sin.astype(np.float64)

    def clear(self) -> None:
        shape = (self.n_layers, self.n_kv, self.max_ctx, self.head_dim)
        self.kc = np.zeros(shape, dtype=np.float64)
        self.vc = np.zeros(shape, dtype=np.float64)

    # -- math ------------------------------------------------------------------
    def W(self, name: str) -> np.ndarray:
        return self.tensors[name].astype(np.float64)

    def act(self, x: np.ndarray, name: str) -> np.ndarray:
        """The activations as the matmul with weight `name` sees them."""
        if self.act_quant == "q8_1" and self.types.get(name) not in (0, 30):
            return q8_1_roundtrip(x)
        return x

    def mm(self, x: np.ndarray, name: str) -> np.ndarray:
        return self.act(x, name) @ self.W(name).T

    def rms(self, x: np.ndarray, w: np.ndarray) -> np.ndarray:
        ms = np.mean(x * x, axis=-1, keepdims=True)
        return x / np.sqrt(ms + self.eps) * w

    def rope(self, x: np.ndarray, positions: Sequence[int]) -> np.ndarray:
        """x [heads, M, hd]; interleaved (rope_i) or rotate-half (rope)."""
        c = self.cos[np.asarray(positions)][None]
        s = self.sin[np.asarray(positions)][None]
        out = np.empty_like(x)
        if self.rope_half:
            h = self.head_dim // 2
            a, b = x[..., :h], x[..., h:]
            out[..., :h] = a * c - b * s
            out[..., h:] = a * s + b * c
        else:
            a, b = x[..., 0::2], x[..., 1::2]
            out[..., 0::2] = a * c - b * s
            out[..., 1::2] = a * s + b * c
        return out

    def embed(self, tokens: Sequence[int]) -> np.ndarray:
        return self.tensors["token_embd.weight"][np.asarray(tokens)].astype(np.float64)

    def forward(self, tokens: Sequence[int], positions: Sequence[int], slots: Sequence[int], prefix: int,
                anc: Sequence[int], collect: Sequence[int] = ()) -> Tuple[np.ndarray, List[np.ndarray]]:
        """Rows of `tokens` at `positions`; K/V written to `slots`; keys [0, prefix)
        visible to all rows, new key j visible to row i iff bit j of anc[i]."""
        n = len(tokens)
        x = self.embed(tokens)
        hd, nq, nkv = self.head_dim, self.n_heads, self.n_kv
        G = nq // nkv
        total = prefix + n
        vis = np.zeros((n, total), dtype=bool)
        vis[:, :prefix] = True
        if list(anc) == causal_anc(n):
            vis[:, prefix:] = np.tril(np.ones((n, n), dtype=bool))
        else:
            for i in range(n):
                for j in range(n):
                    vis[i, prefix + j] = bool((anc[i] >> j) & 1)
        collected = []
        for li in range(self.n_layers):
            p = f"blk.{li}."
            xn = self.rms(x, self.W(p + "attn_norm.weight"))
            q = self.mm(xn, p + "attn_q.weight")
            k = self.mm(xn, p + "attn_k.weight")
            v = self.mm(xn, p + "attn_v.weight")
            if self.arch == "qwen2":
                q = q + self.W(p + "attn_q.bias")
                k = k + self.W(p + "attn_k.bias")
                v = v + self.W(p + "attn_v.bias")
            q = self.rope(q.reshape(n, nq, hd).transpose(1, 0, 2), positions)
            k = self.rope(k.reshape(n, nkv, hd).transpose(1, 0, 2), positions)
            v = v.reshape(n, nkv, hd).transpose(1, 0, 2)
            self.kc[li][:, np.asarray(slots)] = k
            self.vc[li][:, np.asarray(slots)] = v
            kk = self.kc[li][:, :total]
            vv = self.vc[li][:, :total]
            out = np.empty((n, nq, hd))
            for h in range(nq):
                sc = q[h] @ kk[h // G].T / np.sqrt(hd)
                sc = np.where(vis, sc, -np.inf)
                sc = sc - sc.max(axis=-1, keepdims=True)
                pr = np.exp(sc)
                pr /= pr.sum(axis=-1, keepdims=True)
                out[:, h] = pr @ vv[h // G]
            x = x + self.mm(out.reshape(n, nq * hd), p + "attn_output.weight")
            xn = self.rms(x, self.W(p + "ffn_norm.weight"))
            g = self.mm(xn, p + "ffn_gate.weight")
            u = self.mm(xn, p + "ffn_up.weight")
            x = x + self.mm(g / (1.0 + np.exp(-g)) * u, p + "ffn_down.weight")
            if li in collect:
                collected.append(x.copy())
        hfin = self.rms(x, self.W("output_norm.weight"))
        return hfin, collected

    def lm_head(self, hfin: np.ndarray) -> np.ndarray:
        # In row blocks, so a vocabulary-sized head is never materialised in
        # float64 at once (same products; each logit is one dot product).
        name = "output.weight" if "output.weight" in self.tensors else "token_embd.weight"
        w = self.tensors[name]
        hfin = self.act(hfin, name)
        out = np.empty((hfin.shape[0], self.vocab), dtype=np.float64)
        for r0 in range(0, self.vocab, 16384):
            r1 = min(r0 + 16384, self.vocab)
            out[:, r0:r1] = hfin @ w[r0:r1].astype(np.float64).T
        return out


def causal_anc(n: int) -> List[int]:
    return [(1 << (i + 1)) - 1 for i in range(n)]


def tree_anc(parents: Sequence[int]) -> List[int]:
    out = []
    for i in range(len(parents)):
        b, cur = 1 << i, i
        while cur != 0:
            cur = parents[cur]
            b |= 1 << cur
        out.append(b | 1)
    return out


def tree_depth(parents: Sequence[int], i: int) -> int:
    d = 0
    while i != 0:
        i = parents[i]
        d += 1
    return d


class OracleDecoder:
    """The reference decoder protocol (quantized_llama.rs) over OracleModel."""

    def __init__(self, model: OracleModel):
        self.m = model
        self.history: List[int] = []
        self.cache_len = 0
        self.last_logits: Optional[np.ndarray] = None

    def reset(self) -> None:
        self.history = []
        self.cache_len = 0
        self.last_logits = None

    def _advance(self, tokens: Sequence[int], last_only: bool = False) -> np.ndarray:
        # last_only: the caller reads only the last row's logits (observe),
        # so the LM head runs on that row alone; the result is the same row.
        n = len(tokens)
        P = self.cache_len
        h, _ = self.m.forward(tokens, list(range(P, P + n)), list(range(P, P + n)), P, causal_anc(n))
        logits = self.m.lm_head(h[-1:] if last_only else h)
        self.cache_len += n
        self.last_logits = logits[-1].copy()
        return logits

    def observe(self, ids: Sequence[int]) -> None:
        if len(ids) == 0:
            return
        self._advance(ids, last_only=True)
        self.history.extend(int(t) for t in ids)

    def next_logits(self) -> np.ndarray:
        if self.last_logits is not None:
            return self.last_logits.copy()
        last = self.history[-1]
        self.cache_len = len(self.history) - 1
        return self._advance([last], last_only=True)[-1]

    def batched_logits(self, drafts: Sequence[int]) -> np.ndarray:
        if len(drafts) == 0:
            return self.next_logits()[None]
        last = self.history[-1]
        self.cache_len = len(self.history) - 1
        out = self._advance([last, *drafts])
        self.history.extend(int(t) for t in drafts)
        return out

    def rollback_to(self, length: int) -> None:
        if length > len(self.history):
            raise ValueError("CacheRollback")
        self.history = self.history[:length]
        self.last_logits = None
        self.cache_len = length

    def _tree_forward(self, tokens, parents, prefix):
        n = len(tokens)
        pos = [prefix + tree_depth(parents, i) for i in range(n)]
        h, _ = self.m.forward(tokens, pos, list(range(prefix, prefix + n)), prefix, tree_anc(parents))
        return h, self.m.lm_head(h)

    def tree_logits(self, tokens, parents) -> np.ndarray:
        pre = self.cache_len
        prefix = pre - 1
        _, logits = self._tree_forward(tokens, parents, prefix)
        self.cache_len = prefix
        restore = self._advance([self.history[-1]])
        logits[0] = restore[-1]
        return logits

    def tree_logits_keep_kv(self, tokens, parents) -> Tuple[np.ndarray, np.ndarray]:
        self.last_logits = None
        prefix = self.cache_len - 1
        h, logits = self._tree_forward(tokens, parents, prefix)
        self.cache_len = prefix + len(tokens)
        return logits, h

    def commit_tree_path(self, tokens, parents, accepted) -> None:
        self.last_logits = None
        prefix = len(self.history) - 1
        keep = list(range(prefix)) + [prefix + ti for ti in accepted]
        for li in range(self.m.n_layers):
            self.m.kc[li][:, : len(keep)] = self.m.kc[li][:, keep]
            self.m.vc[li][:, : len(keep)] = self.m.vc[li][:, keep]
        self.cache_len = len(keep)
        for ti in accepted[1:]:
            self.history.append(int(tokens[ti]))
