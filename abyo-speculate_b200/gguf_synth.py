"""Seeded synthetic GGUF models for the verify-step backend.

The reference loads real checkpoints from the Hugging Face hub; this container
has no network, so every model here is synthetic: seeded N(0, 0.02) weights
quantized with this module's own GGUF quantizers and written with
``gguf.GGUFWriter`` in exactly the layout the reference's loaders read
(metadata keys and tensor names of
``crates/speculate/src/model/quantized_llama_local.rs:229-281`` and
``crates/speculate/src/model/quantized_qwen2_local.rs:220-275``).

The quantizers are this project's own (``gguf`` 0.19.0 can only quantize
Q8_0).  They produce valid GGUF blocks; the decode of those blocks is the
public GGUF specification and is what every consumer (gguf-py, candle, the
oracle, the CUDA kernels) agrees on.

Quant mixes (recorded in the GGUF under ``speculate_b200.quant_mix``):

* ``Q4_K_M``: Q4_K everywhere; ``attn_v`` and ``ffn_down`` Q6_K on even
  layers; ``output.weight`` Q6_K; norms F32; any tensor whose K is not a
  multiple of 256 falls back to Q8_0.
* ``Q5_K``: Q5_K everywhere, ``output.weight`` Q6_K, same Q8_0 fallback.
* ``Q8_0``: Q8_0 everywhere.
* ``BF16``: BF16 everywhere (norms and biases F32).

Norm weights are ``1 + N(0, 0.02)`` rather than N(0, 0.02): a norm weight near
zero would scale every activation to ~0 and make every logit row flat.
"""

from __future__ import annotations

import dataclasses
import json
from typing import Dict, List, Optional, Tuple

import numpy as np

# GGML type ids (public GGUF specification).
F32, F16, Q8_0, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 8, 12, 13, 14, 30
BLOCK_ELEMS = {Q4_K: 256, Q5_K: 256, Q6_K: 256, Q8_0: 32, F32: 1, F16: 1, BF16: 1}
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210, Q8_0: 34, F32: 4, F16: 2, BF16: 2}
TYPE_NAMES = {F32: "F32", F16: "F16", Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K", BF16: "BF16"}


def _f16(x: np.ndarray) -> np.ndarray:
    return x.astype(np.float16)


def _safe_div(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    out = np.zeros_like(a, dtype=np.float32)
    np.divide(a, b, out=out, where=b != 0)
    return out


def _pack_k4_scales(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Pack 8 six-bit scales and 8 six-bit mins per superblock into 12 bytes."""
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    out = np.zeros(sc.shape[:-1] + (12,), dtype=np.uint8)
    for j in range(4):
        out[..., j] = (sc[..., j] & 63) | ((sc[..., j + 4] >> 4) << 6)
        out[..., j + 4] = (mn[..., j] & 63) | ((mn[..., j + 4] >> 4) << 6)
        out[..., j + 8] = (sc[..., j + 4] & 15) | ((mn[..., j + 4] & 15) << 4)
    return out


def _kquant_affine(x: np.ndarray, levels: int) -> Tuple[np.ndarray, ...]:
    """Shared Q4_K / Q5_K scale search: x [nb, 8, 32] -> (d, dmin, sc, m, q)."""
    lo = np.minimum(x.min(axis=-1), 0.0)
    hi = x.max(axis=-1)
    scale = (hi - lo) / levels
    mins = -lo
    d = _f16(scale.max(axis=-1) / 63.0)
    dmin = _f16(mins.max(axis=-1) / 63.0)
    df = d.astype(np.float32)[:, None]
    dmf = dmin.astype(np.float32)[:, None]
    sc = np.clip(np.rint(_safe_div(scale, df)), 0, 63)
    m = np.clip(np.rint(_safe_div(mins, dmf)), 0, 63)
    s_eff = (df * sc)[..., None]
    c_eff = (dmf * m)[..., None]
    q = np.clip(np.rint(_safe_div(x + c_eff, np.broadcast_to(s_eff, x.shape))), 0, levels)
    return d, dmin, sc, m, q.astype(np.uint8)


def quantize_q4_k(w: np.ndarray) -> np.ndarray:
    """[rows, K] float -> [rows, K/256 * 144] uint8 (Q4_K blocks)."""
    rows, k = w.shape
    x = w.reshape(-1, 8, 32).astype(np.float32)
    d, dmin, sc, m, q = _kquant_affine(x, 15)
    nb = x.shape[0]
    out = np.zeros((nb, 144), dtype=np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = dmin.view(np.uint8).reshape(nb, 2)
    out[:, 4:16] = _pack_k4_scales(sc, m)
    q = q.reshape(nb, 4, 2, 32)  # chunk c: sub-blocks 2c (low nibble), 2c+1 (high)
    out[:, 16:] = (q[:, :, 0, :] | (q[:, :, 1, :] << 4)).reshape(nb, 128)
    return out.reshape(rows, -1)


def quantize_q5_k(w: np.ndarray) -> np.ndarray:
    """[rows, K] float -> [rows, K/256 * 176] uint8 (Q5_K blocks)."""
    rows, k = w.shape
    x = w.reshape(-1, 8, 32).astype(np.float32)
    d, dmin, sc, m, q = _kquant_affine(x, 31)
    nb = x.shape[0]
    out = np.zeros((nb, 176), dtype=np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = dmin.view(np.uint8).reshape(nb, 2)
    out[:, 4:16] = _pack_k4_scales(sc, m)
    q = q.reshape(nb, 4, 2, 32)
    lo = q & 15
    hi = q >> 4
    out[:, 48:] = (lo[:, :, 0, :] | (lo[:, :, 1, :] << 4)).reshape(nb, 128)
    qh = np.zeros((nb, 32), dtype=np.uint8)
    for c in range(4):
        qh |= (hi[:, c, 0, :] << (2 * c)).astype(np.uint8)
        qh |= (hi[:, c, 1, :] << (2 * c + 1)).astype(np.uint8)
    out[:, 16:48] = qh
    return out.reshape(rows, -1)


def quantize_q6_k(w: np.ndarray) -> np.ndarray:
    """[rows, K] float -> [rows, K/256 * 210] uint8 (Q6_K blocks)."""
    rows, k = w.shape
    x = w.reshape(-1, 16, 16).astype(np.float32)
    nb = x.shape[0]
    amax = np.abs(x).max(axis=-1)
    scale = amax / 31.0
    d = _f16(scale.max(axis=-1) / 127.0)
    df = d.astype(np.float32)[:, None]
    sc = np.clip(np.rint(_safe_div(scale, df)), 0, 127).astype(np.int8)
    s_eff = (df * sc.astype(np.float32))[..., None]
    q = np.clip(np.rint(_safe_div(x, np.broadcast_to(s_eff, x.shape))), -32, 31).astype(np.int16) + 32
    q = q.astype(np.uint8).reshape(nb, 2, 4, 32)  # half n, quarter j (q1..q4), l
    out = np.zeros((nb, 210), dtype=np.uint8)
    ql = np.zeros((nb, 2, 64), dtype=np.uint8)
    qh = np.zeros((nb, 2, 32), dtype=np.uint8)
    ql[:, :, 0:32] = (q[:, :, 0, :] & 15) | ((q[:, :, 2, :] & 15) << 4)
    ql[:, :, 32:64] = (q[:, :, 1, :] & 15) | ((q[:, :, 3, :] & 15) << 4)
    qh[:] = ((q[:, :, 0, :] >> 4) | ((q[:, :, 1, :] >> 4) << 2) | ((q[:, :, 2, :] >> 4) << 4)
             | ((q[:, :, 3, :] >> 4) << 6))
    out[:, 0:128] = ql.reshape(nb, 128)
    out[:, 128:192] = qh.reshape(nb, 64)
    out[:, 192:208] = sc.view(np.uint8)
    out[:, 208:210] = d.view(np.uint8).reshape(nb, 2)
    return out.reshape(rows, -1)


def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    """[rows, K] float -> [rows, K/32 * 34] uint8 (Q8_0 blocks)."""
    rows, k = w.shape
    x = w.reshape(-1, 32).astype(np.float32)
    nb = x.shape[0]
    d = _f16(np.abs(x).max(axis=-1) / 127.0)
    q = np.clip(np.rint(_safe_div(x, np.broadcast_to(d.astype(np.float32)[:, None], x.shape))), -127, 127)
    out = np.zeros((nb, 34), dtype=np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    out[:, 2:] = q.astype(np.int8).view(np.uint8)
    return out.reshape(rows, -1)


def to_bf16_bits(w: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (round to nearest even), as uint16."""
    u = np.ascontiguousarray(w, dtype=np.float32).view(np.uint32)
    rounded = u + 0x7FFF + ((u >> 16) & 1)
    return (rounded >> 16).astype(np.uint16)


QUANTIZERS = {Q4_K: quantize_q4_k, Q5_K: quantize_q5_k, Q6_K: quantize_q6_k, Q8_0: quantize_q8_0}


def quantize(w: np.ndarray, qtype: int) -> np.ndarray:
    """Quantize a [rows, K] float matrix into raw GGUF bytes of ``qtype``."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    if qtype == F32:
        return w
    if qtype == F16:
        return w.astype(np.float16)
    if qtype == BF16:
        return to_bf16_bits(w)
    be = BLOCK_ELEMS[qtype]
    if w.shape[-1] % be:
        raise ValueError(f"K={w.shape[-1]} is not a multiple of {be} for {TYPE_NAMES[qtype]}")
    return QUANTIZERS[qtype](w)


@dataclasses.dataclass(frozen=True)
class ModelSpec:
    """Shape of a synthetic Llama / Qwen2 model (the reference's GGUF metadata)."""

    arch: str  # "llama" or "qwen2"
    n_layers: int
    hidden: int
    n_heads: int
    n_kv_heads: int
    ffn: int
    vocab: int
    rope_theta: float
    ctx_len: int = 4096
    eps: float = 1e-5
    quant_mix: str = "Q4_K_M"

    @property
    def head_dim(self) -> int:
        return self.hidden // self.n_heads


# The configurations BASELINE.json names (shapes only; weights are synthetic).
QWEN25_05B = ModelSpec("qwen2", 24, 896, 14, 2, 4864, 151936, 1e6, 32768, 1e-6)
LLAMA3_8B = ModelSpec("llama", 32, 4096, 32, 8, 14336, 128256, 5e5, 8192, 1e-5)
LLAMA32_1B = ModelSpec("llama", 16, 2048, 32, 8, 8192, 128256, 5e5, 8192, 1e-5)
QWEN25_7B = ModelSpec("qwen2", 28, 3584, 28, 4, 18944, 152064, 1e6, 32768, 1e-6, quant_mix="Q5_K")


def tensor_qtype(spec: ModelSpec, name: str, k: int, layer: Optional[int]) -> int:
    """Quant type of one weight matrix under ``spec.quant_mix``."""
    mix = spec.quant_mix
    if mix == "BF16":
        return BF16
    if mix == "Q8_0":
        return Q8_0
    if name == "output.weight":
        base = Q6_K
    elif mix == "Q4_K_M":
        base = Q4_K
        if layer is not None and layer % 2 == 0 and (name.endswith("attn_v.weight") or name.endswith("ffn_down.weight")):
            base = Q6_K
    elif mix == "Q5_K":
        base = Q5_K
    else:
        raise ValueError(f"unknown quant mix {mix}")
    if k % 256:
        return Q8_0
    return base


def layer_tensor_shapes(spec: ModelSpec) -> List[Tuple[str, Tuple[int, int]]]:
    """(name suffix, (rows N, cols K)) of one transformer block's matrices."""
    hd = spec.head_dim
    return [
        ("attn_q.weight", (spec.n_heads * hd, spec.hidden)),
        ("attn_k.weight", (spec.n_kv_heads * hd, spec.hidden)),
        ("attn_v.weight", (spec.n_kv_heads * hd, spec.hidden)),
        ("attn_output.weight", (spec.hidden, spec.n_heads * hd)),
        ("ffn_gate.weight", (spec.ffn, spec.hidden)),
        ("ffn_up.weight", (spec.ffn, spec.hidden)),
        ("ffn_down.weight", (spec.hidden, spec.ffn)),
    ]


def synth_tensors(spec: ModelSpec, seed: int, sigma: float = 0.02) -> Dict[str, Tuple[np.ndarray, int]]:
    """All model tensors as name -> (raw GGUF data, ggml type), seeded.

    Weight matrices are N(0, sigma) (default 0.02) before quantization; norms
    1 + N(0, 0.02); Qwen2 q/k/v biases N(0, 0.02) in F32.
    """
    rng = np.random.default_rng(seed)
    out: Dict[str, Tuple[np.ndarray, int]] = {}

    def mat(name: str, shape: Tuple[int, int], layer: Optional[int]) -> None:
        w = rng.standard_normal(shape, dtype=np.float32) * np.float32(sigma)
        qt = tensor_qtype(spec, name, shape[1], layer)
        out[name] = (quantize(w, qt), qt)

    def vec(name: str, n: int, base: float) -> None:
        v = np.float32(base) + rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)
        out[name] = (v.astype(np.float32), F32)

    mat("token_embd.weight", (spec.vocab, spec.hidden), None)
    for i in range(spec.n_layers):
        vec(f"blk.{i}.attn_norm.weight", spec.hidden, 1.0)
        for suffix, shape in layer_tensor_shapes(spec):
            mat(f"blk.{i}.{suffix}", shape, i)
        if spec.arch == "qwen2":
            hd = spec.head_dim
            vec(f"blk.{i}.attn_q.bias", spec.n_heads * hd, 0.0)
            vec(f"blk.{i}.attn_k.bias", spec.n_kv_heads * hd, 0.0)
            vec(f"blk.{i}.attn_v.bias", spec.n_kv_heads * hd, 0.0)
        vec(f"blk.{i}.ffn_norm.weight", spec.hidden, 1.0)
    vec("output_norm.weight", spec.hidden, 1.0)
    mat("output.weight", (spec.vocab, spec.hidden), None)
    return out


def write_gguf(path: str, spec: ModelSpec, seed: int, rope_style: Optional[str] = None,
               llama3_scaling: bool = False, sigma: float = 0.02) -> Dict[str, Tuple[np.ndarray, int]]:
    """Write a synthetic GGUF for ``spec`` and return its tensors.

    ``rope_style="half"`` marks a Llama whose q/k use rotate-half RoPE (the
    layout of HF BF16 checkpoints read by crates/speculate/src/model/
    llama_local.rs); ``llama3_scaling`` records Llama-3.1 frequency scaling
    (factor 8, low 1, high 4, original context 8192; llama_local.rs:47-75).
    """
    tensors = synth_tensors(spec, seed, sigma)
    write_gguf_tensors(path, spec, tensors, seed, rope_style, llama3_scaling)
    return tensors


def device_synthetic_tensors(spec: ModelSpec, seed: int, device: int = 0, damp_from_layer: int = 0,
                             damp: float = 1.0) -> Dict[str, Tuple[np.ndarray, int]]:
    """The tensors of ``B200Decoder.synthetic(..., seed=seed)`` (spec_create_synthetic),
    rebuilt one by one with the same device generator, numbering and seeds
    (spec_synthetic_seed / spec_synthetic_tensor / spec_synthetic_vector), as
    name -> (raw GGUF data, ggml type).  Writing them with write_gguf_tensors
    gives a GGUF file holding exactly the weights the device model runs on."""
    import ctypes
    from . import _lib
    lib = _lib.load()
    out: Dict[str, Tuple[np.ndarray, int]] = {}
    counter = [0]

    def next_seed() -> int:
        counter[0] += 1
        return int(lib.spec_synthetic_seed(seed, counter[0]))

    def mat(name: str, rows: int, k: int, layer: Optional[int], sigma: float = 0.02) -> None:
        qt = tensor_qtype(spec, name, k, layer)
        nbytes = rows * (k // BLOCK_ELEMS[qt]) * BLOCK_BYTES[qt] if qt in BLOCK_ELEMS else rows * k * 2
        buf = np.empty(nbytes, dtype=np.uint8)
        _lib.check(lib.spec_synthetic_tensor(device, qt, rows, k, next_seed(), sigma, buf.ctypes.data, nbytes))
        if qt == BF16:
            out[name] = (buf.view(np.uint16).reshape(rows, k), qt)
        else:
            out[name] = (buf.reshape(rows, -1), qt)

    def vec(name: str, n: int, base: float) -> np.ndarray:
        v = np.empty(n, dtype=np.float32)
        _lib.check(lib.spec_synthetic_vector(device, n, next_seed(), base, 0.02,
                                             v.ctypes.data_as(ctypes.POINTER(ctypes.c_float))))
        if name:
            out[name] = (v, F32)
        return v

    hd = spec.head_dim
    vec("output_norm.weight", spec.hidden, 1.0)
    mat("token_embd.weight", spec.vocab, spec.hidden, None)
    mat("output.weight", spec.vocab, spec.hidden, None)
    damp_sigma = np.float32(0.02) * np.float32(int(round(damp * 10000))) / np.float32(10000)
    for i in range(spec.n_layers):
        for suffix, (rows, k) in layer_tensor_shapes(spec):
            damped = damp_from_layer > 0 and i >= damp_from_layer and suffix in ("attn_output.weight",
                                                                                 "ffn_down.weight")
            mat(f"blk.{i}.{suffix}", rows, k, i, float(damp_sigma) if damped else 0.02)
        vec(f"blk.{i}.attn_norm.weight", spec.hidden, 1.0)
        vec(f"blk.{i}.ffn_norm.weight", spec.hidden, 1.0)
        if spec.arch == "qwen2":
            b = vec("", (spec.n_heads + 2 * spec.n_kv_heads) * hd, 0.0)
            nq, nk = spec.n_heads * hd, spec.n_kv_heads * hd
            out[f"blk.{i}.attn_q.bias"] = (b[:nq].copy(), F32)
            out[f"blk.{i}.attn_k.bias"] = (b[nq:nq + nk].copy(), F32)
            out[f"blk.{i}.attn_v.bias"] = (b[nq + nk:].copy(), F32)
    return out


def write_device_synthetic_gguf(path: str, spec: ModelSpec, seed: int, device: int = 0,
                                rope_half: bool = False) -> Dict[str, Tuple[np.ndarray, int]]:
    """GGUF file of the device-synthesized model ``B200Decoder.synthetic(spec, seed)``
    (same RoPE style and, for BF16 Llama, the Llama-3.1 scaling that
    spec_create_synthetic applies)."""
    tensors = device_synthetic_tensors(spec, seed, device)
    bf16_llama = spec.quant_mix == "BF16" and spec.arch == "llama"
    rope_style = "half" if (spec.arch == "llama" and rope_half) else None
    write_gguf_tensors(path, spec, tensors, seed, rope_style, bf16_llama)
    return tensors


def write_gguf_tensors(path: str, spec: ModelSpec, tensors: Dict[str, Tuple[np.ndarray, int]], seed: int,
                       rope_style: Optional[str] = None, llama3_scaling: bool = False) -> None:
    """Write ``tensors`` (name -> (raw data, ggml type)) with the model metadata of ``spec``."""
    import gguf

    arch = spec.arch
    w = gguf.GGUFWriter(path, arch)
    w.add_uint32(f"{arch}.attention.head_count", spec.n_heads)
    w.add_uint32(f"{arch}.attention.head_count_kv", spec.n_kv_heads)
    w.add_uint32(f"{arch}.embedding_length", spec.hidden)
    w.add_uint32(f"{arch}.context_length", spec.ctx_len)
    w.add_uint32(f"{arch}.block_count", spec.n_layers)
    w.add_uint32(f"{arch}.feed_forward_length", spec.ffn)
    w.add_uint32(f"{arch}.rope.dimension_count", spec.head_dim)
    w.add_float32(f"{arch}.attention.layer_norm_rms_epsilon", spec.eps)
    w.add_float32(f"{arch}.rope.freq_base", spec.rope_theta)
    w.add_string("speculate_b200.quant_mix", spec.quant_mix)
    if rope_style:
        w.add_string("speculate_b200.rope_style", rope_style)
    if llama3_scaling:
        w.add_string(f"{arch}.rope.scaling.type", "llama3")
        w.add_float32(f"{arch}.rope.scaling.factor", 8.0)
        w.add_float32(f"{arch}.rope.scaling.low_freq_factor", 1.0)
        w.add_float32(f"{arch}.rope.scaling.high_freq_factor", 4.0)
        w.add_uint32(f"{arch}.rope.scaling.original_context_length", 8192)
    w.add_uint32("speculate_b200.seed", seed)
    w.add_array("tokenizer.ggml.tokens", [f"<t{i}>" for i in range(spec.vocab)])
    for name, (data, qt) in tensors.items():
        if qt in (F32, F16):
            w.add_tensor(name, data)
        elif qt == BF16:
            w.add_tensor(name, data.view(np.uint8).reshape(data.shape[0], -1),
                         raw_dtype=gguf.GGMLQuantizationType.BF16)
        else:
            w.add_tensor(name, data, raw_dtype=gguf.GGMLQuantizationType(qt))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def spec_to_json(spec: ModelSpec) -> str:
    return json.dumps(dataclasses.asdict(spec))
