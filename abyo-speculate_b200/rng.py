"""The reference's seeded RNG stream, restated: rand 0.8 ``StdRng``.

The reference seeds its sampling RNG with ``StdRng::seed_from_u64(seed)``
(crates/speculate/src/engine.rs:320-326) and draws uniforms with
``rng.gen::<f32>()`` (sampling/tokens.rs:99-120, methods/vanilla.rs:297-343).
The crates are third-party and not vendored: rand 0.8.6 / rand_core 0.6 /
rand_chacha 0.3.1 (Cargo.lock:2285-2308).  Their published algorithms:

* ``StdRng`` is ``ChaCha12Rng``: the ChaCha stream cipher with 12 rounds
  (6 double rounds), key = the 32-byte seed, a 64-bit block counter starting
  at 0 in state words 12-13 and a 64-bit stream id 0 in words 14-15.  Output
  words are the blocks' 16 little-endian words in order, block after block
  (rand_chacha buffers four blocks at a time; the order is the same).
* ``seed_from_u64(state)`` (rand_core 0.6 ``SeedableRng``) fills the 32-byte
  seed with eight PCG32 outputs: state = state * 6364136223846793005 +
  11634580027462260723 (mod 2^64), then x = rotr32(((state >> 18) ^ state)
  >> 27, state >> 59), stored little-endian.
* ``gen::<f32>()`` (rand 0.8 ``Standard``) takes one ``next_u32`` and keeps
  its top 24 bits: (x >> 8) * 2^-24, in [0, 1).

The block function is checked against the published ChaCha20 test vectors
(tests/test_rng.py); the 12-round stream uses the same code.  This is host
code of the SD loop (it produces the uniforms the device rejection round
consumes), not part of the verify kernels.
"""

from __future__ import annotations

from typing import List

import numpy as np

_MASK32 = 0xFFFFFFFF
_SIGMA = (0x61707865, 0x3320646E, 0x79622D32, 0x6B206574)  # "expand 32-byte k"


def _rotl(x: np.ndarray, n: int) -> np.ndarray:
    return ((x << np.uint32(n)) | (x >> np.uint32(32 - n))).astype(np.uint32)


def chacha_blocks(key_words: List[int], counter: int, nonce_words: List[int], rounds: int, n_blocks: int,
                  nonce96: bool = False) -> np.ndarray:
    """``n_blocks`` ChaCha blocks (uint32 words, [n_blocks][16]) from block
    ``counter``.  Default layout (rand_chacha, original ChaCha): a 64-bit
    counter in words 12-13 and a 64-bit nonce in words 14-15.  ``nonce96``:
    the RFC 7539 layout, a 32-bit counter in word 12 and a 96-bit nonce."""
    if rounds % 2:
        raise ValueError("rounds must be even")
    st = np.zeros((16, n_blocks), dtype=np.uint32)
    for i in range(4):
        st[i] = _SIGMA[i]
    for i in range(8):
        st[4 + i] = key_words[i] & _MASK32
    ctr = np.arange(counter, counter + n_blocks, dtype=np.uint64)
    if nonce96:
        st[12] = (ctr & np.uint64(_MASK32)).astype(np.uint32)
        for i in range(3):
            st[13 + i] = nonce_words[i] & _MASK32
    else:
        st[12] = (ctr & np.uint64(_MASK32)).astype(np.uint32)
        st[13] = (ctr >> np.uint64(32)).astype(np.uint32)
        st[14] = nonce_words[0] & _MASK32
        st[15] = nonce_words[1] & _MASK32
    x = st.copy()

    def qr(a, b, c, d):
        x[a] = x[a] + x[b]
        x[d] = _rotl(x[d] ^ x[a], 16)
        x[c] = x[c] + x[d]
        x[b] = _rotl(x[b] ^ x[c], 12)
        x[a] = x[a] + x[b]
        x[d] = _rotl(x[d] ^ x[a], 8)
        x[c] = x[c] + x[d]
        x[b] = _rotl(x[b] ^ x[c], 7)

    with np.errstate(over="ignore"):
        for _ in range(rounds // 2):
            qr(0, 4, 8, 12)
            qr(1, 5, 9, 13)
            qr(2, 6, 10, 14)
            qr(3, 7, 11, 15)
            qr(0, 5, 10, 15)
            qr(1, 6, 11, 12)
            qr(2, 7, 8, 13)
            qr(3, 4, 9, 14)
        out = (x + st).astype(np.uint32)
    return out.T.copy()


def quarter_round(a: int, b: int, c: int, d: int):
    """One ChaCha quarter round on four 32-bit words (for the RFC 7539 2.1.1 check)."""
    x = np.array([a, b, c, d], dtype=np.uint32).reshape(4, 1)
    with np.errstate(over="ignore"):
        x[0] = x[0] + x[1]
        x[3] = _rotl(x[3] ^ x[0], 16)
        x[2] = x[2] + x[3]
        x[1] = _rotl(x[1] ^ x[2], 12)
        x[0] = x[0] + x[1]
        x[3] = _rotl(x[3] ^ x[0], 8)
        x[2] = x[2] + x[3]
        x[1] = _rotl(x[1] ^ x[2], 7)
    return tuple(int(v) for v in x[:, 0])


def pcg32_seed(state: int) -> bytes:
    """rand_core 0.6 ``seed_from_u64``: the 32-byte seed from eight PCG32 outputs."""
    mul, inc = 6364136223846793005, 11634580027462260723
    out = bytearray()
    for _ in range(8):
        state = (state * mul + inc) & 0xFFFFFFFFFFFFFFFF
        xorshifted = (((state >> 18) ^ state) >> 27) & _MASK32
        rot = state >> 59
        x = ((xorshifted >> rot) | (xorshifted << ((32 - rot) & 31))) & _MASK32
        out += x.to_bytes(4, "little")
    return bytes(out)


class StdRng:
    """rand 0.8 ``StdRng`` (ChaCha12) seeded like ``StdRng::seed_from_u64``.

    ``next_u32`` / ``gen_f32`` advance the stream; ``peek_f32(n)`` returns the
    next ``n`` ``gen::<f32>()`` values without consuming them, and
    ``advance(n)`` consumes them (the device rejection round reports how many
    uniforms it used)."""

    ROUNDS = 12

    def __init__(self, seed: int = 0, key: bytes = None, rounds: int = ROUNDS):
        key = key if key is not None else pcg32_seed(seed & 0xFFFFFFFFFFFFFFFF)
        if len(key) != 32:
            raise ValueError("key must be 32 bytes")
        self._key = [int.from_bytes(key[4 * i:4 * i + 4], "little") for i in range(8)]
        self._rounds = rounds
        self._block = 0
        self._buf = np.zeros(0, dtype=np.uint32)
        self._pos = 0

    def _fill(self, need: int) -> None:
        while len(self._buf) - self._pos < need:
            blocks = chacha_blocks(self._key, self._block, [0, 0], self._rounds, 4).reshape(-1)
            self._block += 4
            self._buf = np.concatenate([self._buf[self._pos:], blocks])
            self._pos = 0

    def next_u32(self) -> int:
        self._fill(1)
        v = int(self._buf[self._pos])
        self._pos += 1
        return v

    def peek_u32(self, n: int) -> np.ndarray:
        self._fill(n)
        return self._buf[self._pos:self._pos + n].copy()

    def advance(self, n: int) -> None:
        self._fill(n)
        self._pos += n

    @staticmethod
    def to_f32(words: np.ndarray) -> np.ndarray:
        """rand 0.8 ``Standard`` f32: the top 24 bits scaled by 2^-24."""
        return ((np.asarray(words, dtype=np.uint32) >> np.uint32(8)).astype(np.float32)
                * np.float32(1.0 / (1 << 24))).astype(np.float32)

    def gen_f32(self) -> float:
        return float(self.to_f32(np.array([self.next_u32()], dtype=np.uint32))[0])

    def peek_f32(self, n: int) -> np.ndarray:
        return self.to_f32(self.peek_u32(n))
