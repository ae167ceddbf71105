"""The restated rand 0.8 StdRng (abyo-speculate_b200/rng.py) against published vectors (CPU).

* RFC 7539 2.1.1: one ChaCha quarter round.
* ChaCha20 with an all-zero key, nonce and counter (the first test vector of
  RFC 7539 A.1, also rand_chacha's own `test_chacha_true_values_a`): the
  first 64 keystream bytes.  The 12-round StdRng stream runs the same code
  with fewer rounds.
* rand 0.8 `gen::<f32>()`: top 24 bits x 2^-24, in [0, 1).
"""

import importlib

import numpy as np


def _rng():
    return importlib.import_module("abyo-speculate_b200.rng")


def test_quarter_round_rfc7539():
    r = _rng()
    assert r.quarter_round(0x11111111, 0x01020304, 0x9B8D6F43, 0x01234567) == (
        0xEA2A92F4, 0xCB1CF8CE, 0x4581472E, 0x5881C4BB)


def test_chacha20_zero_key_block():
    r = _rng()
    words = r.chacha_blocks([0] * 8, 0, [0, 0], 20, 1)[0]
    got = words.astype("<u4").tobytes().hex()
    want = ("76b8e0ada0f13d90405d6ae55386bd28bdd219b8a08ded1aa836efcc8b770dc7"
            "da41597c5157488d7724e03fb8d84a376a43b8f41518a11cc387b669b2ee6586")
    assert got == want
    # The 96-bit-nonce layout gives the same block for a zero nonce and counter.
    words96 = r.chacha_blocks([0] * 8, 0, [0, 0, 0], 20, 1, nonce96=True)[0]
    assert np.array_equal(words, words96)


def test_stream_is_blocks_in_order_and_f32_conversion():
    r = _rng()
    key = bytes(range(32))
    g = r.StdRng(key=key)
    words = [g.next_u32() for _ in range(100)]
    kw = [int.from_bytes(key[4 * i:4 * i + 4], "little") for i in range(8)]
    want = r.chacha_blocks(kw, 0, [0, 0], 12, 7).reshape(-1)[:100]
    assert words == [int(w) for w in want]
    g2 = r.StdRng(key=key)
    peek = g2.peek_f32(5)
    assert np.array_equal(peek, r.StdRng.to_f32(np.array(words[:5], dtype=np.uint32)))
    g2.advance(3)
    assert g2.next_u32() == words[3]
    f = r.StdRng.to_f32(np.array([0, 0xFFFFFFFF, 0x80000000], dtype=np.uint32))
    assert f[0] == 0.0 and f[1] == np.float32(1 - 2.0 ** -24) and f[2] == 0.5


def test_seed_from_u64_pcg32_fill():
    """rand_core 0.6 seed_from_u64: eight PCG32 outputs (restated step by step here)."""
    r = _rng()
    state = 42
    words = []
    for _ in range(8):
        state = (state * 6364136223846793005 + 11634580027462260723) % (1 << 64)
        xs = (((state >> 18) ^ state) >> 27) & 0xFFFFFFFF
        rot = state >> 59
        words.append(((xs >> rot) | (xs << (32 - rot))) & 0xFFFFFFFF if rot else xs)
    assert r.pcg32_seed(42) == b"".join(w.to_bytes(4, "little") for w in words)
    a, b = r.StdRng(42), r.StdRng(42)
    assert [a.next_u32() for _ in range(70)] == [b.next_u32() for _ in range(70)]
    assert r.StdRng(43).next_u32() != r.StdRng(42).next_u32()


def test_library_stream_equals_restatement(pkg):
    """spec_rng (the C++ stream spec_sd_sampled_round draws from) gives the
    same gen::<f32>() values as rng.StdRng for several seeds, across the
    four-block refills."""
    sd = importlib.import_module("abyo-speculate_b200.sd_loop")
    for seed in (0, 7, 42, 2**63 + 12345):
        want = _rng().StdRng(seed).peek_f32(300)
        r = sd.NativeRng(seed)
        got = np.concatenate([r.next_f32(1), r.next_f32(63), r.next_f32(236)])
        r.close()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), seed
