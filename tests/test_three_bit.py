"""CPU checks of the 3-bit residual mode (mode byte 3), this library's extension of the container.

The reference implements raw, 2-bit and 4-bit blocks; its README (README.md:35, :200) measured a
3-bit residual (ratio 0.712120 at block 128) without implementing it.  Here the oracle's 3-bit
encoder is pinned to the reference's own exponent analyser (python/analyze_exponents.py
`policy_size` over {raw, 2, 3, 4}; fixtures in tests/golden/golden_3bit.json, made by
tests/golden/make_golden_3bit.py), and its layout, round trip and the reference's raw == XKV
invariant are checked directly.  The default mode mask stays the reference's {2, 4}.
"""
import json
import os
import struct

import numpy as np
import pytest

import oracle as O
import synth as S
from golden_cases import CASES, inputs
from helpers import make_bf16, mixed_modes

G3 = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "golden_3bit.json")))
ALL = (2, 3, 4)


def payload(nt, hd, mode):
    """Residual code bytes of a coded block: the reference's formula for 2 and 4 bits; for 3 bits
    3 nt hd / 8 rounded up to an even count."""
    if mode == 3:
        return (nt * hd * 3 + 15) // 16 * 2
    return (nt * hd * mode + 7) // 8


def walk(blob):
    """(mode, n_tokens, n_escape, block bytes) per block header."""
    out, off = [], 0
    while off < blob.size:
        mode, nt, ne, hd, _ = struct.unpack_from("<BBHHH", blob, off)
        n = 8 + (2 * nt * hd if mode == 0 else hd + nt * hd + payload(nt, hd, mode) + 2 * ne)
        out.append((mode, nt, ne, n))
        off += n
    assert off == blob.size
    return out


def _check(blob, g):
    hdr = walk(blob)
    assert blob.size == g["container_bytes"]
    assert sum(ne for m, _, ne, _ in hdr if m) == g["escapes"]
    assert {str(m): sum(1 for h in hdr if h[0] == m) for m in (0, 2, 3, 4)} == g["mode_blocks"]


@pytest.mark.parametrize("name", sorted(G3["cases"]))
def test_sizes_match_reference_analyser(oracle, name):
    g = G3["cases"][name]
    if g["kind"] == "case":
        c = CASES[name]
        _, k, v = inputs(c)
        _check(oracle.encode(k, c["block"], code_bits=ALL), g["k"])
        _check(oracle.encode(v, c["block"], code_bits=ALL), g["v"])
    else:
        t = S.synth_bf16(g["seed"], g["stream"], g["seq"], g["dim"], g["profile"])
        _check(oracle.encode(t, g["block"], code_bits=ALL), g["t"])


def test_config1_ratio_drops(oracle):
    """On a config[1]-shaped tensor the {2, 3, 4} policy shrinks the container against {2, 4}
    (the reference README's 0.7536 -> 0.7121 on real activations goes the same way)."""
    g = G3["cases"]["c1_k_s16384"]
    t = S.synth_bf16(g["seed"], g["stream"], g["seq"], g["dim"], g["profile"])
    r24 = oracle.encode(t, 128).size / t.nbytes
    r234 = oracle.encode(t, 128, code_bits=ALL).size / t.nbytes
    assert r234 < r24 - 0.02, (r24, r234)


@pytest.mark.parametrize("seq,dim,block", [(1, 4, 128), (3, 4, 1), (3, 8, 1), (17, 12, 16),
                                           (512, 64, 128), (300, 128, 128), (256, 252, 255),
                                           (640, 256, 128)])
def test_round_trip_every_mode(oracle, seq, dim, block):
    x = mixed_modes(seq, dim, block, seed=seq + dim)
    blob = oracle.encode(x, block, code_bits=ALL)
    assert np.array_equal(oracle.decode(blob, seq, dim), x)
    hdr = walk(blob)
    assert len(hdr) == (seq + block - 1) // block
    assert all(m in (0, 2, 3, 4) for m, *_ in hdr)
    # the default mask is the reference encoder's: never a 3-bit block
    assert all(m in (0, 2, 4) for m, *_ in walk(oracle.encode(x, block)))


def test_mixed_blob_holds_every_mode(oracle):
    x = mixed_modes(1024, 64, 128)
    modes = [m for m, *_ in walk(oracle.encode(x, 128, code_bits=ALL))]
    assert set(modes) == {0, 2, 3, 4}, modes


def test_layout_and_padding(oracle):
    """Element i's code sits in bits [3 i, 3 i + 3) of the code bytes; the code section is padded
    to an even length when 3 n dim / 8 is odd."""
    dim, nt = 8, 16
    # token t: exponent 110 + t mod 7 in every dim (base 110, code t mod 7), except one escape
    e = np.array([[110 + t % 7] * dim for t in range(nt)])
    e[0, 5] = 150
    x = np.array([[make_bf16(int(e[t, d]), 3 * d + t, (t + d) & 1) for d in range(dim)]
                  for t in range(nt)], dtype=np.uint16)
    blob = oracle.encode(x, nt, code_bits=ALL)
    (mode, n, ne, size), = walk(blob)
    assert (mode, n, ne) == (3, nt, 1)
    assert np.all(blob[8:8 + dim] == 110)
    codes = blob[8 + dim + nt * dim: 8 + dim + nt * dim + payload(nt, dim, 3)]
    assert codes.size == 48
    bits = int.from_bytes(codes.tobytes(), "little")
    for i in range(nt * dim):
        t, d = divmod(i, dim)
        assert (bits >> (3 * i)) & 7 == (7 if (t, d) == (0, 5) else t % 7), i
    esc = blob[8 + dim + nt * dim + 48:]
    assert esc.size == 2 and int(esc.view("<u2")[0]) == int(x[0, 5])
    # three tokens of 8 dims: 72 code bits = 9 bytes, stored as 10
    y = np.array([[make_bf16(110 + 2 * t, d, 0) for d in range(dim)] for t in range(3)],
                 dtype=np.uint16)
    blob = oracle.encode(y, 3, code_bits=ALL)
    (mode, n, ne, size), = walk(blob)
    assert (mode, n, ne, size) == (3, 3, 0, 8 + dim + 3 * dim + 10)
    assert blob[-1] == 0
    assert np.array_equal(oracle.decode(blob, 3, dim), y)


def test_raw_and_3bit_inputs_give_same_bits(oracle):
    """The reference's raw == XKV invariant (tests/test_main.cpp:124-157) with 3-bit blocks."""
    c = CASES["c0_d64_s1000"]
    q, k, v = inputs(c)
    kx, vx = oracle.encode(k, 128, code_bits=ALL), oracle.encode(v, 128, code_bits=ALL)
    assert {m for m, *_ in walk(kx)} == {3}
    for threads in (1, 4):
        a = oracle.attention(q, kx=kx, vx=vx, seq=c["seq"], threads=threads)
        b = oracle.attention(q, k=k, v=v, seq=c["seq"], threads=threads)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_mode_mask_is_checked(oracle):
    x = mixed_modes(64, 8, 64)
    with pytest.raises(O.OracleError, match="mode mask"):
        oracle.encode(x, 64, code_bits=(3,))
    with pytest.raises(O.OracleError, match="mode mask"):
        oracle.encode(x, 64, code_bits=(2, 4, 5))


def test_unknown_mode_still_rejected(oracle):
    blob = oracle.encode(mixed_modes(256, 64, 128), 128, code_bits=ALL)
    bad = blob.copy()
    bad[0] = 5
    with pytest.raises(O.OracleError, match="unknown xkv block mode"):
        oracle.decode(bad, 256, 64)
