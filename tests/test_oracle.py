"""CPU checks of the oracle (the C restatement in oracle/) -- no GPU needed.

The oracle is what the GPU parity tests compare against, so it is pinned first:
  * against the golden fixtures made by the reference library itself (tests/golden/), which hold
    for every seeded case the reference encoder's blob hash and the reference attention's output
    bits (scalar backend, and AVX2 where the generating host had it);
  * against the reference's own invariants (tests/test_main.cpp:54-172 of the reference):
    lossless round trip including signed zeros, subnormals, infinities and NaN; container sizes;
    an identity token whose output equals its V row exactly; raw and XKV inputs giving the same
    bits; and its argument and malformed-blob errors;
  * against the compiled reference directly, where oracle/_ref was built on this host.
"""
import base64
import hashlib
import json
import os
import struct

import numpy as np
import pytest

import oracle as O
from golden_cases import CASES, inputs
from helpers import XorShift32, make_bf16

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "golden.json")))


def _bits(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


def _golden_out(entry, tag, n_q, dim):
    return np.frombuffer(base64.b64decode(entry["out_" + tag]), dtype=np.float32).reshape(n_q, dim)


def _sizes(blob):
    """Walk the headers: (bytes per block, modes) -- include/kvexp/bf16.hpp:39-49 arithmetic."""
    sizes, modes, off = [], [], 0
    while off < blob.size:
        mode, nt, ne, hd, _ = struct.unpack_from("<BBHHH", blob, off)
        n = 8 + (2 * nt * hd if mode == 0 else hd + nt * hd + (nt * hd * mode + 7) // 8 + 2 * ne)
        sizes.append(n)
        modes.append(mode)
        off += n
    return sizes, modes


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_golden(oracle, name):
    c, g = CASES[name], GOLDEN["cases"][name]
    q, k, v = inputs(c)
    kx, vx = oracle.encode(k, c["block"]), oracle.encode(v, c["block"])
    assert kx.size == g["k_bytes"] and vx.size == g["v_bytes"]
    assert hashlib.sha256(kx.tobytes()).hexdigest() == g["k_sha256"], "encoder bytes differ"
    assert hashlib.sha256(vx.tobytes()).hexdigest() == g["v_sha256"], "encoder bytes differ"
    assert np.array_equal(oracle.decode(kx, c["seq"], c["dim"]), k)
    assert np.array_equal(oracle.decode(vx, c["seq"], c["dim"]), v)
    out = oracle.attention(q, kx=kx, vx=vx, seq=c["seq"], threads=1, split=c["block"])
    assert np.array_equal(_bits(out), _bits(_golden_out(g, "scalar_t1", c["n_q"], c["dim"])))
    if "out_scalar_t3" in g:
        out3 = oracle.attention(q, kx=kx, vx=vx, seq=c["seq"], threads=3, split=c["block"])
        assert np.array_equal(_bits(out3), _bits(_golden_out(g, "scalar_t3", c["n_q"], c["dim"])))


def test_golden_covers_every_block_mode():
    seen = {m: 0 for m in ("0", "2", "4")}
    for g in GOLDEN["cases"].values():
        for key in ("k_modes", "v_modes"):
            for m, n in g[key].items():
                seen[m] += n
    assert all(n > 0 for n in seen.values()), seen


@pytest.mark.parametrize("name", sorted(CASES))
def test_reference_reproduces_golden(reference, name):
    c, g = CASES[name], GOLDEN["cases"][name]
    q, k, v = inputs(c)
    kx = reference.encode(k, c["block"])
    assert hashlib.sha256(kx.tobytes()).hexdigest() == g["k_sha256"]
    vx = reference.encode(v, c["block"])
    out = reference.attention(q, kx=kx, vx=vx, seq=c["seq"], backend=O.SCALAR, threads=1,
                              split=c["block"])
    assert np.array_equal(_bits(out), _bits(_golden_out(g, "scalar_t1", c["n_q"], c["dim"])))


def _specials(seq, dim, seed=5):
    """Random BF16 bits plus every special class in each block: +-0, subnormals, +-inf, NaN."""
    rng = XorShift32(seed)
    x = np.array([make_bf16(100 + (rng() % 40), rng() & 0x7F, rng() & 1) for _ in range(seq * dim)],
                 dtype=np.uint16)
    specials = np.array([0x0000, 0x8000, 0x0001, 0x807F, 0x0040, 0x7F80, 0xFF80, 0x7FC0, 0xFFC1,
                         0x7F7F, 0xFF7F], dtype=np.uint16)
    for i in range(0, x.size, 97):
        x[i] = specials[(i // 97) % specials.size]
    return x.reshape(seq, dim)


@pytest.mark.parametrize("seq,dim,block", [(1, 4, 128), (17, 8, 16), (300, 64, 128),
                                           (256, 252, 255), (129, 128, 128), (5, 256, 1)])
def test_round_trip_specials_and_sizes(oracle, seq, dim, block):
    x = _specials(seq, dim)
    blob = oracle.encode(x, block)
    assert np.array_equal(oracle.decode(blob, seq, dim), x)
    sizes, modes = _sizes(blob)
    assert sum(sizes) == blob.size
    assert len(sizes) == (seq + block - 1) // block
    assert all(m in (0, 2, 4) for m in modes)


def test_identity_token_is_exact(oracle):
    """One token's score dominates every other by far: the output is its V row, bit for bit."""
    dim, seq, hot = 64, 300, 137
    rng = XorShift32(9)
    k = np.array([make_bf16(110 + (rng() % 8), rng() & 0x7F, rng() & 1) for _ in range(seq * dim)],
                 dtype=np.uint16).reshape(seq, dim)
    v = np.array([make_bf16(120 + (rng() % 8), rng() & 0x7F, rng() & 1) for _ in range(seq * dim)],
                 dtype=np.uint16).reshape(seq, dim)
    q = np.full((2, dim), make_bf16(133, 0, 0), dtype=np.uint16)  # 64.0
    k[hot] = make_bf16(133, 0, 0)
    kx, vx = oracle.encode(k, 128), oracle.encode(v, 128)
    out = oracle.attention(q, kx=kx, vx=vx, seq=seq)
    want = (v[hot].astype(np.uint32) << 16).view(np.float32)
    assert np.array_equal(_bits(out[0]), _bits(want)) and np.array_equal(_bits(out[1]), _bits(want))


@pytest.mark.parametrize("seq,dim,n_q,threads,split", [(1, 64, 1, 1, 128), (17, 64, 7, 1, 128),
                                                       (300, 64, 3, 4, 64), (90, 32, 2, 1, 32),
                                                       (700, 64, 7, 3, 128)])
def test_raw_and_xkv_give_the_same_bits(oracle, seq, dim, n_q, threads, split):
    rng = XorShift32(seq * 31 + dim)
    k = np.array([make_bf16(108 + (rng() % 8), rng() & 0x7F, rng() & 1) for _ in range(seq * dim)],
                 dtype=np.uint16).reshape(seq, dim)
    v = np.array([make_bf16(112 + (rng() % 5), rng() & 0x7F, rng() & 1) for _ in range(seq * dim)],
                 dtype=np.uint16).reshape(seq, dim)
    q = np.array([make_bf16(120, rng() & 0x7F, rng() & 1) for _ in range(n_q * dim)],
                 dtype=np.uint16).reshape(n_q, dim)
    kx, vx = oracle.encode(k, split), oracle.encode(v, split)
    a = oracle.attention(q, k=k, v=v, seq=seq, threads=threads, split=split)
    b = oracle.attention(q, kx=kx, vx=vx, seq=seq, threads=threads, split=split)
    assert np.array_equal(_bits(a), _bits(b))


@pytest.mark.parametrize("seq,dim,block", [(0, 64, 128), (16, 6, 128), (16, 260, 128),
                                           (16, 64, 256), (16, 64, 0)])
def test_encoder_argument_errors(oracle, reference_or_none, seq, dim, block):
    x = np.zeros((max(seq, 1), dim), dtype=np.uint16)
    with pytest.raises(O.OracleError) as e:
        oracle.encode_raw_args(x.ctypes.data_as(O._u16p), seq, dim, block)
    assert e.value.code == 1  # std::invalid_argument
    if reference_or_none is not None:
        with pytest.raises(O.OracleError) as r:
            reference_or_none.encode(x[:max(seq, 1)] if seq else x[:0].reshape(0, dim), block)
        assert r.value.code == e.value.code


def test_malformed_blob_errors(oracle):
    k = _specials(256, 64)
    blob = oracle.encode(k, 128)
    with pytest.raises(O.OracleError, match="truncated"):
        oracle.decode(blob[:blob.size - 3], 256, 64)
    with pytest.raises(O.OracleError, match="ran out of blocks"):
        oracle.decode(blob[:_sizes(blob)[0][0]], 256, 64)
    bad = blob.copy()
    bad[0] = 5  # mode byte of the first header (3 is the library's 3-bit extension)
    with pytest.raises(O.OracleError, match="unknown xkv block mode"):
        oracle.decode(bad, 256, 64)


def test_split_must_align_with_blocks(oracle):
    q = np.full((1, 64), make_bf16(120, 0, 0), dtype=np.uint16)
    k = _specials(256, 64)
    kx = oracle.encode(k, 128)
    with pytest.raises(O.OracleError, match="not aligned"):
        oracle.attention(q, kx=kx, vx=kx, seq=256, threads=2, split=96)


def test_reference_error_grows_with_length(oracle):
    """The reference's scalar kernel (which the oracle restates bit for bit) adds every token into
    fp32 running sums in turn, so its own error against the float64 softmax grows with the
    sequence: at 32K tokens with a flat softmax it is about 20 times the GPU tolerance
    (oracle/parity.py).  This is why the GPU is checked against the float64 truth, and against the
    reference within the reference's own error."""
    import synth as S
    from helpers import soften
    from parity import ATOL, truth_and_scale
    errs = []
    for seq in (1024, 8192, 32768):
        k = S.synth_bf16(31, 0, seq, 64, S.PROFILE_K)
        v = S.synth_bf16(31, 1, seq, 64, S.PROFILE_V)
        q = soften(S.synth_bf16(31, 2, 7, 64, S.PROFILE_Q), 8)
        out = oracle.attention(q, kx=oracle.encode(k, 128), vx=oracle.encode(v, 128), seq=seq)
        ex = truth_and_scale(q, k, v)
        errs.append(float(np.max(np.abs(out - ex.truth) / ex.scale)))
    assert errs[0] < errs[1] < errs[2], errs
    assert errs[2] > 5 * ATOL, errs
