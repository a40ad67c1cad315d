"""Exponent statistics on the GPU (kvx_exponent_stats) and the analyser report built on them.

The checker is a plain numpy restatement of the reference analyser's per-block statistics
(python/analyze_exponents.py:57-72 `block_conditional_entropy`, :117-156 `policy_size`): for each
block and head dim, the best count of exponents in a window of 3, 7 or 15 consecutive values
and the Shannon entropy of the exponents.  The report restricted to 2- and 4-bit codes must also
give exactly the size of the container the (byte-exact) encoder writes."""
import numpy as np
import pytest

import synth as S

pytestmark = pytest.mark.gpu


def _np_stats(x, bt):
    seq, dim = x.shape
    e = (x.astype(np.int64) >> 7) & 0xFF
    nb = (seq + bt - 1) // bt
    best = np.zeros((3, nb, dim), dtype=np.int64)
    ent = np.zeros((nb, dim), dtype=np.float64)
    for b in range(nb):
        piece = e[b * bt:(b + 1) * bt]
        n = piece.shape[0]
        for d in range(dim):
            h = np.bincount(piece[:, d], minlength=256)
            c = np.concatenate([[0], np.cumsum(h)])
            for wi, w in enumerate((3, 7, 15)):
                best[wi, b, d] = int(np.max(c[w:] - c[:-w]))
            p = h[h > 0] / n
            ent[b, d] = float(-(p * np.log2(p)).sum())
    return best, ent


CASES = [
    (64, 1000, 128, S.PROFILE_K),      # tail block of 104 tokens
    (128, 512, 128, S.PROFILE_V),
    (40, 300, 64, S.PROFILE_NARROW),   # head_dim not a multiple of 32
    (256, 256, 255, S.PROFILE_WIDE_K),
]


@pytest.mark.parametrize("dim,seq,bt,profile", CASES)
def test_stats_match_numpy(kvx, cuda, dim, seq, bt, profile):
    x = S.synth_bf16(5, 3, seq, dim, profile)
    best, ent = kvx.exponent_stats(x, seq, dim, bt)
    rb, re = _np_stats(x, bt)
    assert np.array_equal(best, rb)
    assert np.max(np.abs(ent - re)) < 1e-5


@pytest.mark.parametrize("dim,seq,bt,profile", CASES)
def test_report_matches_encoder_size(kvx, cuda, dim, seq, bt, profile):
    x = S.synth_bf16(6, 4, seq, dim, profile)
    rep = kvx.exponent_report(x, seq, dim, bt, bit_widths=(2, 4))
    enc = kvx.encode_bf16(x, seq, dim, bt)
    assert rep["container_bytes"] == enc.bytes.size
    assert rep["tight_bytes"] == 2 * seq * dim
    # every block the encoder wrote carries the mode the report chose for it (header walk:
    # u8 mode, u8 tokens, u16 escapes; sections as in include/kvexp/codec.hpp)
    b = enc.bytes.tobytes()
    off, modes = 0, {}
    while off < len(b):
        mode, nt = b[off], b[off + 1]
        ne = int.from_bytes(b[off + 2:off + 4], "little")
        modes[str(mode)] = modes.get(str(mode), 0) + 1
        off += 8 + 2 * nt * dim if mode == 0 else 8 + dim + nt * dim + (nt * dim * mode + 7) // 8 + 2 * ne
    assert off == len(b)
    assert modes == rep["mode_blocks"]


def test_report_entropy_and_three_bit(kvx, cuda):
    dim, seq, bt = 64, 1000, 128
    x = S.synth_bf16(7, 5, seq, dim, S.PROFILE_K)
    rep = kvx.exponent_report(x, seq, dim, bt)
    _, re = _np_stats(x, bt)
    assert abs(rep["block_conditional_entropy"] - re[: seq // bt].mean()) < 1e-5
    # allowing 3-bit codes never makes the container larger
    assert rep["container_bytes"] <= kvx.exponent_report(x, seq, dim, bt, (2, 4))["container_bytes"]
    assert 0.0 <= rep["escape_rate"] <= 1.0 and 0.0 <= rep["coded_element_fraction"] <= 1.0
