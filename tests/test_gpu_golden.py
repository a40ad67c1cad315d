"""GPU path against the fixtures the reference itself produced (tests/golden/golden.json).

No oracle is involved: the expected blob hashes and attention outputs were written by the
reference library (kvexp, compiled from its sources) through tests/golden/make_golden.py, with
softened queries so that the softmax spreads over many tokens.  Per case:
  * the GPU encoder writes the reference's bytes (same length and SHA-256), and the GPU decoder
    returns the input bits;
  * GPU attention over the XKV blobs is bit-identical to the GPU's BF16-input kernel, within the
    tight tolerance of the float64 truth, and within the reference's own error (plus that
    tolerance) of the reference's scalar output (1 thread), of its AVX2 output, and of its
    3-thread output where the fixture has one (the GPU then runs the same call with
    n_threads=3, which the reference's split rule must accept).
"""
import base64
import hashlib
import json
import os

import numpy as np
import pytest

from golden_cases import CASES, inputs
from helpers import assert_attention_close, truth_and_scale

pytestmark = pytest.mark.gpu

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "golden.json")))


def _golden_out(entry, tag, n_q, dim):
    return np.frombuffer(base64.b64decode(entry["out_" + tag]), dtype=np.float32).reshape(n_q, dim)


def _gpu(kvx, q, seq, kx=None, vx=None, k=None, v=None, threads=1, split=128):
    n_q, dim = q.shape
    out = np.zeros((n_q, dim), dtype=np.float32)
    kvx.attention_decode(0, q, k, v, kx, 0 if kx is None else kx.size, vx,
                         0 if vx is None else vx.size, out, n_q, dim, seq, threads, split)
    return out


@pytest.mark.parametrize("name", sorted(CASES))
def test_codec_matches_reference_fixture(kvx, cuda, name):
    c, g = CASES[name], GOLDEN["cases"][name]
    _, k, v = inputs(c)
    for t, key in ((k, "k"), (v, "v")):
        enc = kvx.encode_bf16(t, c["seq"], c["dim"], c["block"]).bytes
        assert enc.size == g[key + "_bytes"]
        assert hashlib.sha256(enc.tobytes()).hexdigest() == g[key + "_sha256"]
        back = np.zeros_like(t)
        kvx.decode_bf16(enc, enc.size, c["seq"], c["dim"], back)
        assert np.array_equal(back, t)


@pytest.mark.parametrize("name", sorted(CASES))
def test_attention_matches_reference_fixture(kvx, cuda, name):
    c, g = CASES[name], GOLDEN["cases"][name]
    q, k, v = inputs(c)
    seq, dim, n_q, block = c["seq"], c["dim"], c["n_q"], c["block"]
    kx = kvx.encode_bf16(k, seq, dim, block).bytes
    vx = kvx.encode_bf16(v, seq, dim, block).bytes
    truth = truth_and_scale(q, k, v)
    got = _gpu(kvx, q, seq, kx=kx, vx=vx, split=block)
    raw = _gpu(kvx, q, seq, k=k, v=v, split=block)
    assert np.array_equal(got.view(np.uint32), raw.view(np.uint32)), "XKV and BF16 GPU outputs differ"
    assert_attention_close(got, _golden_out(g, "scalar_t1", n_q, dim),
                           what=f"{name} vs reference scalar", truth=truth)
    if "out_avx2_t1" in g:
        assert_attention_close(got, _golden_out(g, "avx2_t1", n_q, dim),
                               what=f"{name} vs reference AVX2", truth=truth)
    if "out_scalar_t3" in g:
        got3 = _gpu(kvx, q, seq, kx=kx, vx=vx, threads=3, split=block)
        assert_attention_close(got3, _golden_out(g, "scalar_t3", n_q, dim),
                               what=f"{name} vs reference scalar, 3 threads", truth=truth)
