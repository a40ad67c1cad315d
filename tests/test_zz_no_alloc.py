"""The allocation-free decode entry point (kvx_attention_decode_noalloc), through the C ABI.

Some callers cannot allocate GPU memory while they run -- serving engines that reserve the
device's memory for their KV-cache pool at start-up, and decode loops that cannot take the
device-wide stall of cudaFree.  This entry point keeps all of its scratch in one fixed device
array inside the library.  The tests check two calls in a row (the second finds the first call's
scratch contents) against the ordinary entry point kvx_attention_decode and against the scalar
oracle directly, with the same float64-anchored tolerance as the other attention tests,
including calls with more blocks than the grid has CTAs (then the entry point splits the blocks
evenly over its CTA ranges, and every range holds several).  The file is named so that pytest collects it
last.
"""
import numpy as np
import pytest

import synth as S
from helpers import assert_attention_close, soften, truth_and_scale

pytestmark = pytest.mark.gpu


def _case(dim, n_q, seq, seed):
    k = S.synth_bf16(seed, 0, seq, dim, S.PROFILE_K)
    v = S.synth_bf16(seed, 1, seq, dim, S.PROFILE_V)
    q = soften(S.synth_bf16(seed, 2, n_q, dim, S.PROFILE_Q), 8)
    return q, k, v


def _device_index(kvx, torch, blob, dim):
    """Device copy of an XKV blob and its device block index."""
    d = torch.from_numpy(blob).cuda()
    idx = torch.empty((blob.size // 8 + 16) * 8, dtype=torch.uint8, device="cuda")
    nb, _ = kvx.xkv_index(d, blob.size, dim, idx, idx.numel() // 8)
    return d, idx, nb


@pytest.mark.parametrize("cases", [
    [(64, 7, 3000, 11), (64, 7, 3000, 12)],     # same shape twice, new data
    [(128, 12, 5000, 13), (64, 3, 700, 14)],    # shape changes between the calls
    # more blocks than CTAs: 2048 blocks at D=64 (an even split over 148 ranges), then 2 query
    # groups x 600 blocks at D=256 (the partial states then cap the ranges below one per SM), and
    # back
    [(64, 7, 2048 * 128, 16), (256, 12, 600 * 128, 17), (64, 7, 2048 * 128 - 37, 18)],
])
def test_noalloc_matches_attention_decode(kvx, cuda, oracle, cases):
    torch = cuda
    for dim, n_q, seq, seed in cases:
        q, k, v = _case(dim, n_q, seq, seed)
        kx, vx = oracle.encode(k, 128), oracle.encode(v, 128)
        want = np.zeros((n_q, dim), dtype=np.float32)
        kvx.attention_decode(0, q, None, None, kx, kx.size, vx, vx.size, want, n_q, dim, seq, 1,
                             128)
        kd, kidx, nb = _device_index(kvx, torch, kx, dim)
        vd, vidx, nbv = _device_index(kvx, torch, vx, dim)
        assert nb == nbv
        qd = torch.from_numpy(q.view(np.int16)).cuda()
        out = torch.full((n_q, dim), float("nan"), dtype=torch.float32, device="cuda")
        kvx.attention_decode_noalloc(qd, kd, kx.size, kidx, vd, vx.size, vidx, nb, out, n_q, dim,
                                     seq)
        got = out.cpu().numpy()
        assert np.all(np.isfinite(got))
        truth = truth_and_scale(q, k, v)
        assert_attention_close(got, want, what=f"noalloc vs attention_decode dim={dim} "
                               f"n_q={n_q} seq={seq}", truth=truth)
        assert_attention_close(got, oracle.attention(q, kx=kx, vx=vx, seq=seq),
                               what=f"noalloc vs oracle dim={dim} n_q={n_q} seq={seq}", truth=truth)


def test_noalloc_rejects_oversize(kvx, cuda):
    torch = cuda
    z = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    q = torch.zeros((4, 64), dtype=torch.int16, device="cuda")
    out = torch.zeros((4, 64), dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError, match="8192 blocks"):
        kvx.attention_decode_noalloc(q, z, 4096, z, z, 4096, z, 8193, out, 4, 64, 8193 * 128)
    with pytest.raises(ValueError, match="64 queries"):
        kvx.attention_decode_noalloc(q, z, 4096, z, z, 4096, z, 1, out, 65, 64, 128)


def test_noalloc_rejects_escape_overflow(kvx, cuda, oracle):
    """Blobs whose escape records do not fit the fixed scratch: the call fails with the
    invalid-argument status and says so; the next ordinary call still works."""
    torch = cuda
    dim, n_q, seq = 128, 4, 192 * 1024  # ~3.5M escape words: over the 3M-entry records
    rng = np.random.default_rng(9)
    e = 120 + rng.integers(0, 18, size=(seq, dim))  # ~17 % escapes in 4-bit blocks
    k = ((rng.integers(0, 2, size=(seq, dim)) << 15) | (e << 7) |
         rng.integers(0, 128, size=(seq, dim))).astype(np.uint16)
    v = S.synth_bf16(9, 1, seq, dim, S.PROFILE_V)
    q = S.synth_bf16(9, 2, n_q, dim, S.PROFILE_Q)
    kx, vx = oracle.encode(k, 128), oracle.encode(v, 128)
    kd, kidx, nb = _device_index(kvx, torch, kx, dim)
    vd, vidx, _ = _device_index(kvx, torch, vx, dim)
    qd = torch.from_numpy(q.view(np.int16)).cuda()
    out = torch.zeros((n_q, dim), dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError, match="escape positions exceed the fixed scratch"):
        kvx.attention_decode_noalloc(qd, kd, kx.size, kidx, vd, vx.size, vidx, nb, out, n_q, dim, seq)
    test_noalloc_matches_attention_decode(kvx, cuda, oracle, [(64, 7, 3000, 15)])
