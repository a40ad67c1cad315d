"""GPU XKV codec parity: decode bit-exact, encode byte-exact to the reference's codec
(src/codec.cpp) as restated in oracle/, including the reference's round-trip specials
(tests/test_main.cpp:54-86)."""
import numpy as np
import pytest

import synth as S
from helpers import XorShift32, clustered

pytestmark = pytest.mark.gpu


def _specials(kv):
    kv = kv.copy()
    flat = kv.reshape(-1)
    flat[0] = 0x0000
    flat[1] = 0x8000
    flat[2] = 0x0001  # subnormal
    flat[3] = 0x7F80  # inf
    flat[4] = 0x7FC1  # nan
    return kv


@pytest.mark.parametrize("block", [16, 32, 64, 128])
def test_roundtrip_specials(kvx, cuda, oracle, block):
    rng = XorShift32()
    seq, dim = 300, 64
    kv = _specials(clustered(rng, seq * dim, 110, 6).reshape(seq, dim))
    enc = kvx.encode_bf16(kv, seq, dim, block)
    ref = oracle.encode(kv, block)
    assert np.array_equal(enc.bytes, ref)
    out = np.zeros((seq, dim), dtype=np.uint16)
    kvx.decode_bf16(enc.bytes, enc.bytes.size, seq, dim, out)
    assert np.array_equal(out, kv)


@pytest.mark.parametrize("seq,dim,block,profile", [
    (128, 64, 128, S.PROFILE_K), (4096, 64, 128, S.PROFILE_NARROW), (1000, 128, 128, S.PROFILE_V),
    (640, 256, 128, S.PROFILE_WIDE_K), (77, 8, 16, S.PROFILE_K), (40, 4, 16, S.PROFILE_V),
    (772, 252, 255, S.PROFILE_K),
])
def test_encode_decode_parity(kvx, cuda, oracle, seq, dim, block, profile):
    if block * dim > 65535:
        block = 65535 // dim
    kv = S.synth_bf16(3, profile, seq, dim, profile)
    ref = oracle.encode(kv, block)
    enc = kvx.encode_bf16(kv, seq, dim, block)
    assert np.array_equal(enc.bytes, ref), "GPU encoder differs from the reference encoder"
    out = np.zeros((seq, dim), dtype=np.uint16)
    kvx.decode_bf16(ref, ref.size, seq, dim, out)
    assert np.array_equal(out, kv)


def test_device_decode_and_index(kvx, cuda, oracle):
    torch = cuda
    seq, dim = 3000, 128
    kv = S.synth_bf16(9, 0, seq, dim, S.PROFILE_K)
    blob = oracle.encode(kv, 128)
    d = torch.from_numpy(blob.view(np.int8)).cuda()
    out = torch.zeros((seq, dim), dtype=torch.int16, device="cuda")
    kvx.decode_bf16(d, blob.size, seq, dim, out)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), kv)
    idx = torch.zeros(64 * 8, dtype=torch.uint8, device="cuda")
    nb, nt = kvx.xkv_index(d, blob.size, dim, idx, 64)
    assert nb == (seq + 127) // 128 and nt == seq


def test_encode_batch_and_append(kvx, cuda, oracle):
    torch = cuda
    seq, dim, n = 1024, 64, 3
    tens = [torch.from_numpy(S.synth_bf16(4, t, seq, dim, t % 2).view(np.int16)).cuda()
            for t in range(n)]
    arena_bytes, entries = kvx.encode_batch_bounds(n, seq, dim)
    arena = torch.zeros(arena_bytes, dtype=torch.uint8, device="cuda")
    index = torch.zeros(entries * 8, dtype=torch.uint8, device="cuda")
    off, nb = kvx.encode_batch(tens, seq, dim, arena, index)
    host = arena.cpu().numpy()
    for t in range(n):
        assert off[t] % 16 == 0
        ref = oracle.encode(tens[t].cpu().numpy().view(np.uint16), 128)
        assert np.array_equal(host[int(off[t]):int(off[t] + nb[t])], ref)
    # append 256 + 256 tokens to an empty device blob
    cap = 1 << 20
    blob = torch.zeros(cap, dtype=torch.uint8, device="cuda")
    idx = torch.zeros(8 * 16, dtype=torch.uint8, device="cuda")
    full = S.synth_bf16(6, 0, 512, dim, S.PROFILE_K)
    at, blocks = 0, 0
    for part in (full[:256], full[256:]):
        t = torch.from_numpy(part.copy().view(np.int16)).cuda()
        bw, kw = kvx.cache_append(t, part.shape[0], dim, blob, at, cap,
                                  idx[blocks * 8:])
        at += bw
        blocks += kw
    ref = oracle.encode(full, 128)
    assert at == ref.size and np.array_equal(blob[:at].cpu().numpy(), ref)


def test_synth_device_matches_numpy(kvx, cuda):
    torch = cuda
    for profile in range(6):
        seq, dim = 300, 64
        out = torch.zeros((seq, dim), dtype=torch.int16, device="cuda")
        rate = {3: S.RATE_8, 4: S.RATE_2, 5: S.RATE_2}.get(profile, S.RATE_0P3)
        kvx.synth_bf16(out, seq, dim, 1234, 77, profile, rate)
        torch.cuda.synchronize()
        ref = S.synth_bf16(1234, 77, seq, dim, profile)
        assert np.array_equal(out.cpu().numpy().view(np.uint16), ref), f"profile {profile}"


def test_encode_errors(kvx, cuda):
    kv = np.zeros((10, 64), dtype=np.uint16)
    with pytest.raises(ValueError, match="empty input"):
        kvx.encode_bf16(kv, 0, 64)
    with pytest.raises(ValueError, match="multiple of 4"):
        kvx.encode_bf16(kv, 10, 62)
    with pytest.raises(ValueError, match="fit in a byte"):
        kvx.encode_bf16(kv, 10, 64, 256)
    # the reference's "escape count would not fit in u16" check (src/codec.cpp:50-52) cannot
    # fire once head_dim <= 256 and block_tokens <= 255 (255 * 256 < 65536): no case to test.
