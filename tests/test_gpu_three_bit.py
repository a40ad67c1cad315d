"""GPU parity of the 3-bit residual mode (mode byte 3, the library's extension), through the C ABI.

The reference has no 3-bit code; the oracle's 3-bit encoder is pinned to the reference's own
exponent analyser (tests/test_three_bit.py).  Here the GPU is checked against that oracle:
  * the GPU encoder (host buffers, batched device tensors, cache append) writes the oracle's bytes
    with the {2, 3, 4} mask, and still the reference's bytes with the default mask;
  * the GPU decoder restores every input bit from 3-bit and mixed-mode blobs;
  * the fused attention kernel reads 3-bit blocks: XKV output == the same kernel on the BF16
    input, bit for bit, and within the float64-anchored tolerance of the oracle, at every fused
    head width, at padded widths, in multi-unit plans and with escape-dense blocks.
"""
import numpy as np
import pytest

import synth as S
from helpers import assert_attention_close, mixed_modes, soften

pytestmark = pytest.mark.gpu
ALL = (2, 3, 4)


def _bits(x):
    return np.asarray(x, dtype=np.float32).view(np.uint32)


def _modes(blob):
    import struct
    out, off = set(), 0
    while off < blob.size:
        mode, nt, ne, hd, _ = struct.unpack_from("<BBHHH", blob, off)
        pay = (nt * hd * 3 + 15) // 16 * 2 if mode == 3 else (nt * hd * mode + 7) // 8
        off += 8 + (2 * nt * hd if mode == 0 else hd + nt * hd + pay + 2 * ne)
        out.add(int(mode))
    return out


def _gpu(kvx, q, k=None, v=None, kx=None, vx=None, seq=None, threads=1, split=128):
    n_q, dim = q.shape
    out = np.zeros((n_q, dim), dtype=np.float32)
    kvx.attention_decode(0, q, k, v, kx, 0 if kx is None else kx.size, vx,
                         0 if vx is None else vx.size, out, n_q, dim, seq, threads, split)
    return out


@pytest.mark.parametrize("seq,dim,block", [(512, 64, 128), (1000, 64, 128), (300, 128, 128),
                                           (640, 256, 128), (90, 32, 32), (17, 12, 16),
                                           (256, 252, 255), (3, 8, 3)])
def test_encode_decode_3bit(kvx, cuda, oracle, seq, dim, block):
    x = mixed_modes(seq, dim, block, seed=seq * 3 + dim)
    want = oracle.encode(x, block, code_bits=ALL)
    got = kvx.encode_bf16(x, seq, dim, block, code_bits=kvx.CODE_BITS_ALL).bytes
    assert np.array_equal(got, want), "GPU 3-bit encoder bytes differ from the oracle"
    assert np.array_equal(kvx.encode_bf16(x, seq, dim, block).bytes, oracle.encode(x, block))
    out = np.zeros((seq, dim), dtype=np.uint16)
    kvx.decode_bf16(want, want.size, seq, dim, out)
    assert np.array_equal(out, x)


def test_encode_batch_and_append_3bit(kvx, cuda, oracle):
    torch = cuda
    dim, seq, block = 64, 1024, 128
    xs = [mixed_modes(seq, dim, block, seed=s) for s in (1, 2, 3)]
    dev = [torch.from_numpy(x.view(np.int16)).cuda() for x in xs]
    arena_bytes, n_index = kvx.encode_batch_bounds(3, seq, dim, block)
    arena = torch.zeros(arena_bytes, dtype=torch.uint8, device="cuda")
    index = torch.zeros(n_index * 8, dtype=torch.uint8, device="cuda")
    off, nb = kvx.encode_batch(dev, seq, dim, arena, index, block, code_bits=kvx.CODE_BITS_ALL)
    host = arena.cpu().numpy()
    for t, x in enumerate(xs):
        want = oracle.encode(x, block, code_bits=ALL)
        assert np.array_equal(host[int(off[t]):int(off[t]) + int(nb[t])], want)
        assert 3 in _modes(want)
    # append two pieces: the blob equals one encode of the whole tensor
    x = xs[0]
    cap = 2 * x.nbytes
    blob = torch.zeros(cap, dtype=torch.uint8, device="cuda")
    idx = torch.zeros(64 * 8, dtype=torch.uint8, device="cuda")
    at, blocks = 0, 0
    for lo, hi in ((0, 512), (512, 1024)):
        piece = torch.from_numpy(np.ascontiguousarray(x[lo:hi]).view(np.int16)).cuda()
        bw, kw = kvx.cache_append(piece, hi - lo, dim, blob, at, cap, idx[blocks * 8:], block,
                                  code_bits=kvx.CODE_BITS_ALL)
        at, blocks = at + bw, blocks + kw
    assert np.array_equal(blob.cpu().numpy()[:at], oracle.encode(x, block, code_bits=ALL))


@pytest.mark.parametrize("dim,n_q,seq,soft", [
    (64, 7, 1000, 6), (64, 7, 4096, 8), (128, 4, 2048, 6), (256, 4, 1500, 7), (32, 8, 700, 5),
    (64, 7, 217, 6), (40, 3, 600, 4), (96, 4, 900, 5),
])
def test_attention_3bit_vs_raw_and_oracle(kvx, cuda, oracle, dim, n_q, seq, soft):
    k = S.synth_bf16(61, 0, seq, dim, S.PROFILE_K)
    v = S.synth_bf16(61, 1, seq, dim, S.PROFILE_V)
    q = soften(S.synth_bf16(61, 2, n_q, dim, S.PROFILE_Q), soft)
    kx, vx = oracle.encode(k, 128, code_bits=ALL), oracle.encode(v, 128, code_bits=ALL)
    assert 3 in _modes(kx) and 3 in _modes(vx)
    g_raw = _gpu(kvx, q, k, v, seq=seq)
    g_xkv = _gpu(kvx, q, kx=kx, vx=vx, seq=seq)
    assert np.array_equal(_bits(g_raw), _bits(g_xkv)), "3-bit XKV and BF16 GPU outputs differ"
    cpu = oracle.attention(q, kx=kx, vx=vx, seq=seq)
    assert_attention_close(g_xkv, cpu, q, k, v, f"3-bit dim={dim} n_q={n_q} seq={seq}")


@pytest.mark.parametrize("dim", [32, 64, 128, 256])
def test_attention_mixed_modes(kvx, cuda, oracle, dim):
    """Blobs holding raw, 2-, 3- and 4-bit blocks side by side, escapes and special values (the
    inputs carry NaN and infinities, so only finiteness-independent bit equality with the BF16
    kernel is checked), then the same with the specials replaced, against the oracle."""
    n_q, seq = 4, 1300
    k = mixed_modes(seq, dim, 128, seed=dim)
    v = mixed_modes(seq, dim, 128, seed=dim + 1)
    q = soften(S.synth_bf16(62, 2, n_q, dim, S.PROFILE_Q), 4)
    kx, vx = oracle.encode(k, 128, code_bits=ALL), oracle.encode(v, 128, code_bits=ALL)
    assert _modes(kx) == {0, 2, 3, 4}
    g_raw = _gpu(kvx, q, k, v, seq=seq)
    g_xkv = _gpu(kvx, q, kx=kx, vx=vx, seq=seq)
    assert np.array_equal(_bits(g_raw), _bits(g_xkv))
    # finite inputs for the tolerance check: clear the specials' exponents to a normal value
    fin = lambda a: np.where(((a >> 7) & 0xFF) >= 0xFF, (a & 0x807F) | (120 << 7), a).astype(np.uint16)
    k, v = fin(k), fin(v)
    kx, vx = oracle.encode(k, 128, code_bits=ALL), oracle.encode(v, 128, code_bits=ALL)
    g = _gpu(kvx, q, kx=kx, vx=vx, seq=seq)
    assert np.array_equal(_bits(g), _bits(_gpu(kvx, q, k, v, seq=seq)))
    assert_attention_close(g, oracle.attention(q, kx=kx, vx=vx, seq=seq), q, k, v,
                           f"mixed modes dim={dim}")


@pytest.mark.parametrize("dim,t_out,p", [(64, 128, 0.15), (128, 64, 0.3), (256, 32, 0.3)])
def test_attention_3bit_escape_dense(kvx, cuda, oracle, dim, t_out, p):
    """3-bit blocks whose first stage holds more escapes than a stage stages (the kernel then
    reads their records from HBM) and tiles with more than 32 escapes: every channel's exponents
    fall in a window of 7 values, and the first t_out tokens of each block carry far outliers
    with probability p (they escape at any code width, so 3 bits still wins)."""
    n_q, seq = 4, 1000

    def tensor(seed):
        r = np.random.default_rng(seed)
        e = 118 + r.integers(0, 7, size=(seq, dim))
        first = (np.arange(seq) % 128 < t_out)[:, None]
        out = first & (r.random((seq, dim)) < p)
        e = np.where(out, 160 + r.integers(0, 8, size=(seq, dim)), e)
        return ((r.integers(0, 2, size=(seq, dim)) << 15) | (e << 7) |
                r.integers(0, 128, size=(seq, dim))).astype(np.uint16)
    k, v = tensor(dim), tensor(dim + 7)
    q = soften(S.synth_bf16(63, 2, n_q, dim, S.PROFILE_Q), 6)
    kx, vx = oracle.encode(k, 128, code_bits=ALL), oracle.encode(v, 128, code_bits=ALL)
    assert _modes(kx) == {3} and _modes(vx) == {3}, (_modes(kx), _modes(vx))
    g = _gpu(kvx, q, kx=kx, vx=vx, seq=seq)
    assert np.array_equal(_bits(g), _bits(_gpu(kvx, q, k, v, seq=seq)))
    assert_attention_close(g, oracle.attention(q, kx=kx, vx=vx, seq=seq), q, k, v,
                           f"3-bit escape-dense dim={dim}")


def test_plan_with_3bit_units(kvx, cuda, oracle):
    """A multi-unit plan (units of different lengths, mixed modes) against the oracle, unit by
    unit, and the host-buffer batched entry on the same blobs gives the same bits."""
    torch = cuda
    dim, n_q = 64, 7
    seqs = [4096, 1000, 37, 2048, 129, 3000, 700, 512, 1500]
    keep, units, cases, outs_h = [], [], [], []
    out = torch.full((len(seqs), n_q, dim), float("nan"), device="cuda")
    for u, seq in enumerate(seqs):
        k = S.synth_bf16(70 + u, 0, seq, dim, S.PROFILE_K if u % 3 else S.PROFILE_NARROW)
        v = mixed_modes(seq, dim, 128, seed=70 + u) if u % 4 == 1 else S.synth_bf16(
            70 + u, 1, seq, dim, S.PROFILE_V)
        v = np.where(((v >> 7) & 0xFF) >= 0xFF, (v & 0x807F) | (120 << 7), v).astype(np.uint16)
        q = soften(S.synth_bf16(70 + u, 2, n_q, dim, S.PROFILE_Q), 6)
        kx, vx = oracle.encode(k, 128, code_bits=ALL), oracle.encode(v, 128, code_bits=ALL)
        cases.append((q, k, v, kx, vx, seq))
        dq = torch.from_numpy(q.view(np.int16)).cuda()
        ent = []
        for blob in (kx, vx):
            d = torch.from_numpy(blob.view(np.int8)).cuda()
            idx = torch.empty(((blob.size // 8) + 16) * 8, dtype=torch.uint8, device="cuda")
            nb, nt = kvx.xkv_index(d, blob.size, dim, idx, idx.numel() // 8)
            assert nt == seq
            ent.append((d, idx, nb))
        (dk, kidx, nb), (dv, vidx, _) = ent
        keep += [dq, dk, kidx, dv, vidx]
        units.append(kvx.make_unit(dk, dv, dq, out[u], k_index=kidx, v_index=vidx, k_bytes=kx.size,
                                   v_bytes=vx.size, n_blocks=nb, seq=seq))
    plan = kvx.Plan(units, n_q, dim, 128)
    try:
        plan.run()
        plan.check()
    finally:
        plan.close()
    got = out.cpu().numpy()
    for u, (q, k, v, kx, vx, seq) in enumerate(cases):
        assert_attention_close(got[u], oracle.attention(q, kx=kx, vx=vx, seq=seq), q, k, v,
                               f"plan unit {u} seq={seq}")
