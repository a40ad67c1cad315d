"""GPU parity of the fused XKV decode attention (the hot path), through the C ABI.

Three checks, mirroring the reference's own invariants (tests/test_main.cpp:124-157):
  * XKV output == uncompressed-BF16 output of the same GPU kernel, bit for bit;
  * GPU output within an FP32 tolerance (helpers.assert_attention_close) of the reference's
    scalar kernel restated in oracle/ (and of the reference library itself when built);
  * the batched plan gives the same bits as the one-unit drop-in call.
"""
import numpy as np
import pytest

import synth as S
from helpers import (XorShift32, assert_attention_close, clustered, measure, truth_and_scale,
                     make_bf16, soften)

pytestmark = pytest.mark.gpu


def _case(dim, n_q, seq, seed=7, k_profile=S.PROFILE_K, soft=0):
    k = S.synth_bf16(seed, 0, seq, dim, k_profile)
    v = S.synth_bf16(seed, 1, seq, dim, S.PROFILE_V)
    q = S.synth_bf16(seed, 2, n_q, dim, S.PROFILE_Q)
    return (soften(q, soft) if soft else q), k, v


def _gpu(kvx, q, k=None, v=None, kx=None, vx=None, seq=None, threads=1, split=128,
         backend=0):
    n_q, dim = q.shape
    out = np.zeros((n_q, dim), dtype=np.float32)
    kvx.attention_decode(backend, q, k, v, kx, 0 if kx is None else kx.size, vx,
                         0 if vx is None else vx.size, out, n_q, dim, seq, threads, split)
    return out


def _bits(x):
    return np.asarray(x, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("dim,n_q,seq,soft", [
    (64, 7, 1, 0), (64, 7, 17, 0), (64, 7, 128, 0), (64, 7, 300, 0), (64, 1, 1000, 0),
    (64, 3, 4096, 0), (32, 2, 90, 0), (128, 4, 513, 0), (256, 4, 300, 0), (64, 14, 700, 0),
    (128, 8, 2048, 0), (64, 5, 8192, 0), (64, 7, 4096, 6), (128, 4, 8192, 6), (256, 4, 3000, 7),
    (32, 8, 5000, 5), (64, 16, 1500, 6),
])
def test_xkv_vs_raw_and_oracle(kvx, cuda, oracle, dim, n_q, seq, soft):
    q, k, v = _case(dim, n_q, seq, soft=soft)
    kx = oracle.encode(k, 128)
    vx = oracle.encode(v, 128)
    g_raw = _gpu(kvx, q, k, v, seq=seq)
    g_xkv = _gpu(kvx, q, kx=kx, vx=vx, seq=seq)
    assert np.array_equal(_bits(g_raw), _bits(g_xkv)), "XKV and BF16 GPU outputs differ"
    cpu = oracle.attention(q, kx=kx, vx=vx, seq=seq)
    assert_attention_close(g_xkv, cpu, q, k, v, f"dim={dim} n_q={n_q} seq={seq}")


@pytest.mark.parametrize("dim,n_q,seq,soft", [(64, 7, 8192, 6), (128, 4, 16384, 7),
                                              (256, 4, 4096, 7), (64, 7, 32768, 8)])
def test_accuracy_vs_float64(kvx, cuda, oracle, dim, n_q, seq, soft):
    """Against the float64 softmax the GPU is within the tight tolerance (oracle/parity.py), and
    no less accurate than the reference's scalar kernel."""
    q, k, v = _case(dim, n_q, seq, seed=21, soft=soft)
    kx, vx = oracle.encode(k, 128), oracle.encode(v, 128)
    g = _gpu(kvx, q, kx=kx, vx=vx, seq=seq)
    cpu = oracle.attention(q, kx=kx, vx=vx, seq=seq)
    m = measure(g, cpu, truth_and_scale(q, k, v))
    assert m["accuracy"] <= 1.0 and m["parity"] <= 1.0, m
    assert m["gpu_err_over_scale"] <= m["ref_err_over_scale"], m


def test_accuracy_vs_float64_1m_tokens(kvx, cuda, oracle):
    """config[4]'s shape on one GPU: one KV head of 1,048,576 tokens at D=256 (2 % escapes, 5 %
    raw blocks), softened queries; the inputs come from the device generator (bit-identical to
    synth.py)."""
    torch = cuda
    dim, n_q, seq = 256, 4, 1 << 20
    kt = torch.empty((seq, dim), dtype=torch.int16, device="cuda")
    vt = torch.empty((seq, dim), dtype=torch.int16, device="cuda")
    kvx.synth_bf16(kt, seq, dim, 41, S.stream_id(0, 0), S.PROFILE_WIDE_K, S.RATE_2)
    kvx.synth_bf16(vt, seq, dim, 41, S.stream_id(0, 1), S.PROFILE_WIDE_V, S.RATE_2)
    k = kt.cpu().numpy().view(np.uint16)
    v = vt.cpu().numpy().view(np.uint16)
    del kt, vt
    q = soften(S.synth_bf16(41, S.stream_id(0, 2), n_q, dim, S.PROFILE_Q), 32)
    kx, modes = oracle.encode(k, 128, with_modes=True)
    assert (modes == 0).any() and (modes == 4).any()
    vx = oracle.encode(v, 128)
    g = _gpu(kvx, q, kx=kx, vx=vx, seq=seq)
    cpu = oracle.attention(q, kx=kx, vx=vx, seq=seq)
    m = measure(g, cpu, truth_and_scale(q, k, v))
    assert m["accuracy"] <= 1.0 and m["parity"] <= 1.0, m
    assert m["gpu_err_over_scale"] <= m["ref_err_over_scale"], m


@pytest.mark.parametrize("dim,n_q,seq,block,threads", [
    (64, 1, 1, 128, 1), (64, 7, 17, 128, 1), (64, 7, 128, 128, 1), (64, 3, 200, 64, 1),
    (64, 7, 300, 64, 4), (32, 2, 90, 32, 1), (64, 7, 256, 128, 4),
])
def test_reference_matrix(kvx, cuda, oracle, dim, n_q, seq, block, threads):
    """The reference test matrix (tests/test_main.cpp:165-172) on clustered data."""
    rng = XorShift32()
    k = clustered(rng, seq * dim, 108, 8).reshape(seq, dim)
    v = clustered(rng, seq * dim, 112, 5).reshape(seq, dim)
    q = np.array([make_bf16(120, rng() & 0x7F, rng() & 1) for _ in range(n_q * dim)],
                 dtype=np.uint16).reshape(n_q, dim)
    kx = oracle.encode(k, block)
    vx = oracle.encode(v, block)
    g_raw = _gpu(kvx, q, k, v, seq=seq, threads=threads, split=block)
    g_xkv = _gpu(kvx, q, kx=kx, vx=vx, seq=seq, threads=threads, split=block)
    assert np.array_equal(_bits(g_raw), _bits(g_xkv))
    cpu = oracle.attention(q, kx=kx, vx=vx, seq=seq, threads=threads, split=block)
    assert_attention_close(g_xkv, cpu, q, k, v, "reference matrix")


def test_narrow_two_bit_blocks(kvx, cuda, oracle):
    """2-bit blocks with 8 % escapes (the config[1] layer-0 K distribution)."""
    q, k, v = _case(64, 7, 2048, seed=11, k_profile=S.PROFILE_NARROW)
    kx, modes = oracle.encode(k, 128, with_modes=True)
    assert (modes == 2).all()
    vx = oracle.encode(v, 128)
    g_raw = _gpu(kvx, q, k, v, seq=2048)
    g_xkv = _gpu(kvx, q, kx=kx, vx=vx, seq=2048)
    assert np.array_equal(_bits(g_raw), _bits(g_xkv))
    cpu = oracle.attention(q, kx=kx, vx=vx, seq=2048)
    assert_attention_close(g_xkv, cpu, q, k, v, "2-bit")


@pytest.mark.parametrize("dim,n_q,seq", [(64, 7, 1000), (128, 4, 600), (256, 4, 300), (32, 8, 700)])
def test_escape_heavy_blocks(kvx, cuda, oracle, dim, n_q, seq):
    """4-bit blocks with ~17 % escapes: more escape words per stage than the kernel stages in
    shared memory (it then reads them from HBM), and tiles with more than 32 escapes."""
    rng = np.random.default_rng(dim + seq)
    e = 120 + rng.integers(0, 18, size=(seq, dim))  # 18 exponents: 15 fit the 4-bit window
    m = rng.integers(0, 128, size=(seq, dim))
    sg = rng.integers(0, 2, size=(seq, dim))
    k = ((sg << 15) | (e << 7) | m).astype(np.uint16)
    v = S.synth_bf16(5, 1, seq, dim, S.PROFILE_V)
    q = soften(S.synth_bf16(5, 2, n_q, dim, S.PROFILE_Q), 6)
    kx, modes = oracle.encode(k, 128, with_modes=True)
    assert (modes == 4).all()
    vx = oracle.encode(v, 128)
    g_raw = _gpu(kvx, q, k, v, seq=seq)
    g_xkv = _gpu(kvx, q, kx=kx, vx=vx, seq=seq)
    assert np.array_equal(_bits(g_raw), _bits(g_xkv))
    cpu = oracle.attention(q, kx=kx, vx=vx, seq=seq)
    assert_attention_close(g_xkv, cpu, q, k, v, f"escape-heavy D{dim}")


def test_raw_blocks(kvx, cuda, oracle):
    """Blocks the encoder stores raw (config[4] distribution), mixed with coded blocks."""
    q, k, v = _case(256, 4, 128 * 40, seed=5, k_profile=S.PROFILE_WIDE_K)
    v = S.synth_bf16(5, 1, 128 * 40, 256, S.PROFILE_WIDE_V)
    kx, modes = oracle.encode(k, 128, with_modes=True)
    assert (modes == 0).any() and (modes == 4).any()
    vx = oracle.encode(v, 128)
    g_raw = _gpu(kvx, q, k, v, seq=k.shape[0])
    g_xkv = _gpu(kvx, q, kx=kx, vx=vx, seq=k.shape[0])
    assert np.array_equal(_bits(g_raw), _bits(g_xkv))
    cpu = oracle.attention(q, kx=kx, vx=vx, seq=k.shape[0])
    assert_attention_close(g_xkv, cpu, q, k, v, "raw blocks")


@pytest.mark.parametrize("backend,dim,n_q,seq,block", [
    (0, 8, 3, 200, 64), (1, 16, 1, 40, 16), (0, 24, 4, 333, 128), (1, 40, 7, 1000, 128),
    (2, 96, 4, 700, 128), (0, 200, 2, 300, 128), (2, 160, 3, 129, 128),
])
def test_padded_head_dims(kvx, cuda, oracle, backend, dim, n_q, seq, block):
    """Head dims the reference's backends take but the fused kernels do not (any multiple of 8,
    of 32 for AVX-512): the drop-in call runs them zero-padded to the next fused width, raw and XKV
    inputs bit-identical, within tolerance of the oracle."""
    k = S.synth_bf16(9, 0, seq, dim, S.PROFILE_K)
    v = S.synth_bf16(9, 1, seq, dim, S.PROFILE_V)
    q = soften(S.synth_bf16(9, 2, n_q, dim, S.PROFILE_Q), 8)
    kx, vx = oracle.encode(k, block), oracle.encode(v, block)
    g_raw = _gpu(kvx, q, k, v, seq=seq, split=block, backend=backend)
    g_xkv = _gpu(kvx, q, kx=kx, vx=vx, seq=seq, split=block, backend=backend)
    assert np.array_equal(_bits(g_raw), _bits(g_xkv))
    cpu = oracle.attention(q, kx=kx, vx=vx, seq=seq, split=block)
    assert_attention_close(g_xkv, cpu, q, k, v, f"padded dim={dim}")


def test_identity_token(kvx, cuda):
    """seq 1, q = k = 1.0: out == v exactly (tests/test_main.cpp:102-122, at dim 32)."""
    dim = 32
    q = np.full((1, dim), 0x3F80, dtype=np.uint16)
    k = q.copy()
    v = np.full((1, dim), 0x3F80, dtype=np.uint16)
    v[0, 0] = 0x4000
    out = _gpu(kvx, q, k, v, seq=1)
    assert out[0, 0] == 2.0 and (out[0, 1:] == 1.0).all()


def test_device_pointers_match_host(kvx, cuda, oracle):
    torch = cuda
    q, k, v = _case(64, 7, 1000)
    kx = oracle.encode(k, 128)
    vx = oracle.encode(v, 128)
    host = _gpu(kvx, q, kx=kx, vx=vx, seq=1000)
    dq = torch.from_numpy(q.view(np.int16)).cuda()
    dk = torch.from_numpy(kx.view(np.int8)).cuda()
    dv = torch.from_numpy(vx.view(np.int8)).cuda()
    out = torch.zeros((7, 64), dtype=torch.float32, device="cuda")
    kvx.attention_decode(0, dq, None, None, dk, kx.size, dv, vx.size, out, 7, 64, 1000, 1)
    assert np.array_equal(_bits(out.cpu().numpy()), _bits(host))


def test_units_batch_matches_single(kvx, cuda, oracle):
    dim, n_q, seq = 64, 7, 1500
    qs, kxs, vxs, singles = [], [], [], []
    for u in range(6):
        q, k, v = _case(dim, n_q, seq, seed=100 + u)
        kx, vx = oracle.encode(k, 128), oracle.encode(v, 128)
        qs.append(q); kxs.append(kx); vxs.append(vx)
        singles.append(_gpu(kvx, q, kx=kx, vx=vx, seq=seq))
    runs = []
    for _ in range(2):
        outs = [np.zeros((n_q, dim), dtype=np.float32) for _ in range(6)]
        kvx.attention_decode_units(0, qs, kxs, [x.size for x in kxs], vxs,
                                   [x.size for x in vxs], outs, n_q, dim, seq)
        runs.append(outs)
    for a, b in zip(*runs):  # deterministic
        assert np.array_equal(_bits(a), _bits(b))
    for a, b, q in zip(runs[0], singles, qs):
        scale = np.maximum(np.abs(b), 1e-3)
        assert np.max(np.abs(a - b) / scale) < 1e-4


def test_units_batch_error_then_recovery(kvx, cuda, oracle):
    """With host buffers the blobs are still being copied when a header walk fails: the call
    reports the reference's error, and the next call (same buffers, fixed) is unaffected."""
    dim, n_q, seq = 64, 7, 700
    qs, kxs, vxs, singles = [], [], [], []
    for u in range(4):
        q, k, v = _case(dim, n_q, seq, seed=300 + u)
        kx, vx = oracle.encode(k, 128), oracle.encode(v, 128)
        qs.append(q); kxs.append(kx); vxs.append(vx)
        singles.append(_gpu(kvx, q, kx=kx, vx=vx, seq=seq))
    outs = [np.zeros((n_q, dim), dtype=np.float32) for _ in range(4)]
    bad = list(kxs)
    bad[2] = kxs[2][:-3]
    with pytest.raises(RuntimeError, match="truncated"):
        kvx.attention_decode_units(0, qs, bad, [x.size for x in bad], vxs, [x.size for x in vxs],
                                   outs, n_q, dim, seq)
    kvx.attention_decode_units(0, qs, kxs, [x.size for x in kxs], vxs, [x.size for x in vxs], outs,
                               n_q, dim, seq)
    for a, b in zip(outs, singles):
        scale = np.maximum(np.abs(b), 1e-3)
        assert np.max(np.abs(a - b) / scale) < 1e-4


def test_errors_mirror_reference(kvx, cuda, oracle):
    q, k, v = _case(64, 7, 300)
    kx = oracle.encode(k, 128)
    vx = oracle.encode(v, 128)
    with pytest.raises(ValueError, match="bad argument"):
        _gpu(kvx, q, kx=kx, vx=vx, seq=0)
    with pytest.raises(ValueError, match="not both"):
        out = np.zeros((7, 64), dtype=np.float32)
        kvx.attention_decode(0, q, k, v, kx, kx.size, vx, vx.size, out, 7, 64, 300, 1)
    with pytest.raises(RuntimeError, match="truncated"):
        _gpu(kvx, q, kx=kx[:-3], vx=vx, seq=300)
    bad = kx.copy()
    bad[4] ^= 1  # head_dim field
    with pytest.raises(RuntimeError, match="dimension or length mismatch"):
        _gpu(kvx, q, kx=bad, vx=vx, seq=300)
    bad = kx.copy()
    bad[0] = 5  # mode (3 is the 3-bit extension)
    with pytest.raises(RuntimeError, match="unknown xkv block mode"):
        _gpu(kvx, q, kx=bad, vx=vx, seq=300)
    with pytest.raises(RuntimeError, match="ran out of blocks"):
        _gpu(kvx, q, kx=kx, vx=vx, seq=301)
    with pytest.raises(RuntimeError, match="not aligned"):
        _gpu(kvx, q, kx=kx, vx=vx, seq=300, threads=3, split=64)


@pytest.mark.parametrize("dim", [64, 128, 256])
def test_plan_mostly_empty_stages(kvx, cuda, oracle, dim):
    """One long unit among hundreds of 1-3 token units.  Every block of a plan takes the stages
    of the longest one, so most stages here are empty and the consumer warps run far ahead of the
    copies: each must still take exactly its own stage (the slot's stage tag, not only the parity
    of its barrier), run after run."""
    torch = cuda
    n_q = 4
    seqs = [1100] + [1 + (u % 3) for u in range(400)]
    keep, units, refs, cases = [], [], [], []
    out = torch.full((len(seqs), n_q, dim), float("nan"), device="cuda")
    for u, seq in enumerate(seqs):
        q, k, v = _case(dim, n_q, seq, seed=900 + u, soft=6)
        kx, vx = oracle.encode(k, 128), oracle.encode(v, 128)
        refs.append(oracle.attention(q, kx=kx, vx=vx, seq=seq))
        cases.append((q, k, v))
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
        first = None
        for _ in range(20):
            plan.run()
            plan.check()
            got = out.cpu().numpy()
            if first is None:
                first = got.copy()
            else:
                assert np.array_equal(_bits(first), _bits(got)), "runs differ"
    finally:
        plan.close()
    for u, (g, r, (q, k, v)) in enumerate(zip(first, refs, cases)):
        assert_attention_close(g, r, q, k, v, f"unit {u} seq={seqs[u]}")
