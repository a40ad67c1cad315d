"""The batched decode paths at a config[1]-like size, unit by unit against the oracle.

16 (layer, KV head) units of 32768 tokens, D=64, GQA 7: unit 0 has config[1]'s layer-0 K (2-bit
blocks, 8 % escapes), the others the 4-bit profile; queries are softened so that the softmax
spreads over many tokens.  4096 blocks over 148 CTA ranges: every range holds many blocks and
several units' segments, ranges are cost-balanced, and units span several CTAs; and 16
units is more than 8, so kvx_attention_decode_units with host buffers runs as two chunks, each
with its own plan behind its own copies.  Every path is checked against the float64 truth and
the scalar oracle's output (helpers.assert_attention_close):
  * kvx_attention_decode_units with host buffers (the end-to-end path bench.py times);
  * the same entry point with device buffers;
  * a kvx_plan over device-resident blobs (the path bench.py's `value` times).
"""
import numpy as np
import pytest

import synth as S
from helpers import assert_attention_close, soften, truth_and_scale

pytestmark = pytest.mark.gpu

N_UNITS, SEQ, DIM, NQ = 16, 32768, 64, 7


@pytest.fixture(scope="module")
def batch(oracle):
    qs, ks, vs, kxs, vxs, want, truths = [], [], [], [], [], [], []
    for u in range(N_UNITS):
        kp = S.PROFILE_NARROW if u == 0 else S.PROFILE_K
        k = S.synth_bf16(0x5EED, S.stream_id(u, 0), SEQ, DIM, kp)
        v = S.synth_bf16(0x5EED, S.stream_id(u, 1), SEQ, DIM, S.PROFILE_V)
        q = soften(S.synth_bf16(0x5EED, S.stream_id(u, 2), NQ, DIM, S.PROFILE_Q),
                   6 if u == 0 else 8)
        kx, modes = oracle.encode(k, 128, with_modes=True)
        if u == 0:
            assert (modes == 2).all(), "layer-0 K should encode as 2-bit blocks"
        vx = oracle.encode(v, 128)
        qs.append(np.ascontiguousarray(q)); ks.append(k); vs.append(v)
        kxs.append(kx); vxs.append(vx)
        want.append(oracle.attention(q, kx=kx, vx=vx, seq=SEQ))
        truths.append(truth_and_scale(q, k, v))
    return dict(q=qs, k=ks, v=vs, kx=kxs, vx=vxs, want=want, truth=truths)


def _check_all(got, b, what):
    for u in range(N_UNITS):
        assert np.all(np.isfinite(got[u])), f"{what}: unit {u} not finite"
        assert_attention_close(got[u], b["want"][u], what=f"{what} unit {u}", truth=b["truth"][u])


def test_units_host_buffers_vs_oracle(kvx, cuda, batch):
    b = batch
    runs = []
    for _ in range(2):
        outs = [np.full((NQ, DIM), np.nan, dtype=np.float32) for _ in range(N_UNITS)]
        kvx.attention_decode_units(0, b["q"], b["kx"], [x.size for x in b["kx"]], b["vx"],
                                   [x.size for x in b["vx"]], outs, NQ, DIM, SEQ)
        runs.append(outs)
    for a, c in zip(*runs):  # deterministic from call to call
        assert np.array_equal(a.view(np.uint32), c.view(np.uint32))
    _check_all(runs[0], b, "units (host buffers, two chunks)")


def test_units_device_buffers_vs_oracle(kvx, cuda, batch):
    torch = cuda
    b = batch
    dq = [torch.from_numpy(q.view(np.int16)).cuda() for q in b["q"]]
    dk = [torch.from_numpy(x).cuda() for x in b["kx"]]
    dv = [torch.from_numpy(x).cuda() for x in b["vx"]]
    do = [torch.full((NQ, DIM), float("nan"), device="cuda") for _ in range(N_UNITS)]
    kvx.attention_decode_units(0, dq, dk, [x.size for x in b["kx"]], dv,
                               [x.size for x in b["vx"]], do, NQ, DIM, SEQ)
    _check_all([o.cpu().numpy() for o in do], b, "units (device buffers)")


def test_plan_vs_oracle(kvx, cuda, batch):
    torch = cuda
    b = batch
    keep, units = [], []
    out = torch.full((N_UNITS, NQ, DIM), float("nan"), device="cuda")
    for u in range(N_UNITS):
        dq = torch.from_numpy(b["q"][u].view(np.int16)).cuda()
        ent = []
        for blob in (b["kx"][u], b["vx"][u]):
            d = torch.from_numpy(blob).cuda()
            idx = torch.empty(((blob.size // 8) + 16) * 8, dtype=torch.uint8, device="cuda")
            nb, nt = kvx.xkv_index(d, blob.size, DIM, idx, idx.numel() // 8)
            assert nt == SEQ
            ent.append((d, idx, nb))
        (dk, kidx, nb), (dv, vidx, _) = ent
        keep += [dq, dk, kidx, dv, vidx]
        units.append(kvx.make_unit(dk, dv, dq, out[u], k_index=kidx, v_index=vidx,
                                   k_bytes=b["kx"][u].size, v_bytes=b["vx"][u].size,
                                   n_blocks=nb, seq=SEQ))
    plan = kvx.Plan(units, NQ, DIM, 128)
    try:
        plan.run()
        plan.check()
        first = out.cpu().numpy().copy()
        plan.run()
        plan.check()
        assert np.array_equal(first.view(np.uint32), out.cpu().numpy().view(np.uint32))
    finally:
        plan.close()
    _check_all(list(first), b, "plan (device-resident)")
