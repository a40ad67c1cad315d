"""KVD1 / QSN1 dump loaders (reference src/bench.cpp:87-164) and the model_heads scope on a dump.

The file formats follow python/dump_kv.py (`write_dump`, the .qsnap writer); the loaders raise the
reference's messages.  The GPU test runs the scope on a small synthetic dump: per unit the XKV and
raw outputs agree bit for bit, and every unit matches the CPU oracle within the suite's
tolerance."""
import numpy as np
import pytest

import dumps
import synth as S
from helpers import assert_attention_close

LAYERS, KV, NQ, DIM, SEQ = 2, 2, 4, 64, 640
POS = [300, 640]


def _make(tmp_path, seed=11):
    k = np.stack([np.stack([S.synth_bf16(seed, 10 * l + h, SEQ, DIM, S.PROFILE_K) for h in range(KV)])
                  for l in range(LAYERS)])
    v = np.stack([np.stack([S.synth_bf16(seed, 100 + 10 * l + h, SEQ, DIM, S.PROFILE_V) for h in range(KV)])
                  for l in range(LAYERS)])
    q = np.stack([np.stack([S.synth_bf16(seed, 1000 + 10 * s + l, NQ, DIM, S.PROFILE_Q) for l in range(LAYERS)])
                  for s in range(len(POS))])
    kd, qd = tmp_path / "cache.kvdump", tmp_path / "cache.qsnap"
    dumps.write_kvd1(str(kd), k, v, q[-1])
    dumps.write_qsn1(str(qd), POS, q)
    return str(kd), str(qd), k, v, q


def test_round_trip(tmp_path):
    kd, qd, k, v, q = _make(tmp_path)
    d, s = dumps.load_kvd1(kd), dumps.load_qsn1(qd)
    assert (d.layers, d.kv, d.nq, d.dim, d.seq) == (LAYERS, KV, NQ, DIM, SEQ)
    assert np.array_equal(d.k, k) and np.array_equal(d.v, v)
    assert s.pos == POS and (s.layers, s.nq, s.dim) == (LAYERS, NQ, DIM)
    assert np.array_equal(s.q, q)
    dumps.check_pair(d, s)
    assert s.index(300) == 0 and s.index(640) == 1
    # head_ptr / query_ptr views
    assert np.array_equal(d.head(d.k, 1, 1, 100), k[1, 1, :100])
    assert np.array_equal(s.query(1, 0, 2, 2), q[1, 0, 2:4])


def test_errors_mirror_reference(tmp_path):
    kd, qd, k, v, q = _make(tmp_path)
    raw = open(kd, "rb").read()
    small = tmp_path / "small"
    small.write_bytes(raw[:31])
    with pytest.raises(RuntimeError, match="dump too small"):
        dumps.load_kvd1(str(small))
    bad = tmp_path / "bad"
    bad.write_bytes(b"KVD2" + raw[4:])
    with pytest.raises(RuntimeError, match="not a KVD1 v1 dump"):
        dumps.load_kvd1(str(bad))
    ver = tmp_path / "ver"
    ver.write_bytes(raw[:4] + (2).to_bytes(4, "little") + raw[8:])
    with pytest.raises(RuntimeError, match="not a KVD1 v1 dump"):
        dumps.load_kvd1(str(ver))
    trunc = tmp_path / "trunc"
    trunc.write_bytes(raw[:32 + LAYERS * KV * SEQ * DIM * 4 - 2])
    with pytest.raises(RuntimeError, match="dump truncated"):
        dumps.load_kvd1(str(trunc))
    with pytest.raises(RuntimeError, match="open qsnap failed"):
        dumps.load_qsn1(str(tmp_path / "missing.qsnap"))
    qraw = open(qd, "rb").read()
    qbad = tmp_path / "qbad"
    qbad.write_bytes(b"QSN2" + qraw[4:])
    with pytest.raises(RuntimeError, match="bad qsnap magic"):
        dumps.load_qsn1(str(qbad))
    qtr = tmp_path / "qtr"
    qtr.write_bytes(qraw[:-2])
    with pytest.raises(RuntimeError, match="truncated qsnap"):
        dumps.load_qsn1(str(qtr))
    d, s = dumps.load_kvd1(kd), dumps.load_qsn1(qd)
    with pytest.raises(RuntimeError, match="no query snapshot for this length"):
        s.index(512)
    other = tmp_path / "other.qsnap"
    dumps.write_qsn1(str(other), POS, q[:, :, :2])
    with pytest.raises(RuntimeError, match="qsnap does not match dump"):
        dumps.check_pair(d, dumps.load_qsn1(str(other)))


@pytest.mark.gpu
def test_model_heads_on_dump(tmp_path, kvx, cuda, oracle):
    kd, qd, k, v, q = _make(tmp_path)
    d, s = dumps.load_kvd1(kd), dumps.load_qsn1(qd)
    group = NQ // KV
    for seq in POS:
        res = dumps.model_heads(kvx, d, s, seq, reps=1)  # raises on a bit or tolerance mismatch
        assert res["seq"] == seq and 0.5 < res["container_ratio"] < 1.0
        m = dumps.prepare_model_heads(kvx, d, s, seq)
        out = dumps.run_model_heads(kvx, m, DIM, "batched")
        for u in range(LAYERS * KV):
            ly, h = divmod(u, KV)
            qq = q[s.index(seq), ly, h * group:(h + 1) * group]
            kk, vv = k[ly, h, :seq], v[ly, h, :seq]
            cpu = oracle.attention(qq, k=kk, v=vv, seq=seq)
            assert_attention_close(out[u], cpu, qq, kk, vv, f"dump unit {u} seq {seq}")


def test_cli(tmp_path, kvx, cuda, capsys):
    kd, qd, _, _, _ = _make(tmp_path)
    assert dumps.main(["--dump", kd, "--qsnap", qd, "--seq", "300", "--reps", "1"]) == 0
    line = capsys.readouterr().out.strip().splitlines()[-1]
    assert '"scope": "model_heads"' in line and '"seq": 300' in line


test_cli = pytest.mark.gpu(test_cli)
