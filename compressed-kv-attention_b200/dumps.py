"""KVD1 / QSN1 dump loaders and the reference benchmark's `model_heads` scope over a real dump.

The reference benchmark (src/bench.cpp:87-143) reads two files written by python/dump_kv.py:

* KVD1 (python/dump_kv.py:157-177 `write_dump`): a 32-byte little-endian header of eight u32
  {"KVD1", version 1, layers, kv_heads, q_heads, head_dim, seq, 0}, then the K plane and the V
  plane, BF16 [layers][kv_heads][seq][head_dim], then the last position's queries (unused here).
* QSN1 (python/dump_kv.py:302-313): u32 {"QSN1", n_snap, layers, q_heads}, n_snap u32 positions
  (the token counts each snapshot attends over), u32 head_dim, then BF16 queries
  [n_snap][layers][q_heads][head_dim].

`load_kvd1` / `load_qsn1` parse them with the reference's checks and messages (RuntimeError, like
its std::runtime_error), memory-mapping the planes.  `model_heads` runs the reference's
model_heads scope on the GPU: every (layer, KV head) at one snapshot length, encoded with the
library's encoder; per unit the XKV and raw BF16 outputs must agree bit for bit
(src/bench.cpp:688-690 "bit mismatch on full model"), and the batched call over all units is
timed too.

    python compressed-kv-attention_b200/dumps.py --dump FILE --qsnap FILE [--seq N]

prints one JSON line per snapshot length: raw, XKV and batched milliseconds, container and tight
bytes.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from dataclasses import dataclass

import numpy as np

KVD1_MAGIC = b"KVD1"
QSN1_MAGIC = b"QSN1"


@dataclass
class Dump:
    layers: int
    kv: int
    nq: int
    dim: int
    seq: int
    k: np.ndarray  # [layers, kv, seq, dim] uint16 (memory-mapped)
    v: np.ndarray

    def head(self, plane: np.ndarray, layer: int, head: int, seq: int) -> np.ndarray:
        """The first `seq` tokens of one KV head (src/bench.cpp:145-148 `head_ptr`)."""
        return plane[layer, head, :seq]


@dataclass
class QSnap:
    pos: list
    layers: int
    nq: int
    dim: int
    q: np.ndarray  # [n_snap, layers, nq, dim] uint16

    def query(self, snap: int, layer: int, q0: int, n: int) -> np.ndarray:
        """Queries q0 .. q0 + n - 1 of one layer at one snapshot (src/bench.cpp:150-155)."""
        return self.q[snap, layer, q0:q0 + n]

    def index(self, seq: int) -> int:
        """src/bench.cpp:157-164 `snap_index`."""
        for i, p in enumerate(self.pos):
            if p == seq:
                return i
        raise RuntimeError("no query snapshot for this length")


def load_kvd1(path: str) -> Dump:
    """src/bench.cpp:87-108 `parse_dump` (the file is mapped, not read)."""
    n = os.path.getsize(path)
    if n < 32:
        raise RuntimeError("dump too small")
    hdr = np.fromfile(path, dtype="<u4", count=8)
    if hdr[:1].tobytes() != KVD1_MAGIC or int(hdr[1]) != 1:
        raise RuntimeError("not a KVD1 v1 dump")
    layers, kv, nq, dim, seq = (int(x) for x in hdr[2:7])
    plane = layers * kv * seq * dim
    if n < 32 + plane * 4:
        raise RuntimeError("dump truncated")
    mm = np.memmap(path, dtype="<u2", mode="r", offset=32, shape=(2 * plane,))
    k = mm[:plane].reshape(layers, kv, seq, dim)
    v = mm[plane:].reshape(layers, kv, seq, dim)
    return Dump(layers, kv, nq, dim, seq, k, v)


def load_qsn1(path: str) -> QSnap:
    """src/bench.cpp:118-143 `load_qsnap`."""
    try:
        f = open(path, "rb")
    except OSError:
        raise RuntimeError("open qsnap failed") from None
    with f:
        hdr = f.read(16)
        if len(hdr) < 16 or hdr[:4] != QSN1_MAGIC:
            raise RuntimeError("bad qsnap magic")
        nsnap, layers, nq = (int(x) for x in np.frombuffer(hdr[4:], dtype="<u4"))
        pos = np.frombuffer(f.read(4 * nsnap), dtype="<u4")
        dimb = f.read(4)
        if len(pos) != nsnap or len(dimb) != 4:
            raise RuntimeError("truncated qsnap")
        dim = int(np.frombuffer(dimb, dtype="<u4")[0])
        count = nsnap * layers * nq * dim
        q = np.frombuffer(f.read(2 * count), dtype="<u2")
        if q.size != count:
            raise RuntimeError("truncated qsnap")
    return QSnap([int(p) for p in pos], layers, nq, dim, q.reshape(nsnap, layers, nq, dim))


def check_pair(dump: Dump, qs: QSnap) -> None:
    """src/bench.cpp:420-423."""
    if qs.layers != dump.layers or qs.nq != dump.nq or qs.dim != dump.dim:
        raise RuntimeError("qsnap does not match dump")


def write_kvd1(path: str, k: np.ndarray, v: np.ndarray, q_last: np.ndarray) -> None:
    """A KVD1 file in python/dump_kv.py's layout (k, v: [layers, kv, seq, dim] uint16; q_last:
    [layers, q_heads, dim] uint16), for tests and for callers that build dumps themselves."""
    hdr = np.zeros(8, dtype="<u4")
    hdr[0] = np.frombuffer(KVD1_MAGIC, dtype="<u4")[0]
    hdr[1] = 1
    hdr[2], hdr[3], hdr[5], hdr[6] = k.shape[0], k.shape[1], k.shape[3], k.shape[2]
    hdr[4] = q_last.shape[1]
    with open(path, "wb") as f:
        f.write(hdr.tobytes())
        f.write(np.ascontiguousarray(k, dtype="<u2").tobytes())
        f.write(np.ascontiguousarray(v, dtype="<u2").tobytes())
        f.write(np.ascontiguousarray(q_last, dtype="<u2").tobytes())


def write_qsn1(path: str, pos, q: np.ndarray) -> None:
    """A QSN1 file in python/dump_kv.py's layout (q: [n_snap, layers, q_heads, dim] uint16)."""
    hdr = np.zeros(4, dtype="<u4")
    hdr[0] = np.frombuffer(QSN1_MAGIC, dtype="<u4")[0]
    hdr[1], hdr[2], hdr[3] = len(pos), q.shape[1], q.shape[2]
    with open(path, "wb") as f:
        f.write(hdr.tobytes())
        f.write(np.asarray(pos, dtype="<u4").tobytes())
        f.write(np.asarray([q.shape[3]], dtype="<u4").tobytes())
        f.write(np.ascontiguousarray(q, dtype="<u2").tobytes())


@dataclass
class ModelHeads:
    """The model_heads scope at one length: inputs prepared for the library."""
    seq: int
    group: int
    qs: list        # per (layer, KV head): [group, dim] uint16
    kraw: list      # per unit: [seq, dim] uint16 (contiguous copies of the planes' prefixes)
    vraw: list
    kxs: list       # per unit: XKV blob (uint8)
    vxs: list
    container_bytes: int
    tight_bytes: int


def prepare_model_heads(kvx, dump: Dump, qs: QSnap, seq: int) -> ModelHeads:
    """Encode every (layer, KV head)'s first `seq` tokens with the library's encoder and pick the
    matching query snapshot (src/bench.cpp:571-690)."""
    check_pair(dump, qs)
    if seq <= 0 or seq > dump.seq:
        raise RuntimeError("bad argument")
    si = qs.index(seq)
    if dump.nq % dump.kv:
        raise RuntimeError("q_heads must be a multiple of kv_heads")
    group = dump.nq // dump.kv
    qv, kr, vr, kx, vx = [], [], [], [], []
    for ly in range(dump.layers):
        for h in range(dump.kv):
            qv.append(np.ascontiguousarray(qs.query(si, ly, h * group, group)))
            k = np.ascontiguousarray(dump.head(dump.k, ly, h, seq))
            v = np.ascontiguousarray(dump.head(dump.v, ly, h, seq))
            kr.append(k)
            vr.append(v)
            kx.append(kvx.encode_bf16(k, seq, dump.dim).bytes)
            vx.append(kvx.encode_bf16(v, seq, dump.dim).bytes)
    cont = sum(x.size for x in kx) + sum(x.size for x in vx)
    tight = 2 * 2 * seq * dump.dim * len(kx)
    return ModelHeads(seq, group, qv, kr, vr, kx, vx, cont, tight)


def run_model_heads(kvx, m: ModelHeads, dim: int, how: str) -> np.ndarray:
    """One step of the scope: outputs [units, group, dim] float32.  how: "raw" (one
    attention_decode call per unit on the BF16 planes), "xkv" (the same on the XKV blobs) or
    "batched" (every unit in one attention_decode_units call)."""
    outs = [np.zeros((m.group, dim), dtype=np.float32) for _ in m.qs]
    if how == "batched":
        kvx.attention_decode_units(0, m.qs, m.kxs, [x.size for x in m.kxs], m.vxs,
                                   [x.size for x in m.vxs], outs, m.group, dim, m.seq)
    elif how == "xkv":
        for q, kx, vx, o in zip(m.qs, m.kxs, m.vxs, outs):
            kvx.attention_decode(0, q, None, None, kx, kx.size, vx, vx.size, o, m.group, dim, m.seq, 1)
    else:
        for q, k, v, o in zip(m.qs, m.kraw, m.vraw, outs):
            kvx.attention_decode(0, q, k, v, None, 0, None, 0, o, m.group, dim, m.seq, 1)
    return np.stack(outs)


def model_heads(kvx, dump: Dump, qs: QSnap, seq: int, reps: int = 5) -> dict:
    """Run the scope at one length.  Per unit, the XKV and raw outputs agree bit for bit (the
    reference's check, src/bench.cpp:688-690); the batched call, whose split of the work over the
    GPU differs, agrees per unit within 1e-4 of the unit's largest output magnitude (fp32 summation
    order).  Returns best-of-`reps` timings."""
    m = prepare_model_heads(kvx, dump, qs, seq)
    raw = run_model_heads(kvx, m, dump.dim, "raw")
    comp = run_model_heads(kvx, m, dump.dim, "xkv")
    if not np.array_equal(raw.view(np.uint32), comp.view(np.uint32)):
        raise RuntimeError("bit mismatch on full model")
    bat = run_model_heads(kvx, m, dump.dim, "batched")
    mag = np.maximum(np.abs(comp).reshape(len(comp), -1).max(axis=1), 1e-30)
    rel = float(np.max(np.abs(bat - comp).reshape(len(comp), -1).max(axis=1) / mag))
    if rel >= 1e-4:
        raise RuntimeError(f"batched outputs differ from the per-unit ones (max {rel:.2e} of the "
                           "unit's largest output)")
    t = {}
    for how in ("raw", "xkv", "batched"):
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            run_model_heads(kvx, m, dump.dim, how)
            ts.append(time.perf_counter() - t0)
        t[how] = 1e3 * min(ts)
    return {"scope": "model_heads", "seq": seq, "layers": dump.layers, "kv_heads": dump.kv,
            "q_heads": dump.nq, "head_dim": dump.dim, "raw_ms": t["raw"], "xkv_ms": t["xkv"],
            "batched_ms": t["batched"], "container_bytes": m.container_bytes,
            "tight_bytes": m.tight_bytes, "container_ratio": m.container_bytes / m.tight_bytes,
            "batched_gbps": m.container_bytes / (t["batched"] * 1e-3) / 1e9}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--dump", required=True)
    ap.add_argument("--qsnap", required=True)
    ap.add_argument("--seq", type=int, action="append", help="lengths (default: every snapshot)")
    ap.add_argument("--reps", type=int, default=5)
    a = ap.parse_args(argv)
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import kvexp_b200 as kvx
    dump, qs = load_kvd1(a.dump), load_qsn1(a.qsnap)
    check_pair(dump, qs)
    for seq in a.seq or [p for p in qs.pos if p <= dump.seq]:
        print(json.dumps(model_heads(kvx, dump, qs, seq, a.reps)), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
