"""Device-resident XKV caches for the benchmark configurations.

A workload is a set of units -- one (layer, KV head[, sequence]) each, with its GQA group of
queries.  K/V are generated on the GPU by the seeded synthetic generator (kvx_synth_bf16,
bit-identical to synth.py) and encoded on the GPU (kvx_encode_batch, byte-identical to the
reference encoder) into one arena with a block index.  This stands in for the reference's
KVD1 dump + per-head encode (src/bench.cpp:584-605).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

import synth as S


@dataclass(frozen=True)
class Config:
    name: str
    layers: int
    kv_heads: int
    group: int        # query heads per KV head (GQA)
    dim: int
    seq: int
    seqs: int = 1     # independent sequences (batched decode)
    k_profile: int = S.PROFILE_K
    v_profile: int = S.PROFILE_V
    layer0_k_profile: int | None = None
    block: int = 128
    # How N GPUs share the workload: "split" (the (layer, KV head) units dealt out in contiguous
    # runs, one per GPU: strong scaling), "replica" (each GPU its own full cache), "units" (the
    # (layer, KV head, sequence) units split over 8 GPU slots) or "sequence" (every KV head's
    # sequence cut into block-aligned shards, folded by log-sum-exp).
    shard: str = "replica"

    @property
    def units(self) -> int:
        return self.layers * self.kv_heads * self.seqs

    @property
    def tight_bytes(self) -> int:
        return 4 * self.seq * self.dim * self.units


CONFIGS = {
    0: Config("config[0]: 1L x 1KV x GQA7 x D64 x S8192", 1, 1, 7, 64, 8192),
    1: Config("config[1]: 24L x 2KV x GQA7 x D64 x S32768 (Qwen2.5-0.5B shape)", 24, 2, 7, 64,
              32768, layer0_k_profile=S.PROFILE_NARROW, shard="split"),
    2: Config("config[2]: config[1] shape at S32731 (91-token tail block)", 24, 2, 7, 64, 32731,
              layer0_k_profile=S.PROFILE_NARROW, shard="split"),
    3: Config("config[3]: 32L x 8KV x GQA4 x D128 x 64 seqs x S32768 (Llama-3-8B shape)", 32, 8,
              4, 128, 32768, seqs=64, shard="units"),
    4: Config("config[4]: 1L x 8KV x GQA4 x D256 x S1048576", 1, 8, 4, 256, 1 << 20,
              k_profile=S.PROFILE_WIDE_K, v_profile=S.PROFILE_WIDE_V, shard="sequence"),
}


def k_profile_of(cfg: Config, unit: int) -> int:
    layer = unit // (cfg.kv_heads * cfg.seqs)
    if layer == 0 and cfg.layer0_k_profile is not None:
        return cfg.layer0_k_profile
    return cfg.k_profile


def rate_of(profile: int) -> int:
    return {S.PROFILE_NARROW: S.RATE_8, S.PROFILE_WIDE_K: S.RATE_2,
            S.PROFILE_WIDE_V: S.RATE_2}.get(profile, S.RATE_0P3)


@dataclass
class DeviceCache:
    cfg: Config
    unit_ids: list
    arenas: list = field(default_factory=list)     # torch uint8 tensors (kept alive)
    indexes: list = field(default_factory=list)
    k: list = field(default_factory=list)          # (arena_idx, offset, bytes) per unit
    v: list = field(default_factory=list)
    q: object = None                               # torch int16 [U, G, D]
    out: object = None                             # torch float32 [U, G, D]
    nb_per: int = 0

    @property
    def compressed_bytes(self) -> int:
        return int(sum(b for _, _, b in self.k) + sum(b for _, _, b in self.v))

    def kvx_units(self, out=None, lse=None):
        """kvx_unit descriptors of every unit; outputs go to self.out unless `out` ([U, G, D]
        FP32) is given; `lse` ([U, G] FP32) optionally receives each query's log-sum-exp."""
        import kvexp_b200 as kvx
        out = self.out if out is None else out
        units = []
        for i in range(len(self.unit_ids)):
            ka, ko, kb = self.k[i]
            va, vo, vb = self.v[i]
            kidx = self._index_of(ka, i, 0)
            vidx = self._index_of(va, i, 1)
            units.append(kvx.kvx_unit(
                self.arenas[ka].data_ptr() + ko, self.arenas[va].data_ptr() + vo,
                kidx, vidx, self.q[i].data_ptr(), out[i].data_ptr(), kb, vb,
                self.nb_per, self.cfg.seq, None if lse is None else lse[i].data_ptr()))
        return units

    def _index_of(self, arena_idx, i, kind):
        # index tensor t of chunk arena_idx: entries for blob (2 * local + kind)
        local = self._local[i]
        base = self.indexes[arena_idx].data_ptr()
        return base + (2 * local + kind) * self.nb_per * 8

    def host_blobs(self, units=None):
        """Host copies (numpy) of the K and V blobs and queries of `units` (local positions;
        default all)."""
        units = range(len(self.unit_ids)) if units is None else units
        ks = [self.arenas[self.k[i][0]][self.k[i][1]:self.k[i][1] + self.k[i][2]].cpu().numpy()
              for i in units]
        vs = [self.arenas[self.v[i][0]][self.v[i][1]:self.v[i][1] + self.v[i][2]].cpu().numpy()
              for i in units]
        qs = [self.q[i].cpu().numpy().view(np.uint16).copy() for i in units]
        return qs, ks, vs


def _torch():
    import torch
    return torch


def build_cache(cfg: Config, unit_ids=None, seed: int = 0x12345678, device="cuda",
                chunk_units: int | None = None, code_bits: int | None = None) -> DeviceCache:
    """Generate and GPU-encode the units `unit_ids` (default: all) of `cfg`; code_bits selects
    the residual widths (default the reference's {2, 4}; kvx.CODE_BITS_ALL adds 3-bit blocks)."""
    import kvexp_b200 as kvx
    torch = _torch()
    if unit_ids is None:
        unit_ids = list(range(cfg.units))
    U = len(unit_ids)
    nb_per = (cfg.seq + cfg.block - 1) // cfg.block
    if chunk_units is None:
        # keep about 4 GiB of tight BF16 in flight while encoding
        per = 4 * cfg.seq * cfg.dim
        chunk_units = max(1, min(U, (4 << 30) // per))
    cache = DeviceCache(cfg, list(unit_ids), nb_per=nb_per)
    cache._local = [0] * U
    cache.q = torch.empty((U, cfg.group, cfg.dim), dtype=torch.int16, device=device)
    cache.out = torch.zeros((U, cfg.group, cfg.dim), dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream().cuda_stream
    for c0 in range(0, U, chunk_units):
        ids = unit_ids[c0:c0 + chunk_units]
        tens = []
        for u in ids:
            kt = torch.empty((cfg.seq, cfg.dim), dtype=torch.int16, device=device)
            vt = torch.empty((cfg.seq, cfg.dim), dtype=torch.int16, device=device)
            kp = k_profile_of(cfg, u)
            kvx.synth_bf16(kt, cfg.seq, cfg.dim, seed, S.stream_id(u, 0), kp, rate_of(kp), stream)
            kvx.synth_bf16(vt, cfg.seq, cfg.dim, seed, S.stream_id(u, 1), cfg.v_profile,
                           rate_of(cfg.v_profile), stream)
            tens += [kt, vt]
        for j, u in enumerate(ids):
            kvx.synth_bf16(cache.q[c0 + j], cfg.group, cfg.dim, seed, S.stream_id(u, 2),
                           S.PROFILE_Q, 0, stream)
        arena_bytes, entries = kvx.encode_batch_bounds(len(tens), cfg.seq, cfg.dim, cfg.block)
        arena = torch.empty(arena_bytes, dtype=torch.uint8, device=device)
        index = torch.empty(entries * 8, dtype=torch.uint8, device=device)
        off, nbytes = kvx.encode_batch(tens, cfg.seq, cfg.dim, arena, index, cfg.block, stream,
                                       code_bits=kvx.CODE_BITS_REFERENCE if code_bits is None
                                       else code_bits)
        del tens
        used = int(off[-1] + nbytes[-1] + 16 + 15) & ~15
        if used < arena_bytes // 2:  # compact large arenas
            small = torch.empty(used, dtype=torch.uint8, device=device)
            small.copy_(arena[:used])
            arena = small
        a = len(cache.arenas)
        cache.arenas.append(arena)
        cache.indexes.append(index)
        for j in range(len(ids)):
            cache.k.append((a, int(off[2 * j]), int(nbytes[2 * j])))
            cache.v.append((a, int(off[2 * j + 1]), int(nbytes[2 * j + 1])))
            cache._local[c0 + j] = j
    torch.cuda.synchronize()
    return cache
