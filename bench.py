#!/usr/bin/env python
"""Benchmark of the fused compressed-KV (XKV) decode attention on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl kvx|reference]

One step = one decode-attention pass over every (layer, KV head) unit of the workload (the
reference's `model_heads` scope, src/bench.cpp:711-728) with the KV cache resident in HBM.
Default workload: BASELINE.json config[1] (24 layers x 2 KV heads x GQA 7 x head_dim 64 x
32768 tokens, block 128), synthetic seeded data.  With N > 1 (torchrun) the 48 (layer, KV head)
units are split over the ranks (strong scaling: one step of the whole config on N GPUs, no
collective on the data path); time is the max over ranks.

--config 3 holds one of 8 layer x KV head shards of config[3] per GPU (the whole config does not
fit one GPU; N GPUs run N/8 of it, no collective).  --config 4 cuts config[4]'s 1M-token
sequence into N block-aligned shards, one per GPU, and ends each step with one NCCL all-gather
of (out, lse) and the rank-ordered fold kernel (strong scaling).

Prints one JSON line (rank 0).  `--impl reference` times the unmodified reference library
(compiled from its own sources into oracle/_ref) on this host's cores on the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in ("compressed-kv-attention_b200", "oracle"):
    sys.path.insert(0, os.path.join(ROOT, p))

METRIC = "compressed-KV decode GB/s and % of HBM peak; µs/step at 32K (1/2/4/8 B200)"
# The reference's published number for this metric: model_heads scope, AVX-512 BF16, 4 threads,
# seq 32768, XKV container bandwidth (reference README.md:159, results/bench.json:172).
PUBLISHED_GBPS = 2.129
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--config", type=int, default=1)
    ap.add_argument("--seq", type=int, default=0,
                    help="attend this many tokens instead of the config's (config[2]'s prefix "
                         "sweep: 8192, 16384, 32731)")
    ap.add_argument("--impl", default="kvx", choices=["kvx", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the check of the timed outputs against the reference")
    ap.add_argument("--e2e-steps", type=int, default=8)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--code-bits", default="24", choices=["24", "234"],
                    help="residual widths of the GPU-encoded cache: the reference's {2, 4} "
                         "(default), or with the library's 3-bit extension")
    ap.add_argument("--units", type=int, default=0,
                    help="only the first N units of this GPU's share (small cases for profilers; "
                         "not a bench line of the config)")
    return ap.parse_args()


def config_of(args):
    """BASELINE.json config[args.config], at args.seq tokens when given."""
    import dataclasses
    import workloads as W
    cfg = W.CONFIGS[args.config]
    if args.seq > 0:
        cfg = dataclasses.replace(cfg, seq=args.seq, name=f"{cfg.name} at S{args.seq}")
    return cfg


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def hbm_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "of measured (MEASURED_PEAKS.json hbm_gbs: copy, read+write)"
    except Exception:
        return FALLBACK_HBM_GBS, "of fallback (6.65 TB/s)"


def ncu_traffic(config, n_units):
    """DRAM bytes per launch of the attention kernel from the committed ncu summary, if any,
    scaled from the captured launch's units to this launch's (the traffic of a unit is fixed)."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(path) as f:
            d = json.load(f)
        e = d.get(str(config))
        if e is None:
            return None
        return float(e["dram_bytes_per_launch"]) * n_units / float(e["units"])
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index, interval_ms=50):
        self.dev = device_index
        self.interval = interval_ms
        self.lines = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.dev), "-lms", str(self.interval)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()
        time.sleep(0.3)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, pw, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
                pw.append(float(parts[3]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None,
                "samples": len(sm), "reasons": sorted(reasons)}


# ---- CPU reference timing ------------------------------------------------------------------------

BACKEND_NAMES = {0: "scalar", 1: "AVX2", 2: "AVX-512 BF16"}


def ref_backends(ref):
    """The reference's backends this host runs, fastest first (AVX-512 BF16, AVX2, scalar)."""
    import oracle as O
    out = [b for b, ok in ((O.AVX512BF16, ref.avx512_bf16), (O.AVX2, ref.avx2)) if ok]
    return out or [O.SCALAR]


def make_ref_step(ref, be, qs, ks, vs, outs, cfg, threads, cores):
    """One pass of the reference over the units: its model_heads scope (one OpenMP thread per
    (layer, KV head) unit, src/bench.cpp:711-728), or for a single unit its head scope (one
    attention_decode over every core, the sequence split at the 128-token blocks)."""
    if len(qs) == 1:
        def step():
            outs[0][...] = ref.attention(qs[0], kx=ks[0], vx=vs[0], seq=cfg.seq, backend=be,
                                         threads=cores, split=cfg.block)
        return step
    return lambda: ref.model_heads(be, qs, ks, vs, outs, cfg.group, cfg.dim, cfg.seq, threads)


def cpu_reference_rate(qs, ks, vs, cfg, seconds, max_passes=50, backend=None):
    """Time the reference library's model_heads loop (oracle/_ref) on all usable host cores with
    `backend` (default: the fastest this host runs); falls back to the C restatement (oracle/)
    when the reference was not built."""
    import numpy as np
    import oracle as O
    n = len(qs)
    outs = [np.zeros((cfg.group, cfg.dim), dtype=np.float32) for _ in range(n)]
    total = sum(k.size for k in ks) + sum(v.size for v in vs)
    threads = max(1, min(n, os.cpu_count() or 1))
    ref = O.reference()
    if ref is not None:
        be = backend if backend is not None else ref_backends(ref)[0]
        bname = BACKEND_NAMES[be]
        run = make_ref_step(ref, be, qs, ks, vs, outs, cfg, threads, os.cpu_count() or 1)
        if n == 1:
            threads = os.cpu_count() or 1
        kind = "reference"
        what = f"reference kvexp model_heads, {bname}, {threads} OpenMP threads"
    else:
        from concurrent.futures import ThreadPoolExecutor
        orc = O.oracle()
        pool = ThreadPoolExecutor(threads)

        def run():
            list(pool.map(lambda u: orc.attention(qs[u], kx=ks[u], vx=vs[u], seq=cfg.seq),
                          range(n)))
        kind = "port"
        what = f"C restatement (oracle/), {threads} threads"
    run()  # warm-up
    t0 = time.perf_counter()
    passes = 0
    while True:
        run()
        passes += 1
        el = time.perf_counter() - t0
        if el >= seconds or passes >= max_passes:
            break
    gbps = total * passes / el / 1e9
    return {"value": gbps, "unit": "GB/s", "cores": threads, "kind": kind,
            "sample": f"{passes} full passes over {n} units of {cfg.name} "
                      f"({total / 1e6:.1f} MB of XKV containers per pass), {what}, "
                      f"{el:.1f} s wall"}, el / passes


def host_workload(cfg, seed, n_units=None):
    """Host-side inputs for the reference arm: numpy synthetic data encoded by the reference's
    own encoder (no GPU code), for the first n_units units (default all)."""
    import numpy as np
    import oracle as O
    import synth as S
    import workloads as W
    ref = O.reference()
    enc = ref.encode if ref is not None else O.oracle().encode
    qs, ks, vs = [], [], []
    for u in range(cfg.units if n_units is None else n_units):
        kp = W.k_profile_of(cfg, u)
        k = S.synth_bf16(seed, S.stream_id(u, 0), cfg.seq, cfg.dim, kp, W.rate_of(kp))
        v = S.synth_bf16(seed, S.stream_id(u, 1), cfg.seq, cfg.dim, cfg.v_profile,
                         W.rate_of(cfg.v_profile))
        q = S.synth_bf16(seed, S.stream_id(u, 2), cfg.group, cfg.dim, S.PROFILE_Q, 0)
        ks.append(enc(k, cfg.block))
        vs.append(enc(v, cfg.block))
        qs.append(np.ascontiguousarray(q))
    return qs, ks, vs


def run_reference(args, rank, world):
    if rank != 0:
        return
    cfg = config_of(args)
    # a workload too large for host memory is timed on its first units (the metric is per byte)
    per_unit = 4 * cfg.seq * cfg.dim
    n_units = cfg.units if cfg.units * per_unit <= 8 << 30 else max(1, (4 << 30) // per_unit)
    qs, ks, vs = host_workload(cfg, 0x12345678, n_units)
    import numpy as np
    import oracle as O
    ref = O.reference()
    if ref is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref was not built"}))
        return
    n = len(qs)
    outs = [np.zeros((cfg.group, cfg.dim), dtype=np.float32) for _ in range(n)]
    cores = os.cpu_count() or 1
    threads = cores if n == 1 else max(1, min(n, cores))
    total = sum(k.size for k in ks) + sum(v.size for v in vs)


    def timed(be, budget_s):
        step = make_ref_step(ref, be, qs, ks, vs, outs, cfg, threads, cores)
        # a step is one model_heads pass; keep the run within a few minutes
        for _ in range(max(1, args.warmup)):
            step()
        t0 = time.perf_counter()
        step()
        one = time.perf_counter() - t0
        steps = max(1, min(args.steps, int(budget_s / max(one, 1e-6))))
        t0 = time.perf_counter()
        for _ in range(steps):
            step()
        el = time.perf_counter() - t0
        return steps, el

    backends = ref_backends(ref)
    be = backends[0]
    bname = BACKEND_NAMES[be]
    steps, el = timed(be, 90.0)
    gbps = total * steps / el / 1e9
    others = {}
    for b in backends[1:]:
        st2, el2 = timed(b, 45.0)
        others[BACKEND_NAMES[b]] = {"value": total * st2 / el2 / 1e9, "unit": "GB/s",
                                    "ms_per_step": el2 / st2 * 1e3, "steps": st2}
    line = {
        "metric": METRIC, "impl": "reference", "value": gbps, "unit": "GB/s", "n_gpus": world,
        "steps": steps, "warmup": max(1, args.warmup), "ms_per_step": el / steps * 1e3,
        "higher_is_better": True,
        "scaling": "strong" if cfg.shard in ("sequence", "split") else "weak",
        "vs_baseline": gbps / PUBLISHED_GBPS, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": cfg.name, "units": n, "compressed_bytes_per_step": total,
                   "units_of_workload": cfg.units, "backend": bname, "threads": threads},
        "other_backends": others,
        "cpu_baseline": {"value": gbps, "unit": "GB/s", "cores": threads, "kind": "reference",
                         "sample": f"{steps} model_heads passes over {n} of {cfg.units} units, "
                                   f"{bname}"},
        "e2e": {"value": gbps, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def parity_check(qs, ks, vs, cfg, plan_out, e2e_out, three_bit=False):
    """Check GPU outputs of the timed units against the float64 truth and the reference
    library's scalar kernel (oracle/_ref, or the C restatement when the reference was not built)
    on the same blobs and queries (oracle/parity.py: |gpu - truth| <= tol, and
    |gpu - ref| <= |ref - truth| + tol).  This is the reference benchmark's own rule of comparing
    before timing (src/bench.cpp:732-734), with a tolerance because the GPU's accumulation order
    is not the reference's."""
    import numpy as np
    import oracle as O
    import parity as P
    n = len(qs)
    # the reference cannot read 3-bit blocks: the oracle's restatement (which can) checks those
    ref = None if three_bit else O.reference()
    outs = [np.zeros((cfg.group, cfg.dim), dtype=np.float32) for _ in range(n)]
    threads = max(1, min(n, os.cpu_count() or 1))
    t0 = time.perf_counter()
    if ref is not None:
        ref.model_heads(O.SCALAR, qs, ks, vs, outs, cfg.group, cfg.dim, cfg.seq, threads)
        what = "reference kvexp (oracle/_ref), scalar backend, one thread per unit"
        decode = ref.decode
    else:
        orc = O.oracle()
        outs = [orc.attention(qs[u], kx=ks[u], vx=vs[u], seq=cfg.seq) for u in range(n)]
        what = "C restatement of the reference's scalar kernel (oracle/)"
        decode = orc.decode
    res = {"reference": what, "units_checked": n, "truth": "float64 softmax(q K^T) V",
           "tolerance": f"tol = {P.ATOL:g} scale + {P.RTOL:g} |truth| + sqrt(D) 2^-24 cond per "
                        "element (scale = p-weighted mean |v|, cond = p-weighted sum_d |q_d k_d| "
                        "(|v| + |truth|), the fp32 score-error term); accuracy = max "
                        "|gpu - truth| / tol, parity = max |gpu - ref| / (|ref - truth| + tol); "
                        "both <= 1 pass"}
    keys = [("plan", plan_out)] + ([("e2e", e2e_out)] if e2e_out is not None else [])
    for key, _ in keys:
        res[key] = {"accuracy": 0.0, "parity": 0.0, "gpu_err_over_scale": 0.0}
    ref_err = 0.0
    for u in range(n):
        k = decode(ks[u], cfg.seq, cfg.dim)
        v = decode(vs[u], cfg.seq, cfg.dim)
        ex = P.exact(qs[u], k, v)
        for key, got in keys:
            m = P.measure(got[u], outs[u], ex)
            r = res[key]
            for f in ("accuracy", "parity", "gpu_err_over_scale"):
                r[f] = max(r[f], m[f])
            ref_err = max(ref_err, m["ref_err_over_scale"])
    res["ref_err_over_scale"] = ref_err
    res["ok"] = all(res[k]["accuracy"] <= 1.0 and res[k]["parity"] <= 1.0 for k, _ in keys)
    res["seconds"] = time.perf_counter() - t0
    return res


# ---- GPU arm ----------------------------------------------------------------------------------------

GPU_SLOTS = 8          # config[3] is cut into 8 unit shards, one per GPU of an 8-GPU box
L2_BYTES = 126 << 20   # B200 L2
MAX_COPIES = 16
SAMPLE_BYTES = 1 << 30  # host sample (CPU baseline, end-to-end) for workloads above this size


def rank_share(cfg, rank, world):
    """This rank's part of the workload: (config to build, unit ids or None, seed, description).

    split    -- GPU r holds units [r*U/N, (r+1)*U/N) of the U (layer, KV head) units (strong
                scaling: the whole config over N GPUs, no collective);
    replica  -- every GPU decodes its own full cache (weak scaling, no collective);
    units    -- GPU r holds unit shard r of GPU_SLOTS (weak scaling: N GPUs run N/8 of the
                config; no collective);
    sequence -- GPU r holds blocks [r*B/N, (r+1)*B/N) of every KV head (strong scaling); one
                NCCL all-gather of (out, lse) and a rank-ordered fold end the step.
    """
    import dataclasses
    import seqsplit
    base = 0x12345678
    if cfg.shard == "units":
        if world > GPU_SLOTS:
            raise SystemExit(f"{cfg.name} is sharded over at most {GPU_SLOTS} GPUs")
        per = cfg.units // GPU_SLOTS
        ids = list(range(rank * per, (rank + 1) * per))
        return cfg, ids, base, (f"layer x KV head shards: GPU r holds units [r*{per}, (r+1)*{per}) "
                                f"of {cfg.units} (one of {GPU_SLOTS} shards, 4 layers each); "
                                "no collective")
    if cfg.shard == "split":
        if world > cfg.units:
            raise SystemExit(f"{cfg.name} has {cfg.units} units: at most that many GPUs")
        u0, u1 = rank * cfg.units // world, (rank + 1) * cfg.units // world
        return cfg, list(range(u0, u1)), base, (
            f"(layer, KV head) units split over the GPUs: GPU r holds units [r*{cfg.units}/N, "
            f"(r+1)*{cfg.units}/N) ({u1 - u0} units here); no collective")
    if cfg.shard == "sequence":
        nb = (cfg.seq + cfg.block - 1) // cfg.block
        b0, b1 = seqsplit.shard_blocks(nb, world, rank)
        sub = dataclasses.replace(cfg, seq=min(b1 * cfg.block, cfg.seq) - b0 * cfg.block)
        how = (f"sequence split: GPU r holds blocks [r*{nb}/N, (r+1)*{nb}/N) of every KV head"
               + ("; one NCCL all-gather of (out, lse) per step, then the rank-ordered fold "
                  "kernel (kvx_fold_shards)" if world > 1 else " (N=1: the whole sequence)"))
        return sub, None, base + 7919 * rank, how
    return cfg, None, base + 7919 * rank, f"dp{world}: an independent cache per GPU, no collective"


def run_kvx(args, rank, world, local):
    import numpy as np
    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    import kvexp_b200 as kvx
    import seqsplit
    import workloads as W
    full = config_of(args)
    cfg, unit_ids, seed, parallelism = rank_share(full, rank, world)
    if args.units > 0:
        unit_ids = list(unit_ids if unit_ids is not None else range(cfg.units))[: args.units]
        parallelism += f"; only the first {len(unit_ids)} units (--units, a profiling case)"
    n_units = cfg.units if unit_ids is None else len(unit_ids)
    code_bits = kvx.CODE_BITS_ALL if args.code_bits == "234" else kvx.CODE_BITS_REFERENCE
    cache = W.build_cache(cfg, unit_ids=unit_ids, seed=seed, code_bits=code_bits)
    caches = [cache]
    # Copies of the cache rotate between steps, enough that a step's blobs were last read at
    # least 3 x L2 bytes earlier: no step finds its inputs in L2.
    n_copies = 1 if cache.compressed_bytes >= 3 * L2_BYTES else min(
        MAX_COPIES, max(2, -(-3 * L2_BYTES // cache.compressed_bytes)))
    while len(caches) < n_copies:
        caches.append(W.build_cache(cfg, unit_ids=unit_ids, seed=seed, code_bits=code_bits))
    exch = None
    if cfg.shard == "sequence" and world > 1:
        exch = seqsplit.ShardExchange(n_units * cfg.group, cfg.dim)
        outs = exch.out_view().view(n_units, cfg.group, cfg.dim)
        lses = exch.lse_view().view(n_units, cfg.group)
        plans = [kvx.Plan(c.kvx_units(out=outs, lse=lses), cfg.group, cfg.dim, cfg.block)
                 for c in caches]
    else:
        plans = [kvx.Plan(c.kvx_units(), cfg.group, cfg.dim, cfg.block) for c in caches]
    comp = cache.compressed_bytes
    tight = 4 * cfg.seq * cfg.dim * n_units
    q_bytes = n_units * cfg.group * cfg.dim * 2
    o_bytes = n_units * cfg.group * cfg.dim * 4
    algo_bytes = comp + q_bytes + o_bytes
    stream = torch.cuda.current_stream()
    h = stream.cuda_stream

    # own device read probe (the reference's peak.hpp read bandwidth, on HBM)
    probe_buf = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    probe_gbs = kvx.hbm_read_probe(probe_buf, reps=5)
    del probe_buf

    def step(i):
        p = plans[i % len(plans)]
        p.run_part(0, h)
        p.run_part(1, h)
        if exch is not None:
            exch.step(h)

    for i in range(max(3, args.warmup)):
        step(i)
    for p in plans:
        p.check()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    sampler = ClockSampler(local)
    sampler.start()
    K = args.steps
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    # The attention kernel's own duration: KA launches of it alone, back to back (each launched as
    # a programmatic dependent of the one before, as in the steps), events only around the loop.
    KA = max(1, min(K, 500))
    torch.cuda.synchronize()
    start.record(stream)
    for i in range(KA):
        plans[i % len(plans)].run_part(0, h)
    end.record(stream)
    end.synchronize()
    kern_ms = start.elapsed_time(end) / KA
    # the timed region: K whole steps, no event between them
    for i in range(2):
        step(i)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    start.record(stream)
    for i in range(K):
        step(i)
    end.record(stream)
    end.synchronize()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = sampler.stop()
    elapsed_ms = start.elapsed_time(end)
    for p in plans:
        p.check()
    comp_all = comp * world
    if dist:
        t = torch.tensor([elapsed_ms, kern_ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms, kern_ms = float(t[0]), float(t[1])
        c = torch.tensor([comp, tight], dtype=torch.float64, device="cuda")
        dist.all_reduce(c, op=dist.ReduceOp.SUM)
        comp_all, tight_all = float(c[0]), float(c[1])
    else:
        tight_all = tight
    ms_step = elapsed_ms / K
    value = comp_all * K / (elapsed_ms * 1e-3) / 1e9

    # the host sample: every unit when the workload is small, else the first units up to about
    # SAMPLE_BYTES of containers
    sample = list(range(n_units))
    if comp > SAMPLE_BYTES:
        per_unit = comp / n_units
        sample = list(range(max(1, min(n_units, int(SAMPLE_BYTES // per_unit)))))

    qs, ks, vs = cache.host_blobs(sample)
    plan_out = cache.out[: len(sample)].cpu().numpy() if exch is None else None

    # end to end through the reference-facing C ABI with pinned host buffers
    e2e = None
    e2e_out = None
    if not args.no_e2e and exch is None:
        pk = [torch.from_numpy(x).pin_memory() for x in ks]
        pv = [torch.from_numpy(x).pin_memory() for x in vs]
        pq = [torch.from_numpy(x.view(np.int16)).pin_memory() for x in qs]
        po = [torch.zeros((cfg.group, cfg.dim), dtype=torch.float32).pin_memory()
              for _ in sample]
        call = lambda: kvx.attention_decode_units(
            0, pq, pk, [x.numel() for x in pk], pv, [x.numel() for x in pv], po, cfg.group,
            cfg.dim, cfg.seq)
        call()
        call()
        ts = []
        for _ in range(args.e2e_steps):
            t0 = time.perf_counter()
            call()
            ts.append(time.perf_counter() - t0)
        e2e_s = sum(ts) / len(ts)
        s_bytes = sum(x.numel() for x in pk) + sum(x.numel() for x in pv)
        if dist:
            t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = float(t[0])
        e2e = {"value": s_bytes * world / e2e_s / 1e9, "unit": "GB/s",
               "h2d_bytes_per_step": s_bytes + len(sample) * cfg.group * cfg.dim * 2,
               "d2h_bytes_per_step": len(sample) * cfg.group * cfg.dim * 4,
               "ms_per_step": e2e_s * 1e3, "steps": args.e2e_steps,
               "units_per_gpu": len(sample),
               "path": "kvx_attention_decode_units (C ABI) with pinned host blobs, one call "
                       "per step: H2D of every blob and query, header walks, decode attention, "
                       "D2H of outputs"}
        e2e_out = np.stack([o.numpy() for o in po])
        if np.array_equal(e2e_out.view(np.uint32), plan_out.view(np.uint32)):
            e2e["vs_plan"] = "bit-identical to the device-resident plan"
        else:
            e2e["vs_plan"] = ("differs from the device-resident plan in fp32 rounding (another "
                              "split of the units over workers); both are checked against the "
                              "reference in `parity`")

    # parity: the timed outputs against the reference's scalar kernel on the same units
    parity = None
    if exch is None and not args.no_parity:
        parity = parity_check(qs, ks, vs, cfg, plan_out, e2e_out, three_bit=args.code_bits == "234")
        if dist:
            keys = [k for k in ("plan", "e2e") if k in parity]
            vals = [parity[k][f] for k in keys for f in ("accuracy", "parity", "gpu_err_over_scale")]
            t = torch.tensor(vals + [parity["ref_err_over_scale"]], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            i = 0
            for k in keys:
                for f in ("accuracy", "parity", "gpu_err_over_scale"):
                    parity[k][f] = float(t[i])
                    i += 1
            parity["ref_err_over_scale"] = float(t[i])
            parity["ok"] = all(parity[k]["accuracy"] <= 1.0 and parity[k]["parity"] <= 1.0
                               for k in keys)
            parity["ranks"] = f"every rank checked its own sample; worst over {world} ranks"

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.code_bits == "24":
        import oracle as O
        cpu, _ = cpu_reference_rate(qs, ks, vs, cfg, args.cpu_seconds)
        ref = O.reference()
        if ref is not None and ref.avx2 and ref.avx512_bf16:
            avx2, _ = cpu_reference_rate(qs, ks, vs, cfg, args.cpu_seconds / 2, backend=O.AVX2)
            cpu["avx2"] = {"value": avx2["value"], "unit": "GB/s", "sample": avx2["sample"]}

    launches = K * plans[0].launches + (K if exch is not None else 0)
    for p in plans:
        p.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    peak, peak_src = hbm_peak()
    achieved = algo_bytes / (kern_ms * 1e-3) / 1e9
    traffic = ncu_traffic(args.config, n_units)
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": K,
        "warmup": max(3, args.warmup), "ms_per_step": ms_step, "us_per_step": ms_step * 1e3,
        "higher_is_better": True,
        "scaling": "strong" if cfg.shard in ("sequence", "split") else "weak",
        "vs_baseline": value / PUBLISHED_GBPS,
        "dtype": "bf16", "data": "synthetic (seeded generator; BASELINE.json distributions)",
        "config": {
            "workload": full.name, "units_per_gpu": n_units, "seq_per_gpu": cfg.seq,
            "block_tokens": cfg.block, "compressed_bytes_per_gpu_step": comp,
            "tight_bytes_per_gpu_step": tight,
            "container_ratio": comp / tight,
            "code_bits": ("{2, 4} (the reference's container)" if args.code_bits == "24" else
                          "{2, 3, 4} (with the library's 3-bit extension; the reference cannot "
                          "read these blobs, so no CPU baseline and parity against the oracle)"),
            "parallelism": parallelism,
            "l2": (f"{len(caches)} cache copies rotate between steps: a step's inputs were last "
                   f"read {(len(caches) - 1) * comp / 1e6:.0f} MB earlier (L2 126 MB)"
                   if len(caches) > 1 else "inputs larger than 3 x L2 (126 MB)"),
        },
        "tight_equiv_gbps": tight_all * K / (elapsed_ms * 1e-3) / 1e9,
        "pct_of_hbm_peak": 100.0 * (value / world) / peak,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "kernel": "attn_kernel (fused XKV decode + QK + online softmax + PV)",
                     "algorithmic_bytes_per_launch": algo_bytes,
                     "kernel_ms_per_launch": kern_ms,
                     "kernel_timing": f"CUDA events around {KA} back-to-back launches of the attention kernel alone (programmatic dependent launches, as in the steps), same plans and clocks as the timed region",
                     "peak_source": peak_src,
                     "device_read_probe_gbs": probe_gbs},
        "cpu_baseline": cpu,
        "parity": parity,
        "e2e": e2e,
        "gpu_launches": launches,
        "clocks": clocks,
        "impl": "kvexp_b200",
    }
    if exch is not None:
        line["exchange"] = {"collective": "NCCL all_gather_into_tensor", "bytes_per_rank":
                            exch.bytes_per_rank, "fold": "kvx_fold_shards, rank order"}
        line["e2e_note"] = ("no end-to-end line for the sequence split: the host-buffer entry "
                            "points return no lse to fold")
    print(json.dumps(line), flush=True)
    if parity is not None and not parity["ok"]:
        print("PARITY FAILURE: the timed GPU outputs are outside the tolerance "
              f"(plan {parity['plan']}" + (f", end to end {parity['e2e']}" if "e2e" in parity else "")
              + "); this line measures a wrong result", file=sys.stderr, flush=True)
        sys.exit(1)


def main():
    args = parse()
    rank, world, local = env_rank()
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_kvx(args, rank, world, local)


if __name__ == "__main__":
    main()
