"""GPU: the per-query log-sum-exp output (kvx_unit.lse) and the sequence split it serves.

  * lse == ln(sum_t exp(q.k_t)) of a float64 softmax, within FP32 tolerance, for whole units and
    for units the plan splits across workers (the combine kernel writes it then);
  * a sequence cut into block-aligned shards (one plan unit per shard, as one rank per shard
    would hold it) and folded by seqsplit.fold gives the single-plan output within the FP32
    attention tolerance -- the multi-GPU config[4] path emulated on one GPU.
"""
import numpy as np
import pytest

import seqsplit
import synth as S
from helpers import assert_attention_close, bf16_to_f64, soften

pytestmark = pytest.mark.gpu


def _case(dim, n_q, seq, seed, soft):
    k = S.synth_bf16(seed, 0, seq, dim, S.PROFILE_K)
    v = S.synth_bf16(seed, 1, seq, dim, S.PROFILE_V)
    q = soften(S.synth_bf16(seed, 2, n_q, dim, S.PROFILE_Q), soft)
    return q, k, v


def _lse_f64(q, k):
    s = bf16_to_f64(q) @ bf16_to_f64(k).T
    m = s.max(axis=1)
    return m + np.log(np.exp(s - m[:, None]).sum(axis=1))


class _Blobs:
    """K/V blobs and block indexes of one sequence, resident on the GPU."""

    def __init__(self, kvx, oracle, k, v, dim):
        import torch
        self.seq = k.shape[0]
        self.dim = dim
        self.kx = torch.from_numpy(oracle.encode(k, 128)).cuda()
        self.vx = torch.from_numpy(oracle.encode(v, 128)).cuda()
        self.n_blocks = (self.seq + 127) // 128
        self.ki = torch.empty(self.n_blocks * 8, dtype=torch.uint8, device="cuda")
        self.vi = torch.empty(self.n_blocks * 8, dtype=torch.uint8, device="cuda")
        assert kvx.xkv_index(self.kx, self.kx.numel(), dim, self.ki, self.n_blocks)[0] == \
            self.n_blocks
        assert kvx.xkv_index(self.vx, self.vx.numel(), dim, self.vi, self.n_blocks)[0] == \
            self.n_blocks

    def unit(self, kvx, q, out, lse, b0=0, b1=None):
        """Unit over blocks [b0, b1): the index entries hold offsets from the blob start, so a
        shard is the same blob with its index advanced to block b0."""
        b1 = self.n_blocks if b1 is None else b1
        t1 = min(b1 * 128, self.seq)
        return kvx.make_unit(self.kx, self.vx, q, out, k_index=self.ki.data_ptr() + 8 * b0,
                             v_index=self.vi.data_ptr() + 8 * b0, k_bytes=self.kx.numel(),
                             v_bytes=self.vx.numel(), n_blocks=b1 - b0, seq=t1 - b0 * 128,
                             lse=lse)


def _run(kvx, units, n_q, dim):
    import torch
    plan = kvx.Plan(units, n_q, dim)
    plan.run()
    plan.check()
    torch.cuda.synchronize()
    split = plan.n_split
    plan.close()
    return split


@pytest.mark.parametrize("dim,n_q,seq,soft", [(64, 7, 3000, 6), (128, 4, 20000, 7),
                                              (256, 4, 40 * 128 + 37, 7), (32, 8, 129, 5)])
def test_lse_matches_float64(kvx, cuda, oracle, dim, n_q, seq, soft):
    import torch
    q, k, v = _case(dim, n_q, seq, 31, soft)
    blobs = _Blobs(kvx, oracle, k, v, dim)
    dq = torch.from_numpy(q.view(np.int16)).cuda()
    out = torch.zeros((n_q, dim), dtype=torch.float32, device="cuda")
    lse = torch.full((n_q,), float("nan"), dtype=torch.float32, device="cuda")
    _run(kvx, [blobs.unit(kvx, dq, out, lse)], n_q, dim)
    want = _lse_f64(q, k)
    got = lse.cpu().numpy().astype(np.float64)
    tol = 2e-5 * np.sqrt(max(1.0, seq / 64)) * (1 + np.abs(want))
    assert np.all(np.abs(got - want) <= tol), (got, want)


def test_lse_of_split_units(kvx, cuda, oracle):
    """Few long units: the plan splits them across workers and the combine kernel writes lse."""
    import torch
    dim, n_q, seq = 64, 7, 64 * 1024
    q, k, v = _case(dim, n_q, seq, 32, 6)
    blobs = _Blobs(kvx, oracle, k, v, dim)
    dq = torch.from_numpy(q.view(np.int16)).cuda()
    out = torch.zeros((n_q, dim), dtype=torch.float32, device="cuda")
    lse = torch.full((n_q,), float("nan"), dtype=torch.float32, device="cuda")
    assert _run(kvx, [blobs.unit(kvx, dq, out, lse)], n_q, dim) > 0, "unit was not split"
    want = _lse_f64(q, k)
    got = lse.cpu().numpy().astype(np.float64)
    tol = 2e-5 * np.sqrt(seq / 64) * (1 + np.abs(want))
    assert np.all(np.abs(got - want) <= tol), (got, want)


@pytest.mark.parametrize("dim,n_q,seq,world", [(256, 4, 64 * 128 + 37, 2), (256, 4, 64 * 128, 8),
                                               (128, 4, 300 * 128, 3), (64, 7, 7 * 128 + 1, 8)])
def test_sequence_split_fold_matches_whole(kvx, cuda, oracle, dim, n_q, seq, world):
    import torch
    q, k, v = _case(dim, n_q, seq, 33, 7)
    blobs = _Blobs(kvx, oracle, k, v, dim)
    dq = torch.from_numpy(q.view(np.int16)).cuda()
    whole = torch.zeros((n_q, dim), dtype=torch.float32, device="cuda")
    _run(kvx, [blobs.unit(kvx, dq, whole, None)], n_q, dim)
    outs = torch.zeros((world, n_q, dim), dtype=torch.float32, device="cuda")
    lses = torch.zeros((world, n_q), dtype=torch.float32, device="cuda")
    units = []
    for r in range(world):
        b0, b1 = seqsplit.shard_blocks(blobs.n_blocks, world, r)
        if b1 == b0:  # an empty shard contributes nothing: weight exp(-inf) = 0
            lses[r] = float("-inf")
            continue
        units.append(blobs.unit(kvx, dq, outs[r], lses[r], b0, b1))
    _run(kvx, units, n_q, dim)
    folded = seqsplit.fold(outs, lses).cpu().numpy()
    cpu = oracle.attention(q, kx=oracle.encode(k, 128), vx=oracle.encode(v, 128), seq=seq)
    assert_attention_close(folded, cpu, q, k, v, f"fold world={world}")
    assert_attention_close(whole.cpu().numpy(), cpu, q, k, v, "whole")


@pytest.mark.parametrize("n_parts,rows,dim", [(1, 3, 64), (2, 32, 256), (8, 32, 256),
                                              (5, 7, 40), (3, 200, 128)])
def test_fold_kernel_matches_rank_order_fold(kvx, cuda, n_parts, rows, dim):
    """kvx_fold_shards against seqsplit.fold (float64), with an empty shard (lse -inf, outputs
    NaN) among the parts when there are three or more."""
    import torch
    gen = torch.Generator().manual_seed(1000 * n_parts + rows)
    outs = torch.randn(n_parts, rows, dim, generator=gen).float()
    lses = (torch.randn(n_parts, rows, generator=gen) * 20).float()
    if n_parts >= 3:
        lses[1] = float("-inf")
        outs[1] = float("nan")
    parts = torch.cat([outs.reshape(n_parts, -1), lses], dim=1).contiguous().cuda()
    out = torch.full((rows, dim), float("nan"), device="cuda")
    lse = torch.full((rows,), float("nan"), device="cuda")
    kvx.fold_shards(parts, n_parts, rows, dim, out, lse)
    torch.cuda.synchronize()
    clean = torch.where(torch.isnan(outs), torch.zeros_like(outs), outs).double()
    want = seqsplit.fold(clean, lses.double())
    scale = clean.abs().amax()
    assert torch.max(torch.abs(out.cpu().double() - want)) <= 2e-6 * scale
    m = lses.double().amax(0)
    want_lse = m + torch.log(torch.exp(lses.double() - m).sum(0))
    assert torch.allclose(lse.cpu().double(), want_lse, rtol=1e-6, atol=1e-5)


def _nccl_rank(rank, world, port, rows, dim, result):
    import datetime
    import os

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        gen = torch.Generator().manual_seed(77 + rank)
        exch = seqsplit.ShardExchange(rows, dim)
        exch.out_view().copy_(torch.randn(rows, dim, generator=gen))
        exch.lse_view().copy_(torch.randn(rows, generator=gen) * 10)
        exch.step()
        torch.cuda.synchronize()
        result[rank] = (exch.out.cpu().numpy(), exch.lse.cpu().numpy())
    finally:
        dist.destroy_process_group()


def test_shard_exchange_over_nccl(cuda):
    """Two ranks on two GPUs: one NCCL all-gather + the fold kernel give every rank the fold of
    both ranks' parts.  Runs only where the box has two GPUs."""
    import socket

    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, rows, dim = 2, 32, 256
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    result = mp.Manager().dict()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_nccl_rank, args=(r, world, port, rows, dim, result))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    outs, lses = [], []
    for r in range(world):
        gen = torch.Generator().manual_seed(77 + r)
        outs.append(torch.randn(rows, dim, generator=gen).double())
        lses.append((torch.randn(rows, generator=gen) * 10).float().double())
    want = seqsplit.fold(torch.stack(outs).float().double(), torch.stack(lses))
    for r in range(world):
        got = torch.from_numpy(result[r][0]).double()
        assert torch.max(torch.abs(got - want)) <= 2e-6 * want.abs().amax()
    assert np.array_equal(result[0][0], result[1][0])


def test_stream_order_with_dependent_launches(kvx, cuda, oracle):
    """The attention and combine kernels are launched as programmatic dependents of the kernel
    before them; each waits for it before reading.  A kernel that rewrites the queries between two
    runs on the same stream, with no synchronisation, must be seen by the second run, and the
    first run's outputs must be complete before the copy that follows it."""
    import torch
    dim, n_q, seq = 64, 7, 6000
    q1, k, v = _case(dim, n_q, seq, 41, 6)
    q2, _, _ = _case(dim, n_q, seq, 42, 6)
    blobs = _Blobs(kvx, oracle, k, v, dim)
    tq1 = torch.from_numpy(q1.view(np.int16)).cuda()
    tq2 = torch.from_numpy(q2.view(np.int16)).cuda()
    q = tq1.clone()
    out = torch.zeros((n_q, dim), dtype=torch.float32, device="cuda")
    plan = kvx.Plan([blobs.unit(kvx, q, out, None)], n_q, dim)
    assert plan.n_split > 0  # the combine pass runs too
    h = torch.cuda.current_stream().cuda_stream
    refs = []
    for tq in (tq1, tq2):  # each query set alone, synchronised
        q.copy_(tq)
        torch.cuda.synchronize()
        plan.run(h)
        torch.cuda.synchronize()
        refs.append(out.clone())
    q.copy_(tq1)
    torch.cuda.synchronize()
    plan.run(h)
    o1 = out.clone()
    torch.add(tq2, 0, out=q)  # a kernel, right before the next attention launch
    plan.run(h)
    o2 = out.clone()
    plan.check()
    torch.cuda.synchronize()
    plan.close()
    assert torch.equal(o1.view(torch.int32), refs[0].view(torch.int32))
    assert torch.equal(o2.view(torch.int32), refs[1].view(torch.int32))
    assert not torch.equal(refs[0], refs[1])
