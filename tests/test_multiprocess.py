"""Multi-rank host logic on CPU (gloo, world size 2) -- no GPU needed.

  * config[4]'s sequence split: two ranks attend over their block-aligned halves of a sequence
    (float64 numpy attention stands in for the GPU kernel), all-gather (out, lse) and fold; the
    result equals single-rank attention over the whole sequence;
  * bench.py's unit sharding of config[1]/[2] (strong) and config[3] (8 shards): the ranks' unit
    sets are disjoint, and for config[1]/[2] cover every unit.
"""
import os
import socket

import numpy as np
import pytest

import seqsplit


def _attend(q, k, v):
    """float64 softmax attention: normalised output and ln of the normaliser per query."""
    s = q @ k.T
    m = s.max(axis=1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=1, keepdims=True)
    return (p @ v) / l, (m + np.log(l))[:, 0]


def _case(seed=3, seq=1000, dim=16, n_q=4):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((n_q, dim)), rng.standard_normal((seq, dim)),
            rng.standard_normal((seq, dim)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        q, k, v = _case()
        block = 128
        n_blocks = (k.shape[0] + block - 1) // block
        b0, b1 = seqsplit.shard_blocks(n_blocks, world, rank)
        t0, t1 = b0 * block, min(b1 * block, k.shape[0])
        o, lse = _attend(q, k[t0:t1], v[t0:t1])
        got = seqsplit.gather_fold(torch.from_numpy(o), torch.from_numpy(lse))
        result[rank] = got.numpy()
    finally:
        dist.destroy_process_group()


def test_sequence_split_fold_over_gloo():
    import torch.multiprocessing as mp
    world = 2
    port = _free_port()
    mgr = mp.Manager()
    result = mgr.dict()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    q, k, v = _case()
    want, _ = _attend(q, k, v)
    for r in range(world):
        np.testing.assert_allclose(result[r], want, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("n_blocks,world", [(8192, 8), (8192, 3), (7, 8), (1, 2), (256, 1)])
def test_shard_blocks_cover_the_sequence(n_blocks, world):
    ranges = [seqsplit.shard_blocks(n_blocks, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n_blocks
    assert all(ranges[i][1] == ranges[i + 1][0] for i in range(world - 1))
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1


def test_fold_is_exact_for_one_rank_and_weights_by_normaliser():
    import torch
    o = torch.tensor([[[1.0, 2.0]], [[3.0, 5.0]]], dtype=torch.float64)
    lse = torch.tensor([[0.0], [np.log(3.0)]], dtype=torch.float64)
    got = seqsplit.fold(o, lse)
    np.testing.assert_allclose(got.numpy(), [[2.5, 4.25]])  # (1*o0 + 3*o1) / 4
    np.testing.assert_allclose(seqsplit.fold(o[:1], lse[:1]).numpy(), o[0].numpy())


@pytest.mark.parametrize("config,world", [(1, 1), (1, 2), (1, 3), (1, 8), (2, 8), (1, 48), (3, 8)])
def test_unit_shards_cover_the_config(config, world):
    """bench.py's unit sharding: config[1]/[2] split their (layer, KV head) units over the ranks
    (contiguous runs, sizes within one, one seed: the ranks together hold exactly the config);
    config[3] gives rank r shard r of 8.  Disjoint in every case."""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    import workloads as W
    cfg = W.CONFIGS[config]
    shares = [bench.rank_share(cfg, r, world) for r in range(world)]
    ids = [s[1] for s in shares]
    flat = [u for x in ids for u in x]
    assert len(flat) == len(set(flat))
    if cfg.shard == "split":
        assert sorted(flat) == list(range(cfg.units))
        assert max(map(len, ids)) - min(map(len, ids)) <= 1
        assert len({s[2] for s in shares}) == 1
    else:
        assert len(flat) == world * (cfg.units // bench.GPU_SLOTS)


def test_unit_split_refuses_more_ranks_than_units():
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    import workloads as W
    with pytest.raises(SystemExit):
        bench.rank_share(W.CONFIGS[1], 48, 49)
