"""Sequence split of one long decode step across GPUs.

Every rank attends over a contiguous, block-aligned slice of the sequence and produces, per
query, its normalised output o_r and the log of its softmax normaliser lse_r = m_r + ln(l_r)
(kvx_unit.lse).  The slices are folded exactly like the reference's merge_state
(src/softmax.hpp:16-30) folds thread ranges, only on normalised outputs:

    M = max_r lse_r,  w_r = exp(lse_r - M),  o = sum_r w_r o_r / sum_r w_r

in rank order.  The exchange is one all-gather of (o, lse): U x G x (D + 1) floats per rank,
33 KB for config[4] -- the only collective on the data path.  On the GPU, ShardExchange lays
each rank's outputs and lse out in one buffer so that the exchange is a single NCCL all-gather,
and folds the gathered parts with one kernel (kvx_fold_shards); fold() is the same arithmetic in
torch, for CPU ranks and as the check.
"""
from __future__ import annotations


def shard_blocks(n_blocks: int, world: int, rank: int) -> tuple[int, int]:
    """Block range [b0, b1) of `rank`: contiguous, as even as whole blocks allow."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world / rank")
    return rank * n_blocks // world, (rank + 1) * n_blocks // world


def fold(outs, lses):
    """Fold per-rank results in rank order.  outs: [R, ..., D], lses: [R, ...] (torch)."""
    import torch
    m = lses.max(dim=0).values
    w = torch.exp(lses - m)
    num = torch.zeros_like(outs[0])
    den = torch.zeros_like(lses[0])
    for r in range(outs.shape[0]):  # rank order
        num = num + w[r].unsqueeze(-1) * outs[r]
        den = den + w[r]
    return num / den.unsqueeze(-1)


def gather_fold(out, lse, group=None):
    """All-gather (out, lse) over the process group and fold them; every rank gets the result."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    outs = [torch.empty_like(out) for _ in range(world)]
    lses = [torch.empty_like(lse) for _ in range(world)]
    dist.all_gather(outs, out.contiguous(), group=group)
    dist.all_gather(lses, lse.contiguous(), group=group)
    return fold(torch.stack(outs), torch.stack(lses))


class ShardExchange:
    """The exchange step of a sequence split on the GPU.

    `pack` holds this rank's results as kvx_fold_shards expects them: outputs [rows, dim] then
    lse [rows], rows = units x queries; point the plan's kvx_unit.out / .lse at `out_view()` /
    `lse_view()`.  step() all-gathers every rank's pack over NCCL (one collective, on the current
    stream) and folds the parts in rank order into `out` [rows, dim] and `lse` [rows].
    """

    def __init__(self, rows: int, dim: int, group=None, device="cuda"):
        import torch
        import torch.distributed as dist
        self.rows, self.dim, self.group = rows, dim, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        n = rows * dim + rows
        self.pack = torch.zeros(n, dtype=torch.float32, device=device)
        self.gathered = torch.zeros(self.world * n, dtype=torch.float32, device=device)
        self.out = torch.zeros((rows, dim), dtype=torch.float32, device=device)
        self.lse = torch.zeros(rows, dtype=torch.float32, device=device)

    def out_view(self):
        return self.pack[: self.rows * self.dim].view(self.rows, self.dim)

    def lse_view(self):
        return self.pack[self.rows * self.dim:]

    @property
    def bytes_per_rank(self) -> int:
        return self.pack.numel() * 4

    def step(self, stream=None):
        import torch.distributed as dist
        import kvexp_b200 as kvx
        if self.world > 1:
            dist.all_gather_into_tensor(self.gathered, self.pack, group=self.group)
            parts = self.gathered
        else:
            parts = self.pack
        kvx.fold_shards(parts, self.world, self.rows, self.dim, self.out, self.lse, stream)
