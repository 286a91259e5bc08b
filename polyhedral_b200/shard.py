"""(batch, head) sharding of one block-sparse attention forward across ranks.

Every (batch, head) of a forward is an independent problem over the same mask, so
one configuration's B*H heads split into contiguous ranges, one per rank (one
process per GPU), with no exchange in the forward: each rank runs the same plans
(block index and work list depend on the mask only) on its slice of Q, K, V and
writes its slice of O and LSE.  The only collective is optional: gathering every
rank's O / LSE onto every rank (NCCL all-gather over NVLink), for a caller that
needs the whole result in one place.  The reference runs one GPU and has no
counterpart; this is the partition its experiments would need to scale out.
"""
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class HeadShard:
    """Rows [start, stop) of the [B*H, N, D] tensors belong to `rank` of `world`."""
    BH: int
    rank: int
    world: int
    start: int
    stop: int

    @property
    def size(self):
        return self.stop - self.start

    def slice(self, x):
        """This shard's view of a [B*H, ...] tensor (no copy)."""
        return x[self.start:self.stop]

    def run(self, forward, q, k, v, out=None, lse_out=None):
        """``forward(q, k, v, out=..., lse_out=...) -> (o, lse)`` on this shard's
        heads of the full-size q, k, v (views, no copy); out / lse_out, when given,
        are full-size too and receive this shard's rows.  Returns the shard's
        (o, lse)."""
        o = self.slice(out) if out is not None else None
        lse = self.slice(lse_out) if lse_out is not None else None
        return forward(self.slice(q), self.slice(k), self.slice(v), out=o, lse_out=lse)


def shard_bh(BH, rank, world):
    """Contiguous (batch, head) range of `rank`: every rank gets BH // world heads and
    the first BH % world ranks one more, so the ranges cover [0, BH) exactly once in
    rank order."""
    BH, rank, world = int(BH), int(rank), int(world)
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    if BH < 1:
        raise ValueError(f"BH={BH} must be positive")
    base, extra = divmod(BH, world)
    start = rank * base + min(rank, extra)
    return HeadShard(BH, rank, world, start, start + base + (1 if rank < extra else 0))


def gather(o_local, lse_local, shard, group=None):
    """All ranks' (o, lse) shards concatenated in head order on every rank, by one
    all-gather per tensor (``all_gather_into_tensor`` when the shards are equal,
    padded to the largest shard otherwise).  Must be called by every rank of the
    group, in the same order as every other collective."""
    import torch.distributed as dist
    world = shard.world
    if world == 1:
        return o_local, lse_local
    big = -(-shard.BH // world)

    def _gather(x):
        if x.shape[0] != big:       # pad to the largest shard
            pad = torch.zeros((big - x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype,
                              device=x.device)
            x = torch.cat([x, pad])
        full = torch.empty((big * world,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(full, x.contiguous(), group=group)
        if big * world == shard.BH:
            return full
        return torch.cat([full[r * big:r * big + shard_bh(shard.BH, r, world).size]
                          for r in range(world)])

    return _gather(o_local), _gather(lse_local)
