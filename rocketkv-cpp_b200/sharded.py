"""Multi-GPU execution of the RocketKV path: one process per GPU, torch.distributed.

Sequences shard with no collective: every rank runs its own items through
`Evictor` / `HsaDecoder` (bench.py's decode workload is weak-scaled that way).

KV heads shard for long contexts.  Stage 2 has no cross-head coupling
(rocket.cpp:190-379); stage 1 couples the heads only through the head-order
sum of the pooled scores (rocket.cpp:142-148).  So:

* stage 1: each rank scores and pools its KV heads, one all-gather assembles
  the pooled rows in head order 0..HK-1, and every rank runs the same
  selection on them -- the kept indices are identical on every rank and equal
  to the single-GPU result, with no second broadcast;
* stage 2: each rank decodes its KV heads; one all-gather assembles O.

The per-rank compute is passed in as callables (the CUDA library in
`HeadShardedRocket`); the partition, the collectives and the assembly order
live here.  Every rank makes the same collective calls in the same order.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Tuple


def head_range(num_heads_kv: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous block of KV heads owned by `rank`: (first head, count).
    The first `num_heads_kv % world` ranks take one extra head."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    base, rem = divmod(num_heads_kv, world)
    return rank * base + min(rank, rem), base + (1 if rank < rem else 0)


def gather_rows(local, counts: List[int], group=None):
    """All-gathers `local` [batch, counts[rank], ...] from every rank and
    returns [batch, sum(counts), ...] with the ranks' rows in rank order.
    Ranks pad to the largest count so every rank sends the same shape."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if len(counts) != world:
        raise ValueError("one count per rank")
    mx = max(max(counts), 1)
    pad = local.new_zeros((local.shape[0], mx) + tuple(local.shape[2:]))
    pad[:, : local.shape[1]] = local
    outs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(outs, pad.contiguous(), group=group)
    return torch.cat([o[:, :c] for o, c in zip(outs, counts)], dim=1)


def sharded_evict(pool_heads: Callable, select_pooled: Callable, num_heads_kv: int, group=None):
    """Stage 1 sharded by KV head.  pool_heads(h0, nh) -> pooled rows
    [batch, nh, nk] (float32) of this rank's heads; select_pooled(pooled
    [batch, HK, nk]) -> the kept indices.  Returns select_pooled's result,
    the same on every rank."""
    import torch.distributed as dist
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    counts = [head_range(num_heads_kv, world, r)[1] for r in range(world)]
    h0, nh = head_range(num_heads_kv, world, rank)
    return select_pooled(gather_rows(pool_heads(h0, nh), counts, group))


def sharded_decode(decode_heads: Callable, num_heads_kv: int, group_size: int, group=None):
    """Stage 2 sharded by KV head.  decode_heads(h0, nh) -> O rows
    [batch, nh * group_size, D] of this rank's query heads.  Returns the full
    O [batch, num_heads_kv * group_size, D] on every rank."""
    import torch.distributed as dist
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    counts = [head_range(num_heads_kv, world, r)[1] * group_size for r in range(world)]
    h0, nh = head_range(num_heads_kv, world, rank)
    return gather_rows(decode_heads(h0, nh), counts, group)


class HeadShardedRocket:
    """The CUDA library behind the sharded drivers, on this rank's GPU.  Inputs
    are this rank's shards: Q rows of its query heads and K/V rows of its KV
    heads (the full-model head indices are only used for the partition)."""

    def __init__(self, cfg, device, group=None):
        import torch.distributed as dist
        self.cfg, self.device, self.group = cfg, device, group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.h0, self.nh = head_range(cfg.num_heads_kv, self.world, self.rank)
        self.G = max(1, cfg.num_heads // cfg.num_heads_kv)
        self._ev = {}
        self._dec = {}

    def _local_cfg(self):
        import rocketkv_b200 as rkv
        c = self.cfg
        return rkv.RocketConfig(num_heads=self.nh * self.G, num_heads_kv=self.nh, dim_head=c.dim_head,
                                window_size=c.window_size, kernel_size=c.kernel_size,
                                prompt_budget=c.prompt_budget, topk_decode=c.topk_decode,
                                chunk_size=c.chunk_size, r_dim=c.r_dim, compression_ratio=c.compression_ratio)

    def evict(self, Q_local, K_local, len_q: int, len_k: int, dtype: int):
        """Q_local [B, nh*G, len_q, D*], K_local [B, nh, len_k, D*] on this
        rank's device -> (kept [B, max_kept] int32, n_kept [B]), equal on all ranks."""
        import torch
        import rocketkv_b200 as rkv
        B = K_local.shape[0]
        key = (len_q, len_k, B, dtype)
        if key not in self._ev:
            # pooling with the local shard; selection over all HK heads
            self._ev[key] = (rkv.Evictor(self._local_cfg(), len_q, len_k, B, dtype, self.device) if self.nh else None,
                             rkv.Evictor(self.cfg, len_q, len_k, B, dtype, self.device))
        local_ev, full_ev = self._ev[key]
        nk = len_k - min(self.cfg.window_size, len_q)

        def pool_heads(h0, nh):
            out = torch.zeros((B, nh, max(nk, 0)), dtype=torch.float32, device=self.device)
            if nh and nk > 0:
                local_ev.pool_heads(Q_local, K_local, 0, nh, out)
            return out

        return sharded_evict(pool_heads, full_ev.select_pooled, self.cfg.num_heads_kv, self.group)

    def decode(self, Q_local, K_local, V_local, len_k: int, recent_window: int = 0):
        """Q_local [B, nh*G, D], K/V_local [B, nh, len_k, D] -> O [B, H, D] on every rank."""
        import torch
        import rocketkv_b200 as rkv
        B = K_local.shape[0]
        key = (len_k, B, recent_window)
        if self.nh and key not in self._dec:
            self._dec[key] = rkv.HsaDecoder(self._local_cfg(), len_k, B, self.device, recent_window=recent_window)

        def decode_heads(h0, nh):
            if not nh:
                return torch.zeros((B, 0, self.cfg.dim_head), dtype=torch.float32, device=self.device)
            return self._dec[key](Q_local, K_local, V_local, want_sel=False)

        return sharded_decode(decode_heads, self.cfg.num_heads_kv, self.G, self.group)
