"""KV-head sharding of the paged-attention path across GPUs.

Rank r of N owns kv heads [r*KV/N, (r+1)*KV/N) and the q heads that read them,
[r*H/N, (r+1)*H/N) (q head h reads kv head h // (H/KV), so whole groups stay on one rank).
Append and attention need no cross-rank traffic; one all-gather of the per-rank outputs
[nt, H/N*d] plus a head permute rebuilds [nt, H*d].
"""

from __future__ import annotations

import torch


def head_ranges(num_heads: int, kv_heads: int, rank: int, world: int):
    """(q head range, kv head range) of `rank`."""
    if kv_heads % world or num_heads % world:
        raise ValueError(f"{world} ranks must divide {kv_heads} kv heads and {num_heads} q heads")
    kv_per, q_per = kv_heads // world, num_heads // world
    return (rank * q_per, (rank + 1) * q_per), (rank * kv_per, (rank + 1) * kv_per)


def shard_columns(x: torch.Tensor, heads: int, head_range, head_size: int) -> torch.Tensor:
    """Columns of the heads in `head_range` from a packed [nt, heads*d] activation."""
    lo, hi = head_range
    return x[:, lo * head_size:hi * head_size].contiguous()


def reassemble(gathered: torch.Tensor) -> torch.Tensor:
    """[N, nt, H/N*d] (rank-major all-gather) -> [nt, H*d] in q-head order."""
    n, nt, w = gathered.shape
    return gathered.permute(1, 0, 2).reshape(nt, n * w)


def all_gather_output(out: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather this rank's [nt, H/N*d] output and reassemble [nt, H*d]."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    buf = torch.empty((world, *out.shape), dtype=out.dtype, device=out.device)
    dist.all_gather_into_tensor(buf, out.contiguous(), group=group)
    return reassemble(buf)
