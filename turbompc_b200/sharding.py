"""Batch sharding over the GPUs of one node (one process per GPU).

MPC problems in a batch are independent, so a batch of Nb problems is split
into contiguous slices, each rank solves its slice with no communication,
and only the final result is gathered (torch.distributed, NCCL over NVLink
on GPUs; gloo in CPU tests).  There is no collective on the solve path.
"""
from __future__ import annotations

from typing import Any, Dict, Iterable, Sequence, Tuple

import torch


def shard_range(nb: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [lo, hi) slice of rank `rank`; the first nb % world ranks get one extra."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(nb, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


# Problem parameters that carry one entry per problem (leading batch axis)
# in the batched API; every other entry is shared by the whole batch.
BATCHED_KEYS = frozenset({
    "initial_state", "initial_guess_final_state", "initial_control", "reference_state_trajectory",
    "reference_control_trajectory", "obstacles_centers", "obstacles_radii", "slack_penalization_weight",
})


def shard_params(params: Dict[str, Any], nb: int, lo: int, hi: int,
                 batched: Iterable[str] = BATCHED_KEYS) -> Dict[str, Any]:
    """Slice the per-problem entries named in ``batched`` (top-level keys, or
    'outer.inner' for entries of nested dicts such as dynamics parameters)
    whose leading dimension is the batch size nb; everything else (weights,
    dynamics matrices, scalars) is shared and passed through unsliced, even
    when a dimension of it happens to equal nb."""
    batched = frozenset(batched)

    def walk(d, prefix):
        out = {}
        for k, v in d.items():
            name = prefix + k
            if isinstance(v, dict):
                out[k] = walk(v, name + ".")
            elif (name in batched and isinstance(v, torch.Tensor) and v.dim() > 0 and v.shape[0] == nb):
                out[k] = v[lo:hi]
            else:
                out[k] = v
        return out

    return walk(params, "")


def gather_batch(local: torch.Tensor, nb: int, group=None):
    """Gather per-rank slices (leading dim = the rank's shard) into the full
    (nb, ...) tensor on every rank (all_gather of equally padded slices)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    sizes = [shard_range(nb, world, r) for r in range(world)]
    cap = max(h - l for l, h in sizes)
    pad = torch.zeros((cap,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    out = torch.empty((world * cap,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, pad, group=group) if hasattr(dist, "all_gather_into_tensor") and \
        local.is_cuda else _gather_list(out, pad, world, group)
    parts = [out[r * cap: r * cap + (h - l)] for r, (l, h) in enumerate(sizes)]
    return torch.cat(parts, 0)


def _gather_list(out, pad, world, group):
    import torch.distributed as dist

    chunks = list(out.chunk(world, 0))
    dist.all_gather(chunks, pad, group=group)
    for i, c in enumerate(chunks):
        out[i * pad.shape[0]:(i + 1) * pad.shape[0]] = c


def gather_fields(tensors: Sequence[torch.Tensor], nb: int, group=None):
    return [gather_batch(t, nb, group) for t in tensors]
