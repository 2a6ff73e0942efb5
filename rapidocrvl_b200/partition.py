"""Request partitioning across GPUs (one process per GPU).

The decode step has no cross-request dependency, so multi-GPU decode is
request parallel: every GPU holds a full model replica and its own paged KV
pool, and a host-side dispatcher assigns whole requests to ranks.  This
replaces the reference's single shared Runtime serving concurrent requests
(cmd/paddleocrvl-server/main.go:357-397, a per-request KV pool in
internal/model/model.go:3286-3344) with one Runtime per GPU.

Assignment is longest-processing-time first on the predicted KV footprint of
each request (prompt + max new tokens), which is what bounds a GPU's pool and
its per-step attention bytes; it is deterministic, so every rank computes the
same plan without communicating.  Only host-side results are gathered.
"""
from __future__ import annotations

from typing import Dict, List, Sequence


def kv_bytes_per_token(cfg) -> int:
    """f32 K and V for every layer: layers * 2 * kv_heads * head_dim * 4 bytes."""
    return cfg.num_hidden_layers * 2 * cfg.num_key_value_heads * cfg.head_dim * 4


def request_cost(cfg, prompt_tokens: int, max_new_tokens: int) -> int:
    """Predicted KV bytes a request holds at its longest."""
    if prompt_tokens < 0 or max_new_tokens < 0:
        raise ValueError("token counts must be >= 0")
    return (prompt_tokens + max_new_tokens) * kv_bytes_per_token(cfg)


def assign(costs: Sequence[int], world_size: int) -> List[List[int]]:
    """Request indices per rank: heaviest request first onto the least
    loaded rank (ties: lower request index first, then lower rank)."""
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    if any(int(c) < 0 for c in costs):
        raise ValueError("request costs must be >= 0")
    order = sorted(range(len(costs)), key=lambda i: (-int(costs[i]), i))
    load = [0] * world_size
    count = [0] * world_size
    plan: List[List[int]] = [[] for _ in range(world_size)]
    for i in order:
        r = min(range(world_size), key=lambda k: (load[k], count[k], k))
        plan[r].append(i)
        load[r] += int(costs[i])
        count[r] += 1
    for p in plan:
        p.sort()
    return plan


def shard(costs: Sequence[int], rank: int, world_size: int) -> List[int]:
    """The request indices rank ``rank`` decodes."""
    if not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside world of {world_size}")
    return assign(costs, world_size)[rank]


def gather_results(local: Dict[int, list], group=None) -> Dict[int, list]:
    """Collects every rank's {request index: tokens} on all ranks through the
    host-side process group (gloo or nccl object collectives); returns the
    merged map.  Raises if two ranks report the same request."""
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return dict(local)
    parts = [None] * dist.get_world_size(group)
    dist.all_gather_object(parts, dict(local), group=group)
    merged: Dict[int, list] = {}
    for p in parts:
        for k, v in p.items():
            if k in merged:
                raise RuntimeError(f"request {k} decoded by more than one rank")
            merged[k] = v
    return merged
