"""Expert parallelism host side: one process per GPU, experts split in
contiguous blocks across the ranks of a torch.distributed group.

The data path is the library's own (expert rows read from their owner GPU
over NVLink inside the combine kernel); torch.distributed only exchanges the
small per-layer peer tables once at set-up, and bench code uses it for
barriers and max-over-ranks timing.

The reference has no counterpart: it runs the whole block on one Apple GPU
(src/engine/mlx_lm/models/deepseek_v2.rs:520-553).  The per-rank forward keeps
DeepseekMoe::forward's signature and result.
"""
from __future__ import annotations

from dataclasses import replace

import torch

from . import MAX_RANKS, DeepseekMoe, MoeArgs, MoeWeights, SenMoeError, SwitchLinear, ERR_BAD_ARG


def expert_bounds(num_experts: int, world_size: int) -> list[int]:
    """Rank r owns experts [b[r], b[r+1]): contiguous, as even as possible."""
    if world_size < 1 or world_size > MAX_RANKS:
        raise SenMoeError(ERR_BAD_ARG, f"world_size {world_size} outside [1, {MAX_RANKS}]")
    if num_experts < world_size:
        raise SenMoeError(ERR_BAD_ARG, f"{num_experts} experts cannot be split over {world_size} ranks")
    return [r * num_experts // world_size for r in range(world_size + 1)]


def _slice(p: SwitchLinear, begin: int, end: int) -> SwitchLinear:
    return SwitchLinear(p.weight[begin:end], p.scales[begin:end], p.biases[begin:end])


def shard_weights(weights: MoeWeights, begin: int, end: int) -> MoeWeights:
    """The rank's view of a layer: experts [begin, end) of the three stacked
    projections (views, no copy); router and shared expert stay whole."""
    return replace(weights, gate_proj=_slice(weights.gate_proj, begin, end),
                   up_proj=_slice(weights.up_proj, begin, end), down_proj=_slice(weights.down_proj, begin, end),
                   _keep=[weights])


def connect(layers: list, group=None) -> None:
    """Exchanges every layer's peer table over ``group`` (one all_gather) and
    connects the layers.  Every rank passes its layers in the same order."""
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    mine = [L.peer_info() for L in layers]
    tables: list = [None] * world
    dist.all_gather_object(tables, mine, group=group)
    for r, t in enumerate(tables):
        if len(t) != len(layers):
            raise SenMoeError(ERR_BAD_ARG, f"rank {r} offered {len(t)} layers, this rank {len(layers)}")
    for i, L in enumerate(layers):
        L.connect_peers(rank, [tables[r][i] for r in range(world)])


def make_layer(args: MoeArgs, weights: MoeWeights, max_tokens: int, rank: int, world_size: int,
               device: int | None = None) -> DeepseekMoe:
    """The rank's (unconnected) layer over its shard of ``weights``.  The full
    expert tensors may live anywhere torch can slice them; only the rank's
    experts need to be on its GPU."""
    b = expert_bounds(args.n_routed_experts, world_size)
    w = shard_weights(weights, b[rank], b[rank + 1])
    dev = torch.cuda.current_device() if device is None else device
    for p in (w.gate_proj, w.up_proj, w.down_proj):
        for t in (p.weight, p.scales, p.biases):
            if not t.is_cuda or t.device.index != dev:
                raise SenMoeError(ERR_BAD_ARG, "the rank's expert tensors must be on its GPU")
    return DeepseekMoe(args, w, max_tokens, device=dev, expert_range=(b[rank], b[rank + 1]))
