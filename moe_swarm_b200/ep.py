"""Expert parallelism for the MoE layer: one process per GPU, 256/N experts per rank.

The reference leaves expert parallelism to its caller: every rank routes all tokens over the
256 global experts, computes only its local experts [local_expert_offset, +E_local), and "the
caller all-reduces across ranks" (reference/kernel_pytorch_v1.py:126-130; the paired
baseline derives its rank as offset // 32, solution/baseline_cutlass_sm90/main.py:133-145).
This module is that caller: rank r of N holds experts [r*256/N, (r+1)*256/N), hidden states
and logits are replicated, and the bf16 partial outputs are combined over NCCL -- by
reduce-scatter (rank r keeps token rows [r*T/N, (r+1)*T/N), the input layout of a following
sequence-sharded layer) or by all-reduce (every rank keeps all rows).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

E_GLOBAL = 256


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    offset: int      # local_expert_offset of this rank
    experts: int     # E_local

    @property
    def expert_range(self):
        return range(self.offset, self.offset + self.experts)


def shard(rank: int, world: int) -> Shard:
    """Contiguous expert shard of `rank` among `world` ranks (256 must divide evenly)."""
    if world < 1 or E_GLOBAL % world:
        raise ValueError(f"expert parallelism needs a world size dividing 256, got {world}")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    n = E_GLOBAL // world
    return Shard(rank, world, rank * n, n)


def row_split(T: int, world: int):
    """Token rows kept by each rank after the reduce-scatter: [(start, stop)] per rank.
    NCCL's reduce-scatter needs T divisible by the world size; other sizes use all-reduce."""
    if T % world:
        raise ValueError(f"reduce-scatter needs T divisible by {world}, got T={T}")
    n = T // world
    return [(r * n, (r + 1) * n) for r in range(world)]


class ExpertParallelMoE:
    """The layer on one rank of an expert-parallel group.

    ``local`` computes this rank's partial output from the layer's ten arguments (by default
    :func:`moe_swarm_b200.run`); the group's collective combines the partials.
    """

    def __init__(self, group=None, local=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.shard = shard(self.rank, self.world)
        if local is None:
            from . import run as local
        self.local = local

    def partial(self, routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, routed_scaling_factor):
        if gemm1_weights.shape[0] != self.shard.experts:
            raise ValueError(f"rank {self.rank} holds {self.shard.experts} experts, got weights for "
                             f"{gemm1_weights.shape[0]}")
        return self.local(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                          gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, self.shard.offset,
                          routed_scaling_factor)

    def forward(self, *args, combine: str = "reduce_scatter", out: torch.Tensor | None = None):
        """Partial layer on this rank, then the combine: "reduce_scatter" returns this rank's
        T/N rows of the full layer output, "all_reduce" returns all T rows."""
        part = self.partial(*args)
        if self.world == 1:
            return part
        if combine == "all_reduce":
            dist.all_reduce(part, group=self.group)
            return part
        if combine != "reduce_scatter":
            raise ValueError(f"unknown combine {combine!r}")
        T = part.shape[0]
        lo, hi = row_split(T, self.world)[self.rank]
        if out is None:
            out = torch.empty((hi - lo,) + tuple(part.shape[1:]), dtype=part.dtype, device=part.device)
        dist.reduce_scatter_tensor(out, part, group=self.group)
        return out
