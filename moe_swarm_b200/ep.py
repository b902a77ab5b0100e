"""Expert parallelism for the MoE layer: one process per GPU, 256/N experts per rank.

The reference leaves expert parallelism to its caller: every rank routes all tokens over the
256 global experts, computes only its local experts [local_expert_offset, +E_local), and "the
caller all-reduces across ranks" (reference/kernel_pytorch_v1.py:126-130; the paired
baseline derives its rank as offset // 32, solution/baseline_cutlass_sm90/main.py:133-145).
This module is that caller: rank r of N holds experts [r*256/N, (r+1)*256/N), hidden states
and logits are replicated, and the bf16 partial outputs are combined over NCCL -- by
reduce-scatter (rank r keeps token rows [r*T/N, (r+1)*T/N), the input layout of a following
sequence-sharded layer) or by all-reduce (every rank keeps all rows).

`forward(..., combine="peer")` keeps the reduce-scatter's result layout but has no separate
collective: the layer's GEMM2 and combine epilogues store each output row straight into the
receive buffer of the rank that owns the row, over NVLink, and each rank sums the N slots of its
rows in rank order (`moe_b200_forward_ep`; buffers in torch symmetric memory).

`forward_dispatch` is the token-dispatch form a deployment uses when each rank owns its own
tokens: a rank routes its tokens, sends each one only to the ranks holding its experts
(all-to-all), computes the tokens it received with the pre-routed layer on its experts, and
sends the partial rows back (all-to-all), where each token's rows are summed in rank order.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

E_GLOBAL = 256
H = 7168


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


def _default_route(routing_logits, routing_bias, routed_scaling_factor, like):
    """Device routing of a rank's own tokens: (topk_idx int32 [T, 8] global ids, topk_w f32)."""
    from . import route
    r = route(routing_logits, routing_bias, like["hidden_states"], like["hidden_states_scale"],
              like["gemm1_weights"], like["gemm1_weights_scale"], like["gemm2_weights"],
              like["gemm2_weights_scale"], 0, routed_scaling_factor)
    return r["topk_idx"].clone(), r["topk_w"].clone()   # copies: route() returns workspace views


class _PeerBuffers:
    """Receive buffers and flag words of the peer-memory combine, mapped on every rank of the
    group (torch symmetric memory): recv bf16 [2][N][tokens/N][7168], flags uint32 [2][8]
    (zeroed before any rank signals).  Creating them is collective."""

    def __init__(self, group, world: int, tokens: int, device):
        import torch.distributed._symmetric_memory as symm
        name = (group or dist.group.WORLD).group_name
        self.tokens = tokens
        self.recv = symm.empty(2 * world * (tokens // world) * H, dtype=torch.bfloat16, device=device)
        self.flags = symm.empty(2 * 8, dtype=torch.int32, device=device)
        self.flags.zero_()
        self._handles = (symm.rendezvous(self.recv, name), symm.rendezvous(self.flags, name))
        self.recv_ptrs = [int(p) for p in self._handles[0].buffer_ptrs]
        self.flag_ptrs = [int(p) for p in self._handles[1].buffer_ptrs]
        torch.cuda.synchronize(device)
        dist.barrier(group)
        self.epoch = 0


class ExpertParallelMoE:
    """The layer on one rank of an expert-parallel group.

    ``local`` computes this rank's partial output from the layer's ten arguments (by default
    :func:`moe_swarm_b200.run`); the group's collective combines the partials.  For
    :meth:`forward_dispatch`, ``route_fn(logits, bias, rsf, like)`` gives a rank's routing and
    ``local_routed`` the pre-routed partial output (by default the device routing and
    :func:`moe_swarm_b200.run_routed`).
    """

    def __init__(self, group=None, local=None, route_fn=None, local_routed=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.shard = shard(self.rank, self.world)
        if local is None:
            from . import run as local
        self.local = local
        if local_routed is None:
            from . import run_routed as local_routed
        self.local_routed = local_routed
        self.route_fn = route_fn or _default_route
        self._peer = None

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
        T/N rows of the full layer output, "all_reduce" returns all T rows, "peer" returns the
        same rows as "reduce_scatter" with the combine done over peer memory inside the call."""
        if combine == "peer":
            return self._forward_peer(*args, out=out)
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

    def _forward_peer(self, routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                      gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, routed_scaling_factor, out=None):
        import ctypes

        from . import _args, _native, _validate, _workspace
        T, E, dev = _validate(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                              gemm1_weights_scale, gemm2_weights, gemm2_weights_scale)
        if E != self.shard.experts:
            raise ValueError(f"rank {self.rank} holds {self.shard.experts} experts, got weights for {E}")
        if T % self.world:
            raise ValueError(f"the peer combine needs T divisible by {self.world}, got T={T}")
        rows = T // self.world
        if out is None:
            out = torch.empty((rows, H), dtype=torch.bfloat16, device=dev)
        elif not (out.dtype == torch.bfloat16 and tuple(out.shape) == (rows, H) and out.is_contiguous()
                  and out.device == dev):
            raise ValueError(f"out must be a contiguous bf16 [{rows}, {H}] tensor on {dev}")
        if T == 0:   # the same T on every rank: all skip together
            return out
        if self._peer is None or self._peer.tokens < T:
            self._peer = _PeerBuffers(self.group, self.world, T, dev)
        pb = self._peer
        pb.epoch += 1
        ep = _native.MoeEp()
        ep.world, ep.rank, ep.shard_tokens, ep.epoch = self.world, self.rank, rows, pb.epoch
        for r in range(self.world):
            ep.recv[r] = pb.recv_ptrs[r]
            ep.signal[r] = pb.flag_ptrs[r]
        ep.out_shard = out.data_ptr()
        stream = torch.cuda.current_stream(dev).cuda_stream
        buf = _workspace(dev, stream).get(T, E, stream)
        a = _args(T, E, routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                  gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, self.shard.offset,
                  routed_scaling_factor, out)
        rc = _native.lib().moe_b200_forward_ep(ctypes.byref(a), ctypes.byref(ep), buf.data_ptr(), buf.numel(),
                                               stream)
        if rc != _native.OK:
            raise RuntimeError(f"moe_b200_forward_ep failed ({rc}): {_native.last_error()}")
        return out

    def _exchange(self, send: torch.Tensor, send_counts, recv_counts) -> torch.Tensor:
        """all_to_all of rows: send's rows grouped by destination rank in rank order."""
        out = torch.empty((int(sum(recv_counts)),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
        dist.all_to_all_single(out, send, output_split_sizes=list(recv_counts),
                               input_split_sizes=list(send_counts), group=self.group)
        return out

    def forward_dispatch(self, routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                         gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, routed_scaling_factor):
        """Token-dispatch expert parallelism over this rank's own T tokens; returns their bf16
        [T, 7168] output rows.  Every rank's weights are its shard of the 256 experts."""
        if gemm1_weights.shape[0] != self.shard.experts:
            raise ValueError(f"rank {self.rank} holds {self.shard.experts} experts, got weights for "
                             f"{gemm1_weights.shape[0]}")
        like = dict(hidden_states=hidden_states, hidden_states_scale=hidden_states_scale,
                    gemm1_weights=gemm1_weights, gemm1_weights_scale=gemm1_weights_scale,
                    gemm2_weights=gemm2_weights, gemm2_weights_scale=gemm2_weights_scale)
        topk_idx, topk_w = self.route_fn(routing_logits, routing_bias, routed_scaling_factor, like)
        T = hidden_states.shape[0]
        dev = hidden_states.device
        # the ranks each token goes to: those holding at least one of its experts
        owner = (topk_idx.long() // self.shard.experts).clamp(0, self.world - 1)
        goes = torch.zeros((self.world, T), dtype=torch.bool, device=dev)
        goes.scatter_(0, owner.t().contiguous(), torch.ones_like(owner.t(), dtype=torch.bool))
        dest_tokens = [goes[d].nonzero().squeeze(1) for d in range(self.world)]   # ascending token ids
        send_counts = torch.tensor([len(x) for x in dest_tokens], dtype=torch.int64, device=dev)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        sel = torch.cat(dest_tokens)
        hs_u8 = hidden_states.view(torch.uint8)
        r_hidden = self._exchange(hs_u8.index_select(0, sel).contiguous(), sc, rc)
        r_scale = self._exchange(hidden_states_scale.t().index_select(0, sel).contiguous(), sc, rc)
        r_idx = self._exchange(topk_idx.index_select(0, sel).contiguous(), sc, rc)
        r_w = self._exchange(topk_w.index_select(0, sel).contiguous(), sc, rc)
        part = self.local_routed(r_idx, r_w, r_hidden.view(hidden_states.dtype), r_scale.t().contiguous(),
                                 gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                                 self.shard.offset)
        back = self._exchange(part.contiguous(), rc, sc)      # this rank's tokens, grouped by source rank
        out = torch.zeros((T, back.shape[1]), dtype=torch.float32, device=dev)
        start = 0
        for d in range(self.world):                             # rank order: deterministic sum
            n = sc[d]
            if n:
                out.index_add_(0, dest_tokens[d], back[start:start + n].float())
            start += n
        return out.to(torch.bfloat16)
