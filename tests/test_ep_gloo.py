"""CPU: expert-parallel decomposition of the layer over gloo ranks (no GPU).

Each rank computes its shard's partial output (here with the oracle on the CPU) and the
ranks' collective combines them; the result must equal the whole layer computed in one
process.  Routing is steered onto 8 experts spread over both ranks' shards so each rank
materialises only the experts it actually runs.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from moe_swarm_b200 import ep
from moe_swarm_b200 import workload as W
from oracle import moe_ref as O

FAVOUR = [3, 5, 40, 42, 130, 131, 200, 201]   # 4 groups (0, 1, 4, 6); ranks 0 and 1 hold 4 each
T, SEED = 6, 17


def test_shards_cover_every_expert_once():
    for world in (1, 2, 4, 8):
        seen = []
        for r in range(world):
            s = ep.shard(r, world)
            assert s.experts == 256 // world and s.offset == r * s.experts
            seen.extend(s.expert_range)
        assert seen == list(range(256))
    with pytest.raises(ValueError):
        ep.shard(0, 3)
    with pytest.raises(ValueError):
        ep.shard(2, 2)


def test_row_split():
    assert ep.row_split(4096, 8)[3] == (1536, 2048)
    assert ep.row_split(8, 2) == [(0, 4), (4, 8)]
    with pytest.raises(ValueError):
        ep.row_split(7, 2)


def _inputs():
    x = W.make_steered_activations(T, SEED, 0, FAVOUR)
    x["routed_scaling_factor"] = 2.5
    return x


def _expert(ge):
    return W.make_expert(SEED, ge)


def _local_fn(experts):
    """This rank's partial output in fp32 from the experts it holds (oracle arithmetic)."""
    def local(logits, bias, hs, hs_scale, w13, s13, w2, s2, offset, rsf):
        idx, w = O.route(logits, bias, rsf)
        A = O.dequant_tokens(hs, hs_scale)
        out = torch.zeros(logits.shape[0], 7168)
        for ge in range(offset, offset + w13.shape[0]):
            sel = (idx == ge).any(dim=1)
            if not sel.any():
                continue
            q13, sc13, q2, sc2 = experts[ge]
            tok = sel.nonzero().squeeze(1)
            o = O.expert_forward(A[tok], O.dequant_blocks(q13, sc13), O.dequant_blocks(q2, sc2))
            out.index_add_(0, tok, o * w[tok, ge].unsqueeze(1))
        return out
    return local


def _rank_main(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = ep.shard(rank, world)
        experts = {ge: _expert(ge) for ge in FAVOUR if ge in sh.expert_range}
        layer = ep.ExpertParallelMoE(local=_local_fn(experts))
        x = _inputs()
        stub = torch.zeros(1, 1, 1).expand(sh.experts, 1, 1)   # shape-only stand-in for the weights
        full = layer.forward(x["routing_logits"], x["routing_bias"], x["hidden_states"],
                             x["hidden_states_scale"], stub, stub, stub, stub, x["routed_scaling_factor"],
                             combine="all_reduce")
        if rank == 0:
            torch.save(full, result_path)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_ranks_combine_to_the_whole_layer(tmp_path):
    path = str(tmp_path / "full.pt")
    mp.start_processes(_rank_main, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
    got = torch.load(path)
    # the whole layer in one process
    x = _inputs()
    want = _local_fn({ge: _expert(ge) for ge in FAVOUR})(
        x["routing_logits"], x["routing_bias"], x["hidden_states"], x["hidden_states_scale"],
        torch.zeros(1, 1, 1).expand(256, 1, 1), None, None, None, 0, x["routed_scaling_factor"])
    idx, _ = O.route(x["routing_logits"], x["routing_bias"], 2.5)
    assert sorted(set(idx.flatten().tolist())) == sorted(FAVOUR)
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)


# ----------------------------------------------------------------------------- token dispatch
T_OWN = 5   # tokens owned by each rank


def _own_inputs(rank):
    """Rank `rank`'s own tokens (different on each rank), steered onto FAVOUR."""
    x = W.make_steered_activations(T_OWN, SEED + 10 * rank, 0, FAVOUR)
    x["routed_scaling_factor"] = 2.5
    return x


def _route_fn(logits, bias, rsf, like):
    idx, w = O.route(logits, bias, rsf)
    return idx.int(), torch.gather(w, 1, idx)


def _local_routed_fn(experts):
    """Pre-routed partial output in fp32 from the experts this rank holds (oracle arithmetic);
    fp32 rows keep the exchange free of rounding, so only the final bf16 cast and the order of
    the rank sums separate the result from the one-process layer."""
    def local(idx, w, hs, hs_scale, w13, s13, w2, s2, offset):
        A = O.dequant_tokens(hs, hs_scale)
        out = torch.zeros(hs.shape[0], 7168)
        for ge in range(offset, offset + w13.shape[0]):
            sel = (idx == ge)
            rows = sel.any(dim=1)
            if not rows.any():
                continue
            q13, sc13, q2, sc2 = experts[ge]
            tok = rows.nonzero().squeeze(1)
            o = O.expert_forward(A[tok], O.dequant_blocks(q13, sc13), O.dequant_blocks(q2, sc2))
            wt = (w * sel.float()).sum(dim=1)[tok]
            out.index_add_(0, tok, o * wt.unsqueeze(1))
        return out
    return local


def _dispatch_main(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = ep.shard(rank, world)
        experts = {ge: _expert(ge) for ge in FAVOUR if ge in sh.expert_range}
        layer = ep.ExpertParallelMoE(route_fn=_route_fn, local_routed=_local_routed_fn(experts))
        x = _own_inputs(rank)
        stub = torch.zeros(1, 1, 1).expand(sh.experts, 1, 1)
        out = layer.forward_dispatch(x["routing_logits"], x["routing_bias"], x["hidden_states"],
                                     x["hidden_states_scale"], stub, stub, stub, stub, x["routed_scaling_factor"])
        torch.save(out, f"{result_path}.{rank}")
    finally:
        dist.destroy_process_group()


def test_token_dispatch_matches_the_whole_layer(tmp_path):
    """Each rank's own tokens, dispatched to the expert owners and the partial rows returned,
    equal the whole layer computed for those tokens in one process."""
    path = str(tmp_path / "out")
    mp.start_processes(_dispatch_main, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
    everything = _local_fn({ge: _expert(ge) for ge in FAVOUR})
    for rank in range(2):
        got = torch.load(f"{path}.{rank}")
        x = _own_inputs(rank)
        want = everything(x["routing_logits"], x["routing_bias"], x["hidden_states"], x["hidden_states_scale"],
                          torch.zeros(1, 1, 1).expand(256, 1, 1), None, None, None, 0, 2.5)
        assert got.dtype == torch.bfloat16
        torch.testing.assert_close(got.float(), want.to(torch.bfloat16).float(), rtol=1e-2, atol=1e-2)
        assert (got.float() - want).abs().max() <= 1e-2 + 1e-2 * want.abs().max()
