"""GPU, 2 ranks: expert parallelism over NCCL.

Each rank runs the layer on its 128-expert shard (``local_expert_offset`` = 128 * rank) with
the CUDA library and the shards' bf16 partial outputs are combined by NCCL -- reduce-scatter
(each rank keeps T/2 token rows) and all-reduce.  Routing is steered onto 8 experts, 4 in each
shard, so both ranks do real work; the other experts' weights are zero and never read.

Two checks.  (1) The collective itself: the combined rows equal, bit for bit, the bf16 sum of
the two shards' outputs computed one after the other on one GPU.  (2) Against the whole layer
over all 256 experts on one GPU: the partials are rounded to bf16 before they are added (the
reference's convention: each rank returns bf16 and the caller all-reduces,
reference/kernel_pytorch_v1.py:126-130), so a cancelling pair of partials can move a few
outputs just past the single-GPU tolerance; at most 0.1 % of the elements may, and none by more
than 5x the absolute tolerance.  Skipped unless two GPUs are visible.
"""

import os
import socket

import pytest
import torch

from tests import _cases as C

FAVOUR = [3, 5, 40, 42, 130, 131, 200, 201]
T, SEED = 64, 23

pytestmark = pytest.mark.gpu


def _layer_inputs(device, offset, experts):
    """Activations plus a zero weight stack of `experts` experts from global expert `offset`,
    with the favoured experts filled from the seeded per-expert generator."""
    from moe_swarm_b200 import workload as W
    x = {k: v.to(device) for k, v in W.make_steered_activations(T, SEED, 0, FAVOUR).items()}
    q13 = torch.zeros(experts, 4096, 7168, dtype=torch.float8_e4m3fn, device=device)
    s13 = torch.ones(experts, 32, 56, dtype=torch.float32, device=device)
    q2 = torch.zeros(experts, 7168, 2048, dtype=torch.float8_e4m3fn, device=device)
    s2 = torch.ones(experts, 56, 16, dtype=torch.float32, device=device)
    for ge in FAVOUR:
        if offset <= ge < offset + experts:
            a, sa, b, sb = W.make_expert(SEED, ge)
            q13[ge - offset].copy_(a)
            s13[ge - offset].copy_(sa)
            q2[ge - offset].copy_(b)
            s2[ge - offset].copy_(sb)
    x.update(gemm1_weights=q13, gemm1_weights_scale=s13, gemm2_weights=q2, gemm2_weights_scale=s2)
    return x


def _rank_main(rank, world, port, out_dir):
    from datetime import timedelta

    import torch.distributed as dist

    from moe_swarm_b200 import ep

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=device)
    try:
        sh = ep.shard(rank, world)
        x = _layer_inputs(device, sh.offset, sh.experts)
        layer = ep.ExpertParallelMoE()
        args = (x["routing_logits"], x["routing_bias"], x["hidden_states"], x["hidden_states_scale"],
                x["gemm1_weights"], x["gemm1_weights_scale"], x["gemm2_weights"], x["gemm2_weights_scale"],
                2.5)
        rows = layer.forward(*args, combine="reduce_scatter")
        full = layer.forward(*args, combine="all_reduce")
        torch.cuda.synchronize()
        torch.save({"rows": rows.cpu(), "full": full.cpu()}, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_nccl_matches_single_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    import moe_swarm_b200 as M

    mp.start_processes(_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    parts = [torch.load(tmp_path / f"rank{r}.pt") for r in range(2)]

    dev = torch.device("cuda", 0)
    shard_out = []
    for r in range(2):
        xs = _layer_inputs(dev, 128 * r, 128)
        shard_out.append(M.run(**xs, local_expert_offset=128 * r, routed_scaling_factor=2.5).float())
        del xs
    summed = (shard_out[0] + shard_out[1]).to(torch.bfloat16).cpu()
    rows = torch.cat([p["rows"] for p in parts])
    for got in (rows, parts[0]["full"], parts[1]["full"]):
        assert torch.equal(got.view(torch.int16), summed.view(torch.int16))

    x = _layer_inputs(dev, 0, 256)
    want = M.run(**x, local_expert_offset=0, routed_scaling_factor=2.5).float().cpu()
    got = rows.float()
    err = (got - want).abs()
    bad = err > C.ATOL + C.RTOL * want.abs()
    assert int(bad.sum()) <= 1e-3 * want.numel(), f"{int(bad.sum())} elements outside tolerance"
    assert float(err.max()) <= 5 * C.ATOL
    assert want.abs().max() > 0


def _dispatch_rank_main(rank, world, port, out_dir):
    from datetime import timedelta

    import torch.distributed as dist

    from moe_swarm_b200 import ep
    from moe_swarm_b200 import workload as W

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=device)
    try:
        sh = ep.shard(rank, world)
        x = _layer_inputs(device, sh.offset, sh.experts)
        own = {k: v.to(device) for k, v in W.make_steered_activations(T, SEED + 1 + rank, 0, FAVOUR).items()}
        layer = ep.ExpertParallelMoE()
        out = layer.forward_dispatch(own["routing_logits"], own["routing_bias"], own["hidden_states"],
                                     own["hidden_states_scale"], x["gemm1_weights"], x["gemm1_weights_scale"],
                                     x["gemm2_weights"], x["gemm2_weights_scale"], 2.5)
        torch.cuda.synchronize()
        torch.save(out.cpu(), os.path.join(out_dir, f"dispatch{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_two_rank_token_dispatch_matches_single_gpu(tmp_path):
    """Token-dispatch EP (each rank routes its own tokens, all-to-all to the expert owners,
    pre-routed layer, all-to-all back): every rank's rows match the single-GPU layer over all
    256 experts for its tokens, within the bar of the broadcast test above."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    import moe_swarm_b200 as M
    from moe_swarm_b200 import workload as W

    mp.start_processes(_dispatch_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    dev = torch.device("cuda", 0)
    full = _layer_inputs(dev, 0, 256)
    for rank in range(2):
        got = torch.load(tmp_path / f"dispatch{rank}.pt").float()
        own = {k: v.to(dev) for k, v in W.make_steered_activations(T, SEED + 1 + rank, 0, FAVOUR).items()}
        want = M.run(**{**full, **own}, local_expert_offset=0, routed_scaling_factor=2.5).float().cpu()
        err = (got - want).abs()
        bad = err > C.ATOL + C.RTOL * want.abs()
        assert int(bad.sum()) <= 1e-3 * want.numel(), f"rank {rank}: {int(bad.sum())} elements outside tolerance"
        assert float(err.max()) <= 5 * C.ATOL
        assert want.abs().max() > 0


PEER_TOKENS = (64, 640)   # the streaming kernels, then the wide ones


def _peer_rank_main(rank, world, port, out_dir):
    from datetime import timedelta

    import torch.distributed as dist

    import moe_swarm_b200 as M
    from moe_swarm_b200 import ep
    from moe_swarm_b200 import workload as W

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=device)
    try:
        sh = ep.shard(rank, world)
        wts = W.make_weights_fast(sh.experts, 900 + rank, device=device)
        layer = ep.ExpertParallelMoE()
        res = {}
        for t in PEER_TOKENS:
            x = {k: v.to(device) for k, v in W.make_activations(t, 31 + t).items()}
            args = (x["routing_logits"], x["routing_bias"], x["hidden_states"], x["hidden_states_scale"],
                    wts["gemm1_weights"], wts["gemm1_weights_scale"], wts["gemm2_weights"],
                    wts["gemm2_weights_scale"], 2.5)
            rows = [layer.forward(*args, combine="peer").clone() for _ in range(3)]   # both phases, reuse
            local = layer.partial(*args)
            torch.cuda.synchronize()
            res[t] = {"rows": [r.cpu() for r in rows], "local": local.cpu(),
                      "status": M.device_status(device, t, sh.experts)}
        torch.save(res, os.path.join(out_dir, f"peer{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_two_rank_peer_combine_equals_sum_of_partials(tmp_path):
    """The combine over peer memory (moe_b200_forward_ep): each rank's GEMM2 and combine
    epilogues store its rows into the owning rank's buffer, and the owner sums the slots in rank
    order.  Random routing (tokens with 0, 1 and several local experts) and random weights on
    both ranks; T = 64 runs the streaming kernels, T = 640 the wide ones; three calls per size
    cover both buffer phases and their reuse.  Every call's rows equal, bit for bit, the bf16
    rounding of the fp32 sum of the two ranks' partial outputs (each computed by the plain
    single-GPU call), and the device status stays 0."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    mp.start_processes(_peer_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    parts = [torch.load(tmp_path / f"peer{r}.pt") for r in range(2)]
    for t in PEER_TOKENS:
        want = (parts[0][t]["local"].float() + parts[1][t]["local"].float()).to(torch.bfloat16)
        assert want.float().abs().max() > 0
        for r in range(2):
            p = parts[r][t]
            assert p["status"] == 0, f"rank {r} T={t}: device status {p['status']:#x}"
            lo, hi = r * t // 2, (r + 1) * t // 2
            for i, got in enumerate(p["rows"]):
                assert torch.equal(got.view(torch.int16), want[lo:hi].view(torch.int16)), (r, t, i)
