"""A bounded device wait that runs out: the peer-memory combine (moe_b200_forward_ep) waiting for a
rank that never signals.

On one GPU, "rank 0" of a two-rank group makes the call with both ranks' receive buffers and flag
words in its own memory.  Nothing plays rank 1, so rank 1's flag never arrives.  With a 10 ms wait
bound the call must come back with the device status 0x107 (peers' rows not received), without a
trap or a fault, and the context must stay usable: after the status is cleared and the workspace
re-initialised, a call whose rank-1 flag is present (set by the host, as if rank 1 had written it)
succeeds and returns rank 0's rows unchanged (rank 1's slot holds zeros).  The host-side analogue
in the reference is the timeout of its gate subprocesses (gates.py:175-180).
"""

import ctypes
import time

import pytest
import torch

import moe_swarm_b200 as M
from moe_swarm_b200 import _native as N
from moe_swarm_b200 import workload as W
from tests import _cases as C

pytestmark = pytest.mark.gpu

WORLD, RANK, T, E = 2, 0, 64, 32
ST_WAIT_PEERS = 0x107


def _call(x, ws, recv, flags, out, epoch, wait_us, device):
    ep = N.MoeEp()
    ep.world, ep.rank, ep.shard_tokens, ep.epoch = WORLD, RANK, T // WORLD, epoch
    for r in range(WORLD):
        ep.recv[r] = recv[r].data_ptr()
        ep.signal[r] = flags[r].data_ptr()
    ep.out_shard = out.data_ptr()
    ep.wait_limit_us = wait_us
    a = M._args(T, E, x["routing_logits"], x["routing_bias"], x["hidden_states"], x["hidden_states_scale"],
                x["gemm1_weights"], x["gemm1_weights_scale"], x["gemm2_weights"], x["gemm2_weights_scale"],
                x["local_expert_offset"], x["routed_scaling_factor"], out)
    stream = torch.cuda.current_stream(device).cuda_stream
    rc = N.lib().moe_b200_forward_ep(ctypes.byref(a), ctypes.byref(ep), ws.data_ptr(), ws.numel(), stream)
    assert rc == N.OK, N.last_error()
    return stream


def test_peer_wait_runs_out_and_reports_status(cuda_device):
    x = C.to_device(C.make_case(T, 701), cuda_device)
    ws = torch.empty(int(N.lib().moe_b200_workspace_size(T, E)), dtype=torch.uint8, device=cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    assert N.lib().moe_b200_workspace_init(ws.data_ptr(), ws.numel(), T, E, stream) == N.OK
    shard = T // WORLD
    recv = [torch.zeros(2 * WORLD * shard * 7168, dtype=torch.bfloat16, device=cuda_device) for _ in range(WORLD)]
    flags = [torch.zeros(2 * 8, dtype=torch.int32, device=cuda_device) for _ in range(WORLD)]
    out = torch.empty((shard, 7168), dtype=torch.bfloat16, device=cuda_device)

    # epoch 1: rank 1 never signals; the 10 ms bound runs out
    t0 = time.perf_counter()
    _call(x, ws, recv, flags, out, 1, 10_000, cuda_device)
    status = N.lib().moe_b200_device_status(ws.data_ptr(), ws.numel(), T, E, stream, 1)
    elapsed = time.perf_counter() - t0
    assert status == ST_WAIT_PEERS, f"device status {status:#x}"
    assert elapsed < 1.5, f"the call took {elapsed:.2f} s: the wait did not end at its bound"
    assert N.lib().moe_b200_device_status(ws.data_ptr(), ws.numel(), T, E, stream, 0) == 0, "status not cleared"

    # the context is still usable: re-initialise, then epoch 2 (phase 0) with rank 1's flag present
    assert N.lib().moe_b200_workspace_init(ws.data_ptr(), ws.numel(), T, E, stream) == N.OK
    for r in range(WORLD):
        recv[r].zero_()
    flags[RANK][0 * 8 + 1] = 2
    _call(x, ws, recv, flags, out, 2, 10_000, cuda_device)
    assert N.lib().moe_b200_device_status(ws.data_ptr(), ws.numel(), T, E, stream, 1) == 0
    ref = M.run(**x)
    torch.cuda.synchronize(cuda_device)
    # rank 0's shard = its own rows + rank 1's (zero) slot, summed in fp32 and rounded once
    assert torch.equal(out.view(torch.int16), ref[:shard].view(torch.int16))
