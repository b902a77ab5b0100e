"""The routing entry point that needs no workspace (moe_b200_route_noalloc).

It exists for callers that cannot allocate device memory when they call in -- inference
engines whose plugin/enqueue path forbids allocations because every byte of device memory
is planned ahead, and latency-critical paths that cannot pay for cudaMalloc's device-wide
synchronisation.  Its scratch is a fixed device array inside the library, shared by every
call.  These tests call it through the C ABI twice in a row (so the second call runs on the
first call's leftovers) and require exactly the results of moe_b200_route, the workspace
entry point; they also check that a batch above its 256-token limit is refused.

This file is named to be collected last, and it passes run alone in a fresh process.
"""

import ctypes

import pytest
import torch

import moe_swarm_b200 as M
from moe_swarm_b200 import _native as N
from moe_swarm_b200 import workload as W

pytestmark = pytest.mark.gpu


def _weights(E, device):
    # shape-valid weights for the workspace entry point (routing never reads them)
    return {
        "gemm1_weights": torch.empty(E, 4096, 7168, dtype=torch.float8_e4m3fn, device=device),
        "gemm1_weights_scale": torch.ones(E, 32, 56, device=device),
        "gemm2_weights": torch.empty(E, 7168, 2048, dtype=torch.float8_e4m3fn, device=device),
        "gemm2_weights_scale": torch.ones(E, 56, 16, device=device),
    }


def _route_noalloc(x, E, offset, device):
    T = x["routing_logits"].shape[0]
    R = T * min(8, E)
    outs = {
        "topk_idx": torch.full((T, 8), -1, dtype=torch.int32, device=device),
        "topk_w": torch.full((T, 8), -1.0, dtype=torch.float32, device=device),
        "e_count": torch.full((E,), -1, dtype=torch.int32, device=device),
        "row_token": torch.full((R,), -1, dtype=torch.int32, device=device),
        "row_weight": torch.full((R,), -1.0, dtype=torch.float32, device=device),
    }
    a = N.MoeArgs()
    a.routing_logits = x["routing_logits"].data_ptr()
    a.routing_bias = x["routing_bias"].data_ptr()
    a.num_tokens, a.num_local_experts, a.local_expert_offset = T, E, offset
    a.routed_scaling_factor = 2.5
    stream = torch.cuda.current_stream(device).cuda_stream
    rc = N.lib().moe_b200_route_noalloc(ctypes.byref(a), outs["topk_idx"].data_ptr(), outs["topk_w"].data_ptr(),
                                        outs["e_count"].data_ptr(), outs["row_token"].data_ptr(),
                                        outs["row_weight"].data_ptr(), stream)
    assert rc == N.OK, N.last_error()
    torch.cuda.synchronize(device)
    return outs


@pytest.mark.parametrize("E,offset", [(32, 0), (64, 128), (256, 0)])
def test_noalloc_routing_equals_workspace_routing_twice(cuda_device, E, offset):
    w = _weights(E, cuda_device)
    # two calls in a row on the shared scratch, the second at the 256-token limit
    for T, seed in ((48, 301), (256, 302)):
        x = {k: v.to(cuda_device) for k, v in W.make_activations(T, seed).items()}
        got = _route_noalloc(x, E, offset, cuda_device)
        ref = M.route(**x, **w, local_expert_offset=offset, routed_scaling_factor=2.5)
        R = int(ref["e_count"].sum())
        assert torch.equal(got["topk_idx"], ref["topk_idx"])
        assert torch.equal(got["topk_w"], ref["topk_w"])
        assert torch.equal(got["e_count"], ref["e_count"])
        assert torch.equal(got["row_token"][:R], ref["row_token"])
        assert torch.equal(got["row_weight"][:R], ref["row_weight"])


def test_noalloc_refuses_batches_above_its_limit(cuda_device):
    x = {k: v.to(cuda_device) for k, v in W.make_activations(257, 303).items()}
    a = N.MoeArgs()
    a.routing_logits = x["routing_logits"].data_ptr()
    a.routing_bias = x["routing_bias"].data_ptr()
    a.num_tokens, a.num_local_experts, a.local_expert_offset, a.routed_scaling_factor = 257, 32, 0, 2.5
    buf = torch.empty(1 << 20, dtype=torch.uint8, device=cuda_device)
    p = buf.data_ptr()
    rc = N.lib().moe_b200_route_noalloc(ctypes.byref(a), p, p, p, p, p, None)
    assert rc == N.ERR_ARG
    assert "256" in N.last_error()
