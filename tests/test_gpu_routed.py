"""GPU: the pre-routed entry point (moe_b200_forward_routed / moe_swarm_b200.run_routed).

Given the routing the layer computes itself -- in any order of a token's picks -- it gives the
same bits as moe_swarm_b200.run; given any other routing it matches the oracle's run_routed
(the official layer from the point its routing is known) within the parity bar.  Covers the
single-CTA (T <= 32) and multi-CTA routing paths and the streaming and wide GEMMs.
"""

import pytest
import torch

import moe_swarm_b200 as M
from oracle import moe_ref as O
from moe_swarm_b200 import workload as W
from tests import _cases as C

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,seed", [(9, 501), (200, 502), (700, 503)])
def test_given_own_routing_equals_run(cuda_device, T, seed):
    x = C.make_case(T, seed)
    d = C.to_device(x, cuda_device)
    r = M.route(**d)                                           # the layer's own device routing
    perm = torch.randperm(8, generator=torch.Generator().manual_seed(seed)).to(cuda_device)
    topk_idx = r["topk_idx"][:, perm].contiguous()             # picks in a scrambled order
    topk_w = r["topk_w"][:, perm].contiguous()
    want = M.run(**d)
    got = M.run_routed(topk_idx, topk_w, d["hidden_states"],
                       d["hidden_states_scale"], d["gemm1_weights"], d["gemm1_weights_scale"],
                       d["gemm2_weights"], d["gemm2_weights_scale"], 0)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    assert M.device_status(cuda_device) == 0


@pytest.mark.parametrize("T,seed", [(24, 511), (600, 512)])
def test_arbitrary_routing_matches_oracle(cuda_device, T, seed):
    g = torch.Generator().manual_seed(seed)
    # 8 distinct experts per token drawn from 12 experts spread over local and remote ids
    pool = torch.tensor([1, 3, 4, 9, 17, 30, 31, 40, 77, 128, 200, 255])
    idx = torch.stack([pool[torch.randperm(len(pool), generator=g)[:8]] for _ in range(T)]).int()
    w = torch.rand(T, 8, generator=g) * 0.5
    act = W.make_activations(T, seed)
    local = sorted({int(e) for e in idx.flatten() if e < 32})
    wts = W.make_weights(32, 0, seed, experts=local)
    want = O.run_routed(idx, w, act["hidden_states"], act["hidden_states_scale"], wts["gemm1_weights"],
                        wts["gemm1_weights_scale"], wts["gemm2_weights"], wts["gemm2_weights_scale"], 0)
    dv = lambda t: t.to(cuda_device)
    got = M.run_routed(dv(idx), dv(w), dv(act["hidden_states"]), dv(act["hidden_states_scale"]),
                       dv(wts["gemm1_weights"]), dv(wts["gemm1_weights_scale"]), dv(wts["gemm2_weights"]),
                       dv(wts["gemm2_weights_scale"]), 0)
    torch.cuda.synchronize()
    r = O.parity_report(got.cpu(), want)
    assert r["bad"] == 0, r
    assert M.device_status(cuda_device) == 0
