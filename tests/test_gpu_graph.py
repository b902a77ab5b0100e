"""GPU: the layer call captured in a CUDA graph (moe_swarm_b200.GraphRunner) replays with the
same bits as eager calls, on new input values copied into the static inputs, on the streaming
(T <= 512) and the wide path."""

import pytest
import torch

import moe_swarm_b200 as M
from tests import _cases as C

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T", [16, 700])
def test_graph_replay_matches_eager(cuda_device, T):
    a = C.to_device(C.make_case(T, 401), cuda_device)
    b = C.to_device(C.make_case(T, 402), cuda_device)
    want_a = M.run(**a).clone()
    want_b = M.run(**{**a, **{k: b[k] for k in ("routing_logits", "routing_bias", "hidden_states",
                                                  "hidden_states_scale")}}).clone()
    static = {k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in a.items()}
    g = M.GraphRunner(**static)
    got_a = g.replay().clone()
    for k in ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale"):
        g.inputs[k].copy_(b[k])
    got_b = g.replay().clone()
    torch.cuda.synchronize()
    assert torch.equal(got_a.view(torch.int16), want_a.view(torch.int16))
    assert torch.equal(got_b.view(torch.int16), want_b.view(torch.int16))
    assert M.device_status(cuda_device) == 0
