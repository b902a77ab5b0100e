"""GPU: properties of the layer the reference's anti-cheat gates check (gates.py:385-463),
in sharper form -- which output rows an input change may move, and that no state survives
between calls or lives outside the caller's workspace.

* Input locality: changing one token's hidden state moves exactly that token's output row
  (if the token has a local expert), and zeroing one local expert's weights moves exactly the
  rows of the tokens routed to it.  Shown on the streaming (T <= 512) and the wide path.
* No hidden state: a second workspace allocated by the caller and driven through the C ABI
  gives the same bits as the package's cached workspace, before and after an unrelated call.
"""

import ctypes

import pytest
import torch

import moe_swarm_b200 as M
from moe_swarm_b200 import _native as N
from oracle import moe_ref as O
from tests import _cases as C

pytestmark = pytest.mark.gpu


def _moved_rows(a, b):
    return (a.view(torch.int16) != b.view(torch.int16)).any(dim=1).cpu()


@pytest.mark.parametrize("T,seed", [(40, 301), (700, 302)])
def test_one_token_change_moves_only_its_row(cuda_device, T, seed):
    x = C.make_case(T, seed)
    idx, _ = O.route(x["routing_logits"], x["routing_bias"], 2.5)
    local = ((idx >= 0) & (idx < 32)).any(dim=1)
    t = int(local.nonzero()[len(local.nonzero()) // 2])
    d = C.to_device(x, cuda_device)
    base = M.run(**d).clone()
    hs = d["hidden_states"].clone()
    hs[t] = (hs[t].float() * -1.0).to(torch.float8_e4m3fn)   # sign flip of every element of row t
    changed = M.run(**{**d, "hidden_states": hs})
    torch.cuda.synchronize()
    moved = _moved_rows(base, changed)
    assert moved[t], "the changed token's output did not move"
    assert int(moved.sum()) == 1, f"{int(moved.sum()) - 1} other rows moved"
    assert M.device_status(cuda_device) == 0


@pytest.mark.parametrize("T,seed", [(40, 311), (700, 312)])
def test_one_expert_change_moves_only_its_tokens(cuda_device, T, seed):
    x = C.make_case(T, seed)
    idx, _ = O.route(x["routing_logits"], x["routing_bias"], 2.5)
    counts = torch.bincount(idx.flatten(), minlength=256)[:32]
    e = int(torch.argmax(counts))
    d = C.to_device(x, cuda_device)
    base = M.run(**d).clone()
    w2 = d["gemm2_weights"].clone()
    w2[e].zero_()
    changed = M.run(**{**d, "gemm2_weights": w2})
    torch.cuda.synchronize()
    moved = _moved_rows(base, changed)
    routed = (idx == e).any(dim=1)
    assert torch.equal(moved, routed), "rows moved that expert e does not feed, or rows it feeds did not"
    assert M.device_status(cuda_device) == 0


def _forward_with(ws, d, out):
    T = d["routing_logits"].shape[0]
    E = d["gemm1_weights"].shape[0]
    a = M._args(T, E, d["routing_logits"], d["routing_bias"], d["hidden_states"], d["hidden_states_scale"],
                d["gemm1_weights"], d["gemm1_weights_scale"], d["gemm2_weights"], d["gemm2_weights_scale"],
                d["local_expert_offset"], d["routed_scaling_factor"], out)
    rc = N.lib().moe_b200_forward(ctypes.byref(a), ws.data_ptr(), ws.numel(),
                                  torch.cuda.current_stream(cuda_device_of(d)).cuda_stream)
    assert rc == 0, N.last_error()


def cuda_device_of(d):
    return d["hidden_states"].device


@pytest.mark.parametrize("T,seed", [(24, 321), (900, 322)])
def test_fresh_workspace_gives_the_same_bits(cuda_device, T, seed):
    d = C.to_device(C.make_case(T, seed), cuda_device)
    other = C.to_device(C.make_case(T, seed + 1000), cuda_device)
    want = M.run(**d).clone()
    n = N.lib().moe_b200_workspace_size(T, 32)
    ws = torch.zeros(n, dtype=torch.uint8, device=cuda_device)   # zeroed = initialised
    got1 = torch.empty_like(want)
    _forward_with(ws, d, got1)
    M.run(**other)                                               # an unrelated call in between
    got2 = torch.empty_like(want)
    _forward_with(ws, d, got2)
    torch.cuda.synchronize()
    assert torch.equal(got1.view(torch.int16), want.view(torch.int16))
    assert torch.equal(got2.view(torch.int16), want.view(torch.int16))
    assert M.device_status(cuda_device) == 0
