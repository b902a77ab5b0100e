"""CPU: the C-ABI library loads, exports every declared entry point, and its host-side
argument/workspace logic behaves (no kernel is launched: no GPU is needed)."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

import moe_swarm_b200 as M
from moe_swarm_b200 import _native as N

HEADER = Path(__file__).resolve().parents[1] / "include" / "moe_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"MOE_B200_API\s+[\w\s\*]+?\b(moe_b200_\w+)\s*\(", text)))


def test_header_declares_the_exported_set():
    assert declared_symbols() == sorted(N.EXPORTED)


def test_library_loads_and_exports_every_declared_symbol():
    lib = N.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name


@pytest.mark.parametrize("T,E", [(1, 32), (16, 32), (129, 32), (4096, 256), (16384, 32), (7, 1)])
def test_workspace_layout_is_consistent(T, E):
    L = N.layout(T, E)
    assert L.total == N.lib().moe_b200_workspace_size(T, E)
    offs = [L.plan, L.topk_idx, L.topk_w, L.tok_nloc, L.tok_rows, L.e_count, L.e_start, L.row_token,
            L.row_weight, L.c_hi, L.c_lo, L.c_scale, L.status]
    assert all(o % 1024 == 0 and o < L.total for o in offs)
    assert len(set(offs)) == len(offs)
    assert L.r_max == T * min(8, E) and L.r_pad >= L.r_max and L.r_pad % 32 == 0


def test_workspace_size_rejects_bad_sizes():
    lib = N.lib()
    assert lib.moe_b200_workspace_size(-1, 32) == 0
    assert lib.moe_b200_workspace_size(4, 0) == 0
    assert lib.moe_b200_workspace_size(4, 257) == 0


def _args(T=4, E=32):
    a = N.MoeArgs()
    a.num_tokens, a.num_local_experts, a.local_expert_offset, a.routed_scaling_factor = T, E, 0, 2.5
    return a


def test_forward_rejects_bad_arguments_without_touching_a_gpu():
    lib = N.lib()
    assert lib.moe_b200_forward(None, None, 0, None) == N.ERR_ARG
    a = _args(T=-1)
    assert lib.moe_b200_forward(ctypes.byref(a), None, 0, None) == N.ERR_ARG
    a = _args(E=300)
    assert lib.moe_b200_forward(ctypes.byref(a), None, 0, None) == N.ERR_ARG
    a = _args(T=4)   # null tensor pointers
    assert lib.moe_b200_forward(ctypes.byref(a), None, 0, None) == N.ERR_ARG
    assert "null" in N.last_error()
    # aligned fake pointers but a missing workspace
    a = _args(T=4)
    for f in ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale", "gemm1_weights",
              "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale", "output"):
        setattr(a, f, 1 << 20)
    assert lib.moe_b200_forward(ctypes.byref(a), None, 0, None) == N.ERR_WORKSPACE
    a.gemm1_weights = (1 << 20) + 8
    assert lib.moe_b200_forward(ctypes.byref(a), None, 0, None) == N.ERR_ARG
    assert "aligned" in N.last_error()
    # a large enough workspace that is not 256-byte aligned (rejected before any CUDA call)
    a.gemm1_weights = 1 << 20
    need = lib.moe_b200_workspace_size(4, 32)
    assert lib.moe_b200_forward(ctypes.byref(a), ctypes.c_void_p((1 << 30) + 16), need, None) == N.ERR_ARG
    assert "256-byte" in N.last_error()
    assert lib.moe_b200_workspace_init(ctypes.c_void_p((1 << 30) + 16), need, 4, 32, None) == N.ERR_ARG


def test_forward_ep_rejects_bad_arguments_without_touching_a_gpu():
    lib = N.lib()
    a = _args(T=8)
    for f in ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale", "gemm1_weights",
              "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale", "output"):
        setattr(a, f, 1 << 20)

    def ep(world=2, rank=0, shard=4, epoch=1, peers=2):
        e = N.MoeEp()
        e.world, e.rank, e.shard_tokens, e.epoch = world, rank, shard, epoch
        for r in range(peers):
            e.recv[r] = (1 << 21) * (r + 1)
            e.signal[r] = (1 << 22) * (r + 1)
        e.out_shard = 1 << 23
        return e

    def rc(e):
        return lib.moe_b200_forward_ep(ctypes.byref(a), ctypes.byref(e), None, 0, None)

    assert lib.moe_b200_forward_ep(ctypes.byref(a), None, None, 0, None) == N.ERR_ARG
    assert rc(ep(world=0)) == N.ERR_ARG
    assert rc(ep(world=9)) == N.ERR_ARG
    assert rc(ep(rank=2)) == N.ERR_ARG
    assert rc(ep(shard=3)) == N.ERR_ARG and "shard_tokens" in N.last_error()
    assert rc(ep(epoch=0)) == N.ERR_ARG and "epoch" in N.last_error()
    assert rc(ep(peers=1)) == N.ERR_ARG and "every rank" in N.last_error()
    e = ep()
    e.recv[1] = (1 << 21) + 4   # misaligned receive buffer
    assert rc(e) == N.ERR_ARG
    assert rc(ep()) == N.ERR_WORKSPACE   # valid EP arguments reach the workspace check


def test_python_entry_validates_like_the_reference():
    T = 2
    x = {
        "routing_logits": torch.zeros(T, 256),
        "routing_bias": torch.zeros(256, dtype=torch.bfloat16),
        "hidden_states": torch.zeros(T, 7168, dtype=torch.float8_e4m3fn),
        "hidden_states_scale": torch.ones(56, T),
        "gemm1_weights": torch.zeros(1, 4096, 7168, dtype=torch.float8_e4m3fn),
        "gemm1_weights_scale": torch.ones(1, 32, 56),
        "gemm2_weights": torch.zeros(1, 7168, 2048, dtype=torch.float8_e4m3fn),
        "gemm2_weights_scale": torch.ones(1, 56, 16),
        "local_expert_offset": 0,
        "routed_scaling_factor": 2.5,
    }
    with pytest.raises(AssertionError, match="CUDA"):   # valid shapes, CPU tensors: no CPU path
        M.run(**x)
    bad = dict(x, hidden_states_scale=torch.ones(T, 56))
    with pytest.raises(M.MoEArgumentError, match="56, T"):
        M.run(**bad)
    bad = dict(x, routing_logits=torch.zeros(T, 128))
    with pytest.raises(AssertionError, match="256"):
        M.run(**bad)
    assert M.kernel is M.run
