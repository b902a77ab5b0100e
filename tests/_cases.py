"""Shared helpers of the test suite: golden fixtures and seeded input regeneration."""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import torch

from moe_swarm_b200 import workload as W
from oracle import moe_ref as O

GOLDEN = Path(__file__).resolve().parent / "golden"
ATOL = 1e-2   # bf16 output tolerance of the layer (north-star parity bar)
RTOL = 2e-2


def layer_fixtures():
    return sorted(GOLDEN.glob("layer_*.npz"))


def route_fixtures():
    return sorted(GOLDEN.glob("route_*.npz"))


def _digest(tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.contiguous().reshape(-1).view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def activation_digest(x) -> str:
    return _digest([x[k] for k in ("routing_logits", "routing_bias", "hidden_states",
                                   "hidden_states_scale")])


def expert_digest(x, le) -> str:
    return _digest([x[k][le] for k in ("gemm1_weights", "gemm1_weights_scale", "gemm2_weights",
                                       "gemm2_weights_scale")])


def load_layer_case(path, fill_missing_nan=False):
    """Regenerates a golden layer case's inputs (routed experts only) on the CPU and
    checks them against the fixture's digests before they are trusted."""
    z = np.load(path)
    T, seed, offset = int(z["T"]), int(z["seed"]), int(z["offset"])
    skew, rsf = float(z["skew"]), float(z["rsf"])
    favour = [int(e) for e in z["favour"]]
    if favour:
        x = W.make_steered_activations(T, seed, offset, favour)
    else:
        x = W.make_activations(T, seed, skew=skew)
    active = [int(e) for e in z["active"]]
    x.update(W.make_weights(32, offset, seed, experts=active, fill_missing_nan=fill_missing_nan))
    x["local_expert_offset"] = offset
    x["routed_scaling_factor"] = rsf
    assert activation_digest(x) == str(z["act_sha"]), f"{path.name}: activation generator drifted"
    for le, d in zip(active, z["expert_sha"]):
        assert expert_digest(x, le) == str(d), f"{path.name}: expert {le} generator drifted"
    golden = {
        "official": torch.from_numpy(z["out_official"]).view(torch.bfloat16),
        "v1": torch.from_numpy(z["out_v1"]).view(torch.bfloat16),
        "topk_sorted": torch.from_numpy(z["topk_sorted"].astype(np.int64)),
        "w_sorted": torch.from_numpy(z["w_sorted"]),
    }
    return x, golden


def make_case(T, seed, E_local=32, offset=0, skew=0.0, rsf=2.5, fill_missing_nan=False):
    """Seeded inputs with only the routed local experts materialised."""
    x = W.make_activations(T, seed, skew=skew)
    idx, w = O.route(x["routing_logits"], x["routing_bias"], rsf)
    _, le, _, counts = O.local_permutation(idx, w, offset, E_local)
    active = [int(e) for e in (counts > 0).nonzero().flatten()]
    x.update(W.make_weights(E_local, offset, seed, experts=active, fill_missing_nan=fill_missing_nan))
    x["local_expert_offset"] = offset
    x["routed_scaling_factor"] = rsf
    return x


def to_device(x, device):
    return {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in x.items()}


class DeviceExperts:
    """A stacked weight tensor on the GPU that the CPU oracle indexes one expert at a time: ``[le]``
    copies only that expert to the host, so the oracle of a large configuration materialises on the
    CPU just the experts its sampled tokens are routed to."""

    def __init__(self, t):
        self.t = t
        self.shape = tuple(t.shape)

    def __getitem__(self, le):
        return self.t[le].cpu()


def sample_tokens(idx, w, offset, E_local, T, limit=24, seed=0):
    """Tokens whose rows exercise the edges of the large-batch path: the first and last rows of the
    128-row token tiles of the most, least and median loaded local experts, tokens with the most
    local experts, tokens with none, and the first and last token."""
    tok, le, _, counts = O.local_permutation(idx, w, offset, E_local)
    starts = torch.cumsum(counts, 0) - counts
    nloc = torch.bincount(tok, minlength=T)
    picks = []
    live = (counts > 0).nonzero().flatten()
    if len(live):
        order = live[torch.argsort(counts[live], stable=True)]
        for e in (int(order[-1]), int(order[0]), int(order[len(order) // 2])):
            n, s = int(counts[e]), int(starts[e])
            for pos in (0, 127, 128, 255, 256, n - 1):
                if 0 <= pos < n:
                    picks.append(int(tok[s + pos]))
    most = int(nloc.max())
    picks += [int(t) for t in (nloc == most).nonzero().flatten()[:4]]
    picks += [int(t) for t in (nloc == 0).nonzero().flatten()[:2]]
    picks += [0, T - 1]
    g = torch.Generator().manual_seed(seed)
    picks += [int(t) for t in torch.randint(0, T, (4,), generator=g)]
    out = []
    for t in picks:
        if t not in out:
            out.append(t)
    return torch.tensor(out[:limit], dtype=torch.long)


def oracle_rows(act, dev_weights, tokens, offset, rsf=2.5):
    """The oracle's output rows (spec/reference_official.py semantics, oracle/moe_ref.py) for the
    given tokens only.  Every output row depends on its own token alone -- its routing, its
    activations and its experts -- so the rows equal those of the whole-batch oracle."""
    idx, w = O.route(act["routing_logits"], act["routing_bias"], rsf)
    A = O.dequant_tokens(act["hidden_states"][tokens], act["hidden_states_scale"][:, tokens])
    with torch.no_grad():
        out = O._experts_fp32(A, idx[tokens], w[tokens],
                              DeviceExperts(dev_weights["gemm1_weights"]),
                              DeviceExperts(dev_weights["gemm1_weights_scale"]),
                              DeviceExperts(dev_weights["gemm2_weights"]),
                              DeviceExperts(dev_weights["gemm2_weights_scale"]), offset)
    return out.to(torch.bfloat16)
