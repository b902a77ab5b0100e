"""Generate the golden vectors that pin the CPU oracle to the reference itself.

Run in a container that holds the reference checkout (pass its root as
``--reference``).  It imports the reference's own code --
``spec/reference_official.py`` (``run``), ``reference/kernel_pytorch_v1.py``
(``kernel``, ``_route``) and ``test_kernel.py`` (``route_reference``, the
routing lifted verbatim from the official reference) -- on seeded inputs from
``moe_swarm_b200.workload`` and stores their outputs here as ``.npz``:

* ``layer_<case>.npz``  official and v1 bf16 outputs (as uint16), the routing
  (per-token sorted expert ids and their weights), and sha256 digests of the
  activations and of every routed expert's weights so a drifted generator is
  caught before a comparison is trusted;
* ``route_<case>.npz``  routing only, for larger T.

The fixtures are small (< 2 MB); the inputs are regenerated from their seeds.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
from moe_swarm_b200 import workload as W  # noqa: E402

# (name, T, seed, offset, skew, steered favour or None)
LAYER_CASES = [
    ("cfg0_T16", 16, 0, 0, 0.0, None),
    ("T1_off32", 1, 3, 32, 0.0, None),
    ("T7_off192", 7, 4, 192, 0.0, None),
    ("steered_T8_off96", 8, 5, 96, 0.0, [3, 17, 5, 30, 11, 0, 22, 9]),
    ("skew_T24", 24, 6, 0, 0.5, None),
]
# (name, T, seed, skew)
ROUTE_CASES = [
    ("T1", 1, 10, 0.0),
    ("T7", 7, 11, 0.0),
    ("T56", 56, 12, 0.0),
    ("T257", 257, 13, 0.0),
    ("T901_skew", 901, 14, 0.5),
    ("T4096", 4096, 15, 0.0),
]


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().reshape(-1).view(torch.uint8).numpy().tobytes()).hexdigest()


def activation_digest(x) -> str:
    h = hashlib.sha256()
    for k in ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale"):
        h.update(x[k].contiguous().reshape(-1).view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def expert_digest(x, le: int) -> str:
    h = hashlib.sha256()
    for k in ("gemm1_weights", "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale"):
        h.update(x[k][le].contiguous().reshape(-1).view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def sorted_routing(topk_idx: torch.Tensor, weights: torch.Tensor):
    idx = topk_idx.sort(dim=1).values
    return idx.to(torch.int16).numpy(), torch.gather(weights, 1, idx).numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout")
    args = ap.parse_args()
    ref = Path(args.reference)
    sys.path.insert(0, str(ref / "spec"))
    sys.path.insert(0, str(ref / "reference"))
    sys.path.insert(0, str(ref))
    cwd = os.getcwd()
    os.chdir(ref)                       # test_kernel.py inserts the relative path "reference"
    import reference_official as RO      # noqa: E402
    import kernel_pytorch_v1 as V1       # noqa: E402
    import test_kernel as TK             # noqa: E402
    os.chdir(cwd)
    torch.set_num_threads(os.cpu_count() or 1)

    for name, T, seed, skew in ROUTE_CASES:
        x = W.make_activations(T, seed, skew=skew)
        idx_o, w_o = TK.route_reference(x["routing_logits"], x["routing_bias"], 2.5)
        idx_v, w_v = V1._route(x["routing_logits"], x["routing_bias"], 2.5)
        ids, ws = sorted_routing(idx_o, w_o)
        ids_v, ws_v = sorted_routing(idx_v, w_v)
        np.savez_compressed(HERE / f"route_{name}.npz", T=T, seed=seed, skew=skew, rsf=2.5,
                            act_sha=activation_digest(x), topk_sorted=ids, w_sorted=ws,
                            topk_sorted_v1=ids_v, w_sorted_v1=ws_v)
        print("route", name, "ok")

    for name, T, seed, offset, skew, favour in LAYER_CASES:
        if favour is None:
            x = W.make_inputs(T, seed=seed, offset=offset, skew=skew)
        else:
            x = W.make_steered_activations(T, seed, offset, favour)
            x.update(W.make_weights(32, offset, seed))
            x["local_expert_offset"] = offset
            x["routed_scaling_factor"] = 2.5
        out_o = RO.run(**x)
        out_v = V1.kernel(**x)
        idx_o, w_o = TK.route_reference(x["routing_logits"], x["routing_bias"], 2.5)
        ids, ws = sorted_routing(idx_o, w_o)
        local = sorted({int(e) - offset for e in idx_o.flatten().tolist()
                        if offset <= int(e) < offset + 32})
        np.savez_compressed(
            HERE / f"layer_{name}.npz", T=T, seed=seed, offset=offset, skew=skew, rsf=2.5,
            favour=np.array(favour if favour is not None else [], dtype=np.int64),
            act_sha=activation_digest(x), active=np.array(local, dtype=np.int64),
            expert_sha=np.array([expert_digest(x, le) for le in local]),
            out_official=out_o.view(torch.int16).numpy(), out_v1=out_v.view(torch.int16).numpy(),
            topk_sorted=ids, w_sorted=ws)
        print("layer", name, "active", local)


if __name__ == "__main__":
    main()
