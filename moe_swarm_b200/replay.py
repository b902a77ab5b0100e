"""Replay of workload files in the flashinfer-bench format this layer is scored on.

A workload file (the reference's ``spec/workloads.jsonl``) holds one JSON object per line::

    {"definition": "moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048",
     "workload": {"uuid": "...", "axes": {"seq_len": T},
                  "inputs": {"routing_logits": {"type": "safetensors", "path": "...", "tensor_key": "..."},
                             "hidden_states": {"type": "random"},
                             "local_expert_offset": {"type": "scalar", "value": 192}, ...}}}

Inputs of type ``safetensors`` are read from that file, its relative ``path`` resolved against
``blob_root`` (the contest's captured routing logits and bias are not shipped with the reference,
so the caller supplies the directory).  Inputs of type ``random`` are generated with this
package's seeded generators (``workload.py``) at the definition's shapes and dtypes.  The result
is the keyword arguments of :func:`moe_swarm_b200.run`.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path

import torch

from . import workload as W

DEFINITION = "moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048"
E_LOCAL = 32
ARGS = ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale", "gemm1_weights",
        "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale", "local_expert_offset",
        "routed_scaling_factor")
WEIGHTS = ("gemm1_weights", "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale")


@dataclass
class Workload:
    uuid: str
    T: int
    inputs: dict = field(default_factory=dict)   # argument name -> input spec (dict)

    @property
    def offset(self) -> int:
        return int(self.inputs["local_expert_offset"]["value"])

    @property
    def rsf(self) -> float:
        return float(self.inputs["routed_scaling_factor"]["value"])


def load(path) -> list:
    """Parses a workload file; rejects other definitions and incomplete input lists."""
    out = []
    for n, line in enumerate(Path(path).read_text().splitlines(), 1):
        if not line.strip():
            continue
        rec = json.loads(line)
        if rec.get("definition") != DEFINITION:
            raise ValueError(f"{path}:{n}: definition {rec.get('definition')!r} is not {DEFINITION}")
        wl = rec["workload"]
        inputs = wl["inputs"]
        missing = [a for a in ARGS if a not in inputs]
        if missing:
            raise ValueError(f"{path}:{n}: inputs missing {missing}")
        for a in ("local_expert_offset", "routed_scaling_factor"):
            if inputs[a].get("type") != "scalar":
                raise ValueError(f"{path}:{n}: {a} must be a scalar input")
        out.append(Workload(uuid=wl.get("uuid", f"line{n}"), T=int(wl["axes"]["seq_len"]), inputs=inputs))
    return out


def _tensor(spec, blob_root, name):
    from safetensors.torch import load_file
    p = Path(spec["path"])
    if not p.is_absolute():
        if blob_root is None:
            raise ValueError(f"{name}: relative blob path {p} needs blob_root")
        p = Path(blob_root) / p
    return load_file(str(p))[spec.get("tensor_key", name)]


def materialize(wl: Workload, blob_root=None, seed: int = 0, device="cpu", weights=None) -> dict:
    """Keyword arguments of ``run`` for one workload.  ``weights`` (the four weight tensors) may
    be passed in to reuse one random-init weight set across workloads; otherwise they are
    generated (on the device when it is a GPU)."""
    dev = torch.device(device)
    act = W.make_activations(wl.T, seed)
    x = {}
    for name in ARGS[:4]:
        spec = wl.inputs[name]
        kind = spec.get("type")
        if kind == "safetensors":
            x[name] = _tensor(spec, blob_root, name)
        elif kind == "random":
            x[name] = act[name]
        else:
            raise ValueError(f"{name}: unsupported input type {kind!r}")
    if weights is None:
        kinds = {wl.inputs[n].get("type") for n in WEIGHTS}
        if kinds != {"random"}:
            raise ValueError("weights given as files are not supported; pass weights=")
        weights = (W.make_weights_fast(E_LOCAL, seed, device=dev) if dev.type == "cuda"
                   else W.make_weights(E_LOCAL, wl.offset, seed))
    x = {k: v.to(dev) for k, v in x.items()}
    x.update({k: weights[k] for k in WEIGHTS})
    x["local_expert_offset"] = wl.offset
    x["routed_scaling_factor"] = wl.rsf
    T = wl.T
    shapes = {"routing_logits": (T, 256), "routing_bias": (256,), "hidden_states": (T, 7168),
              "hidden_states_scale": (56, T)}
    for k, shp in shapes.items():
        if tuple(x[k].shape) != shp:
            raise ValueError(f"{k}: shape {tuple(x[k].shape)} for seq_len {T}, expected {shp}")
    return x
