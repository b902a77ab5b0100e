"""Workload replay (flashinfer-bench jsonl + safetensors blobs) -- moe_swarm_b200/replay.py.

The contest's own blobs are not shipped with the reference; these tests write a small workload
file and blob of the same format (captured-logit inputs for one workload, all-random for the
other) and check parsing, blob resolution, the generated inputs' shapes, the error cases, and
on a GPU that a replayed workload matches the oracle.
"""

import json

import pytest
import torch
from safetensors.torch import save_file

from moe_swarm_b200 import replay as R
from moe_swarm_b200 import workload as W
from oracle import moe_ref as O
from tests import _cases as C


def _write_case(tmp_path):
    blob_dir = tmp_path / "blob" / "workloads"
    blob_dir.mkdir(parents=True)
    g = torch.Generator().manual_seed(5)
    logits = torch.randn(7, 256, generator=g)
    bias = (torch.randn(256, generator=g) * 0.1).to(torch.bfloat16)
    save_file({"routing_logits": logits, "routing_bias": bias}, str(blob_dir / "case7.safetensors"))
    rel = "./blob/workloads/case7.safetensors"
    rand = {"type": "random"}
    captured = {
        "routing_logits": {"type": "safetensors", "path": rel, "tensor_key": "routing_logits"},
        "routing_bias": {"type": "safetensors", "path": rel, "tensor_key": "routing_bias"},
        "hidden_states": rand, "hidden_states_scale": rand, "gemm1_weights": rand,
        "gemm1_weights_scale": rand, "gemm2_weights": rand, "gemm2_weights_scale": rand,
        "local_expert_offset": {"type": "scalar", "value": 192},
        "routed_scaling_factor": {"type": "scalar", "value": 2.5},
    }
    all_random = dict(captured, routing_logits=rand, routing_bias=rand,
                      local_expert_offset={"type": "scalar", "value": 0})
    lines = [{"definition": R.DEFINITION, "solution": None,
              "workload": {"uuid": "w7", "axes": {"seq_len": 7}, "inputs": captured}, "evaluation": None},
             {"definition": R.DEFINITION, "solution": None,
              "workload": {"uuid": "w3", "axes": {"seq_len": 3}, "inputs": all_random}, "evaluation": None}]
    path = tmp_path / "workloads.jsonl"
    path.write_text("\n".join(json.dumps(x) for x in lines) + "\n")
    return path, logits, bias


def test_load_and_materialize(tmp_path):
    path, logits, bias = _write_case(tmp_path)
    wls = R.load(path)
    assert [(w.uuid, w.T, w.offset, w.rsf) for w in wls] == [("w7", 7, 192, 2.5), ("w3", 3, 0, 2.5)]
    stub = {k: torch.empty(0) for k in R.WEIGHTS}
    x = R.materialize(wls[0], blob_root=tmp_path, seed=11, weights=stub)
    assert torch.equal(x["routing_logits"], logits)
    assert torch.equal(x["routing_bias"].view(torch.int16), bias.view(torch.int16))
    assert x["hidden_states"].shape == (7, 7168) and x["hidden_states"].dtype == torch.float8_e4m3fn
    assert x["hidden_states_scale"].shape == (56, 7)
    assert x["local_expert_offset"] == 192 and x["routed_scaling_factor"] == 2.5
    y = R.materialize(wls[1], seed=11, weights=stub)            # all random: no blob needed
    assert y["routing_logits"].shape == (3, 256)


def test_rejects_other_definitions_and_bad_inputs(tmp_path):
    path, _, _ = _write_case(tmp_path)
    recs = [json.loads(s) for s in path.read_text().splitlines()]
    bad = dict(recs[0], definition="moe_something_else")
    p2 = tmp_path / "bad.jsonl"
    p2.write_text(json.dumps(bad) + "\n")
    with pytest.raises(ValueError):
        R.load(p2)
    del recs[0]["workload"]["inputs"]["routing_bias"]
    p3 = tmp_path / "missing.jsonl"
    p3.write_text(json.dumps(recs[0]) + "\n")
    with pytest.raises(ValueError):
        R.load(p3)
    wl = R.load(path)[0]
    with pytest.raises(ValueError):   # relative blob path without a blob root
        R.materialize(wl, blob_root=None, weights={k: torch.empty(0) for k in R.WEIGHTS})


@pytest.mark.gpu
def test_replayed_workload_matches_oracle(tmp_path, cuda_device):
    import moe_swarm_b200 as M
    path, _, _ = _write_case(tmp_path)
    wl = R.load(path)[0]
    stub = {k: torch.empty(0) for k in R.WEIGHTS}
    x = R.materialize(wl, blob_root=tmp_path, seed=13, weights=stub)
    idx, w = O.route(x["routing_logits"], x["routing_bias"], wl.rsf)
    _, _, _, counts = O.local_permutation(idx, w, wl.offset, R.E_LOCAL)
    active = [int(e) for e in (counts > 0).nonzero().flatten()]
    x.update(W.make_weights(R.E_LOCAL, wl.offset, 13, experts=active))
    out = M.run(**C.to_device(x, cuda_device))
    torch.cuda.synchronize()
    want = O.run(**x)
    r = O.parity_report(out.cpu(), want)
    assert r["bad"] == 0, r
    assert M.device_status(cuda_device) == 0
