"""GPU parity of the CUDA path (through the C ABI) against the CPU oracle.

Bars: expert selection and the permutation bit-exact; bf16 outputs within
atol 1e-2 / rtol 2e-2 of spec/reference_official.run (every element); device status 0.
"""

import numpy as np
import pytest
import torch

import moe_swarm_b200 as M
from oracle import moe_ref as O
from moe_swarm_b200 import workload as W
from tests import _cases as C

pytestmark = pytest.mark.gpu


def _status_ok(device):
    assert M.device_status(device) == 0


def _check_routing(r, x, T, E, offset, rsf):
    idx, w = O.route(x["routing_logits"].cpu(), x["routing_bias"].cpu(), rsf)
    ids = idx.sort(dim=1).values
    assert torch.equal(r["topk_idx"].cpu().long(), ids), "expert selection differs"
    torch.testing.assert_close(r["topk_w"].cpu(), torch.gather(w, 1, ids), rtol=2e-6, atol=1e-7)
    tok, le, ww, counts = O.local_permutation(idx, w, offset, E)
    assert torch.equal(r["e_count"].cpu().long(), counts)
    assert torch.equal(r["row_token"].cpu().long(), tok), "permutation differs"
    torch.testing.assert_close(r["row_weight"].cpu(), ww, rtol=2e-6, atol=1e-7)
    nloc = torch.bincount(tok, minlength=T)
    assert torch.equal(r["tok_nloc"].cpu().long(), nloc)
    # each token's rows in ascending expert order point back at the token
    rows = r["tok_rows"].cpu().long()
    for t in range(T):
        k = int(nloc[t])
        if k:
            assert torch.all(tok[rows[t, :k]] == t)
            assert torch.all(rows[t, 1:k] > rows[t, :k - 1])


@pytest.mark.parametrize("path", C.route_fixtures(), ids=lambda p: p.stem)
def test_routing_matches_reference_golden(cuda_device, path):
    z = np.load(path)
    T = int(z["T"])
    x = W.make_activations(T, int(z["seed"]), skew=float(z["skew"]))
    for offset, E in ((0, 32), (96, 32), (0, 256), (128, 64)):
        d = C.to_device(x, cuda_device)
        w = {  # weights are not read by routing; minimal valid tensors
            "gemm1_weights": torch.empty(E, 4096, 7168, dtype=torch.float8_e4m3fn, device=cuda_device),
            "gemm1_weights_scale": torch.ones(E, 32, 56, device=cuda_device),
            "gemm2_weights": torch.empty(E, 7168, 2048, dtype=torch.float8_e4m3fn, device=cuda_device),
            "gemm2_weights_scale": torch.ones(E, 56, 16, device=cuda_device),
        }
        r = M.route(**d, **w, local_expert_offset=offset, routed_scaling_factor=float(z["rsf"]))
        ids = torch.from_numpy(z["topk_sorted"].astype(np.int64))
        assert torch.equal(r["topk_idx"].cpu().long(), ids)
        torch.testing.assert_close(r["topk_w"].cpu(), torch.from_numpy(z["w_sorted"]), rtol=2e-6, atol=1e-7)
        _check_routing(r, x, T, E, offset, float(z["rsf"]))
        del w
    _status_ok(cuda_device)


def _expect_parity(got, ref, what, max_bad=0):
    rep = O.parity_report(got.cpu(), ref, atol=C.ATOL, rtol=C.RTOL)
    assert rep["nan"] == 0, f"{what}: NaN in output {rep}"
    assert rep["bad"] <= max_bad, f"{what}: {rep}"
    return rep


@pytest.mark.parametrize("path", C.layer_fixtures(), ids=lambda p: p.stem)
def test_layer_matches_reference_golden(cuda_device, path):
    x, g = C.load_layer_case(path, fill_missing_nan=True)   # unrouted experts poisoned
    d = C.to_device(x, cuda_device)
    out = M.run(**d)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    _expect_parity(out, g["official"], "vs reference_official")
    # kernel_pytorch_v1 (bf16-dequantised GEMMs) is itself off the official output on up to
    # ~2% of elements at this tolerance (971 of 57344 in the steered case), so against v1 the
    # bar is: no further from v1 than the official reference is.
    v1_vs_official = O.parity_report(g["v1"], g["official"], atol=C.ATOL, rtol=C.RTOL)["bad"]
    _expect_parity(out, g["v1"], "vs kernel_pytorch_v1", max_bad=int(1.25 * v1_vs_official) + 16)


def _intermediate_check(d, x, device):
    """GEMM1 output c = s*(hi + lo) against the oracle's fp32 SwiGLU rows."""
    T = x["routing_logits"].shape[0]
    E = x["gemm1_weights"].shape[0]
    mid = M.read_intermediate(device, T, E)
    r = M.route(**d)
    tok = r["row_token"].cpu().long()
    A = O.dequant_tokens(x["hidden_states"], x["hidden_states_scale"])
    counts = r["e_count"].cpu().long()
    start = 0
    hi = mid["c_hi"].cpu().view(torch.float8_e4m3fn).float()
    lo = mid["c_lo"].cpu().view(torch.float8_e4m3fn).float()
    sc = mid["c_scale"].cpu()                               # [16, R]
    rec = (hi + lo) * sc.t().repeat_interleave(128, dim=1)
    worst = 0.0
    for e in range(E):
        n = int(counts[e])
        if n == 0:
            continue
        W13 = O.dequant_blocks(x["gemm1_weights"][e], x["gemm1_weights_scale"][e])
        G1 = A[tok[start:start + n]] @ W13.t()
        Cref = G1[:, 2048:] / (1 + torch.exp(-G1[:, 2048:])) * G1[:, :2048]
        err = (rec[start:start + n] - Cref).abs().max() / Cref.abs().max().clamp_min(1e-30)
        worst = max(worst, float(err))
        start += n
    assert worst < 1e-2, f"GEMM1+SwiGLU intermediate relative error {worst}"


@pytest.mark.parametrize("T,seed,offset,skew", [
    (1, 21, 0, 0.0), (16, 22, 0, 0.0), (64, 23, 32, 0.0), (80, 24, 224, 0.0),
    (128, 25, 0, 0.0), (129, 26, 64, 0.0), (257, 27, 0, 0.5)])
def test_layer_matches_oracle(cuda_device, T, seed, offset, skew):
    x = C.make_case(T, seed, offset=offset, skew=skew, fill_missing_nan=True)
    d = C.to_device(x, cuda_device)
    out = M.run(**d)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    _intermediate_check(d, x, cuda_device)
    _expect_parity(out, O.run(**x), f"T={T}")


@pytest.mark.parametrize("T,E,offset", [(33, 8, 64), (40, 64, 128), (24, 256, 0)])
def test_layer_other_expert_counts(cuda_device, T, E, offset):
    """E_local != 32: the expert-parallel shard sizes 256/N (N = 1, 4, 32-expert ranks...)."""
    x = C.make_case(T, 31 + E, E_local=E, offset=offset, fill_missing_nan=True)
    d = C.to_device(x, cuda_device)
    out = M.run(**d)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    _expect_parity(out, O.run(**x), f"T={T} E={E}")


def test_mid_batch_skewed_T901(cuda_device):
    """BASELINE config 2 shape: T=901 with skewed expert load, all 32 local experts."""
    x = C.make_case(901, 41, skew=0.5)
    d = C.to_device(x, cuda_device)
    out = M.run(**d)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    _expect_parity(out, O.run(**x), "T=901 skew")


def test_deterministic_and_no_cross_call_state(cuda_device):
    """Bitwise-identical repeats; a result depends only on its own inputs
    (the reference's input-sensitivity and no-cross-call-state gates, gates.py:385-463)."""
    xa = C.to_device(C.make_case(48, 51), cuda_device)
    xb = C.to_device(C.make_case(48, 52), cuda_device)
    a1 = M.run(**xa).clone()
    b1 = M.run(**xb).clone()
    a2 = M.run(**xa).clone()
    torch.cuda.synchronize()
    assert torch.equal(a1.view(torch.int16), a2.view(torch.int16))
    assert not torch.equal(a1.view(torch.int16), b1.view(torch.int16))
    xc = dict(xa)
    xc["hidden_states"] = (xa["hidden_states"].float() * 0.5).to(torch.float8_e4m3fn)
    c1 = M.run(**xc)
    assert not torch.equal(a1.view(torch.int16), c1.view(torch.int16))
    _status_ok(cuda_device)


def test_tokens_without_local_experts_get_zero_rows(cuda_device):
    x = C.make_case(40, 61, offset=224)
    d = C.to_device(x, cuda_device)
    out = torch.full((40, 7168), 7.0, dtype=torch.bfloat16, device=cuda_device)
    M.run(**d, out=out)
    idx, _ = O.route(x["routing_logits"], x["routing_bias"], 2.5)
    none = ~((idx >= 224) & (idx < 256)).any(dim=1)
    assert none.any()
    assert torch.all(out.cpu()[none] == 0)
    _status_ok(cuda_device)


def test_empty_batch(cuda_device):
    x = C.to_device(C.make_case(3, 71), cuda_device)
    for k in ("routing_logits", "hidden_states"):
        x[k] = x[k][:0].contiguous()
    x["hidden_states_scale"] = x["hidden_states_scale"][:, :0].contiguous()
    out = M.run(**x)
    assert out.shape == (0, 7168)


@pytest.mark.parametrize("T,E,offset", [(200, 8, 0), (600, 8, 16)])
def test_every_token_on_eight_local_experts(cuda_device, T, E, offset):
    """Steered routing puts all 8 picks of every token on local experts, so every output row
    is the expert-ordered combine of 8 partial rows (streaming path at T=200, wide at T=600)."""
    from moe_swarm_b200 import workload as W
    favour = list(range(8))
    x = W.make_steered_activations(T, 81 + T, offset, favour)
    x.update(W.make_weights(E, offset, 81 + T))
    x["local_expert_offset"] = offset
    x["routed_scaling_factor"] = 2.5
    d = C.to_device(x, cuda_device)
    out = M.run(**d)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    _expect_parity(out, O.run(**x), f"T={T} E={E} steered")


def test_wide_path_T1500(cuda_device):
    """T above the streaming threshold with 32 local experts at offset 32."""
    x = C.make_case(1500, 91, offset=32)
    d = C.to_device(x, cuda_device)
    out = M.run(**d)
    torch.cuda.synchronize()
    _status_ok(cuda_device)
    _intermediate_check(d, x, cuda_device)
    _expect_parity(out, O.run(**x), "T=1500")
