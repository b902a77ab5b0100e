"""Seeded synthetic inputs for the DeepSeek-V3 FP8 block-scale MoE layer.

The reference scores on the 19 contest workloads of
``spec/workloads.jsonl`` whose routing logits live in safetensors blobs that
are not shipped with it; every other tensor there is ``"random"``.  These
generators stand in for them with the distributions the benchmark configs
name: hidden states N(0,1) quantised to e4m3 with per-token 1x128 fp32 scales
(amax/448), expert weights N(0,0.02) quantised to e4m3 with 128x128 fp32
block scales (amax/448), routing logits N(0,1) (optionally plus a per-expert
N(0,0.5) skew term), routing bias N(0,0.1) in bf16.

Layouts follow ``spec/definition.json:57-145``:

* ``hidden_states``        e4m3  [T, 7168]
* ``hidden_states_scale``  f32   [56, T]            (transposed)
* ``gemm1_weights``        e4m3  [E, 4096, 7168]    (rows 0..2047 = X1, 2048.. = X2)
* ``gemm1_weights_scale``  f32   [E, 32, 56]
* ``gemm2_weights``        e4m3  [E, 7168, 2048]
* ``gemm2_weights_scale``  f32   [E, 56, 16]
* ``routing_logits``       f32   [T, 256]
* ``routing_bias``         bf16  [256]

CPU generation is deterministic for a given seed (torch's CPU Philox/MT
stream), so CPU tests, golden fixtures and GPU parity tests see identical
bytes.  Each expert's weights come from their own generator, so a caller may
materialise only the experts it needs (``experts=...``) and still get the same
bytes for those experts as a full generation.
"""

from __future__ import annotations

import torch

H = 7168
I = 2048
N1 = 2 * I
E_GLOBAL = 256
TOP_K = 8
N_GROUP = 8
TOPK_GROUP = 4
BLOCK = 128
NHB = H // BLOCK    # 56 hidden blocks
NIB = I // BLOCK    # 16 intermediate blocks
NG1B = N1 // BLOCK  # 32 gemm1-output blocks
FP8_MAX = 448.0

FP8 = torch.float8_e4m3fn


def quantize_tokens(x: torch.Tensor):
    """Per-token 1x128 quantisation: x fp32 [T, H] -> (e4m3 [T, H], f32 [H/128, T])."""
    T = x.shape[0]
    xb = x.view(T, NHB, BLOCK)
    amax = xb.abs().amax(dim=2)
    scale = torch.clamp(amax, min=1e-12) / FP8_MAX
    q = (xb / scale.unsqueeze(2)).to(FP8).view(T, H)
    st = torch.empty(NHB, T, dtype=torch.float32, device=x.device)
    st.copy_(scale.t())
    return q, st


def quantize_blocks(w: torch.Tensor):
    """128x128 block quantisation: w fp32 [R, C] -> (e4m3 [R, C], f32 [R/128, C/128])."""
    R, C = w.shape
    wb = w.view(R // BLOCK, BLOCK, C // BLOCK, BLOCK)
    amax = wb.abs().amax(dim=(1, 3))
    scale = torch.clamp(amax, min=1e-12) / FP8_MAX
    q = (wb / scale[:, None, :, None]).to(FP8).view(R, C)
    return q, scale.contiguous()


def _gen(seed: int, stream: int, device="cpu") -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed((int(seed) * 1_000_003 + 7919 * int(stream)) & 0x7FFF_FFFF_FFFF)
    return g


_S_HIDDEN, _S_LOGITS, _S_BIAS, _S_SKEW, _S_EXPERT = 1, 2, 3, 4, 100


def make_activations(T: int, seed: int, skew: float = 0.0, device="cpu"):
    """Routing logits, routing bias and quantised hidden states for one call."""
    hidden = torch.randn(T, H, generator=_gen(seed, _S_HIDDEN), dtype=torch.float32)
    hs, hs_scale = quantize_tokens(hidden)
    logits = torch.randn(T, E_GLOBAL, generator=_gen(seed, _S_LOGITS), dtype=torch.float32)
    if skew:
        per_expert = torch.randn(E_GLOBAL, generator=_gen(seed, _S_SKEW)) * float(skew)
        logits = logits + per_expert.unsqueeze(0)
    bias = (torch.randn(E_GLOBAL, generator=_gen(seed, _S_BIAS)) * 0.1).to(torch.bfloat16)
    return {
        "routing_logits": logits.to(device),
        "routing_bias": bias.to(device),
        "hidden_states": hs.to(device),
        "hidden_states_scale": hs_scale.to(device),
    }


def make_expert(seed: int, global_expert: int):
    """One expert's (W13 e4m3, S13, W2 e4m3, S2) on the CPU, deterministic per expert id."""
    g = _gen(seed, _S_EXPERT + int(global_expert))
    w13 = torch.randn(N1, H, generator=g, dtype=torch.float32) * 0.02
    q13, s13 = quantize_blocks(w13)
    del w13
    w2 = torch.randn(H, I, generator=g, dtype=torch.float32) * 0.02
    q2, s2 = quantize_blocks(w2)
    return q13, s13, q2, s2


def make_weights(E_local: int, offset: int, seed: int, experts=None, device="cpu",
                 fill_missing_nan: bool = False):
    """Stacked weights for local experts [offset, offset+E_local).

    ``experts`` (iterable of local indices) restricts generation to those
    experts; the others are zero (or e4m3 NaN with ``fill_missing_nan`` so a
    kernel that reads an expert routing never selected poisons its output).
    """
    dev = torch.device(device)
    q13 = torch.empty(E_local, N1, H, dtype=torch.uint8, device=dev)
    q2 = torch.empty(E_local, H, I, dtype=torch.uint8, device=dev)
    s13 = torch.ones(E_local, NG1B, NHB, dtype=torch.float32, device=dev)
    s2 = torch.ones(E_local, NHB, NIB, dtype=torch.float32, device=dev)
    want = set(range(E_local)) if experts is None else {int(e) for e in experts}
    filler = 0x7F if fill_missing_nan else 0
    for le in range(E_local):
        if le not in want:
            q13[le].fill_(filler)
            q2[le].fill_(filler)
            continue
        a, sa, b, sb = make_expert(seed, offset + le)
        q13[le].copy_(a.view(torch.uint8))
        s13[le].copy_(sa)
        q2[le].copy_(b.view(torch.uint8))
        s2[le].copy_(sb)
    return {
        "gemm1_weights": q13.view(FP8),
        "gemm1_weights_scale": s13,
        "gemm2_weights": q2.view(FP8),
        "gemm2_weights_scale": s2,
    }


def make_weights_fast(E_local: int, seed: int, device="cuda"):
    """Large weight sets generated on the device (benchmarks only; not CPU-reproducible)."""
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(int(seed) + 12345)
    q13 = torch.empty(E_local, N1, H, dtype=FP8, device=dev)
    q2 = torch.empty(E_local, H, I, dtype=FP8, device=dev)
    s13 = torch.empty(E_local, NG1B, NHB, dtype=torch.float32, device=dev)
    s2 = torch.empty(E_local, NHB, NIB, dtype=torch.float32, device=dev)
    for le in range(E_local):
        w = torch.randn(N1, H, generator=g, device=dev, dtype=torch.float32) * 0.02
        a, sa = quantize_blocks(w)
        q13[le].copy_(a)
        s13[le].copy_(sa)
        w = torch.randn(H, I, generator=g, device=dev, dtype=torch.float32) * 0.02
        a, sa = quantize_blocks(w)
        q2[le].copy_(a)
        s2[le].copy_(sa)
        del w, a, sa
    return {
        "gemm1_weights": q13,
        "gemm1_weights_scale": s13,
        "gemm2_weights": q2,
        "gemm2_weights_scale": s2,
    }


def make_steered_activations(T: int, seed: int, offset: int, favour, device="cpu"):
    """Known-answer routing: logits -5 except a descending ramp 10 - 0.1*rank on the
    ``favour`` local experts, zero bias, so every token selects exactly those experts
    (the steered inputs of the reference's dynamic gates, ``gates.py:164-189``)."""
    logits = torch.full((T, E_GLOBAL), -5.0, dtype=torch.float32)
    for rank, e in enumerate(favour):
        logits[:, offset + int(e)] = 10.0 - 0.1 * rank
    hidden = torch.randn(T, H, generator=_gen(seed, _S_HIDDEN), dtype=torch.float32)
    hs, hs_scale = quantize_tokens(hidden)
    return {
        "routing_logits": logits.to(device),
        "routing_bias": torch.zeros(E_GLOBAL, dtype=torch.bfloat16, device=device),
        "hidden_states": hs.to(device),
        "hidden_states_scale": hs_scale.to(device),
    }


def make_inputs(T: int, seed: int = 0, E_local: int = 32, offset: int = 0, skew: float = 0.0,
                rsf: float = 2.5, experts=None, device="cpu", fill_missing_nan=False):
    """Full argument dict for ``run(**inputs)`` (CPU-deterministic)."""
    d = make_activations(T, seed, skew=skew, device=device)
    d.update(make_weights(E_local, offset, seed, experts=experts, device=device,
                          fill_missing_nan=fill_missing_nan))
    d["local_expert_offset"] = int(offset)
    d["routed_scaling_factor"] = float(rsf)
    return d
