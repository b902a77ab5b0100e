"""CPU oracle for the DeepSeek-V3 FP8 block-scale MoE layer -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import it.  The product path (``moe_swarm_b200.run``) runs hand-written
CUDA and raises when its extension is missing; it never routes through here.

It restates, op for op in fp32 PyTorch on the CPU, the reference's semantic
ground truth ``spec/reference_official.py`` (function ``run``), with one
change that does not alter a single bit of the result: weights are
dequantised one routed expert at a time instead of all 32 up front
(the official's ``:80-92``), since the dequantisation is elementwise and the
per-expert GEMM operands are identical.  ``run_v1`` restates the repo's bf16
PyTorch kernel ``reference/kernel_pytorch_v1.py`` (``kernel``, ``:131-192``).

Parity pin: ``tests/golden/make_golden.py`` imports both reference files in a
container that has them and stores their outputs; ``tests/test_oracle.py``
checks this restatement against those fixtures (routing bit-exact, layer
output bit-exact against ``reference_official.run`` and against
``kernel_pytorch_v1.kernel``).
"""

from __future__ import annotations

import torch

H = 7168
I = 2048
E_GLOBAL = 256
TOP_K = 8
N_GROUP = 8
TOPK_GROUP = 4
BLOCK = 128
NHB = H // BLOCK
NIB = I // BLOCK
NG1B = 2 * I // BLOCK


def route(routing_logits: torch.Tensor, routing_bias: torch.Tensor, routed_scaling_factor: float):
    """DeepSeek-V3 no-aux routing (spec/reference_official.py:95-126).

    Returns ``topk_idx`` int64 [T, 8] (global expert ids, unordered as the
    reference's ``topk(sorted=False)``) and the dense combine-weight matrix
    f32 [T, 256] (zero off the selected experts).
    """
    logits = routing_logits.to(torch.float32)
    bias = routing_bias.to(torch.float32).reshape(-1)
    T, E = logits.shape
    s = 1.0 / (1.0 + torch.exp(-logits))                                   # :99
    s_with_bias = s + bias                                                 # :100
    group_size = E // N_GROUP
    grouped = s_with_bias.view(T, N_GROUP, group_size)                     # :104
    top2_vals, _ = torch.topk(grouped, k=2, dim=2, largest=True, sorted=False)  # :107
    group_scores = top2_vals.sum(dim=2)                                    # :108
    _, group_idx = torch.topk(group_scores, k=TOPK_GROUP, dim=1, largest=True, sorted=False)
    group_mask = torch.zeros_like(group_scores)
    group_mask.scatter_(1, group_idx, 1.0)                                 # :111-113
    score_mask = group_mask.unsqueeze(2).expand(T, N_GROUP, group_size).reshape(T, E)
    neg_inf = torch.finfo(torch.float32).min
    scores_pruned = s_with_bias.masked_fill(score_mask == 0, neg_inf)      # :118
    _, topk_idx = torch.topk(scores_pruned, k=TOP_K, dim=1, largest=True, sorted=False)
    M = torch.zeros_like(s)
    M.scatter_(1, topk_idx, 1.0)                                           # :122-123
    weights = s * M
    weights_sum = weights.sum(dim=1, keepdim=True) + 1e-20
    weights = (weights / weights_sum) * routed_scaling_factor              # :124-126
    return topk_idx, weights


def local_permutation(topk_idx: torch.Tensor, weights: torch.Tensor, local_expert_offset: int,
                      E_local: int):
    """(token, local expert, weight) triples in the layer's row order.

    Rows are grouped by ascending local expert and, within an expert, by
    ascending token id -- the stable sort of ``reference/kernel_pytorch_v1.py``
    ``_compact`` (:100-123).  Returns int64 ``row_token``, ``row_expert``,
    f32 ``row_weight`` and int64 ``counts`` [E_local].
    """
    T = topk_idx.shape[0]
    flat_tok = torch.arange(T).unsqueeze(1).expand(T, TOP_K).reshape(-1)
    flat_exp = topk_idx.reshape(-1)
    flat_w = torch.gather(weights, 1, topk_idx).reshape(-1)
    is_local = (flat_exp >= local_expert_offset) & (flat_exp < local_expert_offset + E_local)
    sel = is_local.nonzero(as_tuple=True)[0]
    tok = flat_tok[sel]
    le = flat_exp[sel] - local_expert_offset
    w = flat_w[sel]
    key = le * T + tok                     # expert-major, token-minor: a total order
    perm = torch.argsort(key)
    counts = torch.bincount(le, minlength=E_local)
    return tok[perm], le[perm], w[perm], counts


def dequant_tokens(hidden_states: torch.Tensor, hidden_states_scale: torch.Tensor):
    """A = fp8 * per-(token,128) scale, fp32 [T, H] (spec/reference_official.py:67-78)."""
    T = hidden_states.shape[0]
    A_fp32 = hidden_states.to(torch.float32)
    A_scale_TH = hidden_states_scale.to(torch.float32).permute(1, 0).contiguous()
    expanded = A_scale_TH.unsqueeze(-1).repeat(1, 1, BLOCK).reshape(T, H).contiguous()
    return A_fp32 * expanded


def dequant_blocks(w: torch.Tensor, scale: torch.Tensor):
    """One expert's block-scaled matrix to fp32 (spec/reference_official.py:80-92)."""
    s = torch.repeat_interleave(scale.to(torch.float32), BLOCK, dim=0)
    s = torch.repeat_interleave(s, BLOCK, dim=1)
    return w.to(torch.float32) * s


def expert_forward(A_e: torch.Tensor, W13_e: torch.Tensor, W2_e: torch.Tensor):
    """GEMM1 -> SwiGLU (silu on the SECOND half) -> GEMM2 (reference_official.py:148-162)."""
    G1 = A_e.matmul(W13_e.t())
    X1 = G1[:, :I]
    X2 = G1[:, I:]
    silu_X2 = X2 / (1.0 + torch.exp(-X2))
    C = silu_X2 * X1
    return C.matmul(W2_e.t())


@torch.no_grad()
def _experts_fp32(A, topk_idx, weights, gemm1_weights, gemm1_weights_scale, gemm2_weights,
                  gemm2_weights_scale, local_expert_offset):
    """The official layer after routing (spec/reference_official.py:128-168): each local expert
    in ascending order runs its routed tokens, weighted rows index_add_ed into f32 [T, H]."""
    T = A.shape[0]
    E_local = gemm1_weights.shape[0]
    output = torch.zeros((T, H), dtype=torch.float32)
    local_start = int(local_expert_offset)
    for le in range(E_local):                                              # :134
        ge = local_start + le
        if ge < 0 or ge >= E_GLOBAL:
            continue
        sel = (topk_idx == ge).any(dim=1)
        if not sel.any():
            continue
        token_idx = torch.nonzero(sel, as_tuple=False).squeeze(1)
        W13_e = dequant_blocks(gemm1_weights[le], gemm1_weights_scale[le])
        W2_e = dequant_blocks(gemm2_weights[le], gemm2_weights_scale[le])
        O = expert_forward(A.index_select(0, token_idx), W13_e, W2_e)
        w_tok = weights.index_select(0, token_idx)[:, ge]
        output.index_add_(0, token_idx, O * w_tok.unsqueeze(1))            # :165-166
    return output


def run_fp32(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
             gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
             routed_scaling_factor):
    """The official layer output before the final bf16 cast, f32 [T, H]."""
    A = dequant_tokens(hidden_states, hidden_states_scale)
    topk_idx, weights = route(routing_logits, routing_bias, routed_scaling_factor)
    return _experts_fp32(A, topk_idx, weights, gemm1_weights, gemm1_weights_scale, gemm2_weights,
                         gemm2_weights_scale, local_expert_offset)


def run_routed(topk_idx, topk_w, hidden_states, hidden_states_scale, gemm1_weights, gemm1_weights_scale,
               gemm2_weights, gemm2_weights_scale, local_expert_offset):
    """The official layer with the routing given instead of computed -- token t's experts
    ``topk_idx[t]`` weighted by ``topk_w[t]`` -- i.e. ``run`` from the point its routing is known
    (spec/reference_official.py:128-168); the oracle of the pre-routed entry point.  bf16."""
    T = hidden_states.shape[0]
    A = dequant_tokens(hidden_states, hidden_states_scale)
    idx = topk_idx.long()
    dense = torch.zeros((T, E_GLOBAL), dtype=torch.float32)
    dense.scatter_(1, idx, topk_w.float())
    return _experts_fp32(A, idx, dense, gemm1_weights, gemm1_weights_scale, gemm2_weights,
                         gemm2_weights_scale, local_expert_offset).to(torch.bfloat16)


def run(*args, **kwargs):
    """``spec/reference_official.run`` restated: bf16 [T, 7168]."""
    return run_fp32(*args, **kwargs).to(torch.bfloat16)


@torch.no_grad()
def run_v1(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
           gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
           routed_scaling_factor):
    """``reference/kernel_pytorch_v1.kernel`` restated (bf16 dequantised GEMMs, :131-192)."""
    T = routing_logits.shape[0]
    E_local = gemm1_weights.shape[0]
    logits = routing_logits.to(torch.float32)
    bias = routing_bias.to(torch.float32).reshape(-1)
    s = torch.sigmoid(logits)                                              # v1 :75
    swb = s + bias
    grouped = swb.view(T, N_GROUP, E_GLOBAL // N_GROUP)
    top2 = torch.topk(grouped, k=2, dim=2, largest=True, sorted=False).values
    gidx = torch.topk(top2.sum(dim=2), k=TOPK_GROUP, dim=1, largest=True, sorted=False).indices
    gmask = torch.zeros(T, N_GROUP)
    gmask.scatter_(1, gidx, 1.0)
    keep = gmask.unsqueeze(2).expand(T, N_GROUP, E_GLOBAL // N_GROUP).reshape(T, E_GLOBAL)
    pruned = swb.masked_fill(keep == 0, torch.finfo(torch.float32).min)
    topk_idx = torch.topk(pruned, k=TOP_K, dim=1, largest=True, sorted=False).indices
    mask = torch.zeros_like(s)
    mask.scatter_(1, topk_idx, 1.0)
    weights = s * mask
    weights = weights / (weights.sum(dim=1, keepdim=True) + 1e-20) * routed_scaling_factor

    tok, le, w, counts = local_permutation(topk_idx, weights, int(local_expert_offset), E_local)
    a_scale = hidden_states_scale.to(torch.float32).t().contiguous()
    act = hidden_states.view(T, NHB, BLOCK).to(torch.float32)
    act.mul_(a_scale.unsqueeze(-1))
    act = act.to(torch.bfloat16).view(T, H)
    out = torch.zeros((T, H), dtype=torch.float32)

    def deq(wq, sc):
        m, k = wq.shape
        o = wq.view(m // BLOCK, BLOCK, k // BLOCK, BLOCK).to(torch.float32)
        o.mul_(sc.view(m // BLOCK, 1, k // BLOCK, 1))
        return o.to(torch.bfloat16).view(m, k)

    off = 0
    for e in range(E_local):
        n = int(counts[e])
        if n == 0:
            continue
        tok_e = tok[off:off + n]
        w_e = w[off:off + n]
        off += n
        g1 = act.index_select(0, tok_e) @ deq(gemm1_weights[e], gemm1_weights_scale[e]).t()
        x1, x2 = g1[:, :I], g1[:, I:]
        c = (torch.nn.functional.silu(x2.float()) * x1.float()).to(torch.bfloat16)
        o = c @ deq(gemm2_weights[e], gemm2_weights_scale[e]).t()
        out.index_add_(0, tok_e, o.float() * w_e.unsqueeze(1))
    return out.to(torch.bfloat16)


def parity_report(got: torch.Tensor, ref: torch.Tensor, atol: float = 1e-2, rtol: float = 2e-2):
    """Element counts outside ``|got-ref| <= atol + rtol*|ref|`` plus the max abs error."""
    g = got.float()
    r = ref.float()
    err = (g - r).abs()
    bad = err > (atol + rtol * r.abs())
    return {
        "bad": int(bad.sum()),
        "total": int(r.numel()),
        "max_abs": float(err.max()) if err.numel() else 0.0,
        "nan": int(torch.isnan(g).sum()),
    }
