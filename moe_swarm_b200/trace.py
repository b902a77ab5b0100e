"""Per-CTA role counters of the traced build, for one layer call.

    python -m moe_swarm_b200.build --trace
    MOE_B200_LIB=moe_swarm_b200/libmoe_b200_trace.so python -m moe_swarm_b200.trace 4096:256 16:32 901:32:0.5

Each argument is T:E_local[:logit skew].  The inputs are the seeded activations of
``moe_swarm_b200.workload`` (seed 5) and device-generated weights, local experts at offset 0.
The call runs a few times after a 256 MB L2 flush each; the last call runs with the trace region
of the workspace cleared, and one JSON line per case gives, per kernel that ran:

* ``start_us`` / ``end_us_min`` / ``end_us_max``: CTA start and end times relative to the first
  recorded CTA start of the call (``globaltimer``; CTAs beyond the first 256 are not recorded);
* GEMM kernels: per K-block medians over CTAs of the role counters (``clock64`` cycles):
  producer wait for a free stage, MMA wait for data and for a free TMEM accumulator, MMA issue,
  promotion wait and work, tile epilogue, stream-K fixup, scale staging; ``ns_per_kb`` (span per
  K-block) and, for the wide kernels, the SM clock the span ran at;
* routing: the phase times of the first token (``rt_marks_us``: start, after the sigmoid, after
  the group ranking, after the top-8, end) and the routing CTA's phase marks;
* wide GEMMs (``wide_g1_timeline`` / ``wide_g2_timeline``): the accumulator handoff of CTA 0 per
  K-block, medians over its K-blocks after the first 20 (cycles): the period, the MMA thread's
  wait for a free accumulator and for its operand stage, its issue of the MMAs and commits, the
  commit -> first promotion warp seeing the accumulator, the promotion until the last warp
  releases it, and each promotion warp's release relative to the first promotion warp's
  (``release_vs_w4``, median and 90th percentile, warps 4..11).

Kernel order of the trace region: stream GEMM1, stream GEMM2, wide GEMM1, wide GEMM2, routing,
scatter, GEMM1 finalize, combine, then the two wide-GEMM timelines (``moe_internal.cuh``,
``kTraceKernels``).
"""

from __future__ import annotations

import json
import sys

import torch

from . import _native as N
from . import run, workload as W
from . import _workspace, device_status

NAMES = ["stream_g1", "stream_g2", "wide_g1", "wide_g2", "route", "scatter", "fin1", "combine"]
SLOTS, CTAS = 16, 256
TL_BLOCKS, TL_KBS, TL_ROWS = 2, 256, 12   # wide GEMM1 / GEMM2 timelines: [row][K-block] stamps


def timeline(tl: torch.Tensor) -> dict | None:
    """Handoff medians of one wide-GEMM timeline ([TL_ROWS][TL_KBS] clock64 stamps, 0 = none)."""
    n = int((tl[2] != 0).sum())
    if n < 40:
        return None
    t = tl[:, 20:n].double()
    t = t[:, (t != 0).all(dim=0)]
    if t.shape[1] < 10:
        return None
    med = lambda x: round(x.median().item(), 1)
    last_rel = t[4:12].max(dim=0).values
    rel = t[4:12] - t[4]
    return {
        "kbs": int(t.shape[1]),
        "period": med(t[2, 1:] - t[2, :-1]),
        "mma_wait_acc": med(t[0, 1:] - t[2, :-1]),
        "mma_wait_stage": med(t[1] - t[0]),
        "mma_issue": med(t[2] - t[1]),
        "commit_to_promotion": med(t[3] - t[2]),
        "promotion_to_last_release": med(last_rel - t[3]),
        "release_vs_w4": [med(rel[w]) for w in range(8)],
        "release_vs_w4_p90": [round(rel[w].quantile(0.9).item(), 1) for w in range(8)],
    }


def run_case(T: int, E: int, skew: float = 0.0, seed: int = 5, calls: int = 4) -> dict:
    dev = torch.device("cuda", 0)
    x = {k: v.to(dev) for k, v in W.make_activations(T, seed, skew=skew).items()}
    x.update(W.make_weights_fast(E, 1, device=dev))
    x["local_expert_offset"] = 0
    x["routed_scaling_factor"] = 2.5
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    L = N.layout(T, E)
    n = (len(NAMES) + TL_BLOCKS) * CTAS * SLOTS * 8
    for i in range(calls):
        flush.zero_()
        if i == calls - 1:
            torch.cuda.synchronize()
            _workspace(dev).buf[L.trace:L.trace + n].zero_()
        run(**x)
    torch.cuda.synchronize()
    allt = _workspace(dev).buf[L.trace:L.trace + n].view(torch.int64).cpu()
    tr = allt[:len(NAMES) * CTAS * SLOTS].view(len(NAMES), CTAS, SLOTS)
    tls = allt[len(NAMES) * CTAS * SLOTS:].view(TL_BLOCKS, CTAS * SLOTS)[:, :TL_ROWS * TL_KBS]
    res = {"T": T, "E": E, "skew": skew, "status": device_status(dev)}
    for b, nm in enumerate(("wide_g1_timeline", "wide_g2_timeline")):
        d = timeline(tls[b].view(TL_ROWS, TL_KBS))
        if d:
            res[nm] = d
    live_any = [tr[k][tr[k][:, 0] != 0] for k in range(len(NAMES))]
    t0 = min(int(r[:, 0].min()) for r in live_any if len(r))
    for k, r in enumerate(live_any):
        if not len(r):
            continue
        r = r.double()
        d = {"ctas": len(r), "start_us": round((r[:, 0].min().item() - t0) / 1e3, 1),
             "end_us_min": round((r[:, 1].min().item() - t0) / 1e3, 1),
             "end_us_max": round((r[:, 1].max().item() - t0) / 1e3, 1)}
        if k < 4:
            kb = r[:, 3].clamp_min(1)
            for i, nm in ((2, "prod_wait"), (4, "mma_wait_full"), (5, "mma_wait_tmem"), (6, "epi_wait"),
                          (7, "promo"), (8, "tile_epi"), (9, "fixup"), (10, "staging")):
                d[nm + "_per_kb"] = round((r[:, i] / kb).median().item(), 1)
            d["kb_median"] = int(r[:, 3].median().item())
            d["first_data_us"] = round((r[:, 11].median().item() - t0) / 1e3, 1)
            span = (r[:, 1] - r[:, 0]).median().item()
            d["ns_per_kb"] = round(span / max(1.0, r[:, 3].median().item()), 1)
            if k >= 2:
                d["mma_issue_per_kb"] = round((r[:, 14] / kb).median().item(), 1)
                d["sm_mhz"] = round(((r[:, 13] - r[:, 12]) / (r[:, 1] - r[:, 0]).clamp_min(1)).median().item() * 1e3, 1)
        elif k == 4:
            d["rt_marks_us"] = [round((r[0, i].item() - t0) / 1e3, 2) for i in range(6, 11)]
        res[NAMES[k]] = d
    return res


def main(argv=None):
    for spec in (argv if argv is not None else sys.argv[1:]):
        parts = spec.split(":")
        print(json.dumps(run_case(int(parts[0]), int(parts[1]), float(parts[2]) if len(parts) > 2 else 0.0)),
              flush=True)


if __name__ == "__main__":
    main()
