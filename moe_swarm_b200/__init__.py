"""B200-native (sm_100a) DeepSeek-V3 FP8 block-scale fused-MoE layer.

``run(...)`` (alias ``kernel``) is a drop-in for the reference's entry point of the
``moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048`` definition
(``spec/reference_official.py:5-16`` ``run``; ``solution/python/kernel.py:1448-1459``
``kernel``): the same ten arguments in the same layouts, a freshly allocated bf16
``[T, 7168]`` result, no host synchronisation.  All arithmetic runs in the
hand-written CUDA of ``libmoe_b200.so`` (``include/moe_b200.h``); when that library
is missing the call raises -- there is no CPU or PyTorch fallback.

Shape/dtype violations raise :class:`MoEArgumentError`, which is an
``AssertionError`` like the reference's own ``assert`` checks
(``spec/reference_official.py:43-58``).
"""

from __future__ import annotations

import ctypes
import threading

import torch

from . import _native

H = 7168
I = 2048
E_GLOBAL = 256
NHB = H // 128
NIB = I // 128
NG1B = 2 * I // 128

__all__ = ["run", "kernel", "run_routed", "route", "device_status", "MoEArgumentError", "Workspace",
           "GraphRunner"]


class MoEArgumentError(AssertionError, ValueError):
    """An input violates the layer definition (spec/definition.json)."""


def _check(cond: bool, msg: str):
    if not cond:
        raise MoEArgumentError(msg)


class Workspace:
    """Scratch of one (device, stream) reused across calls (never results: every call recomputes).

    Grows to the largest (T, E_local) seen; the self-resetting counters are zeroed
    whenever the layout changes.
    """

    def __init__(self, device: torch.device):
        self.device = device
        self.buf = None
        self.key = None

    def get(self, T: int, E: int, stream_ptr: int):
        need = int(_native.lib().moe_b200_workspace_size(T, E))
        if need == 0:
            raise MoEArgumentError(f"unsupported sizes T={T}, E_local={E}")
        if self.buf is None or self.buf.numel() < need:
            self.buf = None
            self.buf = torch.empty(need + (need >> 3), dtype=torch.uint8, device=self.device)
            self.key = None
        if self.key != (T, E):
            rc = _native.lib().moe_b200_workspace_init(self.buf.data_ptr(), self.buf.numel(), T, E,
                                                       stream_ptr)
            if rc != _native.OK:
                raise RuntimeError(f"moe_b200_workspace_init failed ({rc}): {_native.last_error()}")
            self.key = (T, E)
        return self.buf


_ws_lock = threading.Lock()
_workspaces: dict[tuple[int, int], Workspace] = {}


def _workspace(device: torch.device, stream: int | None = None) -> Workspace:
    """The workspace of (device, stream).  Calls on one stream run one after another on the GPU
    and may share scratch; calls on two streams may overlap on the GPU, so each stream gets its
    own (a shared one would let them race on the same counters and permuted rows).  ``stream`` is
    the raw ``cudaStream_t`` value; None means the device's current stream."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if stream is None:
        stream = torch.cuda.current_stream(torch.device("cuda", idx)).cuda_stream
    key = (idx, int(stream))
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None:
            ws = _workspaces[key] = Workspace(torch.device("cuda", idx))
        return ws


def _validate(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
              gemm1_weights_scale, gemm2_weights, gemm2_weights_scale):
    T = routing_logits.shape[0]
    _check(routing_logits.dim() == 2 and routing_logits.shape[1] == E_GLOBAL,
           "num_experts must be 256")
    E = gemm1_weights.shape[0]
    _check(1 <= E <= E_GLOBAL, "num_local_experts must be in [1, 256]")
    _check(tuple(hidden_states.shape) == (T, H), "hidden_size must be 7168")
    _check(tuple(hidden_states_scale.shape) == (NHB, T), "hidden_states_scale must be [56, T]")
    _check(tuple(gemm1_weights.shape) == (E, 2 * I, H), "gemm1_weights must be [E, 4096, 7168]")
    _check(tuple(gemm1_weights_scale.shape) == (E, NG1B, NHB), "gemm1_weights_scale must be [E, 32, 56]")
    _check(tuple(gemm2_weights.shape) == (E, H, I), "gemm2_weights must be [E, 7168, 2048]")
    _check(tuple(gemm2_weights_scale.shape) == (E, NHB, NIB), "gemm2_weights_scale must be [E, 56, 16]")
    _check(routing_bias.numel() == E_GLOBAL, "routing_bias must hold 256 values")
    _check(routing_logits.dtype == torch.float32, "routing_logits must be float32")
    _check(routing_bias.dtype == torch.bfloat16, "routing_bias must be bfloat16")
    for name, t in (("hidden_states", hidden_states), ("gemm1_weights", gemm1_weights),
                    ("gemm2_weights", gemm2_weights)):
        _check(t.dtype in (torch.float8_e4m3fn, torch.uint8), f"{name} must be float8_e4m3fn")
    for name, t in (("hidden_states_scale", hidden_states_scale),
                    ("gemm1_weights_scale", gemm1_weights_scale),
                    ("gemm2_weights_scale", gemm2_weights_scale)):
        _check(t.dtype == torch.float32, f"{name} must be float32")
    tensors = (routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
               gemm1_weights_scale, gemm2_weights, gemm2_weights_scale)
    dev = hidden_states.device
    for t in tensors:
        _check(t.is_cuda, "all tensors must be CUDA tensors (there is no CPU path)")
        _check(t.device == dev, "all tensors must be on one device")
        _check(t.is_contiguous(), "all tensors must be contiguous")
    return T, E, dev


def _args(T, E, routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
          gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
          routed_scaling_factor, out):
    return _native.MoeArgs(
        routing_logits.data_ptr(), routing_bias.data_ptr(), hidden_states.data_ptr(),
        hidden_states_scale.data_ptr(), gemm1_weights.data_ptr(), gemm1_weights_scale.data_ptr(),
        gemm2_weights.data_ptr(), gemm2_weights_scale.data_ptr(), out.data_ptr(), int(T), int(E),
        int(local_expert_offset), float(routed_scaling_factor))


@torch.no_grad()
def run(routing_logits: torch.Tensor, routing_bias: torch.Tensor, hidden_states: torch.Tensor,
        hidden_states_scale: torch.Tensor, gemm1_weights: torch.Tensor,
        gemm1_weights_scale: torch.Tensor, gemm2_weights: torch.Tensor,
        gemm2_weights_scale: torch.Tensor, local_expert_offset: int, routed_scaling_factor: float,
        *, out: torch.Tensor | None = None) -> torch.Tensor:
    """One DeepSeek-V3 FP8 block-scale MoE layer call; returns bf16 ``[T, 7168]``.

    Layouts: ``spec/definition.json:57-145``.  Only local experts
    ``[local_expert_offset, local_expert_offset + E_local)`` are computed; the result is
    this rank's partial sum (``reference/kernel_pytorch_v1.py:126-130``).
    ``out`` (optional, bf16 ``[T, 7168]``) receives the result instead of a new tensor.

    The call is enqueued on the current CUDA stream without a host synchronisation.  Its scratch
    is a workspace kept per (device, stream): calls on different streams of one device may run
    concurrently on the GPU, each with its own scratch.  Calls on one stream from several host
    threads share that stream's workspace, which is safe because the GPU runs them in stream order.
    """
    T, E, dev = _validate(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                          gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale)
    if out is None:
        out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    else:
        _check(out.dtype == torch.bfloat16 and tuple(out.shape) == (T, H) and out.is_contiguous()
               and out.device == dev, "out must be a contiguous bf16 [T, 7168] tensor on the device")
    if T == 0:
        return out
    stream = torch.cuda.current_stream(dev).cuda_stream
    buf = _workspace(dev, stream).get(T, E, stream)
    a = _args(T, E, routing_logits, routing_bias, hidden_states, hidden_states_scale,
              gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
              local_expert_offset, routed_scaling_factor, out)
    rc = _native.lib().moe_b200_forward(ctypes.byref(a), buf.data_ptr(), buf.numel(), stream)
    if rc != _native.OK:
        raise RuntimeError(f"moe_b200_forward failed ({rc}): {_native.last_error()}")
    return out


kernel = run


@torch.no_grad()
def run_routed(topk_idx: torch.Tensor, topk_w: torch.Tensor, hidden_states: torch.Tensor,
               hidden_states_scale: torch.Tensor, gemm1_weights: torch.Tensor,
               gemm1_weights_scale: torch.Tensor, gemm2_weights: torch.Tensor,
               gemm2_weights_scale: torch.Tensor, local_expert_offset: int, *,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """The layer with the routing given instead of computed: token t's experts are
    ``topk_idx[t]`` (int32 ``[T, 8]`` global ids, distinct per token) weighted by ``topk_w[t]``
    (float32 ``[T, 8]``, routed scaling factor already applied).  Only the local experts
    ``[local_expert_offset, local_expert_offset + E_local)`` contribute; returns bf16 ``[T, 7168]``.
    Used by token-dispatch expert parallelism (``ep.ExpertParallelMoE.forward_dispatch``)."""
    T = hidden_states.shape[0]
    dummy_logits = torch.empty((T, E_GLOBAL), dtype=torch.float32, device=hidden_states.device)
    dummy_bias = torch.empty(E_GLOBAL, dtype=torch.bfloat16, device=hidden_states.device)
    T, E, dev = _validate(dummy_logits, dummy_bias, hidden_states, hidden_states_scale, gemm1_weights,
                          gemm1_weights_scale, gemm2_weights, gemm2_weights_scale)
    _check(tuple(topk_idx.shape) == (T, 8) and topk_idx.dtype == torch.int32 and topk_idx.is_contiguous()
           and topk_idx.device == dev, "topk_idx must be a contiguous int32 [T, 8] tensor on the device")
    _check(tuple(topk_w.shape) == (T, 8) and topk_w.dtype == torch.float32 and topk_w.is_contiguous()
           and topk_w.device == dev, "topk_w must be a contiguous float32 [T, 8] tensor on the device")
    if out is None:
        out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    else:
        _check(out.dtype == torch.bfloat16 and tuple(out.shape) == (T, H) and out.is_contiguous()
               and out.device == dev, "out must be a contiguous bf16 [T, 7168] tensor on the device")
    if T == 0:
        return out
    stream = torch.cuda.current_stream(dev).cuda_stream
    buf = _workspace(dev, stream).get(T, E, stream)
    a = _args(T, E, dummy_logits, dummy_bias, hidden_states, hidden_states_scale, gemm1_weights,
              gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset, 1.0, out)
    a.routing_logits = None
    a.routing_bias = None
    rc = _native.lib().moe_b200_forward_routed(ctypes.byref(a), topk_idx.data_ptr(), topk_w.data_ptr(),
                                               buf.data_ptr(), buf.numel(), stream)
    if rc != _native.OK:
        raise RuntimeError(f"moe_b200_forward_routed failed ({rc}): {_native.last_error()}")
    return out


class GraphRunner:
    """One layer call captured in a CUDA graph, for callers that replay a fixed shape (decode
    steps at a given batch size; the reference replays graphs the same way,
    solution/python/kernel.py:1068-1089).

    The arguments are those of :func:`run`; their tensors become the graph's static inputs (new
    values are copied into them before :meth:`replay`).  The runner owns its workspace and its
    output tensor, so later calls of :func:`run` with other sizes cannot move memory the graph
    points at.  The first, eager call outside the graph sets up the tensor maps, the kernels'
    attributes and the workspace's counters; the captured launches keep their programmatic
    dependent-launch edges.
    """

    def __init__(self, routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                 gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
                 routed_scaling_factor):
        T, E, dev = _validate(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                              gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale)
        _check(T > 0, "an empty batch needs no graph")
        self.inputs = dict(routing_logits=routing_logits, routing_bias=routing_bias,
                           hidden_states=hidden_states, hidden_states_scale=hidden_states_scale)
        self.out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        n = int(_native.lib().moe_b200_workspace_size(T, E))
        self.workspace = torch.zeros(n, dtype=torch.uint8, device=dev)   # zeroed = initialised
        self._a = _args(T, E, routing_logits, routing_bias, hidden_states, hidden_states_scale,
                        gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                        local_expert_offset, routed_scaling_factor, self.out)
        self._keep = (gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale)
        self._launch(torch.cuda.current_stream(dev).cuda_stream)     # eager set-up call
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._launch(torch.cuda.current_stream(dev).cuda_stream)

    def _launch(self, stream):
        rc = _native.lib().moe_b200_forward(ctypes.byref(self._a), self.workspace.data_ptr(),
                                            self.workspace.numel(), stream)
        if rc != _native.OK:
            raise RuntimeError(f"moe_b200_forward failed ({rc}): {_native.last_error()}")

    def replay(self) -> torch.Tensor:
        """Runs the captured call on the current values of the static inputs; returns the
        runner's output tensor (overwritten by the next replay)."""
        self.graph.replay()
        return self.out


@torch.no_grad()
def route(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
          gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
          routed_scaling_factor, *, out=None):
    """Runs routing + permutation only and returns its device results (for tests/tools):
    topk_idx [T,8] i32 (ascending), topk_w [T,8], tok_nloc [T], tok_rows [T,8],
    e_count [E], e_start [E+1], row_token [R], row_weight [R], plan [16]."""
    T, E, dev = _validate(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                          gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale)
    if out is None:
        out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    buf = _workspace(dev, stream).get(T, E, stream)
    a = _args(T, E, routing_logits, routing_bias, hidden_states, hidden_states_scale,
              gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
              local_expert_offset, routed_scaling_factor, out)
    rc = _native.lib().moe_b200_route(ctypes.byref(a), buf.data_ptr(), buf.numel(), stream)
    if rc != _native.OK:
        raise RuntimeError(f"moe_b200_route failed ({rc}): {_native.last_error()}")
    return read_routing(buf, T, E)


def read_routing(buf: torch.Tensor, T: int, E: int) -> dict:
    """Views of the routing results inside a workspace buffer (copies, on the device)."""
    L = _native.layout(T, E)

    def view(off, n, dtype):
        nbytes = n * torch.empty((), dtype=dtype).element_size()
        return buf[off:off + nbytes].view(dtype).clone()

    plan = view(L.plan, 16, torch.int32)
    R = int(plan[2].item())
    return {
        "plan": plan,
        "topk_idx": view(L.topk_idx, T * 8, torch.int32).view(T, 8),
        "topk_w": view(L.topk_w, T * 8, torch.float32).view(T, 8),
        "tok_nloc": view(L.tok_nloc, T, torch.int32),
        "tok_rows": view(L.tok_rows, T * 8, torch.int32).view(T, 8),
        "e_count": view(L.e_count, E, torch.int32),
        "e_start": view(L.e_start, E + 1, torch.int32),
        "row_token": view(L.row_token, R, torch.int32),
        "row_weight": view(L.row_weight, R, torch.float32),
    }


def read_intermediate(device, T: int, E: int) -> dict:
    """The GEMM1 output (hi/lo e4m3 pair and scales) left in the device's workspace by
    the last call with these sizes: c_hi/c_lo uint8 [R, 2048], c_scale f32 [16, R]."""
    buf = _workspace(torch.device(device)).buf   # the current stream's workspace
    L = _native.layout(T, E)
    plan = buf[L.plan:L.plan + 64].view(torch.int32)
    R = int(plan[2].item())
    c_hi = buf[L.c_hi:L.c_hi + R * I].view(R, I).clone()
    c_lo = buf[L.c_lo:L.c_lo + R * I].view(R, I).clone()
    sc = buf[L.c_scale:L.c_scale + 16 * L.r_pad * 4].view(torch.float32).view(16, L.r_pad)[:, :R].clone()
    return {"c_hi": c_hi, "c_lo": c_lo, "c_scale": sc}


def device_status(device=None, T: int | None = None, E: int | None = None, clear: bool = True) -> int:
    """Synchronises and returns the device status word of the device's workspace
    (0 = ok; otherwise the code of a bounded device-side wait that gave up)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    ws = _workspace(dev)   # the current stream's workspace
    if ws.buf is None:
        return 0
    T0, E0 = ws.key if T is None else (T, E)
    stream = torch.cuda.current_stream(dev).cuda_stream
    return int(_native.lib().moe_b200_device_status(ws.buf.data_ptr(), ws.buf.numel(), T0, E0, stream,
                                                    1 if clear else 0))
