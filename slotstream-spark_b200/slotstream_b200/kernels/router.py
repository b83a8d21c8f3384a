"""Fused router (additive API): logits, fp32 softmax, stable top-k and renormalise in two sm_100a launches.

Replaces the glue of model/layers.py:336-348 (``lin`` -> ``F.softmax(float)`` -> ``topk_stable`` ->
``tv / tv.sum()``) for callers that opt in; ``topk_stable`` itself stays available unchanged. Logits are an
fp32 sum of exact bf16 products ("router math is fp32"); ``logits_round_bf16=True`` rounds them to bf16
first, as ``lin`` does when it returns the bf16 input dtype (model/layers.py:72-75). ``bias`` (fp32 [E])
is added to the logits before the softmax. When ``sh_gate_w`` (bf16 [H] or [1, H]) is given, the same
launch also produces the shared-expert gate sigmoid(x . sh_gate_w) (model/layers.py:401).
"""
import torch

from .. import _lib
from .gemv_affine import _note


def router_topk(x, w_router, k: int, out_idx=None, out_w=None, *, logits_round_bf16: bool = False, bias=None,
                sh_gate_w=None, out_sh_gate=None, out_probs=None, ws=None):
    """x bf16 [T, H] · w_router bf16 [E, H] -> (ids int32 [T, k], weights fp32 [T, k]).
    ``ws`` (fp32, >= T * (E + 1) elements) holds the logits so nothing is allocated under graph capture."""
    if x.dim() != 2 or x.dtype != torch.bfloat16 or not x.is_contiguous():
        raise ValueError("x must be a contiguous bf16 [T, H] tensor")
    t, h = x.shape
    if w_router.dim() != 2 or w_router.dtype != torch.bfloat16 or w_router.shape[1] != h \
            or not w_router.is_contiguous():
        raise ValueError("w_router must be a contiguous bf16 [E, H] tensor")
    e = w_router.shape[0]
    if not 1 <= k <= min(e, 32):
        raise ValueError(f"need 1 <= k <= min(E, 32), got k={k}")
    ld = e + (1 if sh_gate_w is not None else 0)
    dev = x.device
    if out_idx is None:
        out_idx = torch.empty((t, k), dtype=torch.int32, device=dev)
    if out_w is None:
        out_w = torch.empty((t, k), dtype=torch.float32, device=dev)
    for o, dt, name in ((out_idx, torch.int32, "out_idx"), (out_w, torch.float32, "out_w")):
        if tuple(o.shape) != (t, k) or o.dtype != dt or not o.is_contiguous():
            raise ValueError(f"{name} must be contiguous {dt} [T, k]")
    if bias is not None and (bias.dtype != torch.float32 or bias.numel() != e):
        raise ValueError("bias must be fp32 [E]")
    if sh_gate_w is not None:
        if sh_gate_w.dtype != torch.bfloat16 or sh_gate_w.numel() != h:
            raise ValueError("sh_gate_w must be bf16 [H]")
        if out_sh_gate is None:
            out_sh_gate = torch.empty(t, dtype=torch.float32, device=dev)
    if out_probs is not None and (tuple(out_probs.shape) != (t, e) or out_probs.dtype != torch.float32):
        raise ValueError("out_probs must be fp32 [T, E]")
    if ws is None:
        ws = torch.empty(t * ld, dtype=torch.float32, device=dev)
    elif ws.dtype != torch.float32 or ws.numel() < t * ld:
        raise ValueError("ws too small")
    L = _lib.lib()
    rc = L.ssb_router_logits(_lib.ptr(x), _lib.ptr(w_router), _lib.ptr(sh_gate_w), t, h, e, ld, _lib.ptr(ws),
                             _lib.stream())
    _lib.check(rc, "router_logits")
    flags = (_lib.ROUTER_ROUND_BF16 if logits_round_bf16 else 0) | (_lib.ROUTER_SHARED_GATE if sh_gate_w is not None else 0)
    rc = L.ssb_router_select(_lib.ptr(ws), ld, t, e, k, _lib.ptr(bias), flags, _lib.ptr(out_idx), _lib.ptr(out_w),
                             _lib.ptr(out_probs), _lib.ptr(out_sh_gate), _lib.stream())
    _lib.check(rc, "router_select")
    _note("router_logits")
    _note("router_select")
    if sh_gate_w is not None:
        return out_idx, out_w, out_sh_gate
    return out_idx, out_w
