"""Grouped affine 4-bit MoE for prefill -- drop-in for slotstream_spark/kernels/fused_moe_affine.py.

This module currently carries the rank-order combine; the grouped GEMM entry points follow.
"""
import torch

from .. import _lib
from ..records import BASELINE_LAYOUT
from .gemv_affine import _note

HID, INTER, TOPK = BASELINE_LAYOUT.hidden, BASELINE_LAYOUT.inter, 10
RECORD_BYTES = BASELINE_LAYOUT.record_bytes
(O_GATE_W, O_GATE_S, O_GATE_B, O_UP_W, O_UP_S, O_UP_B, O_DOWN_W, O_DOWN_S, O_DOWN_B) = BASELINE_LAYOUT.offsets()
GROUP_MAX = 32


def combine_rank_order(out_rows, T, K=TOPK, out=None):
    """out_rows fp32 [T*K, H], row = token*K + rank -> fp32 [T, H], summed in router rank order (sequential
    fp32), bit-equal to kernels/fused_moe_affine.py:164-172."""
    if out_rows.shape[0] != T * K:
        raise ValueError("out_rows must have T*K rows")
    if out_rows.dtype != torch.float32 or out_rows.dim() != 2 or not out_rows.is_contiguous():
        raise ValueError("out_rows must be a contiguous fp32 [T*K, H] tensor")
    h = out_rows.shape[1]
    if out is None:
        out = torch.empty((T, h), dtype=torch.float32, device=out_rows.device)
    rc = _lib.lib().ssb_combine_rank_order(_lib.ptr(out_rows), T, K, h, _lib.ptr(out), _lib.stream())
    _lib.check(rc, "combine_rank_order")
    _note("combine_rank_order")
    return out
