"""Stable top-k, ties broken by lower index -- drop-in for slotstream_spark/kernels/topk_stable.py.

Same selection and output order as the reference (kernels/topk_stable.py:1-13): order-preserving uint32
keys (NaN lowest), k-th largest key by an 8-bit radix select, ties at that key taken in index order;
k <= 16 sorted by (value desc, index asc), larger k by index asc; rows with fewer than k valid entries
pad with index -1 / value -inf. `n_valid` is read on the device, so the call is CUDA-graph capturable.
"""
import torch

from .. import _lib
from .gemv_affine import _note

MAX_N = 65536


def topk_stable(scores: torch.Tensor, k: int, n_valid: torch.Tensor | None = None,
                out_idx: torch.Tensor | None = None, out_val: torch.Tensor | None = None):
    """scores f32 [R, N] (N <= MAX_N) -> (out_idx int32 [R, k], out_val f32 [R, k] or None)
    (kernels/topk_stable.py:85-113, same argument checks)."""
    if scores.dim() != 2 or scores.dtype != torch.float32 or not scores.is_contiguous():
        raise ValueError("scores must be a contiguous fp32 [R, N] tensor")
    r, n = scores.shape
    if not 1 <= k <= n or n > MAX_N:
        raise ValueError(f"need 1 <= k <= N <= {MAX_N}, got k={k} N={n}")
    if n_valid is not None and (n_valid.dtype != torch.int32 or tuple(n_valid.shape) != (r,)):
        raise ValueError("n_valid must be int32 [R]")
    if out_idx is None:
        out_idx = torch.empty((r, k), dtype=torch.int32, device=scores.device)
    if out_idx.dtype != torch.int32 or tuple(out_idx.shape) != (r, k) or not out_idx.is_contiguous():
        raise ValueError("out_idx must be contiguous int32 [R, k]")
    if out_val is not None and (out_val.dtype != torch.float32 or tuple(out_val.shape) != (r, k)
                                or not out_val.is_contiguous()):
        raise ValueError("out_val must be contiguous fp32 [R, k]")
    rc = _lib.lib().ssb_topk_stable(_lib.ptr(scores), _lib.ptr(n_valid), r, n, k, _lib.ptr(out_idx),
                                    _lib.ptr(out_val), _lib.stream())
    _lib.check(rc, "topk_stable")
    _note("topk_stable")
    return out_idx, out_val
