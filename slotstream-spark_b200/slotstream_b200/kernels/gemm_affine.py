"""Tensor-core GEMM for the dense prefill rows -- drop-in for slotstream_spark/kernels/gemm_affine.py.

y[m, n] = sum_k x[m, k] * w[n, k], fp32 accumulate (kernels/gemm_affine.py:1-8). The affine 4-bit weight is
dequantised as q*s + b in fp32, rounded to bf16 once, and fed to tcgen05 MMAs (256-row tiles of two M128 N128
halves) with the accumulator in TMEM; a bf16 ``DenseWeight`` goes to the same tensor-core kernel with its rows
copied straight into the operand tiles. Any N (the last 128-column block is partial). Tiles and the k order depend
only on (n, k), never on M, so each output row depends only on its own x row: rows i..j of an M-row call equal a
(j - i)-row call bit for bit.
"""
import torch

from .. import _lib
from .gemv_affine import AffineWeight, DenseWeight, _note

STATS = {"calls": 0, "rows": 0}


def gemm(x: torch.Tensor, w, out: torch.Tensor | None = None, cfg: dict | None = None) -> torch.Tensor:
    """x [M, K] bf16 contiguous -> [M, N] fp32 (kernels/gemm_affine.py:62-98, same argument checks).
    ``cfg`` is validated (block_k must divide K) but the tile is fixed per weight shape."""
    if x.dim() != 2 or x.dtype != torch.bfloat16 or not x.is_contiguous():
        raise ValueError("x must be a contiguous 2-D bf16 tensor")
    m, k = x.shape
    if isinstance(w, AffineWeight):
        if w.bits != 4:
            raise ValueError(f"gemm supports 4-bit affine weights only, got bits={w.bits}")
        n = w.n
    elif isinstance(w, DenseWeight):
        n = w.n
    else:
        raise TypeError("w must be AffineWeight or DenseWeight")
    if k != w.k:
        raise ValueError(f"x has K={k}, weight has K={w.k}")
    if cfg is not None and k % cfg.get("block_k", 64):
        raise ValueError(f"K={k} is not a multiple of block_k={cfg['block_k']}")
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=x.device)
    elif (tuple(out.shape) != (m, n) or out.dtype != torch.float32 or out.device != x.device
          or not out.is_contiguous()):
        raise ValueError(f"out must be a contiguous fp32 [{m}, {n}] tensor on {x.device}, got "
                         f"{tuple(out.shape)} {out.dtype} {out.device}")
    if isinstance(w, DenseWeight):
        if not w.w.is_contiguous():
            raise ValueError("the dense weight must be contiguous")
        rc = _lib.lib().ssb_gemm_dense(_lib.ptr(x), m, k, _lib.ptr(w.w), n, _lib.ptr(out), n, _lib.stream())
        _lib.check(rc, "gemm_dense")
        _note("gemm_tc")
    else:
        rc = _lib.lib().ssb_gemm_affine4(_lib.ptr(x), m, k, _lib.ptr(w.q), _lib.ptr(w.s), _lib.ptr(w.b), n, w.gs,
                                         _lib.ptr(out), _lib.stream())
        _lib.check(rc, "gemm_affine4")
        _note("gemm_affine4")
    STATS["calls"] += 1
    STATS["rows"] += m
    return out
