"""Dense GEMV (MLX affine 4/8-bit, gs 32/64, and bf16 dense) -- drop-in for slotstream_spark/kernels/gemv_affine.py.

y[r, n] = sum_k x[r, k] * (q[n, k] * s[n, k//gs] + b[n, k//gs]), fp32 accumulate, fp32 out
(kernels/gemv_affine.py:1-8). The reference splits K into a workspace and reduces it in a second launch;
here one warp owns a weight row end to end, so there is no split and ``ws`` is only validated. Each output
row is the same op sequence whatever R is (row invariance, tests/t0/test_affine_kernels.py:43-75).
"""
from dataclasses import dataclass

import torch

from .. import _lib

SHARED_BYTES: dict[str, int] = {}


def _note(name, handle=None):
    """Record the shared memory the named kernel launched with (kernels/gemv_affine.py:18-25)."""
    b = _lib.smem(name)
    if b >= 0:
        SHARED_BYTES[name] = b


@dataclass
class AffineWeight:
    q: torch.Tensor   # int32 [n, k*bits/32]
    s: torch.Tensor   # bf16 [n, k/gs]
    b: torch.Tensor   # bf16 [n, k/gs]
    bits: int
    gs: int
    n: int
    k: int

    def __post_init__(self):   # same checks as kernels/gemv_affine.py:36-47
        if self.bits not in (4, 8) or self.gs not in (32, 64):
            raise ValueError(f"unsupported bits={self.bits} gs={self.gs}")
        if self.k % self.gs:
            raise ValueError(f"k={self.k} not a multiple of gs={self.gs}")
        if tuple(self.q.shape) != (self.n, self.k * self.bits // 32) or self.q.dtype != torch.int32:
            raise ValueError(f"q must be int32 {(self.n, self.k * self.bits // 32)}, got {tuple(self.q.shape)} {self.q.dtype}")
        for t in (self.s, self.b):
            if tuple(t.shape) != (self.n, self.k // self.gs) or t.dtype != torch.bfloat16:
                raise ValueError("scales and biases must be bf16 [n, k/gs]")


@dataclass
class DenseWeight:
    w: torch.Tensor  # bf16 [n, k]

    def __post_init__(self):
        if self.w.dtype != torch.bfloat16 or self.w.dim() != 2:
            raise ValueError("DenseWeight needs a 2-D bf16 tensor")

    @property
    def n(self):
        return self.w.shape[0]

    @property
    def k(self):
        return self.w.shape[1]


def gemv(x: torch.Tensor, w, out: torch.Tensor | None = None, ws: torch.Tensor | None = None,
         cfg: dict | None = None) -> torch.Tensor:
    """x [R, K] bf16|fp32 -> [R, N] fp32 (kernels/gemv_affine.py:214-262). ``ws`` is accepted for API parity
    and validated like the reference's split-K workspace; ``cfg`` is validated (block_k must be a multiple
    of gs for 4-bit weights) but the launch shape is fixed per weight shape."""
    if x.dim() != 2 or x.dtype not in (torch.bfloat16, torch.float32) or not x.is_contiguous():
        raise ValueError("x must be a contiguous 2-D bf16 or fp32 tensor")
    r, k = x.shape
    if isinstance(w, AffineWeight):
        n, bits, gs = w.n, w.bits, w.gs
    elif isinstance(w, DenseWeight):
        n, bits, gs = w.n, 16, 0
    else:
        raise TypeError("w must be AffineWeight or DenseWeight")
    if k != w.k:
        raise ValueError(f"x has K={k}, weight has K={w.k}")
    if cfg is not None and bits == 4 and cfg.get("block_k", gs) % gs:
        raise ValueError("block_k must be a multiple of gs")
    if out is None:
        out = torch.empty((r, n), dtype=torch.float32, device=x.device)
    elif tuple(out.shape) != (r, n) or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous fp32 [{r}, {n}] tensor")
    if ws is not None and (ws.dtype != torch.float32 or ws.numel() < r * n):
        raise ValueError("workspace too small")
    L = _lib.lib()
    xd = _lib.F32 if x.dtype == torch.float32 else _lib.BF16
    if isinstance(w, DenseWeight):
        rc = L.ssb_gemv_dense(_lib.ptr(x), xd, r, _lib.ptr(w.w), n, k, _lib.ptr(out), _lib.stream())
        _lib.check(rc, "gemv(dense)")
        _note("gemv_dense")
    else:
        rc = L.ssb_gemv_affine(_lib.ptr(x), xd, r, _lib.ptr(w.q), _lib.ptr(w.s), _lib.ptr(w.b), n, k, bits, gs,
                               _lib.ptr(out), _lib.stream())
        _lib.check(rc, "gemv(affine)")
        _note("gemv_affine4" if bits == 4 else "gemv_affine8")
    return out
