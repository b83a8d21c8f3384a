"""Row alignment for the grouped MoE kernels -- drop-in for slotstream_spark/kernels/moe_align.py.

One CUDA kernel (warp scans + match_any ranking) replaces the reference's ten torch ops: rows are sorted by
local expert (stable: the order inside an expert is the row order), each expert's rows are padded to
`block_m` with the sentinel R, every block of `block_m` positions belongs to exactly one expert. No atomics
on data, no host sync; output sizes depend only on (R, num_local, block_m) (kernels/moe_align.py:1-8).
"""
import torch

from .. import _lib
from .gemv_affine import _note


def padded_rows(r: int, num_local: int, block_m: int) -> int:
    """Upper bound of the padded length, rounded up to a whole number of blocks (kernels/moe_align.py:11-14)."""
    n = r + num_local * (block_m - 1)
    return (n + block_m - 1) // block_m * block_m


def moe_align(local_expert: torch.Tensor, num_local: int, block_m: int, *, expert_map: torch.Tensor | None = None,
              out=None):
    """local_expert int32 [R] (-1 = not in the current group) -> (sorted_rows int32 [P], block_expert int32
    [P // block_m], num_padded int32 [1]) (kernels/moe_align.py:17-48). With ``expert_map`` (int32 [E]) the
    input holds global expert ids and the local expert is expert_map[id] (align_rows of
    kernels/fused_moe_affine.py:130-133, fused into the same kernel). ``out`` may pass preallocated outputs."""
    if local_expert.dtype != torch.int32 or local_expert.dim() != 1:
        raise ValueError("local_expert must be int32 [R]")
    if num_local < 1 or block_m < 1:
        raise ValueError("num_local and block_m must be positive")
    if expert_map is not None and (expert_map.dtype != torch.int32 or expert_map.dim() != 1):
        raise ValueError("expert_map must be int32 [E]")
    r = local_expert.numel()
    dev = local_expert.device
    p = padded_rows(r, num_local, block_m)
    if out is None:
        sorted_rows = torch.empty(p, dtype=torch.int32, device=dev)
        block_expert = torch.empty(p // block_m, dtype=torch.int32, device=dev)
        num_padded = torch.empty(1, dtype=torch.int32, device=dev)
    else:
        sorted_rows, block_expert, num_padded = out
        if sorted_rows.numel() != p or block_expert.numel() != p // block_m or num_padded.numel() != 1:
            raise ValueError("preallocated align outputs have the wrong sizes")
    rc = _lib.lib().ssb_moe_align(_lib.ptr(local_expert.contiguous()), r, _lib.ptr(expert_map),
                                  0 if expert_map is None else expert_map.numel(), num_local, block_m,
                                  _lib.ptr(sorted_rows), _lib.ptr(block_expert), _lib.ptr(num_padded), _lib.stream())
    _lib.check(rc, "moe_align")
    _note("moe_align")
    return sorted_rows, block_expert, num_padded
