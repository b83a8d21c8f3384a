"""Grouped affine 4-bit MoE for prefill -- drop-in for slotstream_spark/kernels/fused_moe_affine.py.

One group = experts whose records sit at ``group_ptr[g]`` (a pool slot or a staging slot; the kernel cannot
tell). ``expert_map[e]`` is the local index g or -1 (rows of such experts are skipped). Two sm_100a launches on
the 5th-generation tensor cores (tcgen05, accumulators in TMEM): gate_up writes h = silu(x Wg^T) * (x Wu^T) as
bf16 [R, I]; down writes y = (h Wd^T) * w as fp32 [R, H] into ``out_rows`` (kernels/fused_moe_affine.py:1-20).

Rounding path, as the reference: the dequantised gate, up and down tiles are rounded to bf16 (q*s + b in fp32
first), products accumulate in fp32, h is stored bf16. Tiles and the k order are constants of the shape, never
functions of R or of the group composition, so a row's bits depend on that row and that record only.

Differences from the reference, all additive: the kernels take the shape from the tensors (hidden = x.shape[1],
inter = h_buf.shape[1] or ``inter=``); the module constants HID / INTER / TOPK / RECORD_BYTES / O_* describe the
shape set by ``slotstream_b200.kernels.configure`` (the reference model's 2560 / 640 until then), and a call
without h_buf whose x does not have HID columns raises instead of guessing I; a group may hold up to 512 experts
(every expert of a layer resident at once); BLOCK_M is 256 (one grouped-GEMM tile: two tcgen05 M128 halves
sharing one dequantised weight tile), so ``aligned`` must come from this module's ``align_rows``.
"""
import torch

from .. import _lib
from ..records import RecordLayout
from . import shape as _shape
from .gemv_affine import _note
from .moe_align import moe_align, padded_rows

# HID, INTER, TOPK, RECORD_BYTES and O_GATE_W .. O_DOWN_B: the configured model shape (kernels/shape.py)
_shape.install(globals())
GROUP_MAX = 512
BLOCK_M, BLOCK_N, BLOCK_K = 256, 128, 64


def layout_for(hidden: int, inter: int) -> RecordLayout:
    return RecordLayout(hidden, inter, 64)


def align_rows(row_expert, expert_map, num_local, out=None):
    """Local expert of every row through ``expert_map`` (-1 outside the group), aligned to BLOCK_M
    (kernels/fused_moe_affine.py:130-133); the gather is fused into the align kernel."""
    return moe_align(row_expert, num_local, BLOCK_M, expert_map=expert_map, out=out)


def launch_gate_up(x, row_token, aligned, group_ptr, h_buf, r, err=None):
    sorted_rows, block_expert, num_padded = aligned
    rc = _lib.lib().ssb_fused_moe_gate_up(
        _lib.ptr(x), x.shape[0], x.shape[1], h_buf.shape[1], _lib.ptr(row_token), r, _lib.ptr(sorted_rows),
        _lib.ptr(block_expert), _lib.ptr(num_padded), sorted_rows.numel(), _lib.ptr(group_ptr), group_ptr.numel(),
        _lib.ptr(h_buf), _lib.ptr(err), _lib.stream())
    _lib.check(rc, "fused_moe gate_up")
    _note("fused_moe_gate_up")


def launch_down(h_buf, row_weight, aligned, group_ptr, out_rows, r, err=None):
    sorted_rows, block_expert, num_padded = aligned
    rc = _lib.lib().ssb_fused_moe_down(
        _lib.ptr(h_buf), r, out_rows.shape[1], h_buf.shape[1], _lib.ptr(row_weight), _lib.ptr(sorted_rows),
        _lib.ptr(block_expert), _lib.ptr(num_padded), sorted_rows.numel(), _lib.ptr(group_ptr), group_ptr.numel(),
        _lib.ptr(out_rows), _lib.ptr(err), _lib.stream())
    _lib.check(rc, "fused_moe down")
    _note("fused_moe_down")


def fused_moe_affine(x, row_token, row_weight, expert_map, group_ptr, out_rows, *, row_expert, h_buf=None,
                     aligned=None, inter=None, err=None):
    """x bf16 [T, H] · row_token int32 [R] · row_weight fp32 [R] · expert_map int32 [512] (local index or -1) ·
    group_ptr int64 [G <= GROUP_MAX] record base addresses · out_rows fp32 [R, H] (rows outside the group are
    left alone) -> None (kernels/fused_moe_affine.py:136-161, same argument checks). ``row_expert`` int32 [R]
    is the global expert of each row; ``aligned`` may carry a precomputed ``align_rows`` result and ``h_buf``
    a bf16 [R, I] buffer; ``inter`` gives I when no h_buf is passed, else I is the configured INTER, which needs
    x to have the configured HID columns (the record offsets follow from both)."""
    r = row_token.numel()
    if x.dtype != torch.bfloat16 or x.dim() != 2 or not x.is_contiguous():
        raise ValueError("x must be a contiguous bf16 [T, H] tensor")
    hid = x.shape[1]
    if row_token.dtype != torch.int32 or row_weight.dtype != torch.float32 or row_weight.numel() != r:
        raise ValueError("row_token must be int32 [R] and row_weight fp32 [R]")
    if row_expert.dtype != torch.int32 or row_expert.numel() != r:
        raise ValueError("row_expert must be int32 [R]")
    if expert_map.dtype != torch.int32 or group_ptr.dtype != torch.int64:
        raise ValueError("expert_map must be int32 and group_ptr int64")
    if not 1 <= group_ptr.numel() <= GROUP_MAX:
        raise ValueError(f"a group holds 1..{GROUP_MAX} experts")
    if tuple(out_rows.shape) != (r, hid) or out_rows.dtype != torch.float32 or not out_rows.is_contiguous():
        raise ValueError(f"out_rows must be contiguous fp32 [R, {hid}]")
    if h_buf is None:
        if inter is None:
            if hid != HID:
                raise ValueError(f"x has {hid} columns but the configured shape is {HID}/{INTER}: call "
                                 "slotstream_b200.kernels.configure(hidden, inter) or pass h_buf or inter")
            inter = INTER
        h_buf = torch.empty((r, inter), dtype=torch.bfloat16, device=x.device)
    elif h_buf.dim() != 2 or h_buf.shape[0] != r or h_buf.dtype != torch.bfloat16 or not h_buf.is_contiguous():
        raise ValueError("h_buf must be bf16 [R, I]")
    if aligned is None:
        aligned = align_rows(row_expert, expert_map, group_ptr.numel())
    elif aligned[0].numel() != padded_rows(r, group_ptr.numel(), BLOCK_M):
        raise ValueError(f"aligned must come from align_rows (BLOCK_M = {BLOCK_M})")
    launch_gate_up(x, row_token, aligned, group_ptr, h_buf, r, err)
    launch_down(h_buf, row_weight, aligned, group_ptr, out_rows, r, err)


def combine_rank_order(out_rows, T, K=None, out=None):
    """out_rows fp32 [T*K, H], row = token*K + rank -> fp32 [T, H], summed in router rank order (sequential
    fp32), bit-equal to kernels/fused_moe_affine.py:164-172. K defaults to the configured TOPK."""
    K = TOPK if K is None else K
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
