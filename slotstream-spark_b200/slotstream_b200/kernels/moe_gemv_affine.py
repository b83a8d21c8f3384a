"""MoE expert GEMVs for one token step, MLX affine 4-bit gs64 -- drop-in for slotstream_spark/kernels/moe_gemv_affine.py.

Experts live in records inside pool slots. The kernels never see a slot index from the host: they read
``slot = map[layer*512 + e]`` and ``base = slot_ptr[slot]`` from device tables, so a CUDA graph depends only
on routing (kernels/moe_gemv_affine.py:1-9). Two sm_100a launches: gate_up (h = silu(G x) * U x, fp32) and
down (o_k = w_k * D h_k, fp32) with the rank-order sum out = o_0 + o_1 + ... fused into the same grid. A
3-row call equals three 1-row calls bit for bit and a record can move between slots without changing bits.

The reference hard-codes 2560/640; here the shape comes from the tensors (hidden = x.shape[1],
inter = h_buf.shape[2], top-k = expert_ids.shape[1]) and the record offsets from
``slotstream_b200.records.RecordLayout``. The module constants (HID, INTER, TOPK, RECORD_BYTES, O_*) describe the
shape set by ``slotstream_b200.kernels.configure``: the reference model's 2560 / 640 until then.
"""
import torch

from .. import _lib
from ..records import EXPERTS_PER_LAYER, RecordLayout
from . import shape as _shape
from .gemv_affine import _note

# HID, INTER, TOPK, RECORD_BYTES and O_GATE_W .. O_DOWN_B: the configured model shape (kernels/shape.py)
_shape.install(globals())
GS = 64
MOE_DEFAULT = {"bn": 4, "br": 32, "bk": 512, "bkd": 128, "num_warps": 4}   # accepted for API parity


def layout_for(hidden: int, inter: int) -> RecordLayout:
    return RecordLayout(hidden, inter, GS)


def moe_decode(x, expert_ids, weights, layer: int, map_t, slot_ptr_t, h_buf, o_buf, out, cfg=None, err=None):
    """x [R, H] bf16|fp32 · expert_ids int32 [R, K] (device) · weights fp32 [R, K] · map_t int32 [49*512] ·
    slot_ptr_t int64 [n_slots] · h_buf [R, K, I] f32 · o_buf [R, K, H] f32 · out [R, H] f32 -> out
    (kernels/moe_gemv_affine.py:113-147, same argument checks). ``err`` (optional int32 [1], device)
    receives SSB error bits for unmapped or out-of-range experts, whose contribution is zero."""
    r = x.shape[0]
    if x.dim() != 2 or x.dtype not in (torch.bfloat16, torch.float32) or not x.is_contiguous():
        raise ValueError("x must be a contiguous [R, H] bf16 or fp32 tensor")
    hid = x.shape[1]
    if expert_ids.dim() != 2 or expert_ids.shape[0] != r or expert_ids.dtype != torch.int32 \
            or not expert_ids.is_contiguous():
        raise ValueError("expert_ids must be contiguous int32 [R, K]")
    topk = expert_ids.shape[1]
    if tuple(weights.shape) != (r, topk) or weights.dtype != torch.float32 or not weights.is_contiguous():
        raise ValueError("weights must be contiguous fp32 [R, K]")
    if map_t.dtype != torch.int32 or slot_ptr_t.dtype != torch.int64:
        raise ValueError("map_t must be int32 and slot_ptr_t int64")
    if h_buf.dim() != 3:
        raise ValueError("h_buf must be fp32 [R, K, I]")
    inter = h_buf.shape[2]
    for t, shape in ((h_buf, (r, topk, inter)), (o_buf, (r, topk, hid)), (out, (r, hid))):
        if tuple(t.shape) != shape or t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError(f"buffer must be contiguous fp32 {shape}")
    c = dict(cfg) if cfg is not None else dict(MOE_DEFAULT)
    c.setdefault("bkd", MOE_DEFAULT["bkd"])
    if c["bk"] % 64 or c["bkd"] % 64:
        raise ValueError("bk and bkd must be multiples of 64")
    if err is not None and (err.dtype != torch.int32 or err.numel() < 1):
        raise ValueError("err must be int32 [1]")
    rc = _lib.lib().ssb_moe_decode(
        _lib.ptr(x), _lib.F32 if x.dtype == torch.float32 else _lib.BF16, _lib.ptr(expert_ids), _lib.ptr(weights),
        r, topk, hid, inter, int(layer), _lib.ptr(map_t), map_t.numel(), _lib.ptr(slot_ptr_t), slot_ptr_t.numel(),
        _lib.ptr(h_buf), _lib.ptr(o_buf), _lib.ptr(out), _lib.ptr(err), _lib.stream())
    _lib.check(rc, "moe_decode")
    for name in ("moe_gate_up", "moe_down", "moe_gate_up_grouped", "moe_down_grouped"):
        _note(name)
    return out


__all__ = ["moe_decode", "layout_for", "HID", "INTER", "TOPK", "RECORD_BYTES", "GS", "EXPERTS_PER_LAYER",
           "O_GATE_W", "O_GATE_S", "O_GATE_B", "O_UP_W", "O_UP_S", "O_UP_B", "O_DOWN_W", "O_DOWN_S", "O_DOWN_B"]
