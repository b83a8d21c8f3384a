"""Fused MoE layer for decode (additive API): router -> routed experts -> shared expert -> bf16 output.

Replaces, for callers that opt in, the per-layer sequence of slotstream_spark/runtime/graphs.py:160-182
(``seg_router`` then ``moe_decode`` + four shared-expert ``lin`` calls + ``routed.to(bf16) + sh``) with four
sm_100a launches that chain by programmatic dependent launch:
router_logits -> router_select -> gate_up (routed + shared) -> down + rank-order sum + shared add.
All buffers are preallocated in ``DecodeLayerBuffers`` so a whole 48-layer step can be captured in a graph.
"""
import torch

from .. import _lib
from .gemv_affine import _note
from .router import router_topk


class DecodeLayerBuffers:
    """Every output and workspace of one decode layer call for `rows` tokens."""

    def __init__(self, rows: int, topk: int, hidden: int, inter: int, experts: int = 512, device="cuda"):
        f32 = dict(dtype=torch.float32, device=device)
        self.rows, self.topk, self.hidden, self.inter, self.experts = rows, topk, hidden, inter, experts
        self.ws = torch.empty(rows * (experts + 1), **f32)
        self.ids = torch.empty(rows, topk, dtype=torch.int32, device=device)
        self.w = torch.empty(rows, topk, **f32)
        self.sh_gate = torch.empty(rows, **f32)
        self.h = torch.empty(rows * (topk + 1) * inter, **f32)
        self.o = torch.empty(rows, topk, hidden, **f32)
        self.out = torch.empty(rows, hidden, **f32)
        self.y = torch.empty(rows, hidden, dtype=torch.bfloat16, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)


def _addr(rec) -> int:
    if isinstance(rec, torch.Tensor):
        if not rec.is_cuda:
            raise ValueError("shared record must be a CUDA tensor")
        return rec.data_ptr()
    return int(rec)


def moe_layer_decode(x, w_router, layer: int, map_t, slot_ptr_t, shared_record, sh_gate_w, k: int,
                     bufs: DecodeLayerBuffers, *, bias=None, logits_round_bf16: bool = False, pdl: bool = True):
    """x bf16 [R, H] -> bufs.y bf16 [R, H] (also fills bufs.ids, bufs.w, bufs.out = routed fp32 sum)."""
    r, h = x.shape
    if (r, k, h) != (bufs.rows, bufs.topk, bufs.hidden) or w_router.shape[0] != bufs.experts:
        raise ValueError("buffers were sized for another call shape")
    if map_t.dtype != torch.int32 or slot_ptr_t.dtype != torch.int64:
        raise ValueError("map_t must be int32 and slot_ptr_t int64")
    router_topk(x, w_router, k, bufs.ids, bufs.w, logits_round_bf16=logits_round_bf16, bias=bias,
                sh_gate_w=sh_gate_w, out_sh_gate=bufs.sh_gate, ws=bufs.ws)
    rc = _lib.lib().ssb_moe_decode_layer(
        _lib.ptr(x), _lib.ptr(bufs.ids), _lib.ptr(bufs.w), r, k, h, bufs.inter, int(layer), _lib.ptr(map_t),
        map_t.numel(), _lib.ptr(slot_ptr_t), slot_ptr_t.numel(), _addr(shared_record), _lib.ptr(bufs.sh_gate),
        _lib.ptr(bufs.h), _lib.ptr(bufs.o), _lib.ptr(bufs.out), _lib.ptr(bufs.y), _lib.DECODE_PDL if pdl else 0,
        _lib.ptr(bufs.err), _lib.stream())
    _lib.check(rc, "moe_decode_layer")
    _note("moe_gate_up")
    _note("moe_down")
    return bufs.y
