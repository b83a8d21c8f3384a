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

FUSED_MAX_ROWS = 2


class DecodeLayerBuffers:
    """Every output and workspace of one decode layer call for `rows` tokens."""

    def __init__(self, rows: int, topk: int, hidden: int, inter: int, experts: int = 512, device="cuda"):
        f32 = dict(dtype=torch.float32, device=device)
        self.rows, self.topk, self.hidden, self.inter, self.experts = rows, topk, hidden, inter, experts
        self.ws = torch.empty(rows * (experts + 1), **f32)
        self.ids = torch.empty(rows, topk, dtype=torch.int32, device=device)
        self.w = torch.empty(rows, topk, **f32)
        self.bases = torch.empty(rows, topk, dtype=torch.int64, device=device)
        self.sh_gate = torch.empty(rows, **f32)
        self.h = torch.empty(rows * (topk + 1) * inter, **f32)
        self.o = torch.empty(rows, topk, hidden, **f32)
        self.out = torch.empty(rows, hidden, **f32)
        self.y = torch.empty(rows, hidden, dtype=torch.bfloat16, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.sync = torch.zeros(2, dtype=torch.int32, device=device)   # grid-barrier words of the fused kernel


class PrefillLayerBuffers:
    """Every output and workspace of one prefill layer call for `tokens` tokens.

    Row r < T*topk is (token r // topk, rank r % topk); rows T*topk + t are the shared expert's rows of token t.
    The router writes its ids / weights / shared gate straight into row_expert / row_weight, so the grouped
    GEMM reads them without any gather or concatenation."""

    def __init__(self, tokens: int, topk: int, hidden: int, inter: int, experts: int = 512, device="cuda"):
        from .moe_align import padded_rows
        from .fused_moe_affine import BLOCK_M
        t, r = tokens, tokens * topk
        self.tokens, self.topk, self.hidden, self.inter, self.experts = tokens, topk, hidden, inter, experts
        self.rows = r + t
        self.ld = experts + 4                                   # column `experts` holds the shared-gate logit
        f32 = dict(dtype=torch.float32, device=device)
        self.logits = torch.empty(t * self.ld, **f32)
        self.row_expert = torch.empty(self.rows, dtype=torch.int32, device=device)
        self.row_expert[r:] = experts                           # the shared expert is local expert `experts`
        self.row_token = torch.cat([torch.arange(r, device=device, dtype=torch.int32) // topk,
                                    torch.arange(t, device=device, dtype=torch.int32)])
        self.row_weight = torch.empty(self.rows, **f32)
        self.ids = self.row_expert[:r].view(t, topk)
        self.w = self.row_weight[:r].view(t, topk)
        self.sh_gate = self.row_weight[r:]
        p = padded_rows(self.rows, experts + 1, BLOCK_M)
        self.sorted_rows = torch.empty(p, dtype=torch.int32, device=device)
        self.block_expert = torch.empty(p // BLOCK_M, dtype=torch.int32, device=device)
        self.num_padded = torch.empty(1, dtype=torch.int32, device=device)
        self.x_sorted = torch.empty(p, hidden, dtype=torch.bfloat16, device=device)   # activation rows in expert order
        self.h = torch.empty(p, inter, dtype=torch.bfloat16, device=device)           # h in the same (sorted) order
        self.out_rows = torch.empty(self.rows, hidden, **f32)
        self.y = torch.empty(t, hidden, dtype=torch.bfloat16, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)


def _route_into(x, w_router, sh_gate_w, k: int, bufs: PrefillLayerBuffers, *, bias=None,
                logits_round_bf16: bool = False):
    """Router of a prefill chunk into the buffers: tcgen05 logits GEMM, the shared-gate logit, then the select writes
    ids / weights / shared gate straight into row_expert / row_weight."""
    t, h = x.shape
    e = bufs.experts
    L = _lib.lib()
    st = _lib.stream()
    lg = bufs.logits
    _lib.check(L.ssb_gemm_dense(_lib.ptr(x), t, h, _lib.ptr(w_router), e, _lib.ptr(lg), bufs.ld, st), "router gemm")
    _lib.check(L.ssb_router_logits(_lib.ptr(x), _lib.ptr(sh_gate_w), None, t, h, 1, bufs.ld, lg.data_ptr() + 4 * e, st),
               "shared gate logits")
    flags = _lib.ROUTER_SHARED_GATE | (_lib.ROUTER_ROUND_BF16 if logits_round_bf16 else 0)
    _lib.check(L.ssb_router_select(_lib.ptr(lg), bufs.ld, t, e, k, _lib.ptr(bias), flags, _lib.ptr(bufs.ids),
                                   _lib.ptr(bufs.w), None, _lib.ptr(bufs.sh_gate), st), "router select")


def moe_layer_prefill(x, w_router, group_ptr, sh_gate_w, k: int, bufs: PrefillLayerBuffers, *, bias=None,
                      logits_round_bf16: bool = False):
    """x bf16 [T, H] -> bufs.y bf16 [T, H]: one MoE layer over a prefill chunk, every expert resident.

    ``group_ptr`` int64 [E + 1]: record base of expert e at index e and of the shared expert at index E.
    Launches: router GEMM (tcgen05, dense bf16) + shared-gate logits, router select, align, row permute into
    expert order, gate_up + down (tcgen05 grouped GEMM, shared expert as local expert E), rank-order combine +
    shared add."""
    from .fused_moe_affine import BLOCK_M
    from .moe_align import moe_align
    t, h = x.shape
    e = bufs.experts
    if (t, h) != (bufs.tokens, bufs.hidden) or k != bufs.topk or tuple(w_router.shape) != (e, h):
        raise ValueError("buffers were sized for another call shape")
    if group_ptr.dtype != torch.int64 or group_ptr.numel() != e + 1:
        raise ValueError("group_ptr must be int64 [E + 1] (routed experts, then the shared expert)")
    if x.dtype != torch.bfloat16 or not x.is_contiguous():
        raise ValueError("x must be a contiguous bf16 [T, H] tensor")
    L = _lib.lib()
    st = _lib.stream()
    _route_into(x, w_router, sh_gate_w, k, bufs, bias=bias, logits_round_bf16=logits_round_bf16)
    aligned = moe_align(bufs.row_expert, e + 1, BLOCK_M, out=(bufs.sorted_rows, bufs.block_expert, bufs.num_padded))
    _lib.check(L.ssb_prefill_experts(
        _lib.ptr(x), t, h, bufs.inter, _lib.ptr(bufs.row_token), _lib.ptr(bufs.row_weight), bufs.rows,
        _lib.ptr(aligned[0]), _lib.ptr(aligned[1]), _lib.ptr(aligned[2]), aligned[0].numel(), _lib.ptr(group_ptr),
        e + 1, e, _lib.ptr(bufs.x_sorted), _lib.ptr(bufs.h), _lib.ptr(bufs.out_rows), _lib.ptr(bufs.err), st),
        "prefill experts")
    r = t * k
    _lib.check(L.ssb_combine_layer(_lib.ptr(bufs.out_rows), t, k, h, bufs.out_rows.data_ptr() + 4 * r * h, None,
                                   _lib.ptr(bufs.y), st), "combine")
    _note("fused_moe_gate_up")
    _note("fused_moe_down")
    return bufs.y


def prefetch_l2(t: torch.Tensor):
    """Bring a device tensor's bytes into L2 on the current stream (ssb_prefetch_l2, a hint: nothing is written)."""
    if not t.is_cuda:
        raise ValueError("prefetch_l2 takes a CUDA tensor")
    _lib.check(_lib.lib().ssb_prefetch_l2(t.data_ptr(), t.numel() * t.element_size(), _lib.stream()), "prefetch_l2")


def decode_layers(x, router_w, sh_gate_w, shared_records, map_t, slot_ptr_t, k: int, bufs, *, bias=None,
                  fused: bool = True, prefetch_next: bool = False, side=None, after_layer=None):
    """The MoE layers of one decode step (x bf16 [layers, R, H], router weights [layers, E, H], shared-gate rows
    [layers, H], shared records [layers, record], one DecodeLayerBuffers per layer). With ``prefetch_next`` a side
    stream brings layer l+1's router weight and shared record -- bytes that do not depend on routing -- into L2
    while layer l streams its experts, so the next layer's router and shared rows read from L2. The side stream
    rejoins the current stream at the end (graph-capture safe). Off by default: in the 48-layer graph at b = 1 it
    measured 7% slower (1.355 vs 1.262 ms per step), the side-stream launches costing more than the L2 hits save.
    ``after_layer(l)`` runs after layer l's launch."""
    main = torch.cuda.current_stream()
    side = side if side is not None else (torch.cuda.Stream(device=x.device) if prefetch_next else None)
    nl = x.shape[0]
    for l in range(nl):
        if prefetch_next and l + 1 < nl:
            ev = torch.cuda.Event()
            ev.record(main)
            side.wait_event(ev)
            with torch.cuda.stream(side):
                prefetch_l2(router_w[l + 1])
                prefetch_l2(shared_records[l + 1])
        moe_layer_decode(x[l], router_w[l], l, map_t, slot_ptr_t, shared_records[l], sh_gate_w[l], k, bufs[l],
                         bias=bias, fused=fused)
        if after_layer is not None:
            after_layer(l)
    if prefetch_next:
        main.wait_stream(side)


def _addr(rec) -> int:
    if isinstance(rec, torch.Tensor):
        if not rec.is_cuda:
            raise ValueError("shared record must be a CUDA tensor")
        return rec.data_ptr()
    return int(rec)


def moe_layer_decode(x, w_router, layer: int, map_t, slot_ptr_t, shared_record, sh_gate_w, k: int,
                     bufs: DecodeLayerBuffers, *, bias=None, logits_round_bf16: bool = False, pdl: bool = True,
                     prefetch_bytes: int = 0, fused: bool = True, cuda_cores: bool = False,
                     tensor_cores: bool = False):
    """x bf16 [R, H] -> bufs.y bf16 [R, H] (also fills bufs.ids, bufs.w, bufs.out = routed fp32 sum).
    ``fused`` (R <= 2): the whole layer in one cooperative launch (ssb_moe_decode_fused): the same ids and weights as
    the four-launch path router_logits -> router_select_resolve -> moe_decode_layer used otherwise. One token runs on
    CUDA cores (every output equal to the four-launch path bit for bit), two on the tensor cores (h and the routed sum
    within the fp32 tolerance); ``cuda_cores`` / ``tensor_cores`` force one of the two.
    ``prefetch_bytes`` > 0 makes the four-launch router prefetch that many bytes of each chosen record into L2."""
    r, h = x.shape
    if (r, k, h) != (bufs.rows, bufs.topk, bufs.hidden) or w_router.shape[0] != bufs.experts:
        raise ValueError("buffers were sized for another call shape")
    if map_t.dtype != torch.int32 or slot_ptr_t.dtype != torch.int64:
        raise ValueError("map_t must be int32 and slot_ptr_t int64")
    if x.dtype != torch.bfloat16 or not x.is_contiguous() or w_router.dtype != torch.bfloat16:
        raise ValueError("x and w_router must be contiguous bf16")
    if sh_gate_w.dtype != torch.bfloat16 or sh_gate_w.numel() != h:
        raise ValueError("sh_gate_w must be bf16 [H]")
    if bias is not None and (bias.dtype != torch.float32 or bias.numel() != bufs.experts):
        raise ValueError("bias must be fp32 [E]")
    L = _lib.lib()
    st = _lib.stream()
    e = bufs.experts
    if fused and r <= FUSED_MAX_ROWS:
        rc = L.ssb_moe_decode_fused(
            _lib.ptr(x), r, k, h, bufs.inter, e, _lib.ptr(w_router), _lib.ptr(sh_gate_w), _lib.ptr(bias),
            (_lib.ROUTER_ROUND_BF16 if logits_round_bf16 else 0) | (_lib.DECODE_FUSED_CUDA_CORES if cuda_cores else 0)
            | (_lib.DECODE_FUSED_TENSOR_CORES if tensor_cores else 0),
            int(layer), _lib.ptr(map_t), map_t.numel(),
            _lib.ptr(slot_ptr_t), slot_ptr_t.numel(), _addr(shared_record), _lib.ptr(bufs.ws), _lib.ptr(bufs.ids),
            _lib.ptr(bufs.w), _lib.ptr(bufs.sh_gate), _lib.ptr(bufs.bases), _lib.ptr(bufs.h), _lib.ptr(bufs.o),
            _lib.ptr(bufs.out), _lib.ptr(bufs.y), _lib.ptr(bufs.sync), _lib.ptr(bufs.err), st)
        if rc != _lib.SSB_EUNSUPPORTED:
            _lib.check(rc, "moe_decode_fused")
            _note("moe_decode_fused")
            return bufs.y
    _lib.check(L.ssb_router_logits(_lib.ptr(x), _lib.ptr(w_router), _lib.ptr(sh_gate_w), r, h, e, e + 1,
                                   _lib.ptr(bufs.ws), st), "router_logits")
    flags = _lib.ROUTER_SHARED_GATE | (_lib.ROUTER_ROUND_BF16 if logits_round_bf16 else 0)
    _lib.check(L.ssb_router_select_resolve(
        _lib.ptr(bufs.ws), e + 1, r, e, k, _lib.ptr(bias), flags, _lib.ptr(bufs.ids), _lib.ptr(bufs.w),
        _lib.ptr(bufs.sh_gate), int(layer), _lib.ptr(map_t), map_t.numel(), _lib.ptr(slot_ptr_t), slot_ptr_t.numel(),
        _lib.ptr(bufs.bases), prefetch_bytes, _lib.ptr(bufs.err), st), "router_select_resolve")
    rc = _lib.lib().ssb_moe_decode_layer(
        _lib.ptr(x), _lib.ptr(bufs.ids), _lib.ptr(bufs.w), r, k, h, bufs.inter, int(layer), _lib.ptr(map_t),
        map_t.numel(), _lib.ptr(slot_ptr_t), slot_ptr_t.numel(), _addr(shared_record), _lib.ptr(bufs.sh_gate),
        _lib.ptr(bufs.bases), _lib.ptr(bufs.h), _lib.ptr(bufs.o), _lib.ptr(bufs.out), _lib.ptr(bufs.y),
        _lib.DECODE_PDL if pdl else 0, _lib.ptr(bufs.err), st)
    _lib.check(rc, "moe_decode_layer")
    for name in ("moe_gate_up", "moe_down", "moe_gate_up_grouped", "moe_down_grouped"):
        _note(name)
    return bufs.y
