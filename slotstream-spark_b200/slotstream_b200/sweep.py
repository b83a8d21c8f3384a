"""Prefill MoE sweep over partially resident experts -- the B200 side of slotstream_spark/model/moe_sweep.py:80-176 and
the group planner of engine/sweep.py:34-58.

A layer's (token, rank) rows are sorted stably by (resident first, expert id) and cut into groups of at most
``group_size`` experts that never mix resident and staged experts (``plan_sweep``). A resident group reads its
records where they already sit in HBM (pool slots). A staged group is copied from pinned host records into one of
``staging_groups`` device staging buffers on a copy stream, ``inflight`` groups ahead of the group being computed;
events order every reuse of a buffer after the kernels that read it. Each group is one align (its expert map selects
its rows) and one ``ssb_prefill_experts`` launch (row permute, tcgen05 gate_up, tcgen05 down) writing its rows of
``out_rows``; the shared expert is one more group, and ``ssb_combine_layer`` sums every token's rows in router rank
order and adds the shared expert. A row's result depends only on that row and its expert's bytes, so the layer equals
the all-resident ``moe_layer_prefill`` bit for bit whatever the residency, the grouping or the staging buffer.
"""
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .kernels.fused_moe_affine import BLOCK_M
from .kernels.moe_align import moe_align, padded_rows

EXPERTS = 512
GROUP_SIZE = 32       # experts per group (engine/sweep.py:18)
STAGING_GROUPS = 4    # staging buffers of GROUP_SIZE records (model/moe_sweep.py:25)
INFLIGHT = 2          # staged groups issued ahead of the one being computed (model/moe_sweep.py:26)


@dataclass(frozen=True)
class Group:
    experts: np.ndarray   # int32, ascending expert ids of the group
    resident: bool
    row_lo: int           # rows [row_lo, row_hi) of SweepPlan.order belong to this group
    row_hi: int


@dataclass(frozen=True)
class SweepPlan:
    order: np.ndarray     # int64 [R]: row ids sorted by (resident first, expert id, row id)
    groups: list


def plan_sweep(expert_ids: np.ndarray, resident: np.ndarray, group_size: int = GROUP_SIZE) -> SweepPlan:
    """The grouping of engine/sweep.py:34-58 (same plan, same field meaning): each row gets the key expert id, plus
    EXPERTS when its expert is not resident; rows are ordered by key, ties in row order; the experts present are
    then taken ``group_size`` at a time, all resident keys before any staged one, so no group mixes the two."""
    ids = np.asarray(expert_ids)
    res = np.asarray(resident, dtype=bool)
    if ids.dtype != np.int32 or ids.ndim != 1:
        raise ValueError("expert_ids: want a 1-D int32 array of row experts")
    if res.shape != (EXPERTS,):
        raise ValueError(f"resident: want a bool mask of {EXPERTS} experts")
    if group_size <= 0:
        raise ValueError("group_size: want at least 1")
    if ids.size and not (0 <= int(ids.min()) and int(ids.max()) < EXPERTS):
        raise ValueError("expert_ids: value outside [0, 512)")
    key = ids.astype(np.int64) + np.where(res[ids], 0, EXPERTS)
    order = np.argsort(key, kind="stable")
    first = np.zeros(2 * EXPERTS + 1, dtype=np.int64)     # first[k] = position in `order` of the first row of key k
    np.cumsum(np.bincount(key, minlength=2 * EXPERTS), out=first[1:])
    groups = []
    for staged in (0, 1):
        base = staged * EXPERTS
        present = base + np.flatnonzero(first[base + 1:base + EXPERTS + 1] > first[base:base + EXPERTS])
        for a in range(0, present.size, group_size):
            keys = present[a:a + group_size]
            groups.append(Group((keys - base).astype(np.int32), staged == 0, int(first[keys[0]]),
                                int(first[keys[-1] + 1])))
    return SweepPlan(order, groups)


class SweepStats:
    def __init__(self):
        self.groups = self.staged_groups = self.records_staged = self.bytes_staged = 0
        self.resident_rows = self.staged_rows = 0

    def as_dict(self):
        return dict(self.__dict__)


class PrefillSweep:
    """Buffers and streams for sweeping layers of up to ``max_tokens`` tokens (every output and workspace allocated
    here, once)."""

    def __init__(self, hidden: int, inter: int, k: int, max_tokens: int, record_bytes: int, *, experts: int = EXPERTS,
                 group_size: int = GROUP_SIZE, staging_groups: int = STAGING_GROUPS, inflight: int = INFLIGHT,
                 device="cuda"):
        from .kernels.moe_layer import PrefillLayerBuffers
        if inflight < 1 or inflight > staging_groups:
            raise ValueError("need 1 <= inflight <= staging_groups")
        self.hidden, self.inter, self.k, self.experts = hidden, inter, k, experts
        self.group_size, self.staging_groups, self.inflight = group_size, staging_groups, inflight
        self.record_bytes = record_bytes
        self.bufs = PrefillLayerBuffers(max_tokens, k, hidden, inter, experts, device)
        rows = self.bufs.rows
        p = padded_rows(rows, group_size, BLOCK_M)
        self.sorted_rows = torch.empty(p, dtype=torch.int32, device=device)
        self.block_expert = torch.empty(p // BLOCK_M, dtype=torch.int32, device=device)
        self.num_padded = torch.empty(1, dtype=torch.int32, device=device)
        self.x_sorted = torch.empty(p, hidden, dtype=torch.bfloat16, device=device)
        self.h_sorted = torch.empty(p, inter, dtype=torch.bfloat16, device=device)
        self.staging = torch.empty((staging_groups, group_size, record_bytes), dtype=torch.uint8, device=device)
        self.copy_stream = torch.cuda.Stream(device=device)
        self.ids_host = torch.empty((max_tokens, k), dtype=torch.int32).pin_memory()
        # per-group expert maps and record pointers go through pinned host buffers (no pageable copies)
        n_max = 2 * ((experts + group_size - 1) // group_size) + 1   # groups of a layer, then the shared expert
        self._emap_host = torch.empty((n_max, experts + 1), dtype=torch.int32).pin_memory()
        self._ptr_host = torch.empty((n_max, group_size), dtype=torch.int64).pin_memory()
        self._emap_dev = torch.empty((n_max, experts + 1), dtype=torch.int32, device=device)
        self._ptr_dev = torch.empty((n_max, group_size), dtype=torch.int64, device=device)
        self.stats = SweepStats()
        self.last_plan = None

    def layer(self, x, w_router, sh_gate_w, shared_ptr: int, resident_ptr: dict, host_record_ptr, *, bias=None):
        """x bf16 [T, H] -> y bf16 [T, H] (a view of the sweep's buffer). ``resident_ptr``: {expert: device address}
        of the layer's resident records; ``host_record_ptr(e)``: address of expert e's pinned host record (staged
        experts); ``shared_ptr``: device address of the shared expert's record."""
        from .kernels.moe_layer import _route_into
        t, h = x.shape
        b = self.bufs
        k, E = self.k, self.experts
        if h != self.hidden or t > b.tokens or x.dtype != torch.bfloat16 or not x.is_contiguous():
            raise ValueError("x must be contiguous bf16 [T <= max_tokens, hidden]")
        if t != b.tokens:
            raise ValueError("this sweep's buffers hold exactly max_tokens tokens per layer")
        st = _lib.stream()
        comp = torch.cuda.current_stream()
        L = _lib.lib()
        _route_into(x, w_router, sh_gate_w, k, b, bias=bias)             # ids, weights, shared gate on the device
        self.ids_host[:t].copy_(b.ids, non_blocking=True)
        comp.synchronize()                                              # the router's ids, on the host
        flat = np.ascontiguousarray(self.ids_host[:t].numpy().reshape(-1), dtype=np.int32)
        resident = np.zeros(E, dtype=bool)
        for e in resident_ptr:
            resident[int(e)] = True
        plan = plan_sweep(flat, resident, self.group_size)
        self.last_plan = plan
        groups = plan.groups
        staged = [gi for gi, g in enumerate(groups) if not g.resident]
        buf_of = {gi: j % self.staging_groups for j, gi in enumerate(staged)}
        copy_done, buf_free = {}, [None] * self.staging_groups
        s = self.stats

        def issue(gi):   # copy a staged group's records into its buffer once the buffer's last reader finished
            bi = buf_of[gi]
            if buf_free[bi] is not None:
                self.copy_stream.wait_event(buf_free[bi])
            with torch.cuda.stream(self.copy_stream):
                for j, e in enumerate(groups[gi].experts):
                    _copy_async(self.staging[bi, j].data_ptr(), host_record_ptr(int(e)), self.record_bytes,
                                self.copy_stream)
                ev = torch.cuda.Event()
                ev.record(self.copy_stream)
            copy_done[gi] = ev
            s.staged_groups += 1
            s.records_staged += int(groups[gi].experts.size)
            s.bytes_staged += int(groups[gi].experts.size) * self.record_bytes

        for gi in staged[:self.inflight]:
            issue(gi)
        pending = staged[self.inflight:]
        for gi, g in enumerate(groups):
            s.groups += 1
            n = int(g.experts.size)
            emap = self._emap_host[gi]
            emap.fill_(-1)
            emap[torch.from_numpy(g.experts.astype(np.int64))] = torch.arange(n, dtype=torch.int32)
            ptrs = self._ptr_host[gi]
            if g.resident:
                for j, e in enumerate(g.experts):
                    ptrs[j] = int(resident_ptr[int(e)])
                s.resident_rows += g.row_hi - g.row_lo
            else:
                bi = buf_of[gi]
                for j in range(n):
                    ptrs[j] = self.staging[bi, j].data_ptr()
                comp.wait_event(copy_done.pop(gi))
                s.staged_rows += g.row_hi - g.row_lo
            self._emap_dev[gi].copy_(emap, non_blocking=True)
            self._ptr_dev[gi, :n].copy_(ptrs[:n], non_blocking=True)
            self._experts(x, self._emap_dev[gi], self._ptr_dev[gi, :n], n, -1, st)
            if not g.resident:
                ev = torch.cuda.Event()
                ev.record(comp)
                buf_free[buf_of[gi]] = ev
                if pending:
                    issue(pending.pop(0))   # keep `inflight` staged groups ahead of the compute
        # the shared expert: one more group (local expert 0, the reference's bf16 rounding between its ops)
        gi = len(groups)
        emap = self._emap_host[gi]
        emap.fill_(-1)
        emap[E] = 0
        self._emap_dev[gi].copy_(emap, non_blocking=True)
        self._ptr_host[gi, 0] = int(shared_ptr)
        self._ptr_dev[gi, :1].copy_(self._ptr_host[gi, :1], non_blocking=True)
        self._experts(x, self._emap_dev[gi], self._ptr_dev[gi, :1], 1, 0, st)
        r = t * k
        _lib.check(L.ssb_combine_layer(_lib.ptr(b.out_rows), t, k, h, b.out_rows.data_ptr() + 4 * r * h, None,
                                       _lib.ptr(b.y), st), "combine")
        return b.y

    def _experts(self, x, emap, gptr, n, shared_local, st):
        """One group: align the layer's rows through the group's expert map, then the grouped GEMMs over them."""
        b = self.bufs
        sr, be, npd = moe_align(b.row_expert, n, BLOCK_M, expert_map=emap,
                                out=(self.sorted_rows[:padded_rows(b.rows, n, BLOCK_M)],
                                     self.block_expert[:padded_rows(b.rows, n, BLOCK_M) // BLOCK_M], self.num_padded))
        _lib.check(_lib.lib().ssb_prefill_experts(
            _lib.ptr(x), x.shape[0], self.hidden, self.inter, _lib.ptr(b.row_token), _lib.ptr(b.row_weight), b.rows,
            _lib.ptr(sr), _lib.ptr(be), _lib.ptr(npd), sr.numel(), _lib.ptr(gptr), n, shared_local,
            _lib.ptr(self.x_sorted), _lib.ptr(self.h_sorted), _lib.ptr(b.out_rows), _lib.ptr(b.err), st),
            "prefill experts (sweep group)")


def _copy_async(dst: int, src: int, nbytes: int, stream):
    """One asynchronous copy of a pinned host record into a staging slot on `stream` (ssb_copy_async)."""
    _lib.check(_lib.lib().ssb_copy_async(dst, src, nbytes, stream.cuda_stream), "record copy")


def resident_from_pool(pool, layer: int) -> dict:
    """{expert: device address} of a SlotPool's resident records of `layer` (one small device-to-host read)."""
    m = pool.map[layer * pool.experts:(layer + 1) * pool.experts].cpu().numpy()
    sp = pool.slot_ptr.cpu().numpy()
    return {int(e): int(sp[s]) for e, s in enumerate(m) if s >= 0}
