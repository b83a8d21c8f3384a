"""Prefill MoE sweep over partially resident experts -- the B200 side of slotstream_spark/model/moe_sweep.py:80-176 and
the group planner of engine/sweep.py:34-58.

A layer's (token, rank) rows are grouped as the reference plans them: resident experts first, then staged ones,
at most ``group_size`` experts per group, never mixing the two (``plan_sweep`` restates that planner over the rows;
``plan_groups`` gives the same groups from the per-expert row counts, which is all the device path needs). A
resident group reads its records where they already sit in HBM (pool slots). A staged group is copied from pinned
host records into one of ``staging_groups`` device staging buffers on a copy stream, ``inflight`` groups ahead of
the group being computed; events order every reuse of a buffer after the kernels that read it.

On the device the layer is one router, one align whose expert map numbers the experts in plan order (so each
group's rows are a contiguous run of 256-row blocks), one permute of the activation rows into that order, then per
group the tcgen05 gate_up and down launches over the group's blocks (resident groups, then the shared expert,
whose blocks close the layout, then the staged groups as their copies land), and one rank-order combine with the
shared add. A row's result depends only on that row and its expert's bytes, so the
layer equals the all-resident ``moe_layer_prefill`` bit for bit whatever the residency, the grouping or the staging
buffer.
"""
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .kernels.fused_moe_affine import BLOCK_M
from .kernels.moe_align import moe_align, padded_rows

EXPERTS = 512
GROUP_SIZE = 32       # experts per group (engine/sweep.py:18)
# Staging: the reference keeps 4 buffers of 32 records with 2 groups in flight (model/moe_sweep.py:25-26) for its
# unified memory. On a B200 eight buffers are 453 MB of the 180 GB (2048/512 records), enough for every staged
# record of a layer whose hottest half is resident, so all of a layer's copies are issued at once and the copy
# engine streams them back to back while the resident groups compute.
STAGING_GROUPS = 8    # staging buffers of GROUP_SIZE records
INFLIGHT = 8          # staged groups issued ahead of the one being computed


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


def plan_groups(counts: np.ndarray, resident: np.ndarray, group_size: int = GROUP_SIZE) -> SweepPlan:
    """The groups of ``plan_sweep`` from per-expert row counts alone (int [512]): the same experts, residency and
    row ranges, without ordering the rows on the host (the device align orders them). ``order`` is None."""
    c = np.asarray(counts, dtype=np.int64)
    res = np.asarray(resident, dtype=bool)
    if c.shape != (EXPERTS,) or res.shape != (EXPERTS,) or (c < 0).any():
        raise ValueError(f"counts and resident: want [{EXPERTS}] arrays, counts >= 0")
    if group_size <= 0:
        raise ValueError("group_size: want at least 1")
    groups, pos = [], 0
    for is_res in (True, False):
        present = np.flatnonzero((c > 0) & (res == is_res))
        for a in range(0, present.size, group_size):
            ex = present[a:a + group_size]
            n = int(c[ex].sum())
            groups.append(Group(ex.astype(np.int32), is_res, pos, pos + n))
            pos += n
    return SweepPlan(None, groups)


class SweepStats:
    def __init__(self):
        self.groups = self.staged_groups = self.records_staged = self.bytes_staged = 0
        self.resident_rows = self.staged_rows = 0

    def as_dict(self):
        return dict(self.__dict__)


class PrefillSweep:
    """Buffers and streams for sweeping layers of ``max_tokens`` tokens (every output and workspace allocated here,
    once).

    Per layer: the router on the device, the per-expert row counts read back (2 KB, one host sync), the plan of
    ``plan_groups``; then ONE align over all rows with local expert ids in plan order (so every group's rows form
    a contiguous run of 256-row blocks), ONE permute of the activation rows into that order, and per group the
    tcgen05 gate_up and down launches over the group's block range, reading its records where they are (HBM for
    resident experts, a staging buffer for staged ones); the shared expert's blocks close the layout and are
    launched between the resident and the staged groups; one rank-order combine."""

    def __init__(self, hidden: int, inter: int, k: int, max_tokens: int, record_bytes: int, *, experts: int = EXPERTS,
                 group_size: int = GROUP_SIZE, staging_groups: int = STAGING_GROUPS, inflight: int = INFLIGHT,
                 device="cuda"):
        from .kernels.moe_layer import PrefillLayerBuffers
        if inflight < 1 or inflight > staging_groups:
            raise ValueError("need 1 <= inflight <= staging_groups")
        if experts != EXPERTS:
            raise ValueError(f"the sweep plans {EXPERTS} experts per layer")
        self.hidden, self.inter, self.k, self.experts = hidden, inter, k, experts
        self.group_size, self.staging_groups, self.inflight = group_size, staging_groups, inflight
        self.record_bytes = record_bytes
        self.bufs = PrefillLayerBuffers(max_tokens, k, hidden, inter, experts, device)
        self.staging = torch.empty((staging_groups, group_size, record_bytes), dtype=torch.uint8, device=device)
        self.copy_stream = torch.cuda.Stream(device=device)
        self.counts = torch.empty(experts, dtype=torch.int64, device=device)
        self.counts_host = torch.empty(experts, dtype=torch.int64).pin_memory()
        n_max = 2 * ((experts + group_size - 1) // group_size) + 1   # groups of a layer, then the shared expert
        # per layer: the expert map (global -> local id in plan order), record bases per local id, and per group
        # its padded row count, through pinned host buffers
        self._emap_host = torch.empty(experts + 1, dtype=torch.int32).pin_memory()
        self._ptr_host = torch.empty(experts + 1, dtype=torch.int64).pin_memory()
        self._npad_host = torch.empty(n_max, dtype=torch.int32).pin_memory()
        self._emap_dev = torch.empty(experts + 1, dtype=torch.int32, device=device)
        self._ptr_dev = torch.empty(experts + 1, dtype=torch.int64, device=device)
        self._npad_dev = torch.empty(n_max, dtype=torch.int32, device=device)
        self.stats = SweepStats()
        self.last_plan = None

    def layer(self, x, w_router, sh_gate_w, shared_ptr: int, resident_ptr: dict, host_record_ptr, *, bias=None):
        """x bf16 [T, H] -> y bf16 [T, H] (a view of the sweep's buffer). ``resident_ptr``: {expert: device address}
        of the layer's resident records; ``host_record_ptr(e)``: address of expert e's pinned host record (staged
        experts); ``shared_ptr``: device address of the shared expert's record."""
        from .kernels.moe_layer import _route_into
        b = self.bufs
        t, h = x.shape
        k, E, H, I = self.k, self.experts, self.hidden, self.inter
        if h != H or t != b.tokens or x.dtype != torch.bfloat16 or not x.is_contiguous():
            raise ValueError("x must be contiguous bf16 [max_tokens, hidden]")
        st = _lib.stream()
        comp = torch.cuda.current_stream()
        L = _lib.lib()
        _route_into(x, w_router, sh_gate_w, k, b, bias=bias)             # ids, weights, shared gate on the device
        self.counts.copy_(torch.bincount(b.ids.reshape(-1), minlength=E))
        self.counts_host.copy_(self.counts, non_blocking=True)
        comp.synchronize()                                              # the per-expert row counts, on the host
        counts = self.counts_host.numpy()
        resident = np.zeros(E, dtype=bool)
        for e in resident_ptr:
            resident[int(e)] = True
        plan = plan_groups(counts, resident, self.group_size)
        self.last_plan = plan
        groups = plan.groups
        staged = [gi for gi, g in enumerate(groups) if not g.resident]
        buf_of = {gi: j % self.staging_groups for j, gi in enumerate(staged)}

        # local ids in plan order, the shared expert last; each local expert's rows padded to 256-row blocks
        emap = self._emap_host.numpy()
        ptrs = self._ptr_host.numpy()
        emap[:] = -1
        blk = [0]
        loc = 0
        for gi, g in enumerate(groups):
            for j, e in enumerate(g.experts):
                emap[int(e)] = loc
                ptrs[loc] = (int(resident_ptr[int(e)]) if g.resident else self.staging[buf_of[gi], j].data_ptr())
                loc += 1
            blk.append(blk[-1] + int(((counts[g.experts] + BLOCK_M - 1) // BLOCK_M).sum()))
        emap[E] = loc
        ptrs[loc] = int(shared_ptr)
        n_local = loc + 1
        blk.append(blk[-1] + (t + BLOCK_M - 1) // BLOCK_M)
        npad = self._npad_host.numpy()
        for gi in range(len(groups) + 1):
            npad[gi] = (blk[gi + 1] - blk[gi]) * BLOCK_M
        self._emap_dev.copy_(self._emap_host, non_blocking=True)
        self._ptr_dev[:n_local].copy_(self._ptr_host[:n_local], non_blocking=True)
        self._npad_dev[:len(groups) + 1].copy_(self._npad_host[:len(groups) + 1], non_blocking=True)

        # the staging copies start now, beside the align, the permute and the resident groups
        copy_done, buf_free = {}, [None] * self.staging_groups
        s = self.stats

        def issue(gi):   # copy a staged group's records into its buffer once the buffer's last reader finished
            bi = buf_of[gi]
            if buf_free[bi] is not None:
                self.copy_stream.wait_event(buf_free[bi])
            for j, e in enumerate(groups[gi].experts):
                _copy_async(self.staging[bi, j].data_ptr(), host_record_ptr(int(e)), self.record_bytes,
                            self.copy_stream)
            ev = torch.cuda.Event()
            ev.record(self.copy_stream)
            copy_done[gi] = ev
            s.staged_groups += 1
            s.records_staged += int(groups[gi].experts.size)
            s.bytes_staged += int(groups[gi].experts.size) * self.record_bytes

        self.copy_stream.wait_stream(comp)   # the staging buffers' previous readers (the last layer) are done
        for gi in staged[:self.inflight]:
            issue(gi)
        pending = staged[self.inflight:]

        p_len = padded_rows(b.rows, n_local, BLOCK_M)
        sr, be, npd = moe_align(b.row_expert, n_local, BLOCK_M, expert_map=self._emap_dev,
                                out=(b.sorted_rows[:p_len], b.block_expert[:p_len // BLOCK_M], b.num_padded))
        _lib.check(L.ssb_permute_rows(_lib.ptr(x), t, H, _lib.ptr(b.row_token), b.rows, _lib.ptr(sr), _lib.ptr(npd),
                                      p_len, _lib.ptr(b.x_sorted), st), "sweep permute")
        # launch order: resident groups, the shared expert (its record is resident too), then the staged groups,
        # so the work that needs no copy runs while the copies cross
        n_res = sum(1 for g in groups if g.resident)
        order = list(range(n_res)) + [len(groups)] + list(range(n_res, len(groups)))
        for gi in order:
            s.groups += 1
            g = groups[gi] if gi < len(groups) else None
            if g is not None and g.resident:
                s.resident_rows += g.row_hi - g.row_lo
            elif g is not None:
                comp.wait_event(copy_done.pop(gi))
                s.staged_rows += g.row_hi - g.row_lo
            self._blocks(blk[gi], blk[gi + 1], gi, n_local, n_local - 1, st)
            if g is not None and not g.resident:
                ev = torch.cuda.Event()
                ev.record(comp)
                buf_free[buf_of[gi]] = ev
                if pending:
                    issue(pending.pop(0))   # keep `inflight` staged groups ahead of the compute
        _lib.check(L.ssb_combine_layer(_lib.ptr(b.out_rows), t, k, H, b.out_rows.data_ptr() + 4 * t * k * H, None,
                                       _lib.ptr(b.y), st), "combine")
        return b.y

    def _blocks(self, lo, hi, gi, n_local, shared_local, st):
        """gate_up and down over 256-row blocks [lo, hi) of the layer's aligned rows (one group)."""
        b = self.bufs
        H, I = self.hidden, self.inter
        L = _lib.lib()
        n = (hi - lo) * BLOCK_M
        sr = b.sorted_rows.data_ptr() + 4 * lo * BLOCK_M
        be = b.block_expert.data_ptr() + 4 * lo
        npd = self._npad_dev.data_ptr() + 4 * gi
        hs = b.h.data_ptr() + 2 * lo * BLOCK_M * I
        _lib.check(L.ssb_sorted_gate_up(b.x_sorted.data_ptr() + 2 * lo * BLOCK_M * H, H, I, _lib.ptr(b.row_token),
                                        b.rows, sr, be, npd, n, _lib.ptr(self._ptr_dev), n_local, shared_local, hs,
                                        _lib.ptr(b.err), st), "sweep gate_up")
        _lib.check(L.ssb_sorted_down(hs, b.rows, H, I, _lib.ptr(b.row_weight), sr, be, npd, n, _lib.ptr(self._ptr_dev),
                                     n_local, shared_local, _lib.ptr(b.out_rows), _lib.ptr(b.err), st), "sweep down")


def _copy_async(dst: int, src: int, nbytes: int, stream):
    """One asynchronous copy of a pinned host record into a staging slot on `stream` (ssb_copy_async)."""
    _lib.check(_lib.lib().ssb_copy_async(dst, src, nbytes, stream.cuda_stream), "record copy")


def resident_from_pool(pool, layer: int) -> dict:
    """{expert: device address} of a SlotPool's resident records of `layer` (one small device-to-host read)."""
    m = pool.map[layer * pool.experts:(layer + 1) * pool.experts].cpu().numpy()
    sp = pool.slot_ptr.cpu().numpy()
    return {int(e): int(sp[s]) for e, s in enumerate(m) if s >= 0}
