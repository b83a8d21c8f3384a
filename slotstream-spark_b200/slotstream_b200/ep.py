"""Expert-parallel prefill MoE layer: experts sharded by id over the ranks of a process group.

The reference runs on one GPU and has no multi-GPU path; this module adds the one exchange the MoE layer has
when its experts are spread over G GPUs. Every rank routes its own tokens (router and shared expert are
replicated), then:

1. plan      -- dedupe (token, destination rank), order rows by destination then token, one metadata row per
                sent token: the local expert and weight of each top-k choice that rank owns (-1 otherwise),
                the row's entry base inside the destination block and its entry count;
2. dispatch  -- all-to-all of the per-destination (rows, entries) counts, then all-to-all-v of the bf16 token
                rows and of the metadata;
3. experts   -- the receiving rank compacts the valid (row, choice) entries and runs the grouped tcgen05
                GEMMs (gate_up + SwiGLU, down x weight) over its own experts;
4. combine   -- default: each received row's entries are summed in rank-k order and that fp32 partial goes
                back; the home rank adds the partials of its destinations in rank order. exact: the entry
                rows themselves go back and the home rank sums every token's k rows in router-rank order,
                which reproduces the one-GPU layer bit for bit (kernels/fused_moe_affine.py:164-172);
5. output    -- y = bf16(bf16(routed) + bf16(shared)), as the one-GPU layer.

Placement: ``strided`` puts expert e on rank e % G (local index e // G), spreading the popular low ids of a
Zipf-skewed router over all ranks; contiguous puts it on rank e // (E / G). ``balanced_labels`` goes further
from measured routing counts: it relabels the experts so that the strided placement of the new labels gives
every rank about the same expected number of rows (the kernels are unchanged; the router's weight rows and
logit bias are permuted into label order, and each rank holds the records of the experts its labels name).

The exchange runs through torch.distributed collectives only (NCCL on GPUs; the same code drives gloo on CPU
tensors in the host-side tests), with the per-destination counts copied to the host to size the all-to-all-v
-- one host synchronisation per layer call, so this path is eager, not graph-captured.
"""
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _lib

MAX_RANKS = 8


def owner(e: int, experts: int, n_ranks: int, strided: bool) -> tuple[int, int]:
    """(rank, local index) of expert e."""
    epr = experts // n_ranks
    return (e % n_ranks, e // n_ranks) if strided else (e // epr, e % epr)


def owned_experts(rank: int, experts: int, n_ranks: int, strided: bool) -> list[int]:
    """Global ids of the experts rank `rank` owns, in local-index order."""
    epr = experts // n_ranks
    return [rank + n_ranks * i for i in range(epr)] if strided else list(range(rank * epr, (rank + 1) * epr))


def balanced_labels(counts, n_ranks: int):
    """Labels that balance the ranks' expected rows under the strided placement: experts are taken in decreasing
    order of their routing count (ties to the lower id) and each goes to the rank with the fewest rows so far that
    still has a free slot (E / G slots per rank); the expert in slot i of rank r gets label r + G * i.
    Returns (label int64 [E]: label of expert e, expert int64 [E]: expert of label l). Apply it by permuting the
    router's weight rows and logit bias with ``expert`` (row l = expert[l]) and giving rank r the records of
    ``expert[owned_experts(r, E, G, True)]``: the layer's outputs are those of the original router, except where
    two logits tie exactly (the stable top-k breaks ties by label)."""
    import numpy as np
    c = np.asarray(counts, dtype=np.int64)
    e_n = c.size
    if n_ranks < 1 or e_n % n_ranks:
        raise ValueError("the experts must divide evenly over the ranks")
    epr = e_n // n_ranks
    load = np.zeros(n_ranks, dtype=np.int64)
    used = np.zeros(n_ranks, dtype=np.int64)
    label = np.empty(e_n, dtype=np.int64)
    for e in np.lexsort((np.arange(e_n), -c)):
        free = np.flatnonzero(used < epr)
        r = int(free[np.argmin(load[free])])
        label[e] = r + n_ranks * used[r]
        used[r] += 1
        load[r] += c[e]
    expert = np.empty(e_n, dtype=np.int64)
    expert[label] = np.arange(e_n)
    return label, expert


@dataclass
class Plan:
    dest_count: torch.Tensor   # int32 [G, 2]: rows, entries per destination
    send_token: torch.Tensor   # int32 [rows sent]
    send_meta: torch.Tensor    # int32 [rows sent, 2k + 2]
    tok_slot: torch.Tensor     # int32 [T, G]: send row of (t, d) or -1
    tok_entry: torch.Tensor    # int32 [T, G]: entry base of (t, d) in d's block or -1


@dataclass
class Entries:
    row_expert: torch.Tensor   # int32 [n]: local expert of entry
    row_token: torch.Tensor    # int32 [n]: received row of entry
    row_weight: torch.Tensor   # fp32 [n]
    row_e0: torch.Tensor       # int64 [received rows]: first entry of the row
    row_cnt: torch.Tensor      # int32 [received rows]


def _prefix(v: list[int]) -> list[int]:
    out, s = [0], 0
    for x in v:
        s += x
        out.append(s)
    return out


class ExchangeError(RuntimeError):
    """The exchanged per-destination counts are inconsistent: this rank stops before posting any transfer sized by
    them (its peers' next collective then fails with the process group's timeout instead of hanging)."""


def _check_counts(counts, k, direction):
    """counts[part][rank] = (rows, entries): every sent row carries 1..k entries of its token."""
    for i, part in enumerate(counts):
        for d, (rows, ent) in enumerate(part):
            if rows < 0 or ent < rows or ent > rows * k:
                raise ExchangeError(f"part {i}: counts {direction} rank {d} are inconsistent: {rows} rows, "
                                    f"{ent} entries (k = {k})")


def _host_read(t: torch.Tensor) -> list:
    """The values of a small tensor on the host. A CUDA tensor is copied by the SMs (ssb_copy_sm) into pinned host
    memory on the current stream, then that stream alone is waited on: a copy-engine transfer would queue behind a
    large transfer of another stream (the previous step's output leaving), and the host would wait for it."""
    if not t.is_cuda:
        return t.tolist()
    t = t.contiguous()
    h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    _lib.check(_lib.lib().ssb_copy_sm(h.data_ptr(), t.data_ptr(), t.numel() * t.element_size(), _lib.stream()),
               "counts to host")
    torch.cuda.current_stream().synchronize()
    return h.tolist()


def ep_forward(ops, x: torch.Tensor, k: int, n_ranks: int, group=None, exact: bool = False,
               micro_batches: int = 1, partials_bf16: bool = False, phases: list | None = None):
    """One expert-parallel MoE layer over this rank's tokens x [T, H] -> y bf16 [T, H].
    ``ops`` supplies the per-rank compute (``CudaOps`` on B200); the exchange is the same for every backend.

    ``micro_batches`` = m > 1 splits the tokens into m contiguous parts with their own plans: the counts of
    all parts go in one all-to-all (still one host sync), every exchange is asynchronous, and part i's expert
    GEMMs are issued after part i+1's dispatch and before part i-1's return, so on NCCL the transfers of one
    part overlap the math of its neighbour. Every token's arithmetic is the same as with m = 1. Every rank must
    pass the same m; parts may be empty (a rank with fewer than m tokens, or none).

    ``partials_bf16`` (default mode only): the per-(token, destination) partial sums are rounded to bf16 before
    they go back, halving the return bytes; routed then differs from the fp32 return by the partials'
    rounding (a relative 2^-9 each).

    ``phases`` (a list, CUDA only) receives (name, event) pairs recorded on the current stream at the phase
    borders -- after routing, the plan, the count exchange and its host read, each part's dispatch, expert GEMMs,
    partial sums, return and combine -- so a caller can time the phases of one call; it also receives
    ("rows", received rows, received entries) of this rank."""
    G = n_ranks
    # every rank must post the same collectives: m depends only on the argument, never on this rank's token count
    # (a rank with fewer tokens than m, or none, sends empty parts)
    m = max(1, int(micro_batches))
    reserve = getattr(ops, "sm_reserve", 0) if m > 1 and G > 1 else 0
    if reserve:
        ops.reserve_sms(reserve)   # the overlapped all-to-alls need SMs beside the persistent GEMMs
    try:
        return _ep_forward(ops, x, k, G, group, exact, m, bool(partials_bf16) and not exact, phases)
    finally:
        if reserve:
            ops.reserve_sms(0)


def _ep_forward(ops, x, k, G, group, exact, m, bf16, phases=None):
    def mark(name):
        if phases is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            phases.append((name, ev))

    mark("start")
    t_all = x.shape[0]
    ids, w, sh_gate = ops.route(x)
    mark("route")
    sh = ops.shared(x, sh_gate)
    bounds = [t_all * i // m for i in range(m + 1)]
    parts = [(bounds[i], bounds[i + 1]) for i in range(m)]
    plans = [ops.plan(ids[a:b], w[a:b]) for a, b in parts]
    mark("plan")
    send_counts = torch.stack([p.dest_count for p in plans], dim=1).contiguous()   # [G, m, 2]: per destination
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts.view(-1), send_counts.view(-1), group=group)
    both = _host_read(torch.cat([send_counts.view(-1), recv_counts.view(-1)]))   # the one host sync
    half = G * m * 2
    sc = [[both[(d * m + i) * 2:(d * m + i) * 2 + 2] for d in range(G)] for i in range(m)]
    rc = [[both[half + (d * m + i) * 2:half + (d * m + i) * 2 + 2] for d in range(G)] for i in range(m)]
    _check_counts(rc, k, "received from")
    _check_counts(sc, k, "sent to")
    if hasattr(ops, "synced"):
        ops.synced()   # every kernel of the previous step has run: its pinned host staging may be released
    mark("counts_exchange_and_host_read")
    if phases is not None:
        phases.append(("rows", sum(c[0] for r in rc for c in r), sum(c[1] for r in rc for c in r)))
    # dispatch every part (asynchronous: the math below waits only for its own part)
    sent = []
    for i, ((a, b), plan) in enumerate(zip(parts, plans)):
        send_rows, send_ent = [c[0] for c in sc[i]], [c[1] for c in sc[i]]
        recv_rows, recv_ent = [c[0] for c in rc[i]], [c[1] for c in rc[i]]
        n_send, n_recv = sum(send_rows), sum(recv_rows)
        plan.send_token, plan.send_meta = plan.send_token[:n_send], plan.send_meta[:n_send]
        send_x = ops.gather(x[a:b], plan.send_token)
        recv_x = x.new_empty((n_recv, x.shape[1]))
        recv_meta = plan.send_meta.new_empty((n_recv, plan.send_meta.shape[1]))
        works = [dist.all_to_all_single(recv_x, send_x, recv_rows, send_rows, group=group, async_op=True),
                 dist.all_to_all_single(recv_meta, plan.send_meta, recv_rows, send_rows, group=group,
                                        async_op=True)]
        sent.append((send_x, recv_x, recv_meta, works, send_rows, send_ent, recv_rows, recv_ent))
    # experts of each part as soon as its rows are in; its results go back asynchronously
    returned = []
    for i, (send_x, recv_x, recv_meta, works, send_rows, send_ent, recv_rows, recv_ent) in enumerate(sent):
        for wk in works:
            wk.wait()
        mark(f"dispatch{i}")
        entries = ops.unpack(recv_meta, _prefix(recv_rows), _prefix(recv_ent), sum(recv_ent))
        out_rows = ops.experts(recv_x, entries)
        mark(f"experts{i}")
        if exact:
            back = out_rows
            ret = out_rows.new_empty((sum(send_ent), out_rows.shape[1]))
            work = dist.all_to_all_single(ret, back, send_ent, recv_ent, group=group, async_op=True)
        else:
            back = ops.combine_rows(out_rows, entries, bf16=bf16)
            mark(f"partial_sums{i}")
            ret = back.new_empty((sum(send_rows), back.shape[1]))
            work = dist.all_to_all_single(ret, back, send_rows, recv_rows, group=group, async_op=True)
        returned.append((ret, back, work))
    ys, routed = [], []
    for i, ((a, b), plan) in enumerate(zip(parts, plans)):
        ret, _, work = returned[i]
        work.wait()
        mark(f"return{i}")
        send_ent = sent[i][5]
        off = _prefix(send_ent)[:G] if exact else None
        ys.append(ops.combine(ret, plan, ids[a:b], off, sh[a:b], exact=exact, bf16=bf16))
        mark(f"combine{i}")
        routed.append(ops.routed)
    if m == 1:
        return ys[0]
    ops.routed = torch.cat(routed)
    return torch.cat(ys)


class CudaOps:
    """The B200 kernels of one rank's share of an expert-parallel layer.

    ``group_ptr`` int64 [E / G]: record base of each owned expert in local-index order; ``shared_ptr``: record
    base of the shared expert; w_router bf16 [E, H] and sh_gate_w bf16 [H] are replicated on every rank."""

    def __init__(self, w_router, sh_gate_w, group_ptr, shared_ptr: int, k: int, inter: int, n_ranks: int,
                 strided: bool = True, bias=None, logits_round_bf16: bool = False, sm_reserve: int = 0):
        e, h = w_router.shape
        if n_ranks < 1 or n_ranks > MAX_RANKS or e % n_ranks:
            raise ValueError(f"need 1 <= n_ranks <= {MAX_RANKS} dividing the expert count")
        if group_ptr.dtype != torch.int64 or group_ptr.numel() != e // n_ranks or not group_ptr.is_cuda:
            raise ValueError("group_ptr must be a CUDA int64 [E / G] tensor")
        self.w_router, self.sh_gate_w, self.group_ptr = w_router, sh_gate_w, group_ptr
        self.k, self.hidden, self.inter, self.n_experts = k, h, inter, e
        self.G, self.epr, self.strided = n_ranks, e // n_ranks, bool(strided)
        self.bias, self.round = bias, logits_round_bf16
        dev = w_router.device
        self.shared_ptr = torch.tensor([int(shared_ptr)], dtype=torch.int64, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self._held = []            # pinned host staging of the current step (see _to_device)
        self._static = {}
        self._side, self._sh_ready = None, None
        self.sm_reserve = int(sm_reserve)   # SMs left to the collectives while micro-batches overlap

    def reserve_sms(self, n: int):
        _lib.check(_lib.lib().ssb_set_gemm_sm_reserve(int(n)), "set gemm sm reserve")

    # ---------------------------------------------------------------- helpers
    def _aligned(self, row_expert, num_local):
        from .kernels.fused_moe_affine import BLOCK_M
        from .kernels.moe_align import moe_align
        return moe_align(row_expert, num_local, BLOCK_M)

    def _experts(self, a, tokens, row_token, row_weight, row_expert, group_ptr, n_groups, shared_local):
        n = row_token.numel()
        out = torch.empty((n, self.hidden), dtype=torch.float32, device=a.device)
        if n == 0:
            return out
        sr, be, npd = self._aligned(row_expert, n_groups)
        x_sorted = torch.empty((sr.numel(), self.hidden), dtype=torch.bfloat16, device=a.device)
        h_sorted = torch.empty((sr.numel(), self.inter), dtype=torch.bfloat16, device=a.device)
        L, P = _lib.lib(), _lib.ptr
        _lib.check(L.ssb_prefill_experts(P(a), tokens, self.hidden, self.inter, P(row_token), P(row_weight), n, P(sr),
                                         P(be), P(npd), sr.numel(), P(group_ptr), n_groups, shared_local, P(x_sorted),
                                         P(h_sorted), P(out), P(self.err), _lib.stream()), "prefill experts")
        return out

    # ---------------------------------------------------------------- the steps of ep_forward
    def route(self, x):
        t, h = x.shape
        e, k = self.n_experts, self.k
        L, P, st = _lib.lib(), _lib.ptr, _lib.stream()
        ld = e + 4
        lg = torch.empty(t * ld, dtype=torch.float32, device=x.device)
        _lib.check(L.ssb_gemm_dense(P(x), t, h, P(self.w_router), e, P(lg), ld, st), "router gemm")
        _lib.check(L.ssb_router_logits(P(x), P(self.sh_gate_w), None, t, h, 1, ld, lg.data_ptr() + 4 * e, st),
                   "shared gate logits")
        ids = torch.empty((t, k), dtype=torch.int32, device=x.device)
        w = torch.empty((t, k), dtype=torch.float32, device=x.device)
        sh_gate = torch.empty(t, dtype=torch.float32, device=x.device)
        flags = _lib.ROUTER_SHARED_GATE | (_lib.ROUTER_ROUND_BF16 if self.round else 0)
        _lib.check(L.ssb_router_select(P(lg), ld, t, e, k, P(self.bias), flags, P(ids), P(w), None, P(sh_gate), st),
                   "router select")
        return ids, w, sh_gate

    def shared(self, x, sh_gate):
        """The shared expert of this rank's tokens, on a side stream: it overlaps the exchange and is joined
        in ``combine``."""
        t = x.shape[0]
        key = ("shared", t)
        if key not in self._static:
            self._static[key] = (torch.arange(t, dtype=torch.int32, device=x.device),
                                 torch.zeros(t, dtype=torch.int32, device=x.device))
        tok, zero = self._static[key]
        main = torch.cuda.current_stream()
        if self._side is None:
            self._side = torch.cuda.Stream()
        self._side.wait_stream(main)
        with torch.cuda.stream(self._side):
            out = self._experts(x, t, tok, sh_gate, zero, self.shared_ptr, 1, 0)
        sh_gate.record_stream(self._side)
        out.record_stream(main)
        self._sh_ready = torch.cuda.Event()
        self._sh_ready.record(self._side)
        return out

    def plan(self, ids, w):
        t, k, G = ids.shape[0], self.k, self.G
        dev = ids.device
        cap = t * min(G, k)
        p = Plan(torch.empty((G, 2), dtype=torch.int32, device=dev), torch.empty(cap, dtype=torch.int32, device=dev),
                 torch.empty((cap, 2 * k + 2), dtype=torch.int32, device=dev),
                 torch.empty((t, G), dtype=torch.int32, device=dev), torch.empty((t, G), dtype=torch.int32, device=dev))
        P = _lib.ptr
        _lib.check(_lib.lib().ssb_ep_plan(P(ids), P(w), t, k, self.epr, G, int(self.strided), P(p.dest_count),
                                          P(p.send_token), P(p.send_meta), P(p.tok_slot), P(p.tok_entry), P(self.err),
                                          _lib.stream()), "ep plan")
        return p   # sized for the worst case; ep_forward trims to the counts it reads back

    def _to_device(self, h: torch.Tensor) -> torch.Tensor:
        """A small host array on the device, copied by the SMs from pinned memory (ssb_copy_sm) so that it does not
        queue on a copy engine behind the next step's activations; the pinned copy is held until the next step's
        host sync (``synced``) proves the kernel has read it."""
        hp = h.contiguous().pin_memory()
        d = torch.empty(hp.shape, dtype=hp.dtype, device=self.group_ptr.device)
        _lib.check(_lib.lib().ssb_copy_sm(d.data_ptr(), hp.data_ptr(), hp.numel() * hp.element_size(), _lib.stream()),
                   "offsets to device")
        self._held.append(hp)
        return d

    def synced(self):
        self._held = []

    def gather(self, x, idx):
        out = x.new_empty((idx.numel(), x.shape[1]))
        P = _lib.ptr
        _lib.check(_lib.lib().ssb_gather_rows(P(x), x.shape[0], P(idx), idx.numel(), x.shape[1] * x.element_size(),
                                              P(out), P(self.err), _lib.stream()), "gather rows")
        return out

    def unpack(self, meta, src_row_off, src_entry_off, n_entries):
        dev, n = meta.device, meta.shape[0]
        ent = Entries(torch.empty(n_entries, dtype=torch.int32, device=dev),
                      torch.empty(n_entries, dtype=torch.int32, device=dev),
                      torch.empty(n_entries, dtype=torch.float32, device=dev),
                      torch.empty(n, dtype=torch.int64, device=dev), torch.empty(n, dtype=torch.int32, device=dev))
        # offsets through pinned host memory: a copy from pageable memory blocks the host until a copy engine
        # takes it, behind whatever large transfer (the next step's activations) that engine is running
        ro = self._to_device(torch.tensor(src_row_off, dtype=torch.int32))
        eo = self._to_device(torch.tensor(src_entry_off, dtype=torch.int64))
        P = _lib.ptr
        _lib.check(_lib.lib().ssb_ep_unpack(P(meta), n, self.k, P(ro), P(eo), self.G, n_entries, P(ent.row_expert),
                                            P(ent.row_token), P(ent.row_weight), P(ent.row_e0), P(ent.row_cnt),
                                            P(self.err), _lib.stream()), "ep unpack")
        return ent

    def experts(self, recv_x, ent):
        return self._experts(recv_x, recv_x.shape[0], ent.row_token, ent.row_weight, ent.row_expert, self.group_ptr,
                             self.epr, -1)

    def combine_rows(self, out_rows, ent, bf16: bool = False):
        n = ent.row_e0.numel()
        partial = torch.empty((n, self.hidden), dtype=torch.bfloat16 if bf16 else torch.float32,
                              device=out_rows.device)
        P = _lib.ptr
        fn = _lib.lib().ssb_combine_rows_bf16 if bf16 else _lib.lib().ssb_combine_rows
        _lib.check(fn(P(out_rows), P(ent.row_e0), P(ent.row_cnt), n, self.hidden, P(partial), _lib.stream()),
                   "combine rows")
        return partial

    def combine(self, ret, plan, ids, ret_entry_off, sh, exact, bf16: bool = False):
        t = ids.shape[0]
        dev = ids.device
        self.routed = torch.empty((t, self.hidden), dtype=torch.float32, device=dev)
        y = torch.empty((t, self.hidden), dtype=torch.bfloat16, device=dev)
        reo = self._to_device(torch.tensor(ret_entry_off, dtype=torch.int64)) if ret_entry_off is not None else None
        if self._sh_ready is not None:
            torch.cuda.current_stream().wait_event(self._sh_ready)   # the shared expert's rows (side stream)
        P = _lib.ptr
        if bf16 and not exact:   # bf16 partial rows
            _lib.check(_lib.lib().ssb_ep_combine_bf16(P(ret), P(plan.tok_slot), P(ids), t, self.k, self.epr, self.G,
                                                      int(self.strided), self.hidden, P(sh), P(self.routed), P(y),
                                                      _lib.stream()), "ep combine")
            return y
        _lib.check(_lib.lib().ssb_ep_combine(P(ret), P(plan.tok_slot), P(plan.tok_entry), P(reo), P(ids), t, self.k,
                                             self.epr, self.G, int(self.strided), int(exact), self.hidden, P(sh),
                                             P(self.routed), P(y), _lib.stream()), "ep combine")
        return y
