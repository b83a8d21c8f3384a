"""Oracle-backed per-rank compute for the expert-parallel exchange tests on CPU (gloo).

Implements the step interface that slotstream_b200.ep.ep_forward drives (route, shared, plan, gather, unpack,
experts, combine_rows, combine) with the numpy oracle, so the real exchange protocol -- counts all-to-all,
all-to-all-v of rows and metadata, the return all-to-all -- runs unchanged on CPU tensors.
"""
import numpy as np
import torch

from oracle import ep_oracle as EO
from oracle import moe_oracle as O
from slotstream_b200.ep import Entries, Plan


def bits_to_bf16(b):
    return torch.from_numpy(np.ascontiguousarray(b, dtype=np.uint16).view(np.int16)).view(torch.bfloat16)


def bf16_to_bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def entry_row(layout, dense, x_row, w):
    """One routed entry in fp64 exact dequant: w * D (silu(G x) * (U x)), returned as fp32."""
    g, u, d = dense
    x = np.asarray(x_row, np.float64)
    h = O.silu64(g @ x) * (u @ x)
    return (w * (d @ h)).astype(np.float32)


class CpuOps:
    def __init__(self, layout, recs, shared_rec, rw_bits, sg_bits, k, experts, n_ranks, rank, strided=True,
                 bias=None):
        self.layout, self.k, self.n_experts, self.G, self.rank, self.strided = layout, k, experts, n_ranks, rank, strided
        self.rw, self.sg, self.bias = rw_bits, sg_bits, bias
        epr = experts // n_ranks
        self.owned = ([rank + n_ranks * i for i in range(epr)] if strided else
                      list(range(rank * epr, (rank + 1) * epr)))
        self.dense = {e: O.record_dense(layout, recs[e]) for e in self.owned}
        self.sh_dense = O.record_dense(layout, shared_rec, np.float32)

    def route(self, x):
        ids, w, _ = O.router(bf16_to_bits(x), self.rw, self.k, bias=self.bias)
        return torch.from_numpy(ids.astype(np.int32)), torch.from_numpy(w.astype(np.float32)), None

    def shared(self, x, sh_gate):
        sh = O.shared_expert(bf16_to_bits(x), *self.sh_dense, self.sg)
        return torch.from_numpy(np.asarray(sh, np.float32))

    def plan(self, ids, w):
        dc, st, sm, ts, te = EO.plan(ids.numpy(), w.numpy(), self.n_experts, self.G, self.strided)
        return Plan(*(torch.from_numpy(a) for a in (dc, st, sm, ts, te)))

    def gather(self, x, idx):
        return x[idx.long()].contiguous()

    def unpack(self, meta, src_row_off, src_entry_off, n_entries):
        arrs = EO.unpack(meta.numpy(), src_row_off, src_entry_off, self.k)
        assert arrs[0].size == n_entries
        return Entries(*(torch.from_numpy(a) for a in arrs))

    def experts(self, recv_x, ent):
        xf = O.bf16_to_f32(bf16_to_bits(recv_x))
        rows = [entry_row(self.layout, self.dense[self.owned[int(le)]], xf[int(r)], float(w))
                for le, r, w in zip(ent.row_expert.numpy(), ent.row_token.numpy(), ent.row_weight.numpy())]
        return torch.from_numpy(np.array(rows, np.float32).reshape(-1, self.layout.hidden))

    def combine_rows(self, out_rows, ent, bf16=False):
        part = EO.combine_rows(out_rows.numpy(), ent.row_e0.numpy(), ent.row_cnt.numpy())
        if bf16:   # the bf16 return, carried as bf16-valued fp32 (gloo moves fp32)
            part = O.round_bf16(part).astype(np.float32)
        return torch.from_numpy(part)

    def combine(self, ret, plan, ids, ret_entry_off, sh, exact, bf16=False):
        routed = EO.combine(ret.numpy(), plan.tok_slot.numpy(), plan.tok_entry.numpy(), ret_entry_off, ids.numpy(),
                            self.n_experts, self.G, self.strided, exact)
        self.routed = torch.from_numpy(routed)
        y = O.round_bf16(O.round_bf16(routed).astype(np.float64) + O.round_bf16(sh.numpy()).astype(np.float64))
        return bits_to_bf16(O.f32_to_bf16(np.asarray(y, np.float32)))


def single_rank_reference(layout, recs, shared_rec, rw_bits, sg_bits, k, x_bits, bias=None):
    """The one-GPU layer on the same tokens: routed = sum over j in rank order of the entry rows, in fp32."""
    ids, w, _ = O.router(x_bits, rw_bits, k, bias=bias)
    xf = O.bf16_to_f32(x_bits)
    dense = {}
    routed = np.zeros((x_bits.shape[0], layout.hidden), np.float32)
    for t in range(x_bits.shape[0]):
        for j in range(k):
            e = int(ids[t, j])
            if e not in dense:
                dense[e] = O.record_dense(layout, recs[e])
            routed[t] = (routed[t] + entry_row(layout, dense[e], xf[t], float(w[t, j]))).astype(np.float32)
    return routed
