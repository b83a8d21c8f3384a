"""CPU restatement of the expert-parallel dispatch/combine bookkeeping -- TEST INFRASTRUCTURE ONLY.

The reference runs on one GPU and has no expert-parallel path, so there is no reference file to follow here;
these functions restate, in plain numpy loops, the plan / unpack / combine contract of the B200 EP kernels
(send rows ordered by destination then token, one metadata row per (token, destination), compacted entries in
rank-k order) so the kernels and the host exchange can be checked. The per-token sums keep the rank order of
the reference's combine_rank_order (slotstream_spark/kernels/fused_moe_affine.py:164-172).
Only tests/ import this module.
"""
import numpy as np


def owner(e, experts, n_ranks, strided):
    epr = experts // n_ranks
    return (e % n_ranks, e // n_ranks) if strided else (e // epr, e % epr)


def plan(ids, w, experts, n_ranks, strided):
    """-> dest_count [G, 2], send_token [n], send_meta [n, 2k+2] int32 (weights as float bits), tok_slot [T, G],
    tok_entry [T, G]."""
    t_n, k = ids.shape
    G = n_ranks
    rows = [[] for _ in range(G)]          # per destination: (token, meta)
    ecount = [0] * G
    tok_entry = np.full((t_n, G), -1, np.int32)
    for t in range(t_n):
        per = {}
        for j in range(k):
            d, le = owner(int(ids[t, j]), experts, G, strided)
            per.setdefault(d, []).append((j, le))
        for d in sorted(per):
            meta = np.zeros(2 * k + 2, np.int32)
            meta[:k] = -1
            for j, le in per[d]:
                meta[j] = le
                meta[k + j] = np.float32(w[t, j]).view(np.int32)
            meta[2 * k] = ecount[d]
            meta[2 * k + 1] = len(per[d])
            tok_entry[t, d] = ecount[d]
            ecount[d] += len(per[d])
            rows[d].append((t, meta))
    dest_count = np.array([[len(rows[d]), ecount[d]] for d in range(G)], np.int32)
    send_token, send_meta = [], []
    tok_slot = np.full((t_n, G), -1, np.int32)
    for d in range(G):
        for t, meta in rows[d]:
            tok_slot[t, d] = len(send_token)
            send_token.append(t)
            send_meta.append(meta)
    meta_arr = np.array(send_meta, np.int32).reshape(-1, 2 * k + 2)
    return dest_count, np.array(send_token, np.int32), meta_arr, tok_slot, tok_entry


def unpack(meta, src_row_off, src_entry_off, k):
    """-> row_expert, row_token, row_weight [n_entries], row_e0, row_cnt [rows]."""
    n = meta.shape[0]
    n_entries = int(src_entry_off[-1])
    row_expert = np.zeros(n_entries, np.int32)
    row_token = np.zeros(n_entries, np.int32)
    row_weight = np.zeros(n_entries, np.float32)
    row_e0 = np.zeros(n, np.int64)
    row_cnt = np.zeros(n, np.int32)
    for r in range(n):
        s = max(i for i in range(len(src_row_off) - 1) if src_row_off[i] <= r)
        e0 = int(src_entry_off[s]) + int(meta[r, 2 * k])
        row_e0[r], row_cnt[r] = e0, meta[r, 2 * k + 1]
        p = e0
        for j in range(k):
            if meta[r, j] >= 0:
                row_expert[p], row_token[p] = meta[r, j], r
                row_weight[p] = meta[r, k + j:k + j + 1].view(np.float32)[0]
                p += 1
    return row_expert, row_token, row_weight, row_e0, row_cnt


def combine_rows(out_rows, row_e0, row_cnt):
    part = np.zeros((len(row_e0), out_rows.shape[1]), np.float32)
    for r in range(len(row_e0)):
        for i in range(int(row_cnt[r])):
            part[r] = (part[r] + out_rows[row_e0[r] + i]).astype(np.float32)
    return part


def combine(ret, tok_slot, tok_entry, ret_entry_off, ids, experts, n_ranks, strided, exact):
    """Routed fp32 [T, H]: partial rows summed over destinations ascending, or (exact) entry rows summed in
    router-rank order."""
    t_n, k = ids.shape
    out = np.zeros((t_n, ret.shape[1]), np.float32)
    for t in range(t_n):
        if exact:
            seen = [0] * n_ranks
            for j in range(k):
                d, _ = owner(int(ids[t, j]), experts, n_ranks, strided)
                out[t] = (out[t] + ret[ret_entry_off[d] + tok_entry[t, d] + seen[d]]).astype(np.float32)
                seen[d] += 1
        else:
            for d in range(n_ranks):
                if tok_slot[t, d] >= 0:
                    out[t] = (out[t] + ret[tok_slot[t, d]]).astype(np.float32)
    return out
