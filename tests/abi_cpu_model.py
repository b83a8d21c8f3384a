"""A CPU model of the C ABI (include/slotstream_b200.h) built from the oracle -- TEST INFRASTRUCTURE ONLY.

``install(monkeypatch)`` points ``slotstream_b200._lib`` at this model: ``ptr`` passes the tensor itself instead
of its device address, every ``ssb_*`` entry point the drop-in modules call is computed here on CPU tensors with
the oracle's arithmetic, and record addresses (``group_ptr`` / ``slot_ptr`` entries) are looked up in a registry
of host records. The Python mirrors then run their own argument checks, buffer handling and C-ABI calls exactly
as on a GPU, so the reference's callers can drive them on a machine without one. It is never used by the product
package; the kernels themselves are checked against the oracle by the ``gpu`` tests.
"""
import numpy as np
import torch

from oracle import moe_oracle as O


def _np(t):
    return t.detach().contiguous().numpy()


def _bits(t):
    """bf16 tensor -> uint16 bit patterns."""
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)


class Records:
    """Host records addressable by integer address (their tensor's data_ptr), like records in pool slots."""

    def __init__(self, layout):
        self.layout = layout
        self.by_addr = {}
        self._f32 = {}
        self._bf = {}

    def add(self, rec_u8: torch.Tensor) -> int:
        a = int(rec_u8.data_ptr())
        self.by_addr[a] = rec_u8
        return a

    def dense_f32(self, addr):
        a = int(addr)
        if a not in self._f32:
            self._f32[a] = O.record_dense(self.layout, _np(self.by_addr[a]), np.float32)
        return self._f32[a]

    def dense_bf16(self, addr):
        """The dequantised pieces rounded to bf16 (the prefill kernels' weight tiles), as fp64."""
        a = int(addr)
        if a not in self._bf:
            self._bf[a] = tuple(O.round_bf16(m).astype(np.float64) for m in self.dense_f32(a))
        return self._bf[a]


class CpuAbi:
    def __init__(self, records: Records):
        self.recs = records
        self.calls = []

    def _log(self, name):
        self.calls.append(name)

    # ---- kernels/topk_stable.py
    def ssb_topk_stable(self, scores, n_valid, rows, n, k, out_idx, out_val, stream):
        self._log("ssb_topk_stable")
        idx, val = O.topk_stable(_np(scores), k, None if n_valid is None else _np(n_valid))
        out_idx.copy_(torch.from_numpy(idx))
        if out_val is not None:
            out_val.copy_(torch.from_numpy(val))
        return 0

    # ---- kernels/moe_align.py (+ align_rows of fused_moe_affine)
    def ssb_moe_align(self, row_expert, rows, expert_map, map_len, num_local, block_m, sorted_rows, block_expert,
                      num_padded, stream):
        self._log("ssb_moe_align")
        le = _np(row_expert).astype(np.int64)
        if expert_map is not None:
            m = _np(expert_map)
            ok = (le >= 0) & (le < map_len)
            le = np.where(ok, m[np.clip(le, 0, map_len - 1)], -1)
        sr, be, npd = O.moe_align(le, num_local, block_m)
        sorted_rows.copy_(torch.from_numpy(sr))
        block_expert.copy_(torch.from_numpy(be))
        num_padded.copy_(torch.from_numpy(npd))
        return 0

    def _aligned_rows(self, sorted_rows, block_expert, num_padded, rows, block_m=256):
        """(row, local expert) of every real row in the aligned blocks."""
        sr, be, n = _np(sorted_rows), _np(block_expert), int(_np(num_padded)[0])
        out = []
        for m in range(n):
            e = int(be[m // block_m])
            r = int(sr[m])
            if e >= 0 and r < rows:
                out.append((r, e))
        return out

    # ---- kernels/fused_moe_affine.py: the reference's prefill rounding path (bf16 weight tiles and h)
    def ssb_fused_moe_gate_up(self, x, tokens, hidden, inter, row_token, rows, sorted_rows, block_expert, num_padded,
                              padded_len, group_ptr, n_groups, h_buf, err, stream):
        self._log("ssb_fused_moe_gate_up")
        xf = O.bf16_to_f32(_bits(x)).astype(np.float64)
        tok, gp = _np(row_token), _np(group_ptr)
        h = _bits(h_buf).copy()
        for r, e in self._aligned_rows(sorted_rows, block_expert, num_padded, rows):
            g, u, _ = self.recs.dense_bf16(gp[e])
            xr = xf[int(tok[r])]
            gg, uu = (g @ xr).astype(np.float32), (u @ xr).astype(np.float32)
            h[r] = O.f32_to_bf16(gg.astype(np.float64) / (1.0 + np.exp(-gg.astype(np.float64))) * uu)
        h_buf.copy_(torch.from_numpy(h.view(np.int16)).view(torch.bfloat16))
        return 0

    def ssb_fused_moe_down(self, h_buf, rows, hidden, inter, row_weight, sorted_rows, block_expert, num_padded,
                           padded_len, group_ptr, n_groups, out_rows, err, stream):
        self._log("ssb_fused_moe_down")
        hb = O.bf16_to_f32(_bits(h_buf)).astype(np.float64)
        wt, gp = _np(row_weight), _np(group_ptr)
        for r, e in self._aligned_rows(sorted_rows, block_expert, num_padded, rows):
            d = self.recs.dense_bf16(gp[e])[2]
            out_rows[r] = torch.from_numpy(((d @ hb[r]).astype(np.float32) * np.float32(wt[r])).astype(np.float32))
        return 0

    def ssb_combine_rank_order(self, rows, tokens, k, hidden, out, stream):
        self._log("ssb_combine_rank_order")
        out.copy_(torch.from_numpy(O.combine_rank_order(_np(rows), tokens, k)))
        return 0

    # ---- kernels/moe_gemv_affine.py: exact dequant, fp32 results
    def ssb_moe_decode(self, x, x_dtype, expert_ids, weights, rows, topk, hidden, inter, layer, map_t, map_len,
                       slot_ptr_t, n_slots, h_buf, o_buf, out, err, stream):
        self._log("ssb_moe_decode")
        xf = _np(x.float()).astype(np.float64)
        ids, w, m, sp = _np(expert_ids), _np(weights), _np(map_t), _np(slot_ptr_t)
        res = np.zeros((rows, hidden), dtype=np.float64)
        for r in range(rows):
            for j in range(topk):
                slot = int(m[layer * 512 + int(ids[r, j])])
                g, u, d = (a.astype(np.float64) for a in self.recs.dense_f32(sp[slot]))
                h = O.silu64(g @ xf[r]) * (u @ xf[r])
                res[r] += float(w[r, j]) * (d @ h)
        out.copy_(torch.from_numpy(res.astype(np.float32)))
        return 0

    # ---- kernels/gemv_affine.py
    def ssb_gemv_affine(self, x, x_dtype, rows, q, s, b, n, k, bits, gs, out, stream):
        self._log("ssb_gemv_affine")
        w = O.dequant(_np(q).view(np.uint32), _bits(s), _bits(b), bits, gs, np.float64)
        out.copy_(torch.from_numpy((_np(x.float()).astype(np.float64) @ w.T).astype(np.float32)))
        return 0

    def ssb_gemv_dense(self, x, x_dtype, rows, w, n, k, out, stream):
        self._log("ssb_gemv_dense")
        wf = O.bf16_to_f32(_bits(w)).astype(np.float64)
        out.copy_(torch.from_numpy((_np(x.float()).astype(np.float64) @ wf.T).astype(np.float32)))
        return 0


def install(monkeypatch, records: Records) -> CpuAbi:
    from slotstream_b200 import _lib
    model = CpuAbi(records)
    monkeypatch.setattr(_lib, "lib", lambda: model)
    monkeypatch.setattr(_lib, "ptr", lambda t: t)
    monkeypatch.setattr(_lib, "stream", lambda: None)
    monkeypatch.setattr(_lib, "smem", lambda name: -1)
    return model
