"""CPU oracle for the routed-expert MoE hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the arithmetic of fortil/slotstream-spark's MoE path so the CUDA kernels
can be checked against it. Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
and reference arms may import it; the product package never does.

Every function cites the reference file:line it restates. Parity is pinned: ``tests/test_oracle.py`` checks
these functions against golden vectors that ``tests/golden/make_golden.py`` produced by importing the
reference's own code (affine_ref, moe_align, combine_rank_order, reference_torch.moe_ref and the stable
top-k rule of its test suite) on the same seeded inputs.

bf16 values travel as uint16 bit patterns; fp32 and fp64 as numpy floats.
"""
import numpy as np


# ------------------------------------------------------------------ bf16 helpers
def bf16_to_f32(b):
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a):
    """Round-to-nearest-even fp32 -> bf16 bits; NaN stays NaN."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32)
    r = ((u >> 16) & 1) + np.uint32(0x7FFF)
    out = ((u + r) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out


def round_bf16(a):
    """fp32/fp64 values -> nearest bf16 value as fp32 (via fp32 first, like torch's .to(bfloat16) of an fp32)."""
    return bf16_to_f32(f32_to_bf16(np.asarray(a, dtype=np.float32)))


# ------------------------------------------------------------------ affine 4-bit (kernels/affine_ref.py)
def unpack(q_u32, bits=4):
    """uint32/int32 [N, K*bits/32] -> uint8 [N, K]; element i at bits [bits*i, bits*(i+1)) of the
    little-endian stream, so the low nibble is the even element (kernels/affine_ref.py:10-19)."""
    b = np.ascontiguousarray(q_u32).view(np.uint8)
    if bits == 8:
        return b.copy()
    if bits != 4:
        raise ValueError("bits must be 4 or 8")
    out = np.empty(b.shape[:-1] + (b.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = b & 15
    out[..., 1::2] = b >> 4
    return out


def dequant(q_u32, s_bits, b_bits, bits=4, gs=64, dtype=np.float32):
    """q [N, K*bits/32], s/b bf16 bits [N, K/gs] -> [N, K] = q*s + b, computed in fp32 like
    kernels/affine_ref.py:22-31 (dtype=np.float64 gives the exact value of q*s + b)."""
    u = unpack(q_u32, bits).astype(dtype)
    n, k = u.shape
    if k % gs or s_bits.shape != (n, k // gs) or b_bits.shape != (n, k // gs):
        raise ValueError("shape mismatch")
    s = np.repeat(bf16_to_f32(s_bits).astype(dtype), gs, axis=1)
    b = np.repeat(bf16_to_f32(b_bits).astype(dtype), gs, axis=1)
    return u * s + b


def gemv_ref64(x, w):
    """x [R, K] @ w[N, K]^T in fp64 (kernels/affine_ref.py:39-40)."""
    return np.asarray(x, dtype=np.float64) @ np.asarray(w, dtype=np.float64).T


# ------------------------------------------------------------------ record access
def record_pieces(layout, rec):
    """uint8 record -> [(q uint32 [n, k/8], s bf16 [n, k/gs], b bf16 [n, k/gs])] of gate, up, down
    in the piece order of kernels/moe_gemv_affine.py:11-13 / :21-25."""
    offs = layout.offsets()
    out = []
    for p, (n, k) in enumerate(layout.piece_shapes()):
        ow, os_, ob = offs[3 * p:3 * p + 3]
        ng = k // layout.gs
        out.append((rec[ow:ow + n * k // 2].view(np.uint32).reshape(n, k // 8),
                    rec[os_:os_ + n * ng * 2].view(np.uint16).reshape(n, ng),
                    rec[ob:ob + n * ng * 2].view(np.uint16).reshape(n, ng)))
    return out


def record_dense(layout, rec, dtype=np.float64):
    """(gate [I, H], up [I, H], down [H, I]) dequantized; fp64 is exact."""
    return tuple(dequant(q, s, b, 4, layout.gs, dtype) for (q, s, b) in record_pieces(layout, rec))


# ------------------------------------------------------------------ stable top-k (kernels/topk_stable.py)
def order_keys(x_f32):
    """Order-preserving uint32 key of fp32 bits, NaN -> 0 (lowest); kernels/topk_stable.py:5-8, :36-41;
    the same rule as tests/t0/test_topk_stable.py:14-19."""
    b = np.ascontiguousarray(x_f32, dtype=np.float32).view(np.uint32).astype(np.int64)
    key = np.where(b >= 0x80000000, (~b) & 0xFFFFFFFF, b ^ 0x80000000)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    return np.where(nan, 0, key)


def topk_stable(scores, k, n_valid=None):
    """scores fp32 [R, N] -> (idx int32 [R, k], val fp32 [R, k]).

    Largest keys first, ties to the lower index; k <= 16 sorted by (value desc, index asc), larger k by
    index asc; rows with fewer than k valid entries pad with (-1, -inf)
    (kernels/topk_stable.py:1-13, :42-82; tests/t0/test_topk_stable.py:22-31)."""
    scores = np.ascontiguousarray(scores, dtype=np.float32)
    r, n = scores.shape
    idx = np.full((r, k), -1, dtype=np.int32)
    val = np.full((r, k), -np.inf, dtype=np.float32)
    for row in range(r):
        nv = n if n_valid is None else max(0, min(int(n_valid[row]), n))
        key = order_keys(scores[row, :nv])
        order = np.argsort(-key, kind="stable")[:k]
        sel = order if k <= 16 else np.sort(order)
        idx[row, :sel.size] = sel
        val[row, :sel.size] = scores[row, sel]
    return idx, val


# ------------------------------------------------------------------ router (model/layers.py:336-348)
def router(x_bf16, w_bf16, k, bias=None, logits_round_bf16=False):
    """Router of one layer: logits = x W^T (+ bias), softmax in fp32, stable top-k, renormalise.

    model/layers.py:339-347 and model/reference_torch.py:121-124. Logits are exact (fp64 sum of exact
    bf16 products) rounded to fp32 -- the "router math is fp32" mode; ``logits_round_bf16`` rounds them to
    bf16 first, as ``lin`` does when it returns the bf16 input dtype (model/layers.py:72-75).
    Returns (ids int32 [T, k], weights fp32 [T, k], logits fp64 [T, E] used for the tie test)."""
    x = bf16_to_f32(x_bf16).astype(np.float64)
    w = bf16_to_f32(w_bf16).astype(np.float64)
    logits = (x @ w.T).astype(np.float32)
    if bias is not None:
        logits = (logits + np.asarray(bias, dtype=np.float32)[None, :]).astype(np.float32)
    if logits_round_bf16:
        logits = round_bf16(logits)
    l64 = logits.astype(np.float64)
    m = l64.max(axis=1, keepdims=True)
    e = np.exp(l64 - m)
    probs = (e / e.sum(axis=1, keepdims=True)).astype(np.float32)
    ids, tv = topk_stable(probs, k)
    tv64 = tv.astype(np.float64)
    weights = (tv64 / tv64.sum(axis=1, keepdims=True)).astype(np.float32)
    return ids, weights, l64


def ids_match(ids_dev, ids_ref, logits_ref, tol=1e-6):
    """Top-k ids equal position by position, except where the two candidates' router logits tie within
    ``tol`` (the only exemption the routing contract allows). Returns the number of exempted positions;
    raises AssertionError on a real mismatch or on duplicate ids in a row."""
    ids_dev = np.asarray(ids_dev)
    exempt = 0
    for t in range(ids_ref.shape[0]):
        if len(set(ids_dev[t].tolist())) != ids_dev.shape[1]:
            raise AssertionError(f"token {t}: duplicate ids {ids_dev[t].tolist()}")
        for j in range(ids_ref.shape[1]):
            a, b = int(ids_dev[t, j]), int(ids_ref[t, j])
            if a == b:
                continue
            if a < 0 or abs(logits_ref[t, a] - logits_ref[t, b]) > tol:
                raise AssertionError(f"token {t} rank {j}: id {a} vs oracle {b} "
                                     f"(logits {logits_ref[t, a] if a >= 0 else None} vs {logits_ref[t, b]})")
            exempt += 1
    return exempt


# ------------------------------------------------------------------ align / sort (kernels/moe_align.py)
def padded_rows(r, num_local, block_m):
    """kernels/moe_align.py:11-14."""
    n = r + num_local * (block_m - 1)
    return (n + block_m - 1) // block_m * block_m


def moe_align(local_expert, num_local, block_m):
    """Stable counting sort of rows by local expert, each expert padded to block_m with sentinel R; entries
    outside [0, num_local) are dropped (kernels/moe_align.py:17-48).
    Returns (sorted_rows int32 [P], block_expert int32 [P/block_m], num_padded int32 [1])."""
    le = np.asarray(local_expert, dtype=np.int64)
    r = le.size
    p = padded_rows(r, num_local, block_m)
    valid = (le >= 0) & (le < num_local)
    counts = np.bincount(le[valid], minlength=num_local)[:num_local]
    padded = (counts + block_m - 1) // block_m * block_m
    pad_end = np.cumsum(padded)
    pad_start = pad_end - padded
    sorted_rows = np.full(p, r, dtype=np.int32)
    key = np.where(valid, le, num_local)
    order = np.argsort(key, kind="stable")
    pos = 0
    for e in range(num_local):
        c = int(counts[e])
        sorted_rows[pad_start[e]:pad_start[e] + c] = order[pos:pos + c]
        pos += c
    nb = p // block_m
    starts = np.arange(nb, dtype=np.int64) * block_m
    be = np.searchsorted(pad_end, starts, side="right")
    block_expert = np.where(be < num_local, be, -1).astype(np.int32)
    num_padded = np.array([pad_end[-1] if num_local else 0], dtype=np.int32)
    return sorted_rows, block_expert, num_padded


# ------------------------------------------------------------------ combine (kernels/fused_moe_affine.py:164-172)
def combine_rank_order(rows, t, k):
    """fp32 [t*k, H] -> fp32 [t, H]: out[i] = rows[i*k] + rows[i*k+1] + ... sequentially in fp32."""
    v = np.asarray(rows, dtype=np.float32).reshape(t, k, -1)
    acc = v[:, 0].copy()
    for j in range(1, k):
        acc = (acc + v[:, j]).astype(np.float32)
    return acc


# ------------------------------------------------------------------ expert products
def silu64(g):
    return g / (1.0 + np.exp(-g))


def moe_decode(layout, x, ids, weights, expert_dense):
    """Routed experts of R rows in fp64: out[r] = sum_k w[r,k] * D(silu(G x) * (U x)) in rank order
    (kernels/moe_gemv_affine.py:113-147 semantics; the fp64 check of tests/t0/test_moe_gemv_affine.py:74-84).
    ``x`` fp32 values [R, H]; ``expert_dense(e) -> (G, U, D)`` fp64."""
    x = np.asarray(x, dtype=np.float64)
    out = np.zeros((x.shape[0], layout.hidden), dtype=np.float64)
    for r in range(x.shape[0]):
        for j in range(ids.shape[1]):
            g, u, d = expert_dense(int(ids[r, j]))
            h = silu64(g @ x[r]) * (u @ x[r])
            out[r] += float(weights[r, j]) * (d @ h)
    return out


def fused_rows_exact(x, row_token, row_weight, row_expert, expert_dense, rows):
    """Prefill rows in fp64 exact dequant: y = (D (silu(G x) * U x)) * w
    (tests/gates/test_fused_moe_affine.py:80-100, fp64 branch)."""
    x = np.asarray(x, dtype=np.float64)
    out = []
    for r in rows:
        g, u, d = expert_dense(int(row_expert[r]))
        xr = x[int(row_token[r])]
        out.append((d @ (silu64(g @ xr) * (u @ xr))) * float(row_weight[r]))
    return np.stack(out) if out else np.zeros((0, x.shape[1]))


def fused_rows_bf16_path(x, row_token, row_weight, row_expert, expert_f32, rows):
    """Prefill rows with the reference kernel's rounding points: dequantized tiles rounded to bf16, fp32
    accumulation, h = silu(g)*u stored bf16, y = (D_bf16 h) * w in fp32
    (kernels/fused_moe_affine.py:14-16, :38-50, :76-80, :103-108). ``expert_f32(e)`` gives fp32 dequant."""
    x = np.asarray(x, dtype=np.float64)
    rows = np.asarray(list(rows), dtype=np.int64)
    out = np.zeros((rows.size, x.shape[1]), dtype=np.float64)
    ex = np.asarray(row_expert)[rows]
    for e in np.unique(ex):          # rows are independent; grouping by expert only batches the products
        sel = np.nonzero(ex == e)[0]
        g, u, d = (round_bf16(m).astype(np.float64) for m in expert_f32(int(e)))
        xr = x[np.asarray(row_token)[rows[sel]].astype(np.int64)]
        gg, uu = (xr @ g.T).astype(np.float32), (xr @ u.T).astype(np.float32)
        h = round_bf16(gg.astype(np.float64) / (1.0 + np.exp(-gg.astype(np.float64))) * uu).astype(np.float64)
        wt = np.asarray(row_weight, dtype=np.float32)[rows[sel]]
        out[sel] = ((h @ d.T).astype(np.float32) * wt[:, None]).astype(np.float64)
    return out


def shared_expert(x_bf16, gate, up, down, sh_gate_bf16):
    """Shared expert with the reference's bf16 roundings between ops: every ``lin`` returns bf16
    (model/layers.py:398-402, model/moe_sweep.py:37-43, model/reference_torch.py:130-131).
    gate/up/down are fp32 dequantized weights; returns bf16-valued fp32 [T, H]."""
    x = bf16_to_f32(x_bf16).astype(np.float64)
    a = round_bf16(x @ gate.astype(np.float64).T)
    b = round_bf16(x @ up.astype(np.float64).T)
    sa = round_bf16(a / (1.0 + np.exp(-a.astype(np.float64))))
    h = round_bf16(sa.astype(np.float64) * b)
    y = round_bf16(h.astype(np.float64) @ down.astype(np.float64).T)
    gl = round_bf16(x @ bf16_to_f32(sh_gate_bf16).astype(np.float64).T)
    sg = round_bf16(1.0 / (1.0 + np.exp(-gl.astype(np.float64))))
    return round_bf16(sg.astype(np.float64) * y)


def moe_layer(layout, x_bf16, router_w_bf16, k, expert_dense, sh_dense, sh_gate_bf16, bias=None,
              logits_round_bf16=False):
    """Whole MoE block (model/reference_torch.py:118-134): router -> routed experts summed in rank order
    in fp64 -> bf16, plus the sigmoid-gated shared expert (bf16 between ops); final add in bf16.
    Returns (out bf16-valued fp32 [T, H], routed fp64 [T, H], shared bf16-valued [T, H], ids, weights, logits)."""
    ids, w, logits = router(x_bf16, router_w_bf16, k, bias=bias, logits_round_bf16=logits_round_bf16)
    x = bf16_to_f32(x_bf16)
    routed = moe_decode(layout, x, ids, w, expert_dense)
    sh = shared_expert(x_bf16, *sh_dense, sh_gate_bf16)
    out = round_bf16(round_bf16(routed).astype(np.float64) + sh)
    return out, routed, sh, ids, w, logits


def moe_layer_prefill(layout, x_bf16, router_w_bf16, k, expert_f32, sh_f32, sh_gate_bf16, bias=None,
                      logits_round_bf16=False, routing=None):
    """Whole MoE block on the reference's prefill rounding path: routed rows as fused_rows_bf16_path
    (kernels/fused_moe_affine.py:14-16) summed in rank order in fp32 (combine_rank_order), the shared expert
    through gemm() with bf16-rounded weight tiles and bf16 between ops (model/moe_sweep.py:37-43,
    kernels/gemm_affine.py:32-37), final add in bf16 (model/moe_sweep.py:161 + engine/prefill.py:201).
    ``expert_f32(e)`` -> fp32 (G, U, D). Returns (out bf16-valued fp32 [T, H], routed fp32 [T, H],
    shared bf16-valued [T, H], ids, weights, logits). ``routing`` = (ids, weights) replaces the router's
    choice, so the expert arithmetic can be compared under a given routing."""
    ids, w, logits = router(x_bf16, router_w_bf16, k, bias=bias, logits_round_bf16=logits_round_bf16)
    if routing is not None:
        ids, w = (np.asarray(a) for a in routing)
    t = ids.shape[0]
    x = bf16_to_f32(x_bf16)
    rows = fused_rows_bf16_path(x, np.repeat(np.arange(t), k), w.reshape(-1), ids.reshape(-1), expert_f32,
                                range(t * k))
    routed = combine_rank_order(rows.astype(np.float32), t, k)
    sh = shared_expert(x_bf16, *(round_bf16(m) for m in sh_f32), sh_gate_bf16)
    out = round_bf16(round_bf16(routed).astype(np.float64) + sh)
    return out, routed, sh, ids, w, logits


def moe_layer_grouped(layout, x_bf16, router_w_bf16, k, expert_dense, sh_f32, sh_gate_bf16, bias=None,
                      logits_round_bf16=False):
    """``moe_layer`` with the routed rows batched per expert, for chunks of thousands of tokens: the same fp64
    arithmetic (exact dequant, y = w * D(silu(G x) * U x) per (token, rank), rank-order fp64 sum,
    model/reference_torch.py:118-134), the same shared expert and bf16 final add. ``expert_dense(e)`` -> fp64
    (G, U, D). Returns (out bf16-valued fp32 [T, H], routed fp64 [T, H], ids, weights, logits)."""
    ids, w, logits = router(x_bf16, router_w_bf16, k, bias=bias, logits_round_bf16=logits_round_bf16)
    t = ids.shape[0]
    x = bf16_to_f32(x_bf16).astype(np.float64)
    rows = np.zeros((t * k, layout.hidden), dtype=np.float64)
    flat = ids.reshape(-1)
    for e in np.unique(flat):
        sel = np.nonzero(flat == e)[0]
        g, u, d = expert_dense(int(e))
        xe = x[sel // k]
        rows[sel] = ((silu64(xe @ g.T) * (xe @ u.T)) @ d.T) * w.reshape(-1)[sel, None].astype(np.float64)
    v = rows.reshape(t, k, -1)
    routed = v[:, 0].copy()
    for j in range(1, k):
        routed = routed + v[:, j]
    sh = shared_expert(x_bf16, *sh_f32, sh_gate_bf16)
    out = round_bf16(round_bf16(routed).astype(np.float64) + sh)
    return out, routed, ids, w, logits


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def bf16_ulp(v):
    """Spacing of bf16 values at |v| (fp64 array)."""
    v = np.abs(np.asarray(v, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(v, 2.0 ** -126)))
    return 2.0 ** (e - 7)


def zipf_counts_note(ids, experts):
    c = np.bincount(np.asarray(ids).reshape(-1), minlength=experts)
    return int(c.max()), int((c == 0).sum())

