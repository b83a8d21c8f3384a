"""Prefill grouped GEMM (tcgen05) and the dense prefill GEMM against the oracle (GPU).

Mirrors the reference's tests/gates/test_fused_moe_affine.py: fp64 exact-dequant reference within
fused_moe_rel_l2_max = 1e-2 with a nibble-swap negative control > 10x the limit (:116-128), bit-identical rows
across R (:131-134), grouping and order invariance (:137-145), pool address = staging address (:148-149),
determinism (:152-153), no atomics on data (:156-158), launch time at 40,960 rows (:161-183); and
tests/t0/test_gemm_affine.py (accuracy, nibble-swap control, row invariance, argument errors).
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from gpu_helpers import bf16_tensor, record
from oracle import moe_oracle as O
from slotstream_b200 import synth
from slotstream_b200.records import BASELINE_LAYOUT, REFERENCE_LAYOUT

pytestmark = pytest.mark.gpu
LIMIT, CONTROL = 1e-2, 10.0
SEED, NEXP, TOK, TOPK = 1729, 32, 4096, 10
RMAX = TOK * TOPK


class World:
    def __init__(self, layout, nexp=NEXP, tok=TOK):
        self.lay = layout
        self.recs = [record(layout, SEED, 0, e) for e in range(nexp)]
        host = np.stack(self.recs)
        self.pool = torch.from_numpy(np.concatenate([host, host])).cuda()       # same bytes twice (pool / staging)
        rb = layout.record_bytes
        self.ptr_all = [self.pool.data_ptr() + i * rb for i in range(2 * nexp)]
        rng = np.random.default_rng(SEED)
        self.x_bits = synth.activations(SEED, tok, layout.hidden)
        self.x = bf16_tensor(self.x_bits)
        r = tok * TOPK
        self.expert = torch.from_numpy(rng.integers(0, nexp, r).astype(np.int32)).cuda()
        self.weight = torch.from_numpy((rng.random(r) + 0.1).astype(np.float32)).cuda()
        self.token = (torch.arange(r, dtype=torch.int32) // TOPK).cuda()
        self._f32 = {}

    def dense_f32(self, e):
        if e not in self._f32:
            self._f32[e] = O.record_dense(self.lay, self.recs[e], np.float32)
        return self._f32[e]

    def run(self, r, order=None, offset=0, out=None):
        from slotstream_b200.kernels import fused_moe_affine as fm
        order = list(range(len(self.recs))) if order is None else list(order)
        m = torch.full((512,), -1, dtype=torch.int32)
        for local, e in enumerate(order):
            m[int(e)] = local
        gp = torch.tensor([self.ptr_all[offset + int(e)] for e in order], dtype=torch.int64).cuda()
        if out is None:
            out = torch.zeros(r, self.lay.hidden, dtype=torch.float32, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        fm.fused_moe_affine(self.x, self.token[:r], self.weight[:r], m.cuda(), gp, out, row_expert=self.expert[:r],
                            inter=self.lay.inter, err=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        return out


@pytest.fixture(scope="module")
def world():
    return World(BASELINE_LAYOUT)


def _refs(w, rows, swap=False):
    x = O.bf16_to_f32(w.x_bits).astype(np.float64)
    tok, wt, ex = w.token.cpu().numpy(), w.weight.cpu().numpy(), w.expert.cpu().numpy()
    exact, bf = [], []
    for r in rows:
        g, u, d = (m.astype(np.float64) for m in w.dense_f32(int(ex[r])))
        if swap:
            g, u, d = (_swap(w, int(ex[r]), i) for i in range(3))
        xr = x[int(tok[r])]
        exact.append((d @ (O.silu64(g @ xr) * (u @ xr))) * float(wt[r]))
        if not swap:
            gb, ub, db = (O.round_bf16(m).astype(np.float64) for m in w.dense_f32(int(ex[r])))
            gg, uu = (gb @ xr).astype(np.float32), (ub @ xr).astype(np.float32)
            h = O.round_bf16(gg.astype(np.float64) / (1 + np.exp(-gg.astype(np.float64))) * uu).astype(np.float64)
            bf.append(((db @ h).astype(np.float32) * np.float32(wt[r])).astype(np.float64))
    return np.stack(exact), (np.stack(bf) if bf else None)


def _swap(w, e, piece):
    q, s, b = O.record_pieces(w.lay, w.recs[e])[piece]
    u = O.unpack(q).reshape(q.shape[0], -1, 2)[:, :, ::-1].reshape(q.shape[0], -1).astype(np.float64)
    return u * np.repeat(O.bf16_to_f32(s).astype(np.float64), 64, 1) + np.repeat(O.bf16_to_f32(b).astype(np.float64), 64, 1)


def test_matches_fp64_reference_floor_and_control(world):
    out = world.run(2560)
    rows = list(range(0, 2560, 10))[:120]
    sel = out[rows].cpu().numpy()
    exact, bf = _refs(world, rows)
    err = O.rel_l2(sel, exact)
    floor = O.rel_l2(sel, bf)
    swap, _ = _refs(world, rows[:40], swap=True)
    ctrl = O.rel_l2(sel[:40], swap)
    print(f"fused_moe rel_l2 vs fp64 {err:.3e} (limit {LIMIT}); vs bf16-path oracle {floor:.3e}; control {ctrl:.3f}")
    assert err <= LIMIT
    assert floor <= 2e-3          # same rounding points as the reference kernel: only fp32 sum order differs
    assert ctrl > CONTROL * LIMIT


def test_reference_shape_2560x640():
    w = World(REFERENCE_LAYOUT, nexp=6, tok=64)
    out = w.run(300)
    rows = list(range(0, 300, 7))
    exact, bf = _refs(w, rows)
    assert O.rel_l2(out[rows].cpu().numpy(), exact) <= LIMIT
    assert O.rel_l2(out[rows].cpu().numpy(), bf) <= 2e-3


def test_bit_identical_across_r(world):
    ref = world.run(17)
    for r in (2560, RMAX):
        assert torch.equal(world.run(r)[:17], ref), r


def test_grouping_and_order_do_not_change_bits(world):
    r = 2560
    base = world.run(r)
    assert torch.equal(world.run(r, order=list(reversed(range(NEXP)))), base)
    first = [3, 17, 5, 29] + [e for e in range(NEXP) if e not in (3, 17, 5, 29)]
    assert torch.equal(world.run(r, order=first), base)
    a, b = world.run(r, order=range(0, 16)), world.run(r, order=range(16, 32))
    assert torch.equal(a + b, base)


def test_pool_address_equals_staging_address(world):
    assert torch.equal(world.run(2560, offset=NEXP), world.run(2560))


def test_two_runs_identical(world):
    assert torch.equal(world.run(2560), world.run(2560))


def test_kernel_source_has_no_data_atomics():
    import re
    src = (Path(__file__).resolve().parents[1] / "slotstream-spark_b200" / "csrc" / "grouped_gemm.cu").read_text()
    for bad in (r"\batomic(Add|Max|Min|Exch|CAS|Sub|Inc|Dec)\b", r"(?<![.\w])red\.", r"(?<![.\w])atom\."):
        assert not re.search(bad, src), bad


def test_launch_time_at_40960_rows(world):
    from slotstream_b200.kernels import fused_moe_affine as fm
    r = RMAX
    m = torch.arange(512, dtype=torch.int32).cuda()
    m[NEXP:] = -1
    gp = torch.tensor(world.ptr_all[:NEXP], dtype=torch.int64).cuda()
    out = torch.zeros(r, world.lay.hidden, dtype=torch.float32, device="cuda")
    h = torch.empty(r, world.lay.inter, dtype=torch.bfloat16, device="cuda")
    aligned = fm.align_rows(world.expert, m, NEXP)
    fm.fused_moe_affine(world.x, world.token, world.weight, m, gp, out, row_expert=world.expert, h_buf=h,
                        aligned=aligned)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    ev[0].record()
    fm.launch_gate_up(world.x, world.token, aligned, gp, h, r)
    ev[1].record()
    fm.launch_down(h, world.weight, aligned, gp, out, r)
    ev[2].record()
    torch.cuda.synchronize()
    gu, dn = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
    flops = 2 * r * 3 * world.lay.hidden * world.lay.inter
    print(f"R={r}: gate_up {gu:.3f} ms, down {dn:.3f} ms, {flops / ((gu + dn) * 1e-3) / 1e12:.1f} TFLOP/s")
    assert max(gu, dn) <= 200.0


# ------------------------------------------------------------------ dense prefill GEMM (gemm_affine.gemm)
def _affine(n, k, gs, seed):
    from slotstream_b200.kernels.gemv_affine import AffineWeight
    rng = np.random.default_rng(seed)
    q = rng.integers(0, 2**32, size=(n, k // 8), dtype=np.uint64).astype(np.uint32)
    s = O.f32_to_bf16((rng.standard_normal((n, k // gs)) * 0.02).astype(np.float32))
    b = O.f32_to_bf16((rng.standard_normal((n, k // gs)) * 0.02).astype(np.float32))
    t = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda()  # noqa: E731
    return AffineWeight(torch.from_numpy(q.view(np.int32)).cuda(), t(s), t(b), 4, gs, n, k), (q, s, b)


@pytest.mark.parametrize("n,k,gs", [(512, 2048, 64), (2048, 512, 64), (2560, 2560, 64), (512, 2560, 32)])
def test_gemm_accuracy_and_control(n, k, gs):
    from slotstream_b200.kernels.gemm_affine import gemm
    w, (q, s, b) = _affine(n, k, gs, n + k)
    g = torch.Generator().manual_seed(7)
    x = torch.randn(64, k, generator=g).to(torch.bfloat16).cuda()
    y = gemm(x, w).cpu().numpy()
    xd = x.float().cpu().numpy().astype(np.float64)
    ref = xd @ O.dequant(q, s, b, 4, gs, np.float64).T
    assert O.rel_l2(y, ref) <= LIMIT
    assert O.rel_l2(y, xd @ O.round_bf16(O.dequant(q, s, b, 4, gs)).astype(np.float64).T) <= 1e-5
    u = O.unpack(q).reshape(n, -1, 2)[:, :, ::-1].reshape(n, -1).astype(np.float64)
    sw = u * np.repeat(O.bf16_to_f32(s).astype(np.float64), gs, 1) + np.repeat(O.bf16_to_f32(b).astype(np.float64), gs, 1)
    assert O.rel_l2(y, xd @ sw.T) > CONTROL * LIMIT


@pytest.mark.parametrize("n,k", [(512, 2048), (2048, 512)])
def test_gemm_row_invariance(n, k):
    from slotstream_b200.kernels.gemm_affine import gemm
    w, _ = _affine(n, k, 64, n + k)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(4096, k, generator=g).to(torch.bfloat16).cuda()
    big = gemm(x, w)
    assert torch.equal(big, gemm(x, w))
    for m in (1, 17, 64, 4096):
        assert torch.equal(big[:m], gemm(x[:m].contiguous(), w))


def test_gemm_errors():
    from slotstream_b200.kernels.gemm_affine import gemm
    w, _ = _affine(512, 2048, 64, 1)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(4, 2048, generator=g).to(torch.bfloat16).cuda()
    with pytest.raises(ValueError):
        gemm(x, w, cfg={"block_m": 64, "block_n": 64, "block_k": 96})
    with pytest.raises(ValueError):
        gemm(x.float(), w)
    with pytest.raises(ValueError):
        gemm(torch.randn(4, 1024, generator=g).to(torch.bfloat16).cuda(), w)
    out = torch.empty(4, 512, dtype=torch.float32, device="cuda")
    assert gemm(x, w, out=out) is out
    for bad in (torch.empty(3, 512, device="cuda"), torch.empty(4, 512, dtype=torch.bfloat16, device="cuda")):
        with pytest.raises(ValueError):
            gemm(x, w, out=bad)


@pytest.mark.parametrize("m,k,n,pad", [(300, 64, 256, 0), (5000, 128, 512, 4), (20000, 256, 512, 0), (129, 2048, 512, 4)])
def test_gemm_dense_matches_fp64(m, k, n, pad):
    """Plain bf16 GEMM (the prefill router logits): fp32 accumulation of exact bf16 products vs fp64; several
    tiles per CTA, one-k-block tiles (k = 64) and a row stride wider than n."""
    from slotstream_b200 import _lib
    g = torch.Generator().manual_seed(m + k)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).cuda()
    out = torch.full((m, n + pad), -5.0, dtype=torch.float32, device="cuda")
    _lib.check(_lib.lib().ssb_gemm_dense(_lib.ptr(x), m, k, _lib.ptr(w), n, _lib.ptr(out), n + pad, _lib.stream()),
               "gemm_dense")
    torch.cuda.synchronize()
    ref = x.double().cpu() @ w.double().cpu().T
    got = out[:, :n].double().cpu()
    assert float((got - ref).norm() / ref.norm()) <= 1e-5
    if pad:
        assert bool((out[:, n:] == -5.0).all())
