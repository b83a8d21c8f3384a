"""Decode grouped GEMV (moe_decode) and the fused decode layer against the fp64 oracle (GPU).

Mirrors the reference's tests/t0/test_moe_gemv_affine.py: fp64 reference within 1e-4 (:91-100), slot-placement
bitwise invariance (:103-116), row invariance with duplicate experts (:119-130), config errors (:133-157),
plus error bits for unmapped experts and the shape-generic record layout.
"""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from gpu_helpers import DevicePool, bf16_tensor, record, to_np_bf16_bits
from oracle import moe_oracle as O
from slotstream_b200 import synth
from slotstream_b200.records import BASELINE_LAYOUT, REFERENCE_LAYOUT

pytestmark = pytest.mark.gpu
LAYER = 3
SEED = 100


def _experts(layout, n):
    return [record(layout, SEED, LAYER, e) for e in range(n)]


def _run(pool, x, ids, w, topk=10, cfg=None, err=None):
    from slotstream_b200.kernels.moe_gemv_affine import moe_decode
    r = x.shape[0]
    lay = pool.layout
    h = torch.empty(r, topk, lay.inter, device="cuda")
    o = torch.empty(r, topk, lay.hidden, device="cuda")
    out = torch.empty(r, lay.hidden, device="cuda")
    moe_decode(x, ids, w, pool.layer, pool.map, pool.slot_ptr, h, o, out, cfg=cfg, err=err)
    torch.cuda.synchronize()
    return out, o


def _inputs(layout, r, seed, n_experts, dtype=torch.bfloat16):
    rng = np.random.default_rng(seed)
    xb = synth.activations(seed, r, layout.hidden)
    x = bf16_tensor(xb)
    if dtype == torch.float32:
        x = x.float() + torch.from_numpy(rng.standard_normal((r, layout.hidden)).astype(np.float32) * 1e-3).cuda()
    ids = np.stack([rng.permutation(n_experts)[:10] for _ in range(r)]).astype(np.int32)
    w = rng.dirichlet(np.ones(10), size=r).astype(np.float32)
    return x, torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda()


def _oracle(layout, recs, x, ids, w):
    dense = {}

    def ex(e):
        if e not in dense:
            dense[e] = O.record_dense(layout, recs[e])
        return dense[e]
    return O.moe_decode(layout, x.float().cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy(), ex)


@pytest.mark.parametrize("layout", [BASELINE_LAYOUT, REFERENCE_LAYOUT], ids=["2048x512", "2560x640"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
def test_matches_fp64_oracle(layout, dtype):
    recs = _experts(layout, 16)
    slots = [(i * 5 + 2) % 16 for i in range(16)]
    pool = DevicePool(layout, recs, range(16), slots, 16, LAYER)
    x, ids, w = _inputs(layout, 3, 1, 16, dtype)
    out, o = _run(pool, x, ids, w)
    ref = _oracle(layout, recs, x, ids, w)
    assert O.rel_l2(out.cpu().numpy(), ref) <= 1e-4
    # o_buf holds the weighted per-rank rows, and out is their rank-order sum (bitwise)
    o_np = o.cpu().numpy()
    acc = o_np[:, 0].copy()
    for k in range(1, 10):
        acc = (acc + o_np[:, k]).astype(np.float32)
    assert np.array_equal(acc.view(np.uint32), out.cpu().numpy().view(np.uint32))


def test_reference_shape_golden():
    """2560/640 against the reference test helper's fp64 output (decode_ref.npz)."""
    g = np.load(GOLDEN / "decode_ref.npz")
    lay = REFERENCE_LAYOUT
    n = int(g["n_exp"])
    recs = [synth.expert_record(lay, int(g["seed"]), 0, e) for e in range(n)]
    pool = DevicePool(lay, recs, range(n), list(range(n)), n, layer=0)
    out, _ = _run(pool, bf16_tensor(g["x_bits"]), torch.from_numpy(g["ids"]).cuda(), torch.from_numpy(g["w"]).cuda())
    assert O.rel_l2(out.cpu().numpy(), g["out"]) <= 1e-4


@pytest.mark.parametrize("n_slots", [13, 64])
def test_placement_bitwise(n_slots):
    lay = BASELINE_LAYOUT
    recs = _experts(lay, 13)
    x, ids, w = _inputs(lay, 2, 2, 13)
    base = DevicePool(lay, recs, range(13), list(range(13)), 13, LAYER)
    ref, _ = _run(base, x, ids, w)
    moved = [(i * 7 + 3) % n_slots for i in range(13)]
    assert len(set(moved)) == 13
    pool = DevicePool(lay, recs, range(13), moved, n_slots, LAYER, pad_bytes=4096)
    out, _ = _run(pool, x, ids, w)
    assert torch.equal(out, ref)


def test_row_invariance_and_duplicates():
    lay = BASELINE_LAYOUT
    recs = _experts(lay, 16)
    pool = DevicePool(lay, recs, range(16), list(range(16)), 16, LAYER)
    x, ids, w = _inputs(lay, 3, 3, 16)
    ids[1] = ids[0]
    ids[2, :5] = ids[0, :5]
    out, _ = _run(pool, x, ids, w)
    for r in range(3):
        one, _ = _run(pool, x[r:r + 1].contiguous(), ids[r:r + 1].contiguous(), w[r:r + 1].contiguous())
        assert torch.equal(one[0], out[r])


def test_grouped_runs_equal_single_rows():
    """20 rows: experts 0..4 chosen by every row (runs of 8, 8, 4 entries), an unmapped id in two rows, the
    rest random. Each row equals its own one-row call bit for bit, and the unmapped choice sets the error."""
    lay = BASELINE_LAYOUT
    recs = _experts(lay, 16)
    pool = DevicePool(lay, recs, range(16), list(range(16)), 16, LAYER)
    R = 20
    x, ids, w = _inputs(lay, R, 8, 16)
    rng = np.random.default_rng(8)
    ids_np = np.stack([np.concatenate([np.arange(5), 5 + rng.permutation(11)[:5]]) for _ in range(R)]).astype(np.int32)
    ids_np[3, 7] = ids_np[11, 2] = 300
    ids = torch.from_numpy(ids_np).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out, o = _run(pool, x, ids, w, err=err)
    assert int(err.item()) & 2
    for r in range(R):
        e1 = torch.zeros(1, dtype=torch.int32, device="cuda")
        one, o1 = _run(pool, x[r:r + 1].contiguous(), ids[r:r + 1].contiguous(), w[r:r + 1].contiguous(), err=e1)
        assert torch.equal(one[0], out[r]), r
        assert torch.equal(o1[0], o[r]), r
    assert torch.all(o[3, 7] == 0) and torch.all(o[11, 2] == 0)


def test_config_errors():
    lay = BASELINE_LAYOUT
    recs = _experts(lay, 16)
    pool = DevicePool(lay, recs, range(16), list(range(16)), 16, LAYER)
    x, ids, w = _inputs(lay, 1, 4, 16)
    with pytest.raises(ValueError):
        _run(pool, x, ids, w, cfg={"bn": 4, "br": 32, "bk": 96, "bkd": 128, "num_warps": 4})
    with pytest.raises(ValueError):
        _run(pool, x, ids.to(torch.int64), w)


def test_unmapped_expert_sets_error_and_contributes_zero():
    lay = BASELINE_LAYOUT
    recs = _experts(lay, 16)
    pool = DevicePool(lay, recs, range(16), list(range(16)), 16, LAYER)
    x, ids, w = _inputs(lay, 1, 6, 16)
    bad = ids.clone()
    bad[0, 3] = 300           # not in the map
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out, _ = _run(pool, x, bad, w, err=err)
    assert int(err.item()) & 2
    w2 = w.clone()
    w2[0, 3] = 0.0
    ref = _oracle(lay, recs, x, ids, w2)
    assert O.rel_l2(out.cpu().numpy(), ref) <= 1e-4


# ------------------------------------------------------------------ fused decode layer
@pytest.fixture(scope="module")
def layer_world():
    """BASELINE config-[0]: 512 experts of layer 0 (seed 0), shared expert = record index 512."""
    lay = BASELINE_LAYOUT
    recs = [record(lay, 0, 0, e) for e in range(513)]
    pool = DevicePool(lay, recs[:512], range(512), list(range(512)), 512, layer=0)
    shared = torch.from_numpy(recs[512]).cuda()
    return lay, recs, pool, shared


def test_decode_layer_matches_reference_moe_ref(layer_world):
    """Routed + shared output of the fused layer vs the reference's moe_ref (fp32 mode, moe_ref.npz)."""
    from slotstream_b200.kernels.moe_layer import DecodeLayerBuffers, moe_layer_decode
    lay, recs, pool, shared = layer_world
    g = np.load(GOLDEN / "moe_ref.npz")
    T = int(g["T"])
    x = synth.activations(0, T, lay.hidden)
    rw = synth.router_weight(0, 512, lay.hidden, 0)
    sg = synth.shared_gate_weight(0, lay.hidden, 0)
    bufs = DecodeLayerBuffers(T, 10, lay.hidden, lay.inter)
    y = moe_layer_decode(bf16_tensor(x), bf16_tensor(rw), 0, pool.map, pool.slot_ptr, shared, bf16_tensor(sg), 10, bufs)
    torch.cuda.synchronize()
    assert int(bufs.err.item()) == 0
    ids_ref, _, logits = O.router(x, rw, 10)
    O.ids_match(bufs.ids.cpu().numpy(), ids_ref, logits)
    assert np.array_equal(ids_ref, g["ids"])
    # fp32 golden (routed + sigmoid-gated shared with no bf16 rounding): the layer output, which rounds like
    # the reference's bf16 callers, is within the layer contract's relative L2
    sh = bufs.out.cpu().numpy()        # routed only
    got_y = O.bf16_to_f32(to_np_bf16_bits(y)).astype(np.float64)
    ref = g["out"].astype(np.float64)
    assert O.rel_l2(got_y, ref) <= 1e-2
    # routed part against the oracle in fp64
    dense = {}

    def ex(e):
        if e not in dense:
            dense[e] = O.record_dense(lay, recs[e])
        return dense[e]
    routed = O.moe_decode(lay, O.bf16_to_f32(x), bufs.ids.cpu().numpy(), bufs.w.cpu().numpy(), ex)
    assert O.rel_l2(sh, routed) <= 1e-4
    assert np.max(np.abs(sh - routed)) <= 2e-2


def test_decode_layer_matches_bf16_oracle_and_is_row_invariant(layer_world):
    from slotstream_b200.kernels.moe_layer import DecodeLayerBuffers, moe_layer_decode
    lay, recs, pool, shared = layer_world
    T = 16
    x = synth.activations(11, T, lay.hidden)
    rw = synth.router_weight(0, 512, lay.hidden, 0)
    sg = synth.shared_gate_weight(0, lay.hidden, 0)
    bias = synth.zipf_bias(512)
    bufs = DecodeLayerBuffers(T, 10, lay.hidden, lay.inter)
    args = (bf16_tensor(rw), 0, pool.map, pool.slot_ptr, shared, bf16_tensor(sg), 10)
    y = moe_layer_decode(bf16_tensor(x), *args, bufs, bias=torch.from_numpy(bias).cuda()).clone()
    torch.cuda.synchronize()
    dense = {}

    def ex(e):
        if e not in dense:
            dense[e] = O.record_dense(lay, recs[e])
        return dense[e]
    out_ref, routed, sh_ref, ids, w, logits = O.moe_layer(lay, x, rw, 10, ex,
                                                          O.record_dense(lay, recs[512], np.float32), sg, bias=bias)
    O.ids_match(bufs.ids.cpu().numpy(), ids, logits)
    got = O.bf16_to_f32(to_np_bf16_bits(y)).astype(np.float64)
    assert O.rel_l2(got, out_ref) <= 1e-2
    # routed fp32 sum: max-abs 2e-2 outright; the bf16 output adds the shared expert's bf16 chain (one straddled
    # intermediate moves it by 2^-8 of its size) and the output's two roundings
    assert np.max(np.abs(bufs.out.cpu().numpy() - routed)) <= 2e-2
    assert np.all(np.abs(got - out_ref) <= 2e-2 + 2.0 ** -6 * np.abs(sh_ref) + 2 * O.bf16_ulp(out_ref))
    # row invariance of the four-launch path (the 16-row call groups entries by expert, the 1-row calls do not); the
    # fused tensor-core layer (the 1- and 2-row default) has its own invariance test below
    one = DecodeLayerBuffers(1, 10, lay.hidden, lay.inter)
    xt = bf16_tensor(x)
    for r in (0, 7, 15):
        y1 = moe_layer_decode(xt[r:r + 1].contiguous(), *args, one, bias=torch.from_numpy(bias).cuda(), fused=False)
        assert torch.equal(y1[0], y[r])


# ------------------------------------------------------------------ fused (one cooperative launch) decode layer
@pytest.mark.parametrize("rows,zipf,round_bf16", [(1, True, False), (2, True, False), (1, False, True), (2, False, False)])
def test_fused_cuda_core_layer_equals_four_launch_layer(layer_world, rows, zipf, round_bf16):
    """ssb_moe_decode_fused on CUDA cores reproduces router_logits -> router_select_resolve -> moe_decode_layer bit
    for bit (ids, weights, shared gate, h, o, routed sum and the bf16 output), on three calls in a row."""
    from slotstream_b200.kernels.moe_layer import DecodeLayerBuffers, moe_layer_decode
    lay, recs, pool, shared = layer_world
    rw = bf16_tensor(synth.router_weight(0, 512, lay.hidden, 0))
    sg = bf16_tensor(synth.shared_gate_weight(0, lay.hidden, 0))
    bias = torch.from_numpy(synth.zipf_bias(512)).cuda() if zipf else None
    fb = DecodeLayerBuffers(rows, 10, lay.hidden, lay.inter)
    sb = DecodeLayerBuffers(rows, 10, lay.hidden, lay.inter)
    for call in range(3):
        x = bf16_tensor(synth.activations(200 + call, rows, lay.hidden))
        args = (x, rw, 0, pool.map, pool.slot_ptr, shared, sg, 10)
        moe_layer_decode(*args, fb, bias=bias, logits_round_bf16=round_bf16, fused=True, cuda_cores=True)
        moe_layer_decode(*args, sb, bias=bias, logits_round_bf16=round_bf16, fused=False)
        torch.cuda.synchronize()
        assert int(fb.err.item()) == 0 and int(sb.err.item()) == 0
        for name in ("ids", "w", "sh_gate", "out", "y", "o"):
            assert torch.equal(getattr(fb, name), getattr(sb, name)), (call, name)
        n = rows * 11 * lay.inter
        assert torch.equal(fb.h[:n], sb.h[:n]), call


def test_fused_layer_reports_unmapped_choice(layer_world):
    """A chosen expert missing from the pool sets SSB_ERR_UNMAPPED and contributes zero, as the four-launch path."""
    from slotstream_b200.kernels.moe_layer import DecodeLayerBuffers, moe_layer_decode
    lay, recs, pool, shared = layer_world
    rw = bf16_tensor(synth.router_weight(0, 512, lay.hidden, 0))
    sg = bf16_tensor(synth.shared_gate_weight(0, lay.hidden, 0))
    x = bf16_tensor(synth.activations(300, 1, lay.hidden))
    probe = DecodeLayerBuffers(1, 10, lay.hidden, lay.inter)
    moe_layer_decode(x, rw, 0, pool.map, pool.slot_ptr, shared, sg, 10, probe)
    torch.cuda.synchronize()
    gone = int(probe.ids[0, 3].item())
    holes = pool.map.clone()
    holes[gone] = -1
    fb = DecodeLayerBuffers(1, 10, lay.hidden, lay.inter)
    sb = DecodeLayerBuffers(1, 10, lay.hidden, lay.inter)
    cb = DecodeLayerBuffers(1, 10, lay.hidden, lay.inter)
    moe_layer_decode(x, rw, 0, holes, pool.slot_ptr, shared, sg, 10, fb, fused=True, tensor_cores=True)
    moe_layer_decode(x, rw, 0, holes, pool.slot_ptr, shared, sg, 10, cb, fused=True, cuda_cores=True)
    moe_layer_decode(x, rw, 0, holes, pool.slot_ptr, shared, sg, 10, sb, fused=False)
    torch.cuda.synchronize()
    assert int(fb.err.item()) & 2 and int(cb.err.item()) & 2 and int(sb.err.item()) & 2
    assert torch.equal(cb.out, sb.out) and torch.equal(cb.y, sb.y)
    assert torch.equal(fb.ids, sb.ids)
    assert float((fb.out - sb.out).norm() / sb.out.norm()) <= 1e-5   # the missing expert contributes zero in both


@pytest.mark.parametrize("rows,zipf,round_bf16", [(1, True, False), (2, True, False), (1, False, True), (2, False, False)])
def test_fused_tensor_core_layer_matches_four_launch_layer(layer_world, rows, zipf, round_bf16):
    """The tensor-core fused layer (the default) against the exact-fp32 four-launch path on three calls in a row:
    ids, weights, shared gate and resolved bases bit for bit; h, o and the routed sum within the fp32 decode
    tolerance (relative L2 1e-4 -- and the routed sum against the fp64 oracle too); the bf16 output within rounding
    flips of the four-launch output."""
    from slotstream_b200.kernels.moe_layer import DecodeLayerBuffers, moe_layer_decode
    lay, recs, pool, shared = layer_world
    rw = bf16_tensor(synth.router_weight(0, 512, lay.hidden, 0))
    sg = bf16_tensor(synth.shared_gate_weight(0, lay.hidden, 0))
    bias = torch.from_numpy(synth.zipf_bias(512)).cuda() if zipf else None
    fb = DecodeLayerBuffers(rows, 10, lay.hidden, lay.inter)
    sb = DecodeLayerBuffers(rows, 10, lay.hidden, lay.inter)
    dense = {}

    def ex(e):
        if e not in dense:
            dense[e] = O.record_dense(lay, recs[e])
        return dense[e]
    for call in range(3):
        xb = synth.activations(200 + call, rows, lay.hidden)
        x = bf16_tensor(xb)
        args = (x, rw, 0, pool.map, pool.slot_ptr, shared, sg, 10)
        moe_layer_decode(*args, fb, bias=bias, logits_round_bf16=round_bf16, fused=True, tensor_cores=True)
        moe_layer_decode(*args, sb, bias=bias, logits_round_bf16=round_bf16, fused=False)
        torch.cuda.synchronize()
        assert int(fb.err.item()) == 0 and int(sb.err.item()) == 0
        for name in ("ids", "w", "sh_gate", "bases"):
            assert torch.equal(getattr(fb, name), getattr(sb, name)), (call, name)
        n = rows * 11 * lay.inter
        for name, a_, b_ in (("h", fb.h[:n], sb.h[:n]), ("o", fb.o, sb.o), ("out", fb.out, sb.out)):
            rel = float((a_.double() - b_.double()).norm() / b_.double().norm())
            assert rel <= 1e-4, (call, name, rel)
        routed = O.moe_decode(lay, O.bf16_to_f32(xb), fb.ids.cpu().numpy(), fb.w.cpu().numpy(), ex)
        assert O.rel_l2(fb.out.cpu().numpy(), routed) <= 1e-4
        y_f = O.bf16_to_f32(to_np_bf16_bits(fb.y)).astype(np.float64)
        y_s = O.bf16_to_f32(to_np_bf16_bits(sb.y)).astype(np.float64)
        sh = np.abs(y_s - O.bf16_to_f32(O.f32_to_bf16(sb.out.cpu().numpy())).astype(np.float64))
        bound = O.bf16_ulp(y_s) + O.bf16_ulp(sb.out.cpu().numpy()) + 2.0 ** -7 * sh + 1e-3
        assert np.all(np.abs(y_f - y_s) <= bound), call


def test_fused_tensor_core_layer_is_row_invariant(layer_world):
    """A two-token call gives each token the bits of a one-token call: the tokens are separate mma columns, and
    the routing, the fold and the combine are per token."""
    from slotstream_b200.kernels.moe_layer import DecodeLayerBuffers, moe_layer_decode
    lay, recs, pool, shared = layer_world
    rw = bf16_tensor(synth.router_weight(0, 512, lay.hidden, 0))
    sg = bf16_tensor(synth.shared_gate_weight(0, lay.hidden, 0))
    bias = torch.from_numpy(synth.zipf_bias(512)).cuda()
    x = bf16_tensor(synth.activations(400, 2, lay.hidden))
    two, one = DecodeLayerBuffers(2, 10, lay.hidden, lay.inter), DecodeLayerBuffers(1, 10, lay.hidden, lay.inter)
    moe_layer_decode(x, rw, 0, pool.map, pool.slot_ptr, shared, sg, 10, two, bias=bias, tensor_cores=True)
    for r in range(2):
        moe_layer_decode(x[r:r + 1].contiguous(), rw, 0, pool.map, pool.slot_ptr, shared, sg, 10, one, bias=bias,
                         tensor_cores=True)
        torch.cuda.synchronize()
        assert torch.equal(one.ids[0], two.ids[r]) and torch.equal(one.w[0], two.w[r])
        assert torch.equal(one.out[0], two.out[r]) and torch.equal(one.y[0], two.y[r])
