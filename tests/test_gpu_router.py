"""Router, top-k and combine kernels against the oracle and the reference's golden vectors (GPU)."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from gpu_helpers import bf16_tensor
from oracle import moe_oracle as O
from slotstream_b200 import synth

pytestmark = pytest.mark.gpu


def _topk(x_np, k, nv=None):
    from slotstream_b200.kernels.topk_stable import topk_stable
    x = torch.from_numpy(np.ascontiguousarray(x_np, dtype=np.float32)).cuda()
    nvt = None if nv is None else torch.tensor(nv, dtype=torch.int32, device="cuda")
    val = torch.empty(x.shape[0], k, dtype=torch.float32, device="cuda")
    idx, val = topk_stable(x, k, nvt, out_val=val)
    torch.cuda.synchronize()
    return idx.cpu().numpy(), val.cpu().numpy()


def test_topk_matches_reference_golden():
    g = np.load(GOLDEN / "topk.npz")
    for ci in range(len(g["names"])):
        x = g[f"c{ci}_x"]
        nv = g[f"c{ci}_nv"]
        nv = None if nv[0] < 0 else nv.tolist()
        for k in (10, 512):
            key = f"c{ci}_k{k}_idx"
            if key not in g:
                continue
            idx, val = _topk(x, k, nv)
            assert np.array_equal(idx, g[key]), (g["names"][ci], k)
            ok = idx >= 0
            for r in range(x.shape[0]):
                assert np.array_equal(val[r][ok[r]].view(np.uint32), x[r][idx[r][ok[r]]].view(np.uint32))
            assert np.all(np.isneginf(val[~ok]))


@pytest.mark.parametrize("n", [512, 513, 8192, 65536])
@pytest.mark.parametrize("k", [10, 512])
def test_topk_random_and_ties_vs_oracle(n, k):
    rng = np.random.default_rng(n + k)
    for levels in (None, 2):
        x = rng.standard_normal((3, n)).astype(np.float32)
        if levels:
            x = (np.round(x * levels) / levels).astype(np.float32)
        idx, _ = _topk(x, k)
        ref, _ = O.topk_stable(x, k)
        assert np.array_equal(idx, ref)


def test_topk_row_invariance():
    rng = np.random.default_rng(21)
    x = (np.round(rng.standard_normal((3, 8192)) * 3) / 3).astype(np.float32)
    both, _ = _topk(x, 512)
    for r in range(3):
        one, _ = _topk(x[r:r + 1], 512)
        assert np.array_equal(one[0], both[r])


def _router_inputs(t, e=512, h=2048, seed=0):
    return synth.activations(seed, t, h), synth.router_weight(seed, e, h), synth.shared_gate_weight(seed, h)


def test_router_logits_are_fp32_exact_sums():
    from slotstream_b200 import _lib
    x, w, sg = _router_inputs(37)
    xt, wt, sgt = bf16_tensor(x), bf16_tensor(w), bf16_tensor(sg)
    ld = 513
    out = torch.empty(37 * ld, dtype=torch.float32, device="cuda")
    rc = _lib.lib().ssb_router_logits(xt.data_ptr(), wt.data_ptr(), sgt.data_ptr(), 37, 2048, 512, ld, out.data_ptr(),
                                      _lib.stream())
    _lib.check(rc, "router_logits")
    got = out.view(37, ld).cpu().numpy().astype(np.float64)
    xf = O.bf16_to_f32(x).astype(np.float64)
    ref = np.concatenate([xf @ O.bf16_to_f32(w).astype(np.float64).T, xf @ O.bf16_to_f32(sg).astype(np.float64).T], 1)
    assert np.max(np.abs(got - ref)) < 2e-5


def test_single_row_logits_equal_staged_kernel():
    """One weight row over >= 1024 tokens (the prefill shared gate) takes the warp-per-token kernel; its sums are
    the bits of the staged kernel that shorter calls use."""
    from slotstream_b200 import _lib
    T = 2048
    x, _, sg = _router_inputs(T, seed=3)
    xt, sgt = bf16_tensor(x), bf16_tensor(sg)
    ld = 5
    big = torch.full((T * ld,), -1.0, dtype=torch.float32, device="cuda")
    _lib.check(_lib.lib().ssb_router_logits(xt.data_ptr(), sgt.data_ptr(), None, T, 2048, 1, ld, big.data_ptr(),
                                            _lib.stream()), "router_logits")
    small = torch.full((T * ld,), -1.0, dtype=torch.float32, device="cuda")
    for t0 in range(0, T, 512):
        _lib.check(_lib.lib().ssb_router_logits(xt[t0:].data_ptr(), sgt.data_ptr(), None, 512, 2048, 1, ld,
                                                small[t0 * ld:].data_ptr(), _lib.stream()), "router_logits")
    torch.cuda.synchronize()
    assert torch.equal(big.view(T, ld)[:, 0], small.view(T, ld)[:, 0])
    assert torch.all(big.view(T, ld)[:, 1:] == -1.0)
    ref = O.bf16_to_f32(x).astype(np.float64) @ O.bf16_to_f32(sg).astype(np.float64).reshape(-1)
    assert np.max(np.abs(big.view(T, ld)[:, 0].cpu().numpy() - ref)) < 2e-5


@pytest.mark.parametrize("zipf", [False, True])
@pytest.mark.parametrize("round_bf16", [False, True])
def test_router_topk_matches_oracle(zipf, round_bf16):
    from slotstream_b200.kernels.router import router_topk
    t = 300
    x, w, sg = _router_inputs(t, seed=5)
    bias = synth.zipf_bias(512) if zipf else None
    ids, wts, shg = router_topk(bf16_tensor(x), bf16_tensor(w), 10, logits_round_bf16=round_bf16,
                                bias=None if bias is None else torch.from_numpy(bias).cuda(),
                                sh_gate_w=bf16_tensor(sg))
    torch.cuda.synchronize()
    ref_ids, ref_w, logits = O.router(x, w, 10, bias=bias, logits_round_bf16=round_bf16)
    ex = O.ids_match(ids.cpu().numpy(), ref_ids, logits, tol=1e-6)
    same = (ids.cpu().numpy() == ref_ids).all(axis=1)
    np.testing.assert_allclose(wts.cpu().numpy()[same], ref_w[same], rtol=2e-5, atol=1e-7)
    assert ex <= t * 10 // 100      # tie exemptions must stay rare
    # shared-expert gate: bf16(sigmoid(bf16(x . g))) like lin() + torch.sigmoid on bf16 (model/layers.py:401)
    xf = O.bf16_to_f32(x).astype(np.float64)
    gl = O.round_bf16(xf @ O.bf16_to_f32(sg).astype(np.float64).T)[:, 0].astype(np.float64)
    want = O.round_bf16(1 / (1 + np.exp(-gl)))
    got = shg.cpu().numpy()
    assert np.all(np.abs(got - want) <= O.bf16_ulp(want))


def test_router_row_invariance():
    from slotstream_b200.kernels.router import router_topk
    x, w, _ = _router_inputs(9, seed=7)
    xt, wt = bf16_tensor(x), bf16_tensor(w)
    ids, wts = router_topk(xt, wt, 10)
    for r in range(9):
        i1, w1 = router_topk(xt[r:r + 1].contiguous(), wt, 10)
        assert torch.equal(i1[0], ids[r]) and torch.equal(w1[0], wts[r])


def test_combine_matches_reference_golden_bitwise():
    from slotstream_b200.kernels.fused_moe_affine import combine_rank_order
    g = np.load(GOLDEN / "combine.npz")
    rows = torch.from_numpy(g["rows"]).cuda()
    out = combine_rank_order(rows, int(g["t"]), int(g["k"]))
    assert np.array_equal(out.cpu().numpy().view(np.uint32), g["out"].view(np.uint32))
    with pytest.raises(ValueError):
        combine_rank_order(rows[:-1], int(g["t"]), int(g["k"]))


def test_combine_rank_order_large_vs_oracle():
    from slotstream_b200.kernels.fused_moe_affine import combine_rank_order
    rng = np.random.default_rng(3)
    t, k, h = 1000, 10, 2048
    rows = (rng.standard_normal((t * k, h)) * np.logspace(-3, 3, k).repeat(1)[np.tile(np.arange(k), t)][:, None]
            ).astype(np.float32)
    got = combine_rank_order(torch.from_numpy(rows).cuda(), t, k).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), O.combine_rank_order(rows, t, k).view(np.uint32))
