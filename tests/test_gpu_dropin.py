"""The drop-in modules called on the GPU the way the reference's callers call them (tests/test_reference_callers.py
runs those callers themselves against a CPU model of the C ABI; here the same calls reach the sm_100a kernels).

* ``lin`` inside ``prefill_gemm()`` (model/layers.py:37-76): ``gemm_affine.gemm(x, DenseWeight(w)).to(x.dtype)`` for
  every bf16 weight, the [1, H] shared-expert gate and the [512, H] router included, and ``gemm(x, AffineWeight)``;
* ``SweepMoE._group`` (model/moe_sweep.py:163-176): ``fused_moe_affine`` per group of at most 32 experts with no
  h_buf, into ``torch.empty(n, fm.HID)``, then ``index_copy_`` into ``out_rows`` and ``combine_rank_order``;
* ``Segments.seg_moe`` (model/layers.py:372-390): ``moe_decode`` per row group into views of ``routed``, with
  ``h_buf [r, topk, moe_intermediate_size]``;
at the BASELINE shape 2048 / 512 and at the reference model's 2560 / 640, against the oracle.
"""
import numpy as np
import pytest
import torch

from gpu_helpers import DevicePool, bf16_tensor, record
from oracle import moe_oracle as O
from slotstream_b200 import synth

pytestmark = pytest.mark.gpu
SHAPES = [(2048, 512), (2560, 640)]
K = 10


@pytest.fixture
def shape_reset():
    yield
    from slotstream_b200.kernels import configure
    configure(2560, 640)


@pytest.mark.parametrize("n,k,m", [(1, 2560, 300), (5, 2048, 64), (200, 2048, 129), (512, 2560, 1000),
                                   (2560, 2560, 17)])
def test_lin_gemm_dense_weight(n, k, m):
    from slotstream_b200.kernels.gemm_affine import gemm
    from slotstream_b200.kernels.gemv_affine import DenseWeight
    g = torch.Generator().manual_seed(n + k)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).cuda()
    y = gemm(x.contiguous(), DenseWeight(w))            # lin under prefill_gemm(), model/layers.py:67-70
    assert tuple(y.shape) == (m, n) and y.dtype == torch.float32
    ref = x.double().cpu() @ w.double().cpu().T
    assert float((y.double().cpu() - ref).norm() / ref.norm()) <= 1e-5
    assert torch.equal(y[: m // 2 + 1], gemm(x[: m // 2 + 1].contiguous(), DenseWeight(w)))   # row invariance
    assert gemm(x, DenseWeight(w)).to(x.dtype).dtype == torch.bfloat16


@pytest.mark.parametrize("n,k,gs", [(100, 2560, 64), (640, 2560, 64), (2560, 640, 32)])
def test_lin_gemm_affine_weight_any_n(n, k, gs):
    from slotstream_b200.kernels.gemm_affine import gemm
    from slotstream_b200.kernels.gemv_affine import AffineWeight
    rng = np.random.default_rng(n)
    q = rng.integers(0, 2**32, size=(n, k // 8), dtype=np.uint64).astype(np.uint32)
    s = O.f32_to_bf16(rng.uniform(0.005, 0.02, (n, k // gs)).astype(np.float32))
    b = O.f32_to_bf16((-8 * O.bf16_to_f32(s) + rng.normal(0, 1e-3, (n, k // gs))).astype(np.float32))
    w = AffineWeight(torch.from_numpy(q.view(np.int32)).cuda(), bf16_tensor(s), bf16_tensor(b), 4, gs, n, k)
    x = torch.randn(77, k, generator=torch.Generator().manual_seed(k)).to(torch.bfloat16).cuda()
    y = gemm(x, w).double().cpu().numpy()
    xd = x.double().cpu().numpy()
    assert O.rel_l2(y, xd @ O.round_bf16(O.dequant(q, s, b, 4, gs)).astype(np.float64).T) <= 1e-5
    assert O.rel_l2(y, xd @ O.dequant(q, s, b, 4, gs, np.float64).T) <= 1e-2


@pytest.mark.parametrize("hidden,inter", SHAPES)
def test_sweep_group_calls(shape_reset, hidden, inter):
    """fused_moe_affine as SweepMoE._group calls it: 40 experts in groups of <= 32, <= 96 rows per launch."""
    from slotstream_b200.kernels import configure
    from slotstream_b200.kernels import fused_moe_affine as fm
    lay = configure(hidden, inter)
    assert fm.HID == hidden and fm.INTER == inter and fm.RECORD_BYTES == lay.record_bytes
    rng = np.random.default_rng(hidden + 1)
    experts = np.sort(rng.choice(512, 40, replace=False)).astype(np.int32)
    recs = {int(e): record(lay, 41, 0, int(e)) for e in experts}
    dev = {e: torch.from_numpy(r).cuda() for e, r in recs.items()}
    T = 64
    ids = np.stack([rng.choice(experts, K, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K)).astype(np.float32)
    x_bits = synth.activations(42, T, hidden)
    x = bf16_tensor(x_bits)
    R = T * K
    flat = ids.reshape(-1)
    row_expert = torch.from_numpy(flat).cuda()
    row_token = torch.div(torch.arange(R, device="cuda"), K, rounding_mode="floor").to(torch.int32)
    row_weight = torch.from_numpy(w.reshape(-1)).cuda()
    out_rows = torch.zeros(R, fm.HID, dtype=torch.float32, device="cuda")
    order = np.argsort(flat, kind="stable")
    for g0 in range(0, experts.size, 32):                       # groups of at most 32 experts
        grp = experts[g0:g0 + 32]
        rows = order[np.isin(flat[order], grp)]
        emap_h = np.full(512, -1, dtype=np.int32)
        emap_h[grp] = np.arange(grp.size, dtype=np.int32)
        emap = torch.from_numpy(emap_h).cuda()
        gptr = torch.tensor([dev[int(e)].data_ptr() for e in grp], dtype=torch.int64, device="cuda")
        for a in range(0, rows.size, 96):
            idx = torch.from_numpy(np.ascontiguousarray(rows[a:a + 96])).cuda()
            tmp = torch.empty(idx.numel(), fm.HID, dtype=torch.float32, device="cuda")
            fm.fused_moe_affine(x, row_token[idx].contiguous(), row_weight[idx].contiguous(), emap, gptr, tmp,
                                row_expert=row_expert[idx].contiguous())
            out_rows.index_copy_(0, idx, tmp)
    routed = fm.combine_rank_order(out_rows, T, K).cpu().numpy()
    f32 = {e: O.record_dense(lay, r, np.float32) for e, r in recs.items()}
    rows_ref = O.fused_rows_bf16_path(O.bf16_to_f32(x_bits), np.repeat(np.arange(T), K), w.reshape(-1), flat,
                                      lambda e: f32[e], range(R))
    ref = O.combine_rank_order(rows_ref.astype(np.float32), T, K)
    # the same rounding points; an h element that rounds to the other bf16 neighbour moves a row by 2^-8 of one term
    assert O.rel_l2(routed, ref) <= 1e-3
    exact = O.fused_rows_exact(O.bf16_to_f32(x_bits), np.repeat(np.arange(T), K), w.reshape(-1), flat,
                               lambda e: O.record_dense(lay, recs[e]), range(R))
    assert O.rel_l2(routed, O.combine_rank_order(exact, T, K)) <= 1e-2
    configure(hidden + 512, inter)
    with pytest.raises(ValueError):   # x of another width than the configured HID, and no h_buf: no guessing
        fm.fused_moe_affine(x, row_token[:8].contiguous(), row_weight[:8].contiguous(), emap, gptr,
                            torch.empty(8, hidden, device="cuda"), row_expert=row_expert[:8].contiguous())


@pytest.mark.parametrize("hidden,inter", SHAPES)
def test_seg_moe_calls(shape_reset, hidden, inter):
    """moe_decode as seg_moe calls it: row groups of <= 2 rows written into views of one routed tensor."""
    from slotstream_b200.kernels import configure
    from slotstream_b200.kernels.moe_gemv_affine import moe_decode
    lay = configure(hidden, inter)
    rng = np.random.default_rng(inter + 2)
    experts = np.sort(rng.choice(512, 24, replace=False))
    recs = [record(lay, 43, 0, int(e)) for e in experts]
    pool = DevicePool(lay, recs, experts, list(range(len(experts))), 32, layer=7)
    T = 5
    ids = np.stack([rng.choice(experts, K, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K)).astype(np.float32)
    x_bits = synth.activations(44, T, hidden)
    mixed, ids_d, w_d = bf16_tensor(x_bits), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda()
    routed = torch.zeros(T, hidden, dtype=torch.float32, device="cuda")
    for a in range(0, T, 2):
        b = min(T, a + 2)
        r = b - a
        h_buf = torch.empty(r, K, inter, dtype=torch.float32, device="cuda")
        o_buf = torch.empty(r, K, hidden, dtype=torch.float32, device="cuda")
        moe_decode(mixed[a:b].contiguous(), ids_d[a:b].to(torch.int32).contiguous(), w_d[a:b].contiguous(), 7,
                   pool.map, pool.slot_ptr, h_buf, o_buf, routed[a:b])
    torch.cuda.synchronize()
    dense = {int(e): O.record_dense(lay, r) for e, r in zip(experts, recs)}
    ref = O.moe_decode(lay, O.bf16_to_f32(x_bits), ids, w, lambda e: dense[e])
    assert O.rel_l2(routed.cpu().numpy(), ref) <= 1e-4
