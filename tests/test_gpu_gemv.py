"""gemv (affine 4/8-bit, bf16 dense) against fp64, with row invariance (GPU).

Mirrors tests/t0/test_affine_kernels.py:43-75 of the reference: rel_l2 <= 1e-4 vs fp64 and bitwise equality of
each row of a 3-row call with a 1-row call.
"""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

SHAPES = [(512, 2048), (2048, 512), (2560, 2560), (640, 2560), (2560, 640), (10240, 2560), (320, 10240), (1, 2048)]


def _affine(n, k, bits, gs, seed):
    from slotstream_b200.kernels.gemv_affine import AffineWeight
    rng = np.random.default_rng(seed)
    q = rng.integers(0, 2**32, size=(n, k * bits // 32), dtype=np.uint64).astype(np.uint32)
    s = O.f32_to_bf16((rng.standard_normal((n, k // gs)) * 0.02).astype(np.float32))
    b = O.f32_to_bf16((rng.standard_normal((n, k // gs)) * 0.02).astype(np.float32))
    t = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda()  # noqa: E731
    w = AffineWeight(torch.from_numpy(q.view(np.int32)).cuda(), t(s), t(b), bits, gs, n, k)
    return w, O.dequant(q, s, b, bits, gs, np.float64)


def _x(r, k, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(r, k, generator=g).to(dtype).cuda()


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("n,k", SHAPES)
def test_affine_vs_fp64_and_row_invariance(n, k, bits):
    from slotstream_b200.kernels.gemv_affine import gemv
    w, deq = _affine(n, k, bits, 64, n + k + bits)
    x = _x(3, k, 7)
    y = gemv(x, w)
    ref = O.gemv_ref64(x.float().cpu().numpy(), deq)
    assert O.rel_l2(y.cpu().numpy(), ref) <= 1e-4
    for r in range(3):
        assert torch.equal(gemv(x[r:r + 1], w)[0], y[r])


@pytest.mark.parametrize("gs", [32, 64])
def test_affine_gs_and_fp32_x(gs):
    from slotstream_b200.kernels.gemv_affine import gemv
    w, deq = _affine(2560, 2560, 4, gs, 3)
    x = _x(3, 2560, 4, torch.float32)
    y = gemv(x, w)
    assert O.rel_l2(y.cpu().numpy(), O.gemv_ref64(x.cpu().numpy(), deq)) <= 1e-4
    assert torch.equal(gemv(x[1:2], w)[0], y[1])


@pytest.mark.parametrize("n,k", [(512, 2048), (48, 2560), (1, 2560), (4, 10240), (513, 2048)])
def test_dense_bf16(n, k):
    from slotstream_b200.kernels.gemv_affine import DenseWeight, gemv
    g = torch.Generator().manual_seed(n)
    wt = torch.randn(n, k, generator=g).to(torch.bfloat16).cuda()
    x = _x(3, k, 9)
    y = gemv(x, DenseWeight(wt))
    ref = O.gemv_ref64(x.float().cpu().numpy(), wt.float().cpu().numpy())
    assert O.rel_l2(y.cpu().numpy(), ref) <= 1e-4
    for r in range(3):
        assert torch.equal(gemv(x[r:r + 1], DenseWeight(wt))[0], y[r])


def test_block_k_multiple_of_gs_and_shared_bytes():
    from slotstream_b200.kernels import gemv_affine
    w, _ = _affine(256, 2560, 4, 64, 2)
    with pytest.raises(ValueError):
        gemv_affine.gemv(_x(1, 2560, 1), w, cfg={"block_n": 16, "block_k": 32, "split_k": 1, "num_warps": 4,
                                                 "num_stages": 2})
    gemv_affine.gemv(_x(1, 2560, 1), w)
    assert 0 <= gemv_affine.SHARED_BYTES["gemv_affine4"] <= 232448
