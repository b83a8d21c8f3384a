"""Empty and ragged inputs through the public functions (GPU): the reference's functions accept zero rows and
zero tokens; these must too, and agree with the oracle on them."""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nl,bm", [(512, 64), (33, 256), (1, 16)])
def test_align_of_no_rows_equals_oracle(nl, bm):
    from slotstream_b200.kernels.moe_align import moe_align
    sr, be, npad = moe_align(torch.empty(0, dtype=torch.int32, device="cuda"), nl, bm)
    torch.cuda.synchronize()
    rs, rb, rn = O.moe_align(np.empty(0, dtype=np.int32), nl, bm)
    assert np.array_equal(sr.cpu().numpy(), rs)
    assert np.array_equal(be.cpu().numpy(), rb)
    assert np.array_equal(npad.cpu().numpy(), rn)


def test_align_of_rows_outside_every_group_equals_oracle():
    """Every row -1 or >= num_local (not in the current group): nothing is sorted, nothing is padded."""
    from slotstream_b200.kernels.moe_align import moe_align
    le = np.array([-1, 7, 9, -1, 8] * 41, dtype=np.int32)
    sr, be, npad = moe_align(torch.from_numpy(le).cuda(), 7, 64)
    torch.cuda.synchronize()
    rs, rb, rn = O.moe_align(le, 7, 64)
    assert np.array_equal(sr.cpu().numpy(), rs) and np.array_equal(be.cpu().numpy(), rb)
    assert int(npad.item()) == int(rn[0]) == 0


def test_topk_of_no_rows():
    from slotstream_b200.kernels.topk_stable import topk_stable
    idx, val = topk_stable(torch.empty((0, 512), dtype=torch.float32, device="cuda"), 10,
                           out_val=torch.empty((0, 10), dtype=torch.float32, device="cuda"))
    torch.cuda.synchronize()
    assert tuple(idx.shape) == (0, 10) and tuple(val.shape) == (0, 10)


def test_topk_with_zero_valid_entries_pads_every_slot():
    from slotstream_b200.kernels.topk_stable import topk_stable
    s = np.random.default_rng(5).standard_normal((3, 300)).astype(np.float32)
    nv = np.array([0, 4, 300], dtype=np.int32)
    idx, val = topk_stable(torch.from_numpy(s).cuda(), 10, n_valid=torch.from_numpy(nv).cuda(),
                           out_val=torch.empty((3, 10), dtype=torch.float32, device="cuda"))
    ri, rv = O.topk_stable(s, 10, nv)
    assert np.array_equal(idx.cpu().numpy(), ri)
    assert np.array_equal(val.cpu().numpy(), rv)


def test_combine_of_no_tokens():
    from slotstream_b200.kernels.fused_moe_affine import combine_rank_order
    out = combine_rank_order(torch.empty((0, 2048), dtype=torch.float32, device="cuda"), 0, 10)
    torch.cuda.synchronize()
    assert tuple(out.shape) == (0, 2048)


def test_fused_decode_of_no_rows_launches_nothing():
    from slotstream_b200 import _lib
    rc = _lib.lib().ssb_moe_decode_fused(None, 0, 10, 2048, 512, 512, None, None, None, 0, 0, None, 0, None, 0, None,
                                         None, None, None, None, None, None, None, None, None, None, None,
                                         _lib.stream())
    assert rc == _lib.SSB_OK


def test_router_entry_points_accept_no_tokens():
    """Zero tokens with the null pointers of empty tensors: nothing to do, SSB_OK (the reference's router runs on
    empty batches)."""
    from slotstream_b200 import _lib
    L, st = _lib.lib(), _lib.stream()
    w = torch.zeros((512, 2048), dtype=torch.bfloat16, device="cuda")
    assert L.ssb_router_logits(None, _lib.ptr(w), None, 0, 2048, 512, 512, None, st) == _lib.SSB_OK
    assert L.ssb_router_select(None, 513, 0, 512, 10, None, _lib.ROUTER_SHARED_GATE, None, None, None, None,
                               st) == _lib.SSB_OK
    assert L.ssb_router_topk_static(None, _lib.ptr(w), None, 0, 2048, 512, 10, None, 0, None, None, None,
                                    st) == _lib.SSB_OK
    from slotstream_b200.kernels.fused_moe_affine import combine_rank_order
    assert L.ssb_combine_layer(None, 0, 10, 2048, None, None, None, st) == _lib.SSB_OK
    combine_rank_order(torch.empty((0, 64), dtype=torch.float32, device="cuda"), 0, 4)
    torch.cuda.synchronize()
