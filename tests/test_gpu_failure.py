"""Failure paths of the cooperative decode kernels, made without any GPU fault (GPU).

The grid barriers of ssb_moe_decode_fused wait a bounded time (ssb_set_wait_limit_ns, default 250 ms). With the
bound set to zero the barrier waits run out at once: the kernel must set SSB_ERR_TIMEOUT in the caller's error word
and return instead of hanging, and the context must stay usable -- after the bound is restored and the sync word
zeroed, the next call computes the layer exactly as before."""
import pytest
import torch

from gpu_helpers import DevicePool, bf16_tensor, record
from slotstream_b200 import _lib, synth
from slotstream_b200.records import BASELINE_LAYOUT

pytestmark = pytest.mark.gpu
E, K = 512, 10


@pytest.fixture(scope="module")
def world():
    lay = BASELINE_LAYOUT
    recs = [record(lay, 9, 0, e) for e in range(E + 1)]
    pool = DevicePool(lay, recs[:E], range(E), list(range(E)), E, layer=0)
    shared = torch.from_numpy(recs[E]).cuda()
    return lay, pool, shared


@pytest.mark.parametrize("rows,kernel", [(1, "cuda_cores"), (2, "tensor_cores"), (1, "tensor_cores")])
def test_barrier_wait_runs_out_and_context_recovers(world, rows, kernel):
    from slotstream_b200.kernels.moe_layer import DecodeLayerBuffers, moe_layer_decode
    lay, pool, shared = world
    rw = bf16_tensor(synth.router_weight(9, E, lay.hidden, 0))
    sg = bf16_tensor(synth.shared_gate_weight(9, lay.hidden, 0))
    x = bf16_tensor(synth.activations(90, rows, lay.hidden))
    kw = {kernel: True}
    good = DecodeLayerBuffers(rows, K, lay.hidden, lay.inter)
    moe_layer_decode(x, rw, 0, pool.map, pool.slot_ptr, shared, sg, K, good, **kw)
    torch.cuda.synchronize()
    assert int(good.err.item()) == 0
    bad = DecodeLayerBuffers(rows, K, lay.hidden, lay.inter)
    L = _lib.lib()
    try:
        _lib.check(L.ssb_set_wait_limit_ns(0), "wait limit")
        moe_layer_decode(x, rw, 0, pool.map, pool.slot_ptr, shared, sg, K, bad, **kw)
        torch.cuda.synchronize()                 # returns: no hang, no fault
    finally:
        _lib.check(L.ssb_set_wait_limit_ns(250_000_000), "wait limit")
    assert int(bad.err.item()) & _lib.ERR_TIMEOUT
    bad.err.zero_()
    bad.sync.zero_()                             # the sync word must be zeroed after a timed-out call
    moe_layer_decode(x, rw, 0, pool.map, pool.slot_ptr, shared, sg, K, bad, **kw)
    torch.cuda.synchronize()
    assert int(bad.err.item()) == 0
    for name in ("ids", "w", "out", "y"):
        assert torch.equal(getattr(bad, name), getattr(good, name)), name
    assert L.ssb_set_wait_limit_ns(-1) == _lib.SSB_EINVAL
