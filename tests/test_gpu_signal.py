"""Router readback signal and the whole-step decode graph (GPU): the host follows a captured multi-layer decode step
layer by layer through the pinned readback (slotstream_spark/kernels/signal.py:15-37, runtime/readback.py:1-70),
with no stream synchronisation, and reads every layer's ids and weights as the graph wrote them."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
E, K = 512, 10


def test_signal_publishes_ids_then_sequence():
    from slotstream_b200.kernels.signal import SLOT, signal
    from slotstream_b200.readback import Readback
    rb = Readback(layers=4)
    ids = torch.arange(20, dtype=torch.int32, device="cuda").view(2, 10) * 3
    w = torch.linspace(0, 1, 20, device="cuda").view(2, 10).contiguous()
    rb.begin(7, 1000)
    signal(ids, w, rb.ids, rb.w, rb.seq, rb.ctrl, 2)
    rb.wait(1002)
    assert int(rb.seq[0]) == 1002
    assert np.array_equal(rb.layer_ids(2, 20), ids.cpu().numpy().reshape(-1))
    assert np.array_equal(rb.layer_weights(2, 20), w.cpu().numpy().reshape(-1))
    signal(None, None, rb.ids, rb.w, rb.seq, rb.ctrl, 3)   # the final segment publishes only
    rb.wait(1003)
    with pytest.raises(ValueError):
        signal(torch.zeros(SLOT + 1, dtype=torch.int32, device="cuda"), torch.zeros(SLOT + 1, device="cuda"),
               rb.ids, rb.w, rb.seq, rb.ctrl, 0)
    torch.cuda.synchronize()


@pytest.mark.parametrize("batch", [1, 2])
def test_host_follows_a_captured_decode_step(batch):
    from slotstream_b200 import synth
    from slotstream_b200.decode_step import DecodeStep
    from slotstream_b200.readback import Readback
    from slotstream_b200.records import BASELINE_LAYOUT as LAY, MAP_LAYERS
    NL = 6
    recs = torch.empty((NL * E, LAY.record_bytes), dtype=torch.uint8, device="cuda")
    synth.fill_records_device(LAY, recs, 77)
    shared = torch.empty((NL, LAY.record_bytes), dtype=torch.uint8, device="cuda")
    synth.fill_records_device(LAY, shared, 78)
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    router_w = (torch.randn(NL, E, LAY.hidden, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    sh_gate_w = (torch.randn(NL, LAY.hidden, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    map_t = torch.full((MAP_LAYERS * E,), -1, dtype=torch.int32, device="cuda")
    map_t[:NL * E] = torch.arange(NL * E, dtype=torch.int32, device="cuda")
    slot_ptr = recs.data_ptr() + torch.arange(NL * E, dtype=torch.int64, device="cuda") * LAY.record_bytes
    bias = torch.from_numpy(synth.zipf_bias(E)).cuda()
    x = torch.randn(NL, batch, LAY.hidden, device="cuda", generator=g).to(torch.bfloat16)
    rb = Readback(layers=NL)
    step = DecodeStep(x, router_w, sh_gate_w, shared, map_t, slot_ptr, K, LAY.inter, bias=bias, readback=rb)
    for t in range(3):                       # three steps, each with its own sequence base
        base = 49 * (t + 1)
        x.copy_(torch.randn(NL, batch, LAY.hidden, device="cuda", generator=g).to(torch.bfloat16))
        step.replay(base=base, pos=t)
        seen = []
        for l in range(NL):                  # the host follows the step layer by layer, no stream synchronisation
            rb.wait(base + l)
            seen.append((rb.layer_ids(l, batch * K), rb.layer_weights(l, batch * K)))
        torch.cuda.synchronize()
        assert int(rb.seq[0]) == base + NL - 1
        for l in range(NL):
            assert np.array_equal(seen[l][0], step.bufs[l].ids.cpu().numpy().reshape(-1)), (t, l)
            assert np.array_equal(seen[l][1], step.bufs[l].w.cpu().numpy().reshape(-1)), (t, l)
            assert int(step.bufs[l].err.item()) == 0
    # the graph computed what the eager layers compute
    from slotstream_b200.kernels.moe_layer import DecodeLayerBuffers, moe_layer_decode
    one = DecodeLayerBuffers(batch, K, LAY.hidden, LAY.inter, E)
    moe_layer_decode(x[NL - 1], router_w[NL - 1], NL - 1, map_t, slot_ptr, shared[NL - 1], sh_gate_w[NL - 1], K, one,
                     bias=bias)
    torch.cuda.synchronize()
    assert torch.equal(one.y, step.bufs[NL - 1].y) and torch.equal(one.ids, step.bufs[NL - 1].ids)


@pytest.mark.parametrize("nbytes", [0, 7, 16, 4096 + 3, 1 << 20])
def test_copy_sm_moves_bytes_between_device_and_pinned_host(nbytes):
    """ssb_copy_sm (the SMs' loads and stores, no copy engine): device -> pinned host, pinned host -> device and
    device -> device give the bytes back unchanged, aligned and odd sizes alike."""
    from slotstream_b200 import _lib
    L, st = _lib.lib(), _lib.stream()
    src = torch.randint(0, 256, (max(nbytes, 1),), dtype=torch.uint8, device="cuda")[:nbytes]
    host = torch.full((max(nbytes, 1),), 7, dtype=torch.uint8).pin_memory()[:nbytes]
    back = torch.zeros(max(nbytes, 1), dtype=torch.uint8, device="cuda")[:nbytes]
    dd = torch.zeros(max(nbytes, 1), dtype=torch.uint8, device="cuda")[:nbytes]
    _lib.check(L.ssb_copy_sm(host.data_ptr(), src.data_ptr(), nbytes, st), "d2h")
    torch.cuda.synchronize()
    assert torch.equal(host, src.cpu())
    _lib.check(L.ssb_copy_sm(back.data_ptr(), host.data_ptr(), nbytes, st), "h2d")
    _lib.check(L.ssb_copy_sm(dd.data_ptr(), back.data_ptr(), nbytes, st), "d2d")
    torch.cuda.synchronize()
    assert torch.equal(back, src) and torch.equal(dd, src)
    assert L.ssb_copy_sm(None, src.data_ptr(), 16, st) == _lib.SSB_EINVAL
    assert L.ssb_copy_sm(back.data_ptr(), src.data_ptr(), (1 << 24) + 1, st) == _lib.SSB_EINVAL


def test_prefetch_l2_is_a_hint_that_changes_nothing():
    """ssb_prefetch_l2 on aligned and unaligned ranges returns SSB_OK and leaves the bytes as they were."""
    from slotstream_b200 import _lib
    from slotstream_b200.kernels.moe_layer import prefetch_l2
    t = torch.randint(0, 256, (3 << 20,), dtype=torch.uint8, device="cuda")
    ref = t.clone()
    prefetch_l2(t)
    L, st = _lib.lib(), _lib.stream()
    for off, n in ((1, 100), (7, (1 << 20) + 5), (0, 0), (16, 15)):
        assert L.ssb_prefetch_l2(t.data_ptr() + off, n, st) == _lib.SSB_OK
    torch.cuda.synchronize()
    assert torch.equal(t, ref)
