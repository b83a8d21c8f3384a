"""experts.bin into host pinned memory and HBM (ExpertsFile.to_pinned / to_device / resident_tables) on a B200:
the bytes arrive unchanged whatever the bounce-chunk size, and a decode layer reading the loaded records through
resident_tables equals the same layer reading records placed in HBM directly."""
import numpy as np
import pytest
import torch

from gpu_helpers import bf16_tensor
from slotstream_b200 import synth
from slotstream_b200.experts_file import ExpertsFile, write_experts_bin
from slotstream_b200.records import BASELINE_LAYOUT, MAP_LAYERS

pytestmark = pytest.mark.gpu
E, K = 512, 10


@pytest.fixture(scope="module")
def packed(tmp_path_factory):
    lay = BASELINE_LAYOUT
    d = tmp_path_factory.mktemp("packed")
    recs = {L: np.stack([synth.expert_record(lay, 11, L, e) for e in range(E)]) for L in range(2)}
    write_experts_bin(d, 2, E, [lay.w_bytes, lay.sb_bytes, lay.sb_bytes] * 3, lambda L: recs[L])
    return d, recs


@pytest.mark.parametrize("chunk", [1 << 20, 96 << 20, 1 << 30])
def test_to_device_and_pinned_bytes_unchanged(packed, chunk):
    d, recs = packed
    ef = ExpertsFile(d, hidden=BASELINE_LAYOUT.hidden)
    dev = ef.to_device(chunk_bytes=chunk)
    for L in range(2):
        assert torch.equal(dev[L].cpu(), torch.from_numpy(recs[L]))
    pin = ef.to_pinned([1])
    assert pin.is_pinned() and torch.equal(pin[0], torch.from_numpy(recs[1]))


def test_decode_through_resident_tables(packed):
    from slotstream_b200.kernels.moe_layer import DecodeLayerBuffers, moe_layer_decode
    d, recs = packed
    lay = BASELINE_LAYOUT
    ef = ExpertsFile(d, hidden=lay.hidden)
    dev = ef.to_device()
    map_t, slot_ptr = ef.resident_tables(dev[1:], first_layer=1)
    assert map_t.numel() == MAP_LAYERS * E and int(map_t[E]) == 0 and int(map_t[0]) == -1
    # the same layer-1 records placed in HBM directly, with hand-built tables
    direct = torch.from_numpy(recs[1]).cuda()
    map_d = torch.full((MAP_LAYERS * E,), -1, dtype=torch.int32, device="cuda")
    map_d[E:2 * E] = torch.arange(E, dtype=torch.int32, device="cuda")
    ptr_d = direct.data_ptr() + torch.arange(E, dtype=torch.int64, device="cuda") * lay.record_bytes
    shared = torch.from_numpy(synth.expert_record(lay, 11, 1, E)).cuda()
    rw = bf16_tensor(synth.router_weight(11, E, lay.hidden, 1))
    sg = bf16_tensor(synth.shared_gate_weight(11, lay.hidden, 1))
    x = bf16_tensor(synth.activations(12, 1, lay.hidden))
    outs = []
    for m, p in ((map_t, slot_ptr), (map_d, ptr_d)):
        bufs = DecodeLayerBuffers(1, K, lay.hidden, lay.inter, E)
        moe_layer_decode(x, rw, 1, m, p, shared, sg, K, bufs)
        torch.cuda.synchronize()
        assert int(bufs.err.item()) == 0
        outs.append((bufs.y.clone(), bufs.ids.clone()))
    assert torch.equal(outs[0][1], outs[1][1])
    assert torch.equal(outs[0][0].view(torch.int16), outs[1][0].view(torch.int16))
