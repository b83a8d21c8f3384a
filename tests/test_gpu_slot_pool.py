"""HBM slot pool (streaming decode) on the GPU.

The decode layer through a pool far smaller than the experts it touches (misses copied from pinned host
records, CLOCK eviction, event-ordered reuse) equals the same layer with every record resident, bit for bit;
ensure returns each expert's slot, counts hits and misses, and refuses a request that cannot fit."""
import numpy as np
import pytest
import torch

from gpu_helpers import DevicePool, bf16_tensor, record
from slotstream_b200 import synth
from slotstream_b200.records import BASELINE_LAYOUT

pytestmark = pytest.mark.gpu
E, K = 512, 10


@pytest.fixture(scope="module")
def store():
    lay = BASELINE_LAYOUT
    recs = np.stack([record(lay, 0, 0, e) for e in range(E)])
    host = torch.from_numpy(recs).pin_memory()
    return lay, recs, host


def test_streaming_decode_equals_resident(store):
    from slotstream_b200.kernels.moe_layer import DecodeLayerBuffers, moe_layer_decode
    from slotstream_b200.slot_pool import SlotPool, decode_layer_streaming, host_table
    lay, recs, host = store
    layers = 3
    pool = SlotPool(lay.record_bytes, layers, E, chunk_bytes=16 * lay.record_bytes)
    pool.resize(24)                                  # 24 slots for 3 layers x 512 experts
    table = host_table(host.data_ptr(), lay.record_bytes, layers, E, per_layer=False)
    resident = DevicePool(lay, list(recs), range(E), list(range(E)), E, layer=0)
    shared = torch.from_numpy(record(lay, 0, 0, E)).cuda()
    copy = torch.cuda.Stream()
    totals = np.zeros(3, dtype=np.int64)
    for step in range(4):
        for l in range(layers):
            rw = bf16_tensor(synth.router_weight(l, E, lay.hidden, 0))
            sg = bf16_tensor(synth.shared_gate_weight(l, lay.hidden, 0))
            x = bf16_tensor(synth.activations(100 * step + l, 2, lay.hidden))
            sb = DecodeLayerBuffers(2, K, lay.hidden, lay.inter)
            y, stats = decode_layer_streaming(pool, table, x, rw, l, shared, sg, K, sb, copy_stream=copy)
            totals += stats
            # the same records, all resident (map of layer 0 used for every layer: the store is shared)
            rb = DecodeLayerBuffers(2, K, lay.hidden, lay.inter)
            y_ref = moe_layer_decode(x, rw, 0, resident.map, resident.slot_ptr, shared, sg, K, rb, fused=False)
            torch.cuda.synchronize()
            assert int(sb.err.item()) == 0 and int(rb.err.item()) == 0
            assert torch.equal(sb.ids, rb.ids)
            assert torch.equal(y, y_ref), (step, l)
    hits, misses, copied = pool.counters()
    assert (hits, misses, copied) == tuple(int(v) for v in totals)
    assert misses > 0 and copied == misses * lay.record_bytes
    pool.close()


def test_ensure_slots_hits_and_capacity(store):
    from slotstream_b200.slot_pool import SlotPool, host_table
    lay, recs, host = store
    pool = SlotPool(lay.record_bytes, 2, E, chunk_bytes=8 * lay.record_bytes)
    pool.resize(8)
    table = host_table(host.data_ptr(), lay.record_bytes, 2, E, per_layer=False)
    slots, st = pool.ensure(1, [5, 7, 5, 9], table)
    assert st == (0, 3, 3 * lay.record_bytes) and slots[0] == slots[2] and len(set(slots.tolist())) == 3
    slots2, st2 = pool.ensure(1, [9, 5], table)
    assert st2[:2] == (2, 0) and slots2.tolist() == [slots[3], slots[0]]
    m = pool.map.cpu().numpy()
    assert m[E + 5] == slots[0] and m[E + 7] == slots[1] and m[5] == -1
    with pytest.raises(RuntimeError, match="exhausted"):
        pool.ensure(0, list(range(9)), table)     # 9 distinct experts, 8 slots: refused, nothing changed
    assert np.array_equal(pool.map.cpu().numpy(), m)
    torch.cuda.synchronize()
    pool.close()
