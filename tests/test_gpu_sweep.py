"""The prefill sweep over partially resident experts (slotstream_b200.sweep.PrefillSweep, the B200 side of
model/moe_sweep.py:80-176) against the all-resident layer (moe_layer_prefill) on the same inputs.

A row's result depends only on the row and its expert's record bytes, and the combine sums every token's rows in rank
order whatever group wrote them, so the sweep must equal the all-resident layer bit for bit for every residency mask,
group size and staging configuration; resident records are read where they lie in HBM, the others are staged from
pinned host memory."""
import numpy as np
import pytest
import torch

from gpu_helpers import bf16_tensor, record
from slotstream_b200 import synth
from slotstream_b200.records import BASELINE_LAYOUT
from slotstream_b200.sweep import PrefillSweep

pytestmark = pytest.mark.gpu
E, K, SEED = 512, 10, 0


@pytest.fixture(scope="module")
def layer():
    lay = BASELINE_LAYOUT
    recs = np.stack([record(lay, SEED, 0, e) for e in range(E + 1)])
    host = torch.from_numpy(recs).pin_memory()
    dev = host.cuda()
    gp = (dev.data_ptr() + torch.arange(E + 1, dtype=torch.int64) * lay.record_bytes).cuda()
    return dict(lay=lay, host=host, dev=dev, gp=gp, rw=bf16_tensor(synth.router_weight(SEED, E, lay.hidden, 0)),
                sg=bf16_tensor(synth.shared_gate_weight(SEED, lay.hidden, 0)),
                bias=torch.from_numpy(synth.zipf_bias(E)).cuda())


def _resident_layer(L, x):
    from slotstream_b200.kernels.moe_layer import PrefillLayerBuffers, moe_layer_prefill
    lay = L["lay"]
    bufs = PrefillLayerBuffers(x.shape[0], K, lay.hidden, lay.inter, E)
    y = moe_layer_prefill(x, L["rw"], L["gp"], L["sg"], K, bufs, bias=L["bias"]).clone()
    torch.cuda.synchronize()
    assert int(bufs.err.item()) == 0
    return y, bufs.ids.clone()


def _sweep(L, x, resident, **kw):
    lay = L["lay"]
    sw = PrefillSweep(lay.hidden, lay.inter, K, x.shape[0], lay.record_bytes, **kw)
    dev_base, host_base, rb = L["dev"].data_ptr(), L["host"].data_ptr(), lay.record_bytes
    res_ptr = {int(e): dev_base + int(e) * rb for e in np.flatnonzero(resident)}
    y = sw.layer(x, L["rw"], L["sg"], dev_base + E * rb, res_ptr, lambda e: host_base + e * rb, bias=L["bias"])
    torch.cuda.synchronize()
    assert int(sw.bufs.err.item()) == 0
    return y.clone(), sw


@pytest.mark.parametrize("frac,kw", [
    (0.3, {}),                                              # 32-expert groups, 4 staging buffers, 2 in flight
    (0.0, {"staging_groups": 2, "inflight": 1}),            # nothing resident, buffers reused back to back
    (1.0, {}),                                              # everything resident: no staging at all
    (0.5, {"group_size": 7, "staging_groups": 3, "inflight": 3}),
])
def test_sweep_equals_all_resident_layer_bit_for_bit(layer, frac, kw):
    t = 2048
    x = bf16_tensor(synth.activations(900, t, layer["lay"].hidden))
    y_ref, ids_ref = _resident_layer(layer, x)
    resident = np.random.default_rng(int(frac * 10)).random(E) < frac
    y, sw = _sweep(layer, x, resident, **kw)
    assert torch.equal(sw.bufs.ids, ids_ref)
    assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))
    st = sw.stats
    assert st.resident_rows + st.staged_rows == t * K
    staged_experts = {int(e) for g in sw.last_plan.groups if not g.resident for e in g.experts}
    assert st.records_staged == len(staged_experts)
    assert st.bytes_staged == len(staged_experts) * layer["lay"].record_bytes
    if frac == 1.0:
        assert st.staged_groups == 0


def test_sweep_repeats_and_reuses_its_buffers(layer):
    """Two layers in a row through the same sweep object: the second call must not see anything of the first."""
    lay = layer["lay"]
    sw = PrefillSweep(lay.hidden, lay.inter, K, 512, lay.record_bytes, staging_groups=2, inflight=2)
    dev_base, host_base, rb = layer["dev"].data_ptr(), layer["host"].data_ptr(), lay.record_bytes
    resident = np.random.default_rng(5).random(E) < 0.25
    res_ptr = {int(e): dev_base + int(e) * rb for e in np.flatnonzero(resident)}
    for seed in (901, 902):
        x = bf16_tensor(synth.activations(seed, 512, lay.hidden))
        y_ref, _ = _resident_layer(layer, x)
        y = sw.layer(x, layer["rw"], layer["sg"], dev_base + E * rb, res_ptr, lambda e: host_base + e * rb,
                     bias=layer["bias"])
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))


def test_sweep_reads_resident_records_from_a_slot_pool(layer):
    """Resident records where a SlotPool put them (resident_from_pool), the rest staged: still bit-equal."""
    from slotstream_b200.slot_pool import SlotPool, host_table
    from slotstream_b200.sweep import resident_from_pool
    lay = layer["lay"]
    rb = lay.record_bytes
    pool = SlotPool(rb, 1, max_slots=200)
    try:
        pool.resize(200)
        table = host_table(layer["host"].data_ptr(), rb, 1, E)
        want = np.sort(np.random.default_rng(9).choice(E, 150, replace=False)).astype(np.int32)
        pool.ensure(0, want, table)
        torch.cuda.synchronize()
        res_ptr = resident_from_pool(pool, 0)
        assert sorted(res_ptr) == want.tolist()
        x = bf16_tensor(synth.activations(903, 1024, lay.hidden))
        y_ref, _ = _resident_layer(layer, x)
        sw = PrefillSweep(lay.hidden, lay.inter, K, 1024, rb)
        host_base, dev_base = layer["host"].data_ptr(), layer["dev"].data_ptr()
        y = sw.layer(x, layer["rw"], layer["sg"], dev_base + E * rb, res_ptr, lambda e: host_base + e * rb,
                     bias=layer["bias"])
        pool.release()
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))
        assert sw.stats.resident_rows > 0 and sw.stats.staged_rows > 0
    finally:
        pool.close()
