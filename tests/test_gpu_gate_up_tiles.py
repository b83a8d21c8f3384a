"""The two tiles of the sorted gate_up GEMM (ssb_set_gate_up_tile: 256 B-rows with M128 x N256 tensor-core
instructions, or 128 with M128 x N128) give the same bits for every row: same dequantised B values, same k order.
Checked through the whole prefill layer (h in sorted order, the fp32 expert rows, the bf16 output) at sizes where
most experts fill less than one 128-row half (37 tokens), some fill one half exactly, and thousands of rows span
many tiles (8,192 tokens)."""
import numpy as np
import pytest
import torch

from gpu_helpers import bf16_tensor, record
from slotstream_b200 import _lib, synth
from slotstream_b200.records import BASELINE_LAYOUT

pytestmark = pytest.mark.gpu
E, K = 512, 10


@pytest.fixture(scope="module")
def layer():
    lay = BASELINE_LAYOUT
    pool = torch.from_numpy(np.stack([record(lay, 0, 0, e) for e in range(E + 1)])).cuda()
    gp = (pool.data_ptr() + torch.arange(E + 1, dtype=torch.int64) * lay.record_bytes).cuda()
    return dict(lay=lay, pool=pool, gp=gp, rw=bf16_tensor(synth.router_weight(0, E, lay.hidden, 0)),
                sg=bf16_tensor(synth.shared_gate_weight(0, lay.hidden, 0)),
                bias=torch.from_numpy(synth.zipf_bias(E)).cuda())


def _layer(L, x, tile):
    from slotstream_b200.kernels.moe_layer import PrefillLayerBuffers, moe_layer_prefill
    lay = L["lay"]
    _lib.check(_lib.lib().ssb_set_gate_up_tile(tile), "gate_up tile")
    try:
        bufs = PrefillLayerBuffers(x.shape[0], K, lay.hidden, lay.inter, E)
        y = moe_layer_prefill(x, L["rw"], L["gp"], L["sg"], K, bufs, bias=L["bias"])
        torch.cuda.synchronize()
    finally:
        _lib.lib().ssb_set_gate_up_tile(256)
    assert int(bufs.err.item()) == 0
    n = int(bufs.num_padded.item())
    sr = bufs.sorted_rows[:n]
    valid = (sr >= 0) & (sr < bufs.rows)
    return y.clone(), bufs.out_rows.clone(), bufs.h[:n][valid].clone()


@pytest.mark.parametrize("tokens", [37, 300, 8192])
def test_wide_and_narrow_gate_up_tiles_agree_bit_for_bit(layer, tokens):
    x = bf16_tensor(synth.activations(400 + tokens, tokens, layer["lay"].hidden))
    y256, rows256, h256 = _layer(layer, x, 256)
    y128, rows128, h128 = _layer(layer, x, 128)
    assert torch.equal(h256.view(torch.int16), h128.view(torch.int16))
    assert torch.equal(rows256.view(torch.int32), rows128.view(torch.int32))
    assert torch.equal(y256.view(torch.int16), y128.view(torch.int16))


def test_gate_up_tile_setting_is_checked():
    assert _lib.lib().ssb_set_gate_up_tile(64) == _lib.SSB_EINVAL
    assert _lib.lib().ssb_set_gate_up_tile(256) == _lib.SSB_OK
