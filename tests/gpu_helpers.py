"""Helpers shared by the GPU parity tests: device pools of records with their slot tables."""
import numpy as np
import torch

from slotstream_b200 import synth
from slotstream_b200.records import MAP_LAYERS, EXPERTS_PER_LAYER

_REC_CACHE = {}


def record(layout, seed, layer, e):
    key = (layout, seed, layer, e)
    if key not in _REC_CACHE:
        _REC_CACHE[key] = synth.expert_record(layout, seed, layer, e)
    return _REC_CACHE[key]


class DevicePool:
    """`n_slots` record-sized slots in one CUDA buffer; expert e of `layer` sits in slot slots[i]."""

    def __init__(self, layout, recs, experts, slots, n_slots, layer=3, pad_bytes=0):
        self.layout, self.layer = layout, layer
        stride = layout.record_bytes + pad_bytes
        self.stride = stride
        host = np.zeros((n_slots, stride), dtype=np.uint8)
        for rec, s in zip(recs, slots):
            host[s, :layout.record_bytes] = rec
        self.buf = torch.from_numpy(host).cuda()
        m = torch.full((MAP_LAYERS * EXPERTS_PER_LAYER,), -1, dtype=torch.int32)
        for e, s in zip(experts, slots):
            m[layer * EXPERTS_PER_LAYER + int(e)] = int(s)
        self.map = m.cuda()
        base = self.buf.data_ptr()
        self.slot_ptr = torch.tensor([base + i * stride for i in range(n_slots)], dtype=torch.int64).cuda()


def bf16_tensor(bits, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def to_np_bf16_bits(t):
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)
