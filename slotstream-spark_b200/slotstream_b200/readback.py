"""Pinned readback of the CUDA-graph decode path -- the B200 side of slotstream_spark/runtime/readback.py.

One sequence word, one control word pair and one slot per layer, all in pinned host memory the GPU writes through
its mapping (runtime/readback.py:1-13):
  seq     int64 [1]            published by ``kernels.signal`` as base + layer after the layer's ids are in its slot
  ctrl    int64 [2]            (position of the first row, step base) written by the host before the step launches
  ids / w [LAYERS * SLOT]      top-k expert ids (int32) and weights (fp32) of each layer, rows back to back
The host waits with ``wait`` (acquire loads in a bounded spin, ``ssb_wait_seq``), with no stream synchronisation, so it
can act on layer l's routing (ensure the next layer's experts, log the routing) while the graph keeps running.
"""
import torch

from . import _lib
from .kernels.signal import SLOT

LAYERS = 49           # 48 layers plus the final segment (runtime/readback.py:20)


class Readback:
    def __init__(self, layers: int = LAYERS, timeout_s: float = 2.0):
        self.layers = layers
        self.timeout_ns = int(timeout_s * 1e9)
        self.base = 0
        self.seq = torch.zeros(1, dtype=torch.int64).pin_memory()
        self.ctrl = torch.zeros(2, dtype=torch.int64).pin_memory()
        self.ids = torch.zeros(layers * SLOT, dtype=torch.int32).pin_memory()
        self.w = torch.zeros(layers * SLOT, dtype=torch.float32).pin_memory()
        self._ids_np = self.ids.numpy()
        self._w_np = self.w.numpy()

    @property
    def seq_addr(self):
        return self.seq.data_ptr()

    def set_seq(self, value):
        self.seq[0] = int(value)

    def begin(self, pos, base):
        """Before a step's graphs launch: its position and sequence base (runtime/readback.py:35-37)."""
        self.ctrl[0] = int(pos)
        self.ctrl[1] = int(base)

    def wait(self, target):
        """Spin until seq >= target; RuntimeError (SSB_ETIMEDOUT) after the bound (runtime/readback.py:39-41)."""
        _lib.check(_lib.lib().ssb_wait_seq(self.seq_addr, int(target), self.timeout_ns), f"wait for seq {target}")

    def layer_ids(self, layer, n):
        """The first n ids of a layer slot (a copy)."""
        o = layer * SLOT
        return self._ids_np[o:o + n].copy()

    def layer_weights(self, layer, n):
        o = layer * SLOT
        return self._w_np[o:o + n].copy()
