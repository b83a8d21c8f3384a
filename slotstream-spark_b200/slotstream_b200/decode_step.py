"""A whole decode step of MoE layers in one CUDA graph, each layer followed by its readback signal.

The B200 counterpart of the decode MoE segments of slotstream_spark/runtime/graphs.py:92-200 for this path: the
MoE layers of one token step (``moe_layer_decode`` per layer, resident experts read through the slot tables) are
captured once per batch size with every buffer preallocated, and after layer l the graph publishes layer l's
routing through ``kernels.signal`` (seq = base + l), so the host can follow the step layer by layer with
``Readback.wait`` while it runs. Replaying the graph is the step.
"""
import torch

from .kernels.moe_layer import DecodeLayerBuffers, decode_layers
from .kernels.signal import signal
from .readback import Readback


class DecodeStep:
    """``layers`` MoE layers for ``batch`` tokens. ``x`` bf16 [layers, batch, H] holds each layer's input (the
    attention and hyper-connection segments between MoE layers are outside this path); the outputs are
    ``bufs[l].y``. Router weights [layers, E, H], shared-gate rows [layers, H], shared records [layers, record]."""

    def __init__(self, x, router_w, sh_gate_w, shared_records, map_t, slot_ptr_t, k: int, inter: int, *, bias=None,
                 readback: Readback | None = None, fused: bool = True, prefetch_next: bool = False):
        self.x = x
        nl, b, h = x.shape
        e = router_w.shape[1]
        if readback is not None and readback.layers < nl:
            raise ValueError("the readback has fewer layer slots than the step has layers")
        self.layers, self.batch, self.k = nl, b, k
        self.readback = readback
        self.ctrl_dev = torch.zeros(2, dtype=torch.int64, device=x.device)
        self.bufs = [DecodeLayerBuffers(b, k, h, inter, e, x.device) for _ in range(nl)]
        self._args = (router_w, sh_gate_w, shared_records, map_t, slot_ptr_t, bias, fused)
        self.prefetch_next = prefetch_next
        self._side = torch.cuda.Stream(device=x.device) if prefetch_next else None
        self.step()                      # eager warm-up: first-use setup happens outside the capture
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.step()
        torch.cuda.synchronize()

    def step(self):
        router_w, sh_gate_w, shared_records, map_t, slot_ptr_t, bias, fused = self._args
        rb = self.readback

        def publish(l):
            if rb is not None:
                bf = self.bufs[l]
                signal(bf.ids, bf.w, rb.ids, rb.w, rb.seq, rb.ctrl, l)

        decode_layers(self.x, router_w, sh_gate_w, shared_records, map_t, slot_ptr_t, self.k, self.bufs, bias=bias,
                      fused=fused, prefetch_next=self.prefetch_next, side=self._side, after_layer=publish)

    def replay(self, base: int = 0, pos: int = 0):
        """Launch the captured step (asynchronously); layer l's routing is readable once seq >= base + l."""
        if self.readback is not None:
            self.readback.begin(pos, base)
        self.graph.replay()
