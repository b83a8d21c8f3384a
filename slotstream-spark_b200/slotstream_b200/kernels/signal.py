"""Router readback signal -- drop-in for slotstream_spark/kernels/signal.py.

At the end of a layer's segment graph one warp copies the layer's top-k expert ids and weights into that layer's slot
of the pinned readback buffers and then publishes ``seq = base + layer`` with a system-scope release exchange
(kernels/signal.py:1-7), so a host thread that observes the word with an acquire load also sees the ids. ``base``
is ``ctrl[1]``, written by the host before the step's first graph launches. Layer 48 has no ids (``ids=None``): it
only publishes. Graph-capturable: it reads ``ctrl`` on the device at replay time.
"""
import torch

from .. import _lib
from .gemv_affine import _note

SLOT = 32      # elements per layer slot: 3 rows x 10 experts at most (kernels/signal.py:11)


def signal(ids, w, slot_ids, slot_w, seq, ctrl, layer):
    """ids int32 [R, 10] and w fp32 [R, 10] (device, contiguous) or None; slot_ids / slot_w / seq are the pinned
    readback buffers (int32 [49*SLOT], float32 [49*SLOT], int64 [1]); ctrl int64 [2] (pos, base), pinned or on the
    device (kernels/signal.py:29-37, same argument check)."""
    n = 0 if ids is None else ids.numel()
    if n > SLOT:
        raise ValueError(f"at most {SLOT} ids per layer slot")
    if ids is not None and (ids.dtype != torch.int32 or w is None or w.dtype != torch.float32 or w.numel() != n
                            or not ids.is_contiguous() or not w.is_contiguous()):
        raise ValueError("ids must be contiguous int32 and w contiguous fp32 of the same size")
    for t, dt in ((slot_ids, torch.int32), (slot_w, torch.float32), (seq, torch.int64), (ctrl, torch.int64)):
        if t.dtype != dt:
            raise ValueError("readback buffers: slot_ids int32, slot_w fp32, seq and ctrl int64")
    rc = _lib.lib().ssb_signal(_lib.ptr(ids), _lib.ptr(w), n, slot_ids.data_ptr(), slot_w.data_ptr(), seq.data_ptr(),
                               ctrl.data_ptr(), int(layer), _lib.stream())
    _lib.check(rc, "signal")
    _note("signal")
