"""Model shape behind the module constants of the drop-in kernel modules.

The reference's kernel modules carry the model's shape as constants (``HID, INTER, TOPK = 2560, 640, 10``,
``RECORD_BYTES`` and the nine ``O_*`` piece offsets; kernels/fused_moe_affine.py:28-32,
kernels/moe_gemv_affine.py:21-25), and its callers read them: ``SweepMoE.layer`` / ``_group`` size ``out_rows``
and their per-launch buffers as ``[rows, fm.HID]`` and count staging bytes with ``fm.RECORD_BYTES``
(model/moe_sweep.py:100, :123, :173). Here the kernels take every shape from their tensors; the constants only
answer such callers, so they follow one configured shape. They start at the reference model's 2560 / 640 (the
values of the modules these replace); ``configure`` switches them, e.g. to BASELINE's 2048 / 512, before the
caller runs.
"""
import sys

from ..records import REFERENCE_LAYOUT, RecordLayout

_MODULES = ("slotstream_b200.kernels.fused_moe_affine", "slotstream_b200.kernels.moe_gemv_affine")
_CURRENT = {"layout": REFERENCE_LAYOUT, "topk": 10}


def constants(layout: RecordLayout, topk: int) -> dict:
    """The module constants of one shape: HID, INTER, TOPK, RECORD_BYTES, O_GATE_W .. O_DOWN_B."""
    names = ("O_GATE_W", "O_GATE_S", "O_GATE_B", "O_UP_W", "O_UP_S", "O_UP_B", "O_DOWN_W", "O_DOWN_S", "O_DOWN_B")
    c = dict(zip(names, layout.offsets()))
    c.update(HID=layout.hidden, INTER=layout.inter, TOPK=int(topk), RECORD_BYTES=layout.record_bytes)
    return c


def current() -> RecordLayout:
    return _CURRENT["layout"]


def configure(hidden: int, inter: int, topk: int = 10, gs: int = 64) -> RecordLayout:
    """Set the shape the module constants describe (hidden size, expert intermediate size, router top-k, group
    size) in every drop-in module, loaded now or later. Returns the record layout of that shape."""
    if topk < 1:
        raise ValueError(f"topk must be positive, got {topk}")
    lay = RecordLayout(int(hidden), int(inter), int(gs))
    _CURRENT["layout"], _CURRENT["topk"] = lay, int(topk)
    c = constants(lay, topk)
    for name in _MODULES:
        mod = sys.modules.get(name)
        if mod is not None:
            for k, v in c.items():
                setattr(mod, k, v)
    return lay


def install(module_globals: dict) -> None:
    """Called by each drop-in module at import: its constants start at the configured shape."""
    module_globals.update(constants(_CURRENT["layout"], _CURRENT["topk"]))
