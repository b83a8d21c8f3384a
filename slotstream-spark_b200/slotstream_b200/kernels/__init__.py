"""Drop-in mirrors of slotstream_spark/kernels on the MoE hot path, backed by the sm_100a C-ABI library.

``configure(hidden, inter, topk=10, gs=64)`` sets the model shape that the modules' constants (HID, INTER, TOPK,
RECORD_BYTES, O_*) report to callers that read them; the kernels themselves take every shape from their tensors."""
from .shape import configure

__all__ = ["configure"]
