"""The C-ABI library loads without a GPU and exports every entry point include/*.h declares (CPU)."""
import ctypes
import re
from pathlib import Path

import pytest

from conftest import ROOT

HEADER_DIR = ROOT / "include"


def _declared():
    names = set()
    for h in HEADER_DIR.glob("*.h"):
        txt = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(ssb_\w+)\s*\(", txt))
    return sorted(names)


def test_header_declares_entry_points():
    names = _declared()
    for must in ("ssb_topk_stable", "ssb_router_logits", "ssb_router_select", "ssb_moe_align", "ssb_moe_decode",
                 "ssb_moe_decode_layer", "ssb_combine_rank_order", "ssb_gemv_affine", "ssb_gemv_dense"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from slotstream_b200 import _lib
    if not _lib.LIB_PATH.exists():
        pytest.skip("library not built (run slotstream-spark_b200/build.py)")
    h = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in _declared() if not hasattr(h, n)]
    assert not missing, missing
    assert b"sm_100a" in _lib.lib().ssb_version()


def test_python_binding_covers_header():
    from slotstream_b200 import _lib
    declared = set(_declared()) - {"ssb_version"}
    assert declared <= set(_lib.SIGNATURES), declared - set(_lib.SIGNATURES)


def test_argument_errors_need_no_gpu():
    """Argument checks fire before any launch, with the reference's exception types."""
    import torch
    from slotstream_b200.kernels.topk_stable import topk_stable
    from slotstream_b200.kernels.moe_align import moe_align, padded_rows
    with pytest.raises(ValueError):
        topk_stable(torch.zeros(2, 8, dtype=torch.float64), 3)
    with pytest.raises(ValueError):
        topk_stable(torch.zeros(2, 8), 9)
    with pytest.raises(ValueError):
        moe_align(torch.zeros(4, dtype=torch.int64), 2, 64)
    with pytest.raises(ValueError):
        moe_align(torch.zeros(4, dtype=torch.int32), 0, 64)
    assert padded_rows(0, 4, 64) == 256 and padded_rows(10, 1, 1) == 10


def test_no_cpu_fallback():
    """A CPU tensor reaching a kernel raises instead of silently computing on the host."""
    import torch
    from slotstream_b200.kernels.topk_stable import topk_stable
    from slotstream_b200 import _lib
    if not _lib.LIB_PATH.exists():
        pytest.skip("library not built")
    with pytest.raises(ValueError, match="CUDA"):
        topk_stable(torch.zeros(2, 8), 3)


def test_wait_seq_is_host_side_and_bounded():
    """ssb_wait_seq is host code (acquire loads on a pinned word): it returns when the word reaches the target and
    gives up with SSB_ETIMEDOUT after its bound, with no GPU involved."""
    import torch
    from slotstream_b200 import _lib
    if not _lib.LIB_PATH.exists():
        pytest.skip("library not built")
    seq = torch.tensor([41], dtype=torch.int64)
    L = _lib.lib()
    assert L.ssb_wait_seq(seq.data_ptr(), 41, 10_000_000) == _lib.SSB_OK
    assert L.ssb_wait_seq(seq.data_ptr(), 42, 5_000_000) == _lib.SSB_ETIMEDOUT
    assert L.ssb_wait_seq(None, 1, 1) == _lib.SSB_EINVAL


def test_signal_argument_errors_need_no_gpu():
    import torch
    from slotstream_b200.kernels.signal import SLOT, signal
    with pytest.raises(ValueError):
        signal(torch.zeros(SLOT + 1, dtype=torch.int32), torch.zeros(SLOT + 1), torch.zeros(64, dtype=torch.int32),
               torch.zeros(64), torch.zeros(1, dtype=torch.int64), torch.zeros(2, dtype=torch.int64), 0)


def test_copy_async_argument_errors_need_no_gpu():
    """ssb_copy_async checks its arguments on the host before any CUDA call; a zero-byte copy is a no-op."""
    import ctypes
    from slotstream_b200 import _lib
    L = _lib.lib()
    buf = ctypes.create_string_buffer(16)
    addr = ctypes.addressof(buf)
    assert L.ssb_copy_async(None, addr, 16, None) == _lib.SSB_EINVAL
    assert L.ssb_copy_async(addr, None, 16, None) == _lib.SSB_EINVAL
    assert L.ssb_copy_async(addr, addr, -1, None) == _lib.SSB_EINVAL
    assert L.ssb_copy_async(addr, addr, 0, None) == _lib.SSB_OK
