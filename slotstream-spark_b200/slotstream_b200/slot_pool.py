"""HBM expert slot pool for streaming decode (additive): the B200 side of slotio's Pool + Ensurer
(slotio/include/slotio/pool.hpp:23-160, slotio/src/ensure.cpp), over the C entry points ssb_pool_*.

Records live in slots of 1 GiB device chunks; ``map`` (int32 [layers * experts], -1 = absent) and ``slot_ptr``
(int64 [slots]) are device tables the decode kernels read every expert through. ``ensure(layer, experts)``
makes a layer's experts resident: misses are copied from pinned host records (``host_table``) on a copy stream
into CLOCK victims and published in ``map``; the compute stream waits for them. ``release()`` after the layer's
kernels records the event a victim's next copy waits for, so no slot is overwritten while a kernel reads it.
"""
import ctypes

import numpy as np
import torch

from . import _lib


class _DeviceArray:
    """Zero-copy view of device memory the pool owns, for torch.as_tensor."""

    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}


class SlotPool:
    def __init__(self, record_bytes: int, layers: int, experts: int = 512, chunk_bytes: int = 1 << 30,
                 max_slots: int | None = None):
        self.record_bytes, self.layers, self.experts = record_bytes, layers, experts
        self.max_slots = max_slots or layers * experts
        L = _lib.lib()
        self.h = L.ssb_pool_create(record_bytes, chunk_bytes, layers, experts, self.max_slots)
        if not self.h:
            raise RuntimeError("ssb_pool_create failed (bad sizes or no CUDA device)")
        self.map = self.slot_ptr = None
        self._tables()

    def _tables(self):
        m, sp = ctypes.c_void_p(), ctypes.c_void_p()
        ml, ns, nc = ctypes.c_int64(), ctypes.c_int32(), ctypes.c_int32()
        _lib.check(_lib.lib().ssb_pool_tables(self.h, ctypes.byref(m), ctypes.byref(sp), ctypes.byref(ml),
                                              ctypes.byref(ns), ctypes.byref(nc)), "pool tables")
        self.map = torch.as_tensor(_DeviceArray(m.value, ml.value, "<i4"), device="cuda")
        self.slot_ptr = torch.as_tensor(_DeviceArray(sp.value, self.max_slots, "<i8"), device="cuda")
        self.slots, self.chunks = ns.value, nc.value

    def resize(self, n_slots: int):
        _lib.check(_lib.lib().ssb_pool_resize(self.h, n_slots), "pool resize")
        self._tables()

    def ensure(self, layer: int, experts, host_table, copy_stream=None, compute_stream=None):
        """-> (slot per requested expert (numpy int32), (hits, misses, bytes))."""
        ex = np.ascontiguousarray(np.asarray(experts, dtype=np.int32).reshape(-1))
        out = np.empty(ex.size, dtype=np.int32)
        st = np.zeros(3, dtype=np.int64)
        cs = copy_stream.cuda_stream if copy_stream is not None else _lib.stream()
        ks = compute_stream.cuda_stream if compute_stream is not None else _lib.stream()
        rc = _lib.lib().ssb_pool_ensure(self.h, layer, ex.ctypes.data, ex.size, ctypes.cast(host_table, ctypes.c_void_p),
                                        cs, ks, out.ctypes.data, st.ctypes.data)
        if rc == _lib.SSB_ETOOBIG:
            raise RuntimeError("pool exhausted: the misses of this layer do not fit in the unpinned slots")
        _lib.check(rc, "pool ensure")
        return out, tuple(int(v) for v in st)

    def release(self, compute_stream=None):
        ks = compute_stream.cuda_stream if compute_stream is not None else _lib.stream()
        _lib.check(_lib.lib().ssb_pool_release(self.h, ks), "pool release")

    def counters(self):
        h, m, b = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        _lib.check(_lib.lib().ssb_pool_counters(self.h, ctypes.byref(h), ctypes.byref(m), ctypes.byref(b)), "counters")
        return h.value, m.value, b.value

    def close(self):
        if self.h:
            self.map = self.slot_ptr = None
            _lib.lib().ssb_pool_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def host_table(records_ptr: int, record_bytes: int, layers: int, experts: int, per_layer: bool = True):
    """ctypes array of host record addresses indexed layer * experts + e: ``records_ptr`` holds ``layers *
    experts`` records (per_layer) or ``experts`` records shared by every layer."""
    t = (ctypes.c_void_p * (layers * experts))()
    for l in range(layers):
        for e in range(experts):
            t[l * experts + e] = records_ptr + ((l * experts + e) if per_layer else e) * record_bytes
    return t


def decode_layer_streaming(pool: SlotPool, table, x, w_router, layer: int, shared_record, sh_gate_w, k: int, bufs,
                           *, bias=None, copy_stream=None, ids_host=None):
    """One decode MoE layer whose routed experts stream through the pool (ssb_pool_decode_layer): router (logits
    + select), the chosen ids to the host, ensure (misses copied on ``copy_stream``), then gate_up / down /
    combine through the pool's tables on the current stream, and release, with the host side in native code.
    ``ids_host``: pinned int32 [rows, k] buffer for the ids' readback (allocated when None).
    Returns (y, (hits, misses, bytes))."""
    from .kernels.moe_layer import _addr
    r, h = x.shape
    if x.dtype != torch.bfloat16 or not x.is_contiguous() or (r, k, h) != (bufs.rows, bufs.topk, bufs.hidden):
        raise ValueError("x must be contiguous bf16 [rows, hidden] matching the buffers")
    if ids_host is None:
        ids_host = torch.empty((r, k), dtype=torch.int32).pin_memory()
    st = np.zeros(3, dtype=np.int64)
    P = _lib.ptr
    cs = copy_stream.cuda_stream if copy_stream is not None else _lib.stream()
    rc = _lib.lib().ssb_pool_decode_layer(
        pool.h, int(layer), P(x), r, k, h, bufs.inter, bufs.experts, P(w_router), P(sh_gate_w), P(bias),
        ctypes.cast(table, ctypes.c_void_p), _addr(shared_record), P(bufs.ws), P(bufs.ids), P(bufs.w),
        P(bufs.sh_gate), ids_host.data_ptr(), P(bufs.h), P(bufs.o), P(bufs.out), P(bufs.y), P(bufs.err), cs,
        _lib.stream(), st.ctypes.data)
    if rc == _lib.SSB_ETOOBIG:
        raise RuntimeError("pool exhausted: the misses of this layer do not fit in the unpinned slots")
    _lib.check(rc, "pool_decode_layer")
    return bufs.y, tuple(int(v) for v in st)
