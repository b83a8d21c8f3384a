"""ctypes binding of libslotstream_b200.so (the C ABI declared in include/slotstream_b200.h).

There is no CPU fallback: if the library is missing, or a tensor is not on a CUDA device, the call raises.
Launches go to torch's current CUDA stream, so the Python wrappers are CUDA-graph capturable as long as
the caller provides every output and workspace.
"""
import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libslotstream_b200.so"

SSB_OK, SSB_EINVAL, SSB_EUNSUPPORTED, SSB_ENODEVICE, SSB_ETOOBIG, SSB_ETIMEDOUT = 0, -1, -2, -3, -4, -5
ERR_EXPERT_RANGE, ERR_UNMAPPED, ERR_SLOT_RANGE, ERR_MISALIGNED, ERR_TIMEOUT = 1, 2, 4, 8, 16
BF16, F32 = 0, 1
ROUTER_ROUND_BF16, ROUTER_SHARED_GATE = 1, 2
DECODE_PDL = 1
DECODE_FUSED_CUDA_CORES = 4
DECODE_FUSED_TENSOR_CORES = 8

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64

# name -> argtypes (every entry point returns int)
SIGNATURES = {
    "ssb_device_check": [],
    "ssb_kernel_smem": [ctypes.c_char_p],
    "ssb_set_gemm_sm_reserve": [_I32],
    "ssb_set_gate_up_tile": [_I32],
    "ssb_set_wait_limit_ns": [_I64],
    "ssb_topk_stable": [_P, _P, _I64, _I32, _I32, _P, _P, _P],
    "ssb_router_logits": [_P, _P, _P, _I64, _I32, _I32, _I32, _P, _P],
    "ssb_router_select": [_P, _I32, _I64, _I32, _I32, _P, _I32, _P, _P, _P, _P, _P],
    "ssb_moe_align": [_P, _I64, _P, _I32, _I32, _I32, _P, _P, _P, _P],
    "ssb_moe_decode": [_P, _I32, _P, _P, _I64, _I32, _I32, _I32, _I32, _P, _I64, _P, _I64, _P, _P, _P, _P, _P],
    "ssb_moe_decode_layer": [_P, _P, _P, _I64, _I32, _I32, _I32, _I32, _P, _I64, _P, _I64, _P, _P, _P, _P, _P, _P,
                             _P, _I32, _P, _P],
    "ssb_router_select_resolve": [_P, _I32, _I64, _I32, _I32, _P, _I32, _P, _P, _P, _I32, _P, _I64, _P, _I64, _P,
                                  _I64, _P, _P],
    "ssb_ep_plan": [_P, _P, _I64, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P],
    "ssb_gather_rows": [_P, _I64, _P, _I64, _I64, _P, _P, _P],
    "ssb_ep_unpack": [_P, _I64, _I32, _P, _P, _I32, _I64, _P, _P, _P, _P, _P, _P, _P],
    "ssb_combine_rows": [_P, _P, _P, _I64, _I32, _P, _P],
    "ssb_combine_rows_bf16": [_P, _P, _P, _I64, _I32, _P, _P],
    "ssb_ep_combine": [_P, _P, _P, _P, _P, _I64, _I32, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _P],
    "ssb_ep_combine_bf16": [_P, _P, _P, _I64, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _P],
    "ssb_moe_decode_fused": [_P, _I64, _I32, _I32, _I32, _I32, _P, _P, _P, _I32, _I32, _P, _I64, _P, _I64, _P, _P, _P,
                             _P, _P, _P, _P, _P, _P, _P, _P, _P, _P],
    "ssb_pool_create": [_I64, _I64, _I32, _I32, _I32],
    "ssb_pool_destroy": [_P],
    "ssb_pool_resize": [_P, _I32],
    "ssb_pool_tables": [_P, _P, _P, _P, _P, _P],
    "ssb_pool_ensure": [_P, _I32, _P, _I32, _P, _P, _P, _P, _P],
    "ssb_pool_release": [_P, _P],
    "ssb_pool_counters": [_P, _P, _P, _P],
    "ssb_copy_async": [_P, _P, _I64, _P],
    "ssb_pool_decode_layer": [_P, _I32, _P, _I64, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                              _P, _P, _P, _P, _P, _P, _P, _P],
    "ssb_router_topk_static": [_P, _P, _P, _I64, _I32, _I32, _I32, _P, _I32, _P, _P, _P, _P],
    "ssb_signal": [_P, _P, _I32, _P, _P, _P, _P, _I32, _P],
    "ssb_wait_seq": [_P, _I64, _I64],
    "ssb_copy_sm": [_P, _P, _I64, _P],
    "ssb_prefetch_l2": [_P, _I64, _P],
    "ssb_combine_rank_order": [_P, _I64, _I32, _I32, _P, _P],
    "ssb_combine_layer": [_P, _I64, _I32, _I32, _P, _P, _P, _P],
    "ssb_gemv_affine": [_P, _I32, _I64, _P, _P, _P, _I32, _I32, _I32, _I32, _P, _P],
    "ssb_gemv_dense": [_P, _I32, _I64, _P, _I32, _I32, _P, _P],
    "ssb_fused_moe_gate_up": [_P, _I64, _I32, _I32, _P, _I64, _P, _P, _P, _I64, _P, _I32, _P, _P, _P],
    "ssb_fused_moe_down": [_P, _I64, _I32, _I32, _P, _P, _P, _P, _I64, _P, _I32, _P, _P, _P],
    "ssb_gemm_affine4": [_P, _I64, _I32, _P, _P, _P, _I32, _I32, _P, _P],
    "ssb_prefill_experts": [_P, _I64, _I32, _I32, _P, _P, _I64, _P, _P, _P, _I64, _P, _I32, _I32, _P, _P, _P, _P, _P],
    "ssb_permute_rows": [_P, _I64, _I32, _P, _I64, _P, _P, _I64, _P, _P],
    "ssb_sorted_gate_up": [_P, _I32, _I32, _P, _I64, _P, _P, _P, _I64, _P, _I32, _I32, _P, _P, _P],
    "ssb_sorted_down": [_P, _I64, _I32, _I32, _P, _P, _P, _P, _I64, _P, _I32, _I32, _P, _P, _P],
    "ssb_gemm_dense": [_P, _I64, _I32, _P, _I32, _P, _I64, _P],
}

_lib = None


def lib():
    """Load the library once; raises if it has not been built (run slotstream-spark_b200/build.py)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH.name} is not built: run `python slotstream-spark_b200/build.py` "
                               "(no CPU fallback exists)")
        h = ctypes.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            f = getattr(h, name)
            f.argtypes = args
            f.restype = ctypes.c_int
        h.ssb_version.argtypes = []
        h.ssb_version.restype = ctypes.c_char_p
        h.ssb_pool_create.restype = ctypes.c_void_p
        h.ssb_pool_destroy.restype = None
        _lib = h
    return _lib


def ptr(t):
    """Device address of a tensor (None -> NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("tensor must live on a CUDA device (this library has no CPU path)")
    return t.data_ptr()


def stream():
    return torch.cuda.current_stream().cuda_stream


_NAMES = {SSB_EINVAL: "SSB_EINVAL (bad argument)", SSB_EUNSUPPORTED: "SSB_EUNSUPPORTED (shape not handled)",
          SSB_ENODEVICE: "SSB_ENODEVICE (not an sm_100 device)",
          SSB_ETOOBIG: "SSB_ETOOBIG (request exceeds a fixed capacity: static scratch or slot pool)",
          SSB_ETIMEDOUT: "SSB_ETIMEDOUT (a bounded wait gave up)"}


def check(rc, what):
    if rc != SSB_OK:
        name = _NAMES.get(rc, f"cudaError {rc}")
        raise RuntimeError(f"{what} failed: {name}")


def smem(name: str) -> int:
    return int(lib().ssb_kernel_smem(name.encode()))
