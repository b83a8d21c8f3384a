"""Router with statically reserved logits (ssb_router_topk_static) against the workspace router (GPU).

The entry point takes no workspace and allocates nothing; this file is collected last so it also runs after
every other GPU test has used the same process and device. It calls the C ABI directly.
"""
import numpy as np
import pytest
import torch

from gpu_helpers import bf16_tensor
from slotstream_b200 import _lib, synth

pytestmark = pytest.mark.gpu
E, K, H = 512, 10, 2048
STATIC_LOGITS = 65536          # capacity of the static logits array, in floats


def _static(x, rw, sg, bias, flags=0):
    t = x.shape[0]
    idx = torch.full((t, K), -7, dtype=torch.int32, device="cuda")
    w = torch.full((t, K), -7.0, dtype=torch.float32, device="cuda")
    sh = torch.full((t,), -7.0, dtype=torch.float32, device="cuda")
    rc = _lib.lib().ssb_router_topk_static(_lib.ptr(x), _lib.ptr(rw), _lib.ptr(sg), t, H, E, K, _lib.ptr(bias),
                                           flags, _lib.ptr(idx), _lib.ptr(w), _lib.ptr(sh) if sg is not None else None,
                                           _lib.stream())
    _lib.check(rc, "router_topk_static")
    torch.cuda.synchronize()
    return idx, w, sh


def _workspace(x, rw, sg, bias, round_bf16=False):
    from slotstream_b200.kernels.router import router_topk
    out = router_topk(x, rw, K, bias=bias, sh_gate_w=sg, logits_round_bf16=round_bf16)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("tokens", [1, 16, 127])
def test_static_router_matches_workspace_router_twice(tokens):
    rw = bf16_tensor(synth.router_weight(0, E, H, 0))
    sg = bf16_tensor(synth.shared_gate_weight(0, H, 0))
    bias = torch.from_numpy(synth.zipf_bias(E)).cuda()
    for call in range(2):   # two calls in a row, different inputs: nothing may carry over between them
        x = bf16_tensor(synth.activations(50 + call, tokens, H))
        idx, w, sh = _static(x, rw, sg, bias)
        ridx, rwt, rsh = _workspace(x, rw, sg, bias)
        assert torch.equal(idx, ridx)
        torch.testing.assert_close(w, rwt, rtol=1e-6, atol=0.0)
        torch.testing.assert_close(sh, rsh, rtol=1e-6, atol=0.0)


def test_static_router_allocates_nothing():
    """With its outputs allocated up front, a call leaves torch's allocator and the device's free memory as
    they were: the logits live in the library's own device array."""
    rw = bf16_tensor(synth.router_weight(0, E, H, 0))
    sg = bf16_tensor(synth.shared_gate_weight(0, H, 0))
    x = bf16_tensor(synth.activations(70, 64, H))
    idx = torch.empty((64, K), dtype=torch.int32, device="cuda")
    w = torch.empty((64, K), dtype=torch.float32, device="cuda")
    sh = torch.empty((64,), dtype=torch.float32, device="cuda")

    def call():
        _lib.check(_lib.lib().ssb_router_topk_static(_lib.ptr(x), _lib.ptr(rw), _lib.ptr(sg), 64, H, E, K, None, 0,
                                                     _lib.ptr(idx), _lib.ptr(w), _lib.ptr(sh), _lib.stream()),
                   "router_topk_static")
        torch.cuda.synchronize()

    call()                                   # the first call on the device looks the array's address up
    alloc0, free0 = torch.cuda.memory_allocated(), torch.cuda.mem_get_info()[0]
    for _ in range(3):
        call()
    assert torch.cuda.memory_allocated() == alloc0
    assert torch.cuda.mem_get_info()[0] == free0


def test_static_router_without_shared_gate_and_bf16_logits():
    rw = bf16_tensor(synth.router_weight(0, E, H, 0))
    x = bf16_tensor(synth.activations(60, 8, H))
    for _ in range(2):
        idx, w, _ = _static(x, rw, None, None, flags=_lib.ROUTER_ROUND_BF16)
        ridx, rwt = _workspace(x, rw, None, None, round_bf16=True)
        assert torch.equal(idx, ridx)
        torch.testing.assert_close(w, rwt, rtol=1e-6, atol=0.0)


def test_static_router_refuses_more_than_its_capacity():
    rw = bf16_tensor(synth.router_weight(0, E, H, 0))
    sg = bf16_tensor(synth.shared_gate_weight(0, H, 0))
    t = STATIC_LOGITS // (E + 1) + 1
    x = torch.zeros(t, H, dtype=torch.bfloat16, device="cuda")
    idx = torch.full((t, K), -7, dtype=torch.int32, device="cuda")
    w = torch.zeros(t, K, dtype=torch.float32, device="cuda")
    sh = torch.zeros(t, dtype=torch.float32, device="cuda")
    rc = _lib.lib().ssb_router_topk_static(_lib.ptr(x), _lib.ptr(rw), _lib.ptr(sg), t, H, E, K, None, 0,
                                           _lib.ptr(idx), _lib.ptr(w), _lib.ptr(sh), _lib.stream())
    assert rc == _lib.SSB_ETOOBIG
    with pytest.raises(RuntimeError, match="static scratch"):
        _lib.check(rc, "router_topk_static")
    torch.cuda.synchronize()
    assert bool((idx == -7).all())          # nothing was launched
