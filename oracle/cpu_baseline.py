"""Timed CPU baseline of the MoE path -- TEST/BENCH INFRASTRUCTURE ONLY (bench.py's cpu_baseline leg and
its ``--impl reference`` arm).

A torch-CPU restatement of the reference's own CPU path, timed on the host's cores:
* decode: model/reference_torch.py:118-134 (``moe_ref``): router F.linear, fp32 softmax, top-k, renormalise,
  then per routed expert ``affine_ref.dequant`` (kernels/affine_ref.py:22-31) of its record and
  silu(G x) * (U x) -> D h, summed in rank order, plus the sigmoid-gated shared expert. Dequantisation is
  inside the timed region, as on the reference's CPU branch (model/layers.py:391-397 reads pool.slot_weights
  per call).
* prefill: the same dequant + matmul grouped per expert (the HF experts loop the reference's oracle follows,
  third_party/transformers-5.19.0-qwen4_exp/...modeling_qwen4_exp.py:925-949), over a bounded token sample.
"""
import os
import time

import numpy as np
import torch
import torch.nn.functional as F

from . import moe_oracle as O


def _t_bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def dequant_t(q_u32, s_bits, b_bits, gs=64):
    """torch restatement of kernels/affine_ref.py:22-31 (unpack + q*s + b in fp32)."""
    b = torch.from_numpy(np.ascontiguousarray(q_u32)).view(torch.uint8)
    u = torch.stack([b & 15, b >> 4], dim=-1).reshape(b.shape[0], -1).to(torch.float32)
    s = _t_bf16(s_bits).to(torch.float32).repeat_interleave(gs, dim=1)
    bb = _t_bf16(b_bits).to(torch.float32).repeat_interleave(gs, dim=1)
    return u * s + bb


def _expert_t(layout, rec):
    return [dequant_t(q, s, b, layout.gs) for (q, s, b) in O.record_pieces(layout, rec)]


class CpuLayer:
    """One MoE layer's weights on the host: 512 routed records, the shared record, router and gate rows."""

    def __init__(self, layout, seed, layer=0, experts=512):
        from slotstream_b200 import synth
        self.layout = layout
        self.recs = [synth.expert_record(layout, seed, layer, e) for e in range(experts)]
        self.shared = synth.expert_record(layout, seed, layer, experts)
        self.rw = _t_bf16(synth.router_weight(seed, experts, layout.hidden, layer)).float()
        self.sg = _t_bf16(synth.shared_gate_weight(seed, layout.hidden, layer)).float()
        self.bias = torch.from_numpy(synth.zipf_bias(experts))


def decode_token_layer(L: CpuLayer, x, k=10):
    """One token through one layer (x fp32 [1, H]); dequantisation inside."""
    logits = F.linear(x, L.rw) + L.bias
    probs = F.softmax(logits, dtype=torch.float, dim=-1)
    tv, ti = torch.topk(probs, k, dim=-1)
    tv = tv / tv.sum(-1, keepdim=True)
    out = torch.zeros_like(x)
    for r in range(k):
        g, u, d = _expert_t(L.layout, L.recs[int(ti[0, r])])
        h = F.silu(g @ x[0]) * (u @ x[0])
        out[0] += tv[0, r] * (d @ h)
    g, u, d = _expert_t(L.layout, L.shared)
    sh = d @ (F.silu(g @ x[0]) * (u @ x[0]))
    sh = torch.sigmoid(F.linear(x, L.sg)) * sh
    return out + sh


def prefill_chunk(L: CpuLayer, x, k=10):
    """T tokens through one layer, experts grouped (each routed expert dequantised once per call)."""
    logits = F.linear(x, L.rw) + L.bias
    probs = F.softmax(logits, dtype=torch.float, dim=-1)
    tv, ti = torch.topk(probs, k, dim=-1)
    tv = tv / tv.sum(-1, keepdim=True)
    out = torch.zeros_like(x)
    flat = ti.reshape(-1)
    for e in torch.unique(flat).tolist():
        rows = torch.nonzero(flat == e).squeeze(1)
        tok, rank = rows // k, rows % k
        g, u, d = _expert_t(L.layout, L.recs[e])
        xe = x[tok]
        y = (F.silu(xe @ g.T) * (xe @ u.T)) @ d.T
        out.index_add_(0, tok, y * tv[tok, rank][:, None])
    g, u, d = _expert_t(L.layout, L.shared)
    sh = (F.silu(x @ g.T) * (x @ u.T)) @ d.T
    return out + torch.sigmoid(F.linear(x, L.sg)) * sh


def time_decode(layout, seed=0, seconds=10.0, threads=None, layers_per_token=48):
    """Tokens/s of the CPU decode path over a bounded sample: token-layers are timed until `seconds` pass;
    tokens/s = 1 / (mean seconds per token-layer * layers_per_token)."""
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    L = CpuLayer(layout, seed)
    rng = np.random.default_rng(seed)
    n, t0 = 0, time.perf_counter()
    with torch.no_grad():
        while True:
            x = torch.from_numpy(rng.standard_normal((1, layout.hidden)).astype(np.float32)).bfloat16().float()
            decode_token_layer(L, x)
            n += 1
            if time.perf_counter() - t0 >= seconds:
                break
    per = (time.perf_counter() - t0) / n
    return {"value": 1.0 / (per * layers_per_token), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n} token-layers of the config[0] layer (b=1, Zipf routing), dequant inside; "
                      f"tokens/s = 1/(mean token-layer time x {layers_per_token} layers); torch {torch.__version__}"}


def time_prefill(layout, tokens, seed=0, seconds=10.0, threads=None, sample_tokens=1024, layer=None):
    """Tokens/s of the CPU prefill path on chunks of `sample_tokens` tokens until `seconds` pass."""
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    L = layer if layer is not None else CpuLayer(layout, seed)
    rng = np.random.default_rng(seed + 1)
    n, t0 = 0, time.perf_counter()
    with torch.no_grad():
        while True:
            x = torch.from_numpy(rng.standard_normal((sample_tokens, layout.hidden)).astype(np.float32)).bfloat16().float()
            prefill_chunk(L, x)
            n += sample_tokens
            if time.perf_counter() - t0 >= seconds:
                break
    el = time.perf_counter() - t0
    return {"value": n / el, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n} tokens in chunks of {sample_tokens} (workload chunk {tokens}) of the config[0] layer, "
                      f"Zipf routing, experts grouped and dequantised once per chunk; torch {torch.__version__}"}
