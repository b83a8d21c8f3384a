"""Timed CPU baseline of the MoE path -- TEST/BENCH INFRASTRUCTURE ONLY (bench.py's cpu_baseline leg and
its ``--impl reference`` arm).

A torch-CPU restatement of the reference's own CPU path, timed on the host's cores:
* decode: model/reference_torch.py:118-134 (``moe_ref``): router F.linear, fp32 softmax, stable top-k
  (kernels/topk_stable.py:1-13: ties to the lower index), renormalise, then per routed expert
  ``affine_ref.dequant`` (kernels/affine_ref.py:22-31) of its record and silu(G x) * (U x) -> D h, summed in rank
  order, plus the sigmoid-gated shared expert. Dequantisation is inside the timed region, as on the reference's CPU
  branch (model/layers.py:391-397 reads pool.slot_weights per call).
* prefill: the same arithmetic with each routed expert dequantised once per chunk and its rows batched (the HF
  experts loop the reference's oracle follows, third_party/transformers-5.19.0-qwen4_exp/...modeling_qwen4_exp.py
  :925-949), over whole chunks of the benchmark's token count.

The layer can be built from the seeded generator (``CpuLayer.from_seed``) or from the benchmark's own inputs copied
back from the GPU (``CpuLayer.from_tensors``), so the CPU result of a timed chunk doubles as a parity check of the
GPU output on the same bytes (``parity``).
"""
import os
import platform
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


def host_info(threads):
    """The host the CPU numbers come from: threads used, logical CPUs, CPU model, torch version."""
    model = platform.processor() or ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cores": threads, "nproc": os.cpu_count(), "cpu_model": model, "torch": torch.__version__}


class CpuLayer:
    """One MoE layer's weights on the host: E routed records and the shared record (uint8 [E + 1, record_bytes]),
    the router (fp32 values of bf16 [E, H]), the shared-expert gate (fp32 values of bf16 [1, H]), the logit bias."""

    def __init__(self, layout, recs, router_w, sh_gate_w, bias):
        self.layout = layout
        self.recs = recs
        self.shared = recs[-1]
        self.rw = router_w
        self.sg = sh_gate_w
        self.bias = bias

    @classmethod
    def from_seed(cls, layout, seed, layer=0, experts=512):
        from slotstream_b200 import synth
        recs = np.stack([synth.expert_record(layout, seed, layer, e) for e in range(experts + 1)])
        return cls(layout, recs, _t_bf16(synth.router_weight(seed, experts, layout.hidden, layer)).float(),
                   _t_bf16(synth.shared_gate_weight(seed, layout.hidden, layer)).float(),
                   torch.from_numpy(synth.zipf_bias(experts)))

    @classmethod
    def from_tensors(cls, layout, recs_u8, router_w, sh_gate_w, bias):
        """recs_u8 uint8 [E + 1, record_bytes] (shared last), router_w bf16 [E, H], sh_gate_w bf16 [H] or [1, H],
        bias fp32 [E] or None: CPU tensors copied from the device."""
        return cls(layout, recs_u8.numpy(), router_w.float(), sh_gate_w.float().reshape(1, -1),
                   None if bias is None else bias.float())


def route(L: CpuLayer, x, k):
    """Router (model/layers.py:339-347 in fp32): logits, softmax, stable top-k, renormalise -> (ids, weights)."""
    logits = F.linear(x, L.rw)
    if L.bias is not None:
        logits = logits + L.bias
    probs = F.softmax(logits, dtype=torch.float, dim=-1)
    v, i = torch.sort(probs, dim=-1, descending=True, stable=True)   # ties to the lower index
    tv, ti = v[:, :k], i[:, :k]
    return ti, tv / tv.sum(-1, keepdim=True)


def decode_token_layer(L: CpuLayer, x, k=10):
    """One token through one layer (x fp32 [1, H]); dequantisation inside."""
    ti, tv = route(L, x, k)
    out = torch.zeros_like(x)
    for r in range(k):
        g, u, d = _expert_t(L.layout, L.recs[int(ti[0, r])])
        h = F.silu(g @ x[0]) * (u @ x[0])
        out[0] += tv[0, r] * (d @ h)
    g, u, d = _expert_t(L.layout, L.shared)
    sh = d @ (F.silu(g @ x[0]) * (u @ x[0]))
    sh = torch.sigmoid(F.linear(x, L.sg)) * sh
    return out + sh, ti


def prefill_chunk(L: CpuLayer, x, k=10):
    """T tokens through one layer, experts grouped (each routed expert dequantised once per call). x fp32 [T, H]
    -> (y fp32 [T, H] = routed + shared, ids int64 [T, k])."""
    ti, tv = route(L, x, k)
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
    return out + torch.sigmoid(F.linear(x, L.sg)) * sh, ti


def parity(y_gpu, ids_gpu, y_cpu, ids_cpu):
    """The GPU layer output against the CPU path on the same inputs: share of tokens whose top-k ids are equal
    (near-tie routings may differ), relative L2 over those tokens and over all, max-abs over those tokens."""
    same = (ids_gpu.long() == ids_cpu.long()).all(dim=1)
    a, b = y_gpu.double(), y_cpu.double()
    rel_all = float((a - b).norm() / b.norm())
    if bool(same.any()):
        d = (a[same] - b[same])
        rel_same, mx = float(d.norm() / b[same].norm()), float(d.abs().max())
    else:
        rel_same, mx = float("nan"), float("nan")
    return {"tokens": int(same.numel()), "ids_equal_frac": round(float(same.float().mean()), 6),
            "rel_l2": round(rel_same, 6), "max_abs": round(mx, 5), "rel_l2_all_tokens": round(rel_all, 6),
            "bar": "rel_l2 <= 1e-2 (layer contract); ids differ only where router logits nearly tie"}


def time_decode(L: CpuLayer, seconds=10.0, threads=None, layers_per_token=48, seed=0):
    """Tokens/s of the CPU decode path over a bounded sample: token-layers are timed until `seconds` pass;
    tokens/s = 1 / (mean seconds per token-layer * layers_per_token)."""
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    rng = np.random.default_rng(seed)
    n, t0 = 0, time.perf_counter()
    with torch.no_grad():
        while True:
            x = torch.from_numpy(rng.standard_normal((1, L.layout.hidden)).astype(np.float32)).bfloat16().float()
            decode_token_layer(L, x)
            n += 1
            if time.perf_counter() - t0 >= seconds:
                break
    per = (time.perf_counter() - t0) / n
    out = {"value": 1.0 / (per * layers_per_token), "unit": "tokens/s", "kind": "port",
           "sample": f"{n} token-layers of the config[0] layer (b=1, Zipf routing), dequant inside; "
                     f"tokens/s = 1/(mean token-layer time x {layers_per_token} layers)"}
    out.update(host_info(threads))
    return out


def time_prefill_chunks(L: CpuLayer, x_chunk, n_chunks=1, threads=None):
    """Tokens/s of the CPU prefill path over n_chunks passes of one whole chunk x_chunk (bf16 [T, H]): the same
    chunk size as the GPU workload, each expert dequantised once per pass. Returns (record, y of the last pass,
    ids)."""
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    x = x_chunk.float()
    t = x.shape[0]
    times = []
    with torch.no_grad():
        for _ in range(n_chunks):
            t0 = time.perf_counter()
            y, ids = prefill_chunk(L, x)
            times.append(time.perf_counter() - t0)
    out = {"value": t * len(times) / sum(times), "unit": "tokens/s", "kind": "port",
           "sample": f"{len(times)} pass(es) over the whole {t}-token chunk of the config[0] layer (the GPU "
                     f"workload's chunk), experts grouped and dequantised once per pass",
           "seconds": round(sum(times), 3)}
    out.update(host_info(threads))
    return out, y, ids
