"""Seeded synthetic workload for the MoE hot path (no checkpoint exists on these machines).

Distributions (BASELINE config-[0]):
* codes uniform 0..15, packed 8 per uint32 word, low nibble first;
* scales bf16 ~ U(0.005, 0.02); biases bf16 = -8 * scale + N(0, 1e-3);
* activations bf16 ~ N(0, 1); router weight bf16 ~ N(0, 0.02);
* optional per-expert Zipf(s) logit bias, ranked by expert id: bias[e] = -s * ln(e + 1), so the softmax
  probability of expert e is multiplied by (e + 1) ** -s before renormalisation.

Two generators with the same distributions:
* ``expert_record`` (numpy PCG64, seeded per (seed, layer, expert)) is bit-reproducible on any host and is
  what parity tests and golden fixtures use;
* ``fill_records_device`` (torch CUDA RNG) fills tens of GB of HBM quickly for benchmarks; its bytes are
  copied back to the host whenever a benchmark run is compared with the oracle.
"""
import math

import numpy as np

from .records import RecordLayout


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16, returned as uint16 bit patterns (finite inputs)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + r) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _rng(*key):
    return np.random.default_rng(np.random.SeedSequence([int(k) & 0xFFFFFFFF for k in key]))


def _piece(rng, n, k, gs):
    words = rng.integers(0, 2**32, size=(n, k // 8), dtype=np.uint64).astype(np.uint32)
    s = f32_to_bf16_bits(rng.uniform(0.005, 0.02, size=(n, k // gs)).astype(np.float32))
    b = f32_to_bf16_bits((-8.0 * bf16_bits_to_f32(s) + rng.normal(0.0, 1e-3, size=(n, k // gs))).astype(np.float32))
    return words, s, b


def expert_record(layout: RecordLayout, seed: int, layer: int, expert: int) -> np.ndarray:
    """One record (uint8 [record_bytes]) in the reference byte layout."""
    rng = _rng(seed, 0x5EC0, layer, expert)
    rec = np.empty(layout.record_bytes, dtype=np.uint8)
    offs = layout.offsets()
    for p, (n, k) in enumerate(layout.piece_shapes()):
        w, s, b = _piece(rng, n, k, layout.gs)
        for t, off in zip((w, s, b), offs[3 * p:3 * p + 3]):
            raw = t.view(np.uint8).reshape(-1)
            rec[off:off + raw.size] = raw
    return rec


def split_record(layout: RecordLayout, rec: np.ndarray):
    """uint8 record -> [(words uint32 [n, k/8], s uint16 [n, k/gs], b uint16 [n, k/gs])] for gate, up, down."""
    offs = layout.offsets()
    out = []
    for p, (n, k) in enumerate(layout.piece_shapes()):
        ow, os_, ob = offs[3 * p:3 * p + 3]
        w = rec[ow:ow + n * k // 2].view(np.uint32).reshape(n, k // 8)
        s = rec[os_:os_ + n * (k // layout.gs) * 2].view(np.uint16).reshape(n, k // layout.gs)
        b = rec[ob:ob + n * (k // layout.gs) * 2].view(np.uint16).reshape(n, k // layout.gs)
        out.append((w, s, b))
    return out


def pack_record(layout: RecordLayout, pieces) -> np.ndarray:
    """Inverse of split_record."""
    rec = np.zeros(layout.record_bytes, dtype=np.uint8)
    offs = layout.offsets()
    for p, (w, s, b) in enumerate(pieces):
        for t, off in zip((w, s, b), offs[3 * p:3 * p + 3]):
            raw = np.ascontiguousarray(t).view(np.uint8).reshape(-1)
            rec[off:off + raw.size] = raw
    return rec


def activations(seed: int, t: int, hidden: int, tag: int = 0) -> np.ndarray:
    """bf16 bits [t, hidden] ~ N(0, 1)."""
    return f32_to_bf16_bits(_rng(seed, 0xA11, tag).standard_normal((t, hidden)).astype(np.float32))


def router_weight(seed: int, experts: int, hidden: int, layer: int = 0) -> np.ndarray:
    """bf16 bits [experts, hidden] ~ N(0, 0.02)."""
    return f32_to_bf16_bits((_rng(seed, 0x7A7E, layer).standard_normal((experts, hidden)) * 0.02).astype(np.float32))


def shared_gate_weight(seed: int, hidden: int, layer: int = 0) -> np.ndarray:
    """bf16 bits [1, hidden] ~ N(0, 0.02): the sigmoid gate of the shared expert."""
    return f32_to_bf16_bits((_rng(seed, 0x5A6E, layer).standard_normal((1, hidden)) * 0.02).astype(np.float32))


def zipf_bias(experts: int, s: float = 1.1) -> np.ndarray:
    """fp32 [experts]: -s * ln(e + 1)."""
    return np.array([-s * math.log(e + 1) for e in range(experts)], dtype=np.float32)


# ------------------------------------------------------------------ device-side bulk generation (benchmarks)
def fill_records_device(layout: RecordLayout, out, seed: int):
    """Fill a uint8 CUDA tensor [n, record_bytes] with records of the same distributions (torch CUDA RNG).

    Generates one projection piece at a time for every record at once, so the peak extra memory is a few
    piece-sized fp32 temporaries."""
    import torch
    n = out.shape[0]
    g = torch.Generator(device=out.device)
    g.manual_seed(int(seed))
    offs = layout.offsets()
    chunk = max(1, min(n, (1 << 30) // max(layout.w_bytes, 1)))
    for p, (pn, pk) in enumerate(layout.piece_shapes()):
        ow, os_, ob = offs[3 * p:3 * p + 3]
        ng = pk // layout.gs
        for a in range(0, n, chunk):
            b_ = min(n, a + chunk)
            m = b_ - a
            w = torch.randint(-2**31, 2**31 - 1, (m, pn * pk // 8), dtype=torch.int32, device=out.device, generator=g)
            out[a:b_, ow:ow + layout.w_bytes].copy_(w.view(torch.uint8).view(m, -1))
            del w
            s = torch.empty(m, pn * ng, device=out.device).uniform_(0.005, 0.02, generator=g).to(torch.bfloat16)
            bias = (-8.0 * s.float() + torch.randn(m, pn * ng, device=out.device, generator=g) * 1e-3).to(torch.bfloat16)
            out[a:b_, os_:os_ + layout.sb_bytes].copy_(s.view(torch.uint8).view(m, -1))
            out[a:b_, ob:ob + layout.sb_bytes].copy_(bias.view(torch.uint8).view(m, -1))
            del s, bias
    return out
