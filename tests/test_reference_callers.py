"""The reference's own callers of the kernel modules, run unchanged against the drop-in mirrors (CPU).

INTEGRATION.md's module swap puts ``slotstream_b200.kernels.*`` in place of ``slotstream_spark.kernels.*``; then the
reference's code that calls them -- ``SweepMoE.layer`` / ``SweepMoE._group`` (model/moe_sweep.py:80-176: resident
and staged expert groups of at most 32, launches split at ``max_rows_per_launch``, ``out_rows`` sized
``[R, fm.HID]``, ``combine_rank_order``), the CUDA branch of ``Segments.seg_moe`` (model/layers.py:372-402: row groups,
``moe_decode`` into views of ``routed``, the shared expert through ``gemv`` of AffineWeights) and the CUDA branch of
``Segments.seg_router`` (model/layers.py:336-348: ``topk_stable`` with ``out_val``) -- runs as written, at the
BASELINE shape 2048 / 512 and at the reference model's 2560 / 640 (``kernels.configure``).

The reference cannot be present where the GPU tests run, so here the C ABI underneath the mirrors is the CPU model
of tests/abi_cpu_model.py (the oracle's arithmetic): this checks the mirrors' signatures, constants, argument checks
and the C-ABI calls they make for these callers, and the results against the oracle. The kernels behind the same
calls are checked on the GPU by tests/test_gpu_dropin.py. Skipped where no reference checkout exists.
"""
import importlib
import os
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from abi_cpu_model import Records, install
from oracle import moe_oracle as O
from slotstream_b200 import synth

REF = Path(os.environ.get("SLOTSTREAM_SPARK_REF", "/root/reference"))
pytestmark = pytest.mark.skipif(not (REF / "slotstream_spark" / "model" / "moe_sweep.py").is_file(),
                                reason="no slotstream-spark checkout on this machine")
MIRRORS = ("topk_stable", "moe_align", "fused_moe_affine", "moe_gemv_affine", "gemv_affine", "gemm_affine")
SHAPES = [(2048, 512), (2560, 640)]
K = 10


class _HostEvent:
    """Stands in for torch.cuda.Event on a machine without a GPU (the CPU model runs synchronously)."""

    def __init__(self, *a, **k):
        pass

    def record(self, *a, **k):
        pass

    def synchronize(self):
        pass


@pytest.fixture
def swapped(monkeypatch):
    """The module swap of INTEGRATION.md, undone after the test; reference modules imported during the test are
    dropped again so no other test sees them bound to the mirrors."""
    monkeypatch.syspath_prepend(str(REF))
    mods = {n: importlib.import_module(f"slotstream_b200.kernels.{n}") for n in MIRRORS}
    refk = importlib.import_module("slotstream_spark.kernels")
    for n, m in mods.items():
        monkeypatch.setitem(sys.modules, f"slotstream_spark.kernels.{n}", m)
        monkeypatch.setattr(refk, n, m, raising=False)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: None)
    monkeypatch.setattr(torch.cuda, "Event", _HostEvent)
    before = {k for k in sys.modules if k.startswith("slotstream_spark.model") or k.startswith("slotstream_spark.engine")}
    yield mods
    for k in [k for k in sys.modules if (k.startswith("slotstream_spark.model") or k.startswith("slotstream_spark.engine"))
              and k not in before]:
        del sys.modules[k]
    from slotstream_b200.kernels import configure
    configure(2560, 640)


def _records(lay, seed, experts):
    recs = {int(e): torch.from_numpy(synth.expert_record(lay, seed, 0, int(e))) for e in experts}
    return recs


@pytest.mark.parametrize("hidden,inter", SHAPES)
def test_sweep_moe_layer_runs_unchanged(swapped, monkeypatch, hidden, inter):
    from slotstream_b200.kernels import configure
    lay = configure(hidden, inter)
    from slotstream_spark.model import moe_sweep
    assert moe_sweep.fm is swapped["fused_moe_affine"] and moe_sweep.fm.HID == hidden
    rng = np.random.default_rng(hidden)
    experts = np.sort(rng.choice(512, 40, replace=False)).astype(np.int32)
    recs = _records(lay, 11, experts)
    reg = Records(lay)
    addr = {e: reg.add(r) for e, r in recs.items()}
    model = install(monkeypatch, reg)
    resident = set(int(e) for e in experts[::2])          # half of the experts sit in pool slots, half are staged
    T = 24
    ids_host = np.stack([rng.choice(experts, K, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    x_bits = synth.activations(12, T, hidden)
    mixed = torch.from_numpy(x_bits.view(np.int16)).view(torch.bfloat16)

    class Pool:   # ExpertPool facade: the layer's map row (slot >= 0 = resident) and the slot count
        pool = SimpleNamespace(map_numpy=lambda: np.array([(i if (i < 512 and i in resident) else -1)
                                                           for i in range(49 * 512)], dtype=np.int32),
                               stats=lambda: {"slots": len(resident)})

    staged = {}

    class Sweep:  # slotio.Sweep facade: resident addresses, and staged copies of the group's records
        def set_generation(self, gen):
            pass

        def resident_ptr_nopin_touch(self, L, e):
            return addr[int(e)] if int(e) in resident else None

        def read_group(self, L, exps, buf, adm):
            copies = [recs[int(e)].clone() for e in exps]
            staged[id(copies[0])] = copies
            return SimpleNamespace(copies=[reg.add(c) for c in copies], keep=copies, admitted=0, admit_refused=0)

        def wait(self, t, ms):
            return True

        def record_dev(self, t, i):
            return t.copies[i]

    seg = SimpleNamespace(gen=0, progress=np.zeros(1, dtype=np.uint64), _done=lambda g: None)
    sm = moe_sweep.SweepMoE(seg, Pool(), max_rows_per_launch=64, staging=object(), sweep=Sweep())
    routed = sm.layer(0, mixed, ids_host, torch.from_numpy(w))
    assert tuple(routed.shape) == (T, hidden) and routed.dtype == torch.float32
    st = sm.stats
    assert st.resident_rows > 0 and st.staged_rows > 0 and st.resident_rows + st.staged_rows == T * K
    assert st.launches > st.groups and st.max_launch_rows <= 64
    assert st.bytes_requested == st.records_read * lay.record_bytes
    assert model.calls.count("ssb_fused_moe_gate_up") == st.launches
    assert model.calls[-1] == "ssb_combine_rank_order"
    f32 = {e: O.record_dense(lay, r.numpy(), np.float32) for e, r in recs.items()}
    rows = O.fused_rows_bf16_path(O.bf16_to_f32(x_bits), np.repeat(np.arange(T), K), w.reshape(-1),
                                  ids_host.reshape(-1), lambda e: f32[e], range(T * K))
    ref = O.combine_rank_order(rows.astype(np.float32), T, K)
    np.testing.assert_allclose(routed.numpy(), ref, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("hidden,inter", SHAPES)
def test_seg_moe_cuda_branch_runs_unchanged(swapped, monkeypatch, hidden, inter):
    from slotstream_b200.kernels import configure
    from slotstream_b200.kernels.gemv_affine import AffineWeight
    lay = configure(hidden, inter)
    from slotstream_spark.model import layers
    rng = np.random.default_rng(inter)
    experts = np.sort(rng.choice(512, 30, replace=False)).astype(np.int32)
    recs = _records(lay, 21, experts)
    reg = Records(lay)
    model = install(monkeypatch, reg)
    L, n_slots = 3, 64
    slot_of = {int(e): i for i, e in enumerate(experts)}
    slot_ptr = torch.zeros(n_slots, dtype=torch.int64)
    for e, s in slot_of.items():
        slot_ptr[s] = reg.add(recs[e])
    map_t = torch.full((49 * 512,), -1, dtype=torch.int32)
    for e, s in slot_of.items():
        map_t[L * 512 + e] = s

    class Pool:   # ExpertPool facade: ensure() returns the slot of each unique expert; the device tables
        map_tensor, slot_ptr_tensor = map_t, slot_ptr

        def ensure(self, L_, uniq, gen):
            return [slot_of[int(e)] for e in uniq]

    sh_rec = synth.expert_record(lay, 21, 0, 512)
    pieces = synth.split_record(lay, sh_rec)
    bt = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)  # noqa: E731
    aw = [AffineWeight(torch.from_numpy(np.ascontiguousarray(q).view(np.int32)), bt(s), bt(b), 4, 64, n, k)
          for (q, s, b), (n, k) in zip(pieces, lay.piece_shapes())]
    sg_bits = synth.shared_gate_weight(21, hidden)
    p = f"layers.{L}.mlp."
    W = {p + "shared_expert.gate_proj.weight": aw[0], p + "shared_expert.up_proj.weight": aw[1],
         p + "shared_expert.down_proj.weight": aw[2], p + "shared_expert_gate.weight": bt(sg_bits)}
    seg = layers.Segments.__new__(layers.Segments)
    seg.W, seg.pool, seg.cuda, seg.H, seg.topk, seg.max_rows = W.__getitem__, Pool(), True, hidden, K, 2
    seg.cfg = {"moe_intermediate_size": inter}
    seg.gen, seg.progress, seg.last_routing, seg._tables, seg.rowwise = 0, np.zeros(1, np.uint64), {}, None, False
    T = 5
    ids = np.stack([rng.choice(experts, K, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    x_bits = synth.activations(22, T, hidden)
    out = seg.seg_moe(L, bt(x_bits), torch.from_numpy(ids), torch.from_numpy(w))
    assert tuple(out.shape) == (T, hidden) and out.dtype == torch.bfloat16
    assert model.calls.count("ssb_moe_decode") == len(layers.row_groups(ids, 2)) >= 3
    assert model.calls.count("ssb_gemv_affine") == 3
    dense = {e: O.record_dense(lay, r.numpy()) for e, r in recs.items()}
    routed = O.moe_decode(lay, O.bf16_to_f32(x_bits), ids, w, lambda e: dense[e])
    sh = O.shared_expert(x_bits, *O.record_dense(lay, sh_rec, np.float32), sg_bits)
    ref = O.round_bf16(O.round_bf16(routed).astype(np.float64) + sh)
    got = out.float().numpy().astype(np.float64)
    assert O.rel_l2(got, ref) < 2e-3
    assert np.all(np.abs(got - ref) <= 3 * O.bf16_ulp(ref) + 2.0 ** -6 * np.abs(sh))


def test_seg_router_cuda_branch_runs_unchanged(swapped, monkeypatch):
    from slotstream_b200.kernels import configure
    lay = configure(2048, 512)
    from slotstream_spark.model import layers
    model = install(monkeypatch, Records(lay))
    L, T = 5, 7
    rw = synth.router_weight(31, 512, lay.hidden)
    bt = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)  # noqa: E731
    seg = layers.Segments.__new__(layers.Segments)
    seg.W, seg.cuda, seg.topk, seg.rowwise = {f"layers.{L}.mlp.gate.weight": bt(rw)}.__getitem__, True, K, False
    seg.hc_mix = lambda prefix, hyp: (hyp, None)     # the hyper-connection mix is outside the MoE path
    x = bt(synth.activations(32, T, lay.hidden))
    mixed, _, ids, tv = seg.seg_router(L, x)
    assert model.calls == ["ssb_topk_stable"]
    probs = torch.softmax(torch.nn.functional.linear(x, bt(rw)).float(), dim=-1).numpy()
    ids_ref, val_ref = O.topk_stable(probs, K)
    assert np.array_equal(ids.numpy(), ids_ref)
    np.testing.assert_allclose(tv.numpy(), val_ref / val_ref.sum(1, keepdims=True), rtol=1e-6)
