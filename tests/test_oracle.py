"""The CPU oracle against the golden vectors that the reference's own code produced (make_golden.py)."""
import numpy as np
import pytest

from oracle import moe_oracle as O
from slotstream_b200 import synth
from slotstream_b200.records import BASELINE_LAYOUT, REFERENCE_LAYOUT
from conftest import GOLDEN

import hashlib


def _sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def test_nibble_order_known_answer():
    g = np.load(GOLDEN / "affine.npz")
    assert O.unpack(g["kat_words"]).tolist() == [[0, 1, 2, 3, 4, 5, 6, 7]]
    assert np.array_equal(O.unpack(g["kat_words"]), g["kat_unpacked"])


@pytest.mark.parametrize("gs", [32, 64])
def test_dequant_matches_reference_bitwise(gs):
    g = np.load(GOLDEN / "affine.npz")
    deq = O.dequant(g[f"gs{gs}_q"], g[f"gs{gs}_s"], g[f"gs{gs}_b"], 4, gs)
    assert np.array_equal(deq.view(np.uint32), g[f"gs{gs}_deq"].view(np.uint32))


def test_topk_rule_matches_reference():
    g = np.load(GOLDEN / "topk.npz")
    n_cases = len(g["names"])
    checked = 0
    for ci in range(n_cases):
        x = g[f"c{ci}_x"]
        nv = g[f"c{ci}_nv"]
        nv = None if nv[0] < 0 else nv
        for k in (10, 512):
            key = f"c{ci}_k{k}_idx"
            if key not in g:
                continue
            idx, val = O.topk_stable(x, k, nv)
            assert np.array_equal(idx, g[key]), (g["names"][ci], k)
            ok = idx >= 0
            for r in range(x.shape[0]):
                assert np.array_equal(val[r][ok[r]].view(np.uint32), x[r][idx[r][ok[r]]].view(np.uint32))
            assert np.all(np.isneginf(val[~ok]))
            checked += 1
    assert checked >= 15


def test_align_matches_reference():
    g = np.load(GOLDEN / "align.npz")
    for i, name in enumerate(g["names"]):
        nl, bm = (int(v) for v in g[f"c{i}_meta"])
        sr, be, npad = O.moe_align(g[f"c{i}_in"], nl, bm)
        assert np.array_equal(sr, g[f"c{i}_sorted"]), name
        assert np.array_equal(be, g[f"c{i}_block"]), name
        assert np.array_equal(npad, g[f"c{i}_npad"]), name


def test_combine_matches_reference_bitwise():
    g = np.load(GOLDEN / "combine.npz")
    out = O.combine_rank_order(g["rows"], int(g["t"]), int(g["k"]))
    assert np.array_equal(out.view(np.uint32), g["out"].view(np.uint32))


def test_generator_is_pinned():
    g = np.load(GOLDEN / "moe_ref.npz")
    lay, seed, layer, T, E = BASELINE_LAYOUT, int(g["seed"]), int(g["layer"]), int(g["T"]), int(g["E"])
    x = synth.activations(seed, T, lay.hidden)
    rw = synth.router_weight(seed, E, lay.hidden, layer)
    sg = synth.shared_gate_weight(seed, lay.hidden, layer)
    assert _sha(x, rw, sg, synth.expert_record(lay, seed, layer, E),
                synth.expert_record(lay, seed, layer, 0)) == str(g["inputs_sha"])


def test_moe_layer_fp32_matches_reference_moe_ref():
    """The oracle's routed + shared sum equals the reference moe_ref (fp32 mode) at config-[0] shapes."""
    g = np.load(GOLDEN / "moe_ref.npz")
    lay, seed, layer, T, E, K = BASELINE_LAYOUT, int(g["seed"]), int(g["layer"]), int(g["T"]), int(g["E"]), int(g["K"])
    x = synth.activations(seed, T, lay.hidden)
    rw = synth.router_weight(seed, E, lay.hidden, layer)
    sg = synth.shared_gate_weight(seed, lay.hidden, layer)
    ids, w, logits = O.router(x, rw, K)
    O.ids_match(ids, g["ids"], logits)
    dense = {}

    def expert(e):
        if e not in dense:
            dense[e] = O.record_dense(lay, synth.expert_record(lay, seed, layer, e))
        return dense[e]

    routed = O.moe_decode(lay, O.bf16_to_f32(x), ids, w, expert)
    shg, shu, shd = O.record_dense(lay, synth.expert_record(lay, seed, layer, E))
    xf = O.bf16_to_f32(x).astype(np.float64)
    a, b = xf @ shg.T, xf @ shu.T
    sh = (O.silu64(a) * b) @ shd.T
    sh = sh / (1.0 + np.exp(-(xf @ O.bf16_to_f32(sg).astype(np.float64).T)))
    out = routed + sh
    assert O.rel_l2(out, g["out"]) < 1e-5
    assert np.max(np.abs(out - g["out"])) < 1e-3


def test_decode_fp64_matches_reference_helper():
    g = np.load(GOLDEN / "decode_ref.npz")
    lay = REFERENCE_LAYOUT
    recs = [synth.expert_record(lay, int(g["seed"]), 0, e) for e in range(int(g["n_exp"]))]
    assert _sha(*recs) == str(g["inputs_sha"])
    out = O.moe_decode(lay, O.bf16_to_f32(g["x_bits"]), g["ids"], g["w"], lambda e: O.record_dense(lay, recs[e]))
    assert O.rel_l2(out, g["out"]) < 1e-12


def test_fused_rows_match_reference_helpers():
    g = np.load(GOLDEN / "fused_ref.npz")
    lay = REFERENCE_LAYOUT
    recs = [synth.expert_record(lay, int(g["seed"]), 0, e) for e in range(int(g["n_exp"]))]
    assert _sha(*recs) == str(g["inputs_sha"])
    x = O.bf16_to_f32(g["x_bits"])
    rows = list(range(g["expert"].size))
    exact = O.fused_rows_exact(x, g["token"], g["weight"], g["expert"], lambda e: O.record_dense(lay, recs[e]), rows)
    assert O.rel_l2(exact, g["exact"]) < 1e-6
    bf = O.fused_rows_bf16_path(x, g["token"], g["weight"], g["expert"],
                                lambda e: O.record_dense(lay, recs[e], np.float32), rows)
    assert O.rel_l2(bf, g["bf16_path"]) < 1e-5
    # the reference's own contract numbers, reproduced by the oracle: bf16 path within 1e-2 of exact,
    # nibble-swap control far outside
    assert O.rel_l2(bf, exact) < 1e-2
    assert O.rel_l2(g["swap"], exact) > 10 * 1e-2


def test_grouped_layer_equals_per_token_layer():
    """moe_layer_grouped (rows batched per expert, used for chunks of thousands of tokens) is the same fp64
    arithmetic as moe_layer's per-(token, rank) loop: equal up to fp64 summation order."""
    lay, E, K = BASELINE_LAYOUT, 512, 10
    x = synth.activations(5, 6, lay.hidden, tag=6)
    rw = synth.router_weight(5, E, lay.hidden)
    sg = synth.shared_gate_weight(5, lay.hidden)
    bias = synth.zipf_bias(E)
    dense = {}

    def expert(e):
        if e not in dense:
            dense[e] = O.record_dense(lay, synth.expert_record(lay, 5, 0, e))
        return dense[e]
    sh = O.record_dense(lay, synth.expert_record(lay, 5, 0, E), np.float32)
    out1, routed1, _, ids1, w1, _ = O.moe_layer(lay, x, rw, K, expert, sh, sg, bias=bias)
    out2, routed2, ids2, w2, _ = O.moe_layer_grouped(lay, x, rw, K, expert, sh, sg, bias=bias)
    assert np.array_equal(ids1, ids2) and np.array_equal(w1, w2)
    assert O.rel_l2(routed2, routed1) < 1e-13
    assert np.array_equal(out1, out2)
