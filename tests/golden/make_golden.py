"""Generate the golden fixtures of this directory by running the REFERENCE's own code on CPU.

Usage (in a container that has a slotstream-spark checkout; the GPU box never runs this):

    python tests/golden/make_golden.py --reference <path to the slotstream-spark checkout>

What each fixture pins (reference file:line of the code that produced the expected values):
* ``affine.npz``      -- kernels/affine_ref.py:10-31 (unpack nibble order, dequant q*s+b) on seeded pieces,
                         plus the known answer 0x76543210 -> [0..7] of tests/t0/test_affine_kernels.py:35-40.
* ``topk.npz``        -- the stable top-k rule of tests/t0/test_topk_stable.py:14-31 (``_ref_row``) on random,
                         tied, NaN/inf/+-0 and n_valid-masked rows, k in {10, 512}.
* ``align.npz``       -- kernels/moe_align.py:17-48 (``moe_align``) over empty, ragged, -1 and out-of-range
                         inputs and block_m in {1, 16, 64, 128}.
* ``combine.npz``     -- kernels/fused_moe_affine.py:164-172 (``combine_rank_order``).
* ``moe_ref.npz``     -- model/reference_torch.py:118-134 (``moe_ref``) at BASELINE config-[0] shapes
                         (hidden 2048, intermediate 512, 512 experts, top-10), fp32 router and experts, T = 4.
* ``decode_ref.npz``  -- the fp64 decode reference of tests/t0/test_moe_gemv_affine.py:74-84 at the
                         reference's own 2560/640 shape (that helper hard-codes 2560 columns).
* ``fused_ref.npz``   -- the fp64 exact and bf16-path references of tests/gates/test_fused_moe_affine.py:68-100
                         at 2560/640, with the nibble-swap control.
* ``experts_bin/``    -- tools/repack_experts.py run unmodified on the reference's own synthetic MLX checkpoint
                         (tests/t0/synth_ckpt.py:43-92; 2 layers, 16 experts, hidden 64, ff 64): the packed
                         experts.bin and its manifest, plus pieces.json = SHA-256 of every source tensor slice
                         (layer, expert, piece) the repacker read.
* ``sweep_plan.npz``  -- engine/sweep.py:34-58 (``plan_sweep``): row order and groups for empty, all-resident,
                         none-resident, mixed and Zipf-skewed rows at group sizes 1, 7 and 32.

Inputs come from ``slotstream_b200.synth`` (numpy PCG64, seeded), so tests regenerate them bit for bit; each
fixture stores a SHA-256 of its inputs to catch generator drift.
"""
import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "slotstream-spark_b200"))

from slotstream_b200 import synth  # noqa: E402
from slotstream_b200.records import BASELINE_LAYOUT, REFERENCE_LAYOUT  # noqa: E402

SEED = 0


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def t_bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def make_affine(ref):
    affine_ref = ref["affine_ref"]
    out = {}
    kat = affine_ref.unpack(torch.tensor([[0x76543210]], dtype=torch.int32), 4)
    out["kat_words"] = np.array([[0x76543210]], dtype=np.uint32)
    out["kat_unpacked"] = kat.numpy().astype(np.uint8)
    rng = np.random.default_rng(7)
    for gs in (32, 64):
        n, k = 24, 256
        q = rng.integers(0, 2**32, size=(n, k // 8), dtype=np.uint64).astype(np.uint32)
        s = synth.f32_to_bf16_bits(rng.uniform(0.005, 0.02, (n, k // gs)).astype(np.float32))
        b = synth.f32_to_bf16_bits(rng.normal(0, 0.02, (n, k // gs)).astype(np.float32))
        deq = affine_ref.dequant(torch.from_numpy(q.view(np.int32)), t_bf16(s), t_bf16(b), 4, gs)
        out[f"gs{gs}_q"], out[f"gs{gs}_s"], out[f"gs{gs}_b"] = q, s, b
        out[f"gs{gs}_deq"] = deq.numpy()
    np.savez_compressed(HERE / "affine.npz", **out)


def make_topk(ref):
    tt = ref["test_topk"]
    rows, ks, nvs, names = [], [], [], []
    g = torch.Generator().manual_seed(11)
    cases = []
    for n in (512, 513, 2048):
        cases.append(("randn", torch.randn(3, n, generator=g), None))
        cases.append(("ties", torch.round(torch.randn(3, n, generator=g) * 2) / 2, None))
    x = torch.randn(4, 512, generator=g)
    x[0, :20] = float("nan")
    x[1, 5:15] = float("-inf")
    x[1, 100:104] = float("inf")
    x[2, ::2] = 0.0
    x[2, 1::2] = -0.0
    x[3, :] = float("nan")
    cases.append(("special", x, None))
    cases.append(("equal", torch.full((2, 600), 1.5), None))
    xm = torch.round(torch.randn(5, 2048, generator=g) * 4) / 4
    xm[:, 700:] = 1e9
    cases.append(("nvalid", xm, [2048, 700, 513, 10, 3]))
    out = {}
    for ci, (name, xs, nv) in enumerate(cases):
        for k in (10, 512):
            if k > xs.shape[1]:
                continue
            idx = []
            for r in range(xs.shape[0]):
                v = xs.shape[1] if nv is None else min(nv[r], xs.shape[1])
                idx.append(tt._ref_row(xs[r], k, v).numpy())
            out[f"c{ci}_k{k}_idx"] = np.stack(idx).astype(np.int32)
        out[f"c{ci}_x"] = xs.numpy().astype(np.float32)
        out[f"c{ci}_nv"] = np.array(nv if nv is not None else [-1], dtype=np.int32)
        names.append(name)
    out["names"] = np.array(names)
    np.savez_compressed(HERE / "topk.npz", **out)


def make_align(ref):
    moe_align = ref["moe_align"]
    rng = np.random.default_rng(5)
    cases = [
        ("empty", np.zeros(0, dtype=np.int32), 4, 64),
        ("one", np.array([0], dtype=np.int32), 1, 64),
        ("all_minus1", np.full(37, -1, dtype=np.int32), 8, 16),
        ("random_g32", rng.integers(-1, 32, 2560).astype(np.int32), 32, 64),
        ("out_of_range", rng.integers(-3, 40, 1000).astype(np.int32), 32, 64),
        ("bm1", rng.integers(0, 7, 100).astype(np.int32), 7, 1),
        ("bm128_skew", np.minimum(rng.zipf(1.5, 5000) - 1, 63).astype(np.int32), 64, 128),
        ("big_e512", rng.integers(0, 512, 40960).astype(np.int32), 512, 64),
        ("bm16_sparse", np.where(rng.random(3000) < 0.9, -1, rng.integers(0, 300, 3000)).astype(np.int32), 300, 16),
    ]
    out = {}
    for i, (name, le, nl, bm) in enumerate(cases):
        sr, be, npad = moe_align.moe_align(torch.from_numpy(le), nl, bm)
        out[f"c{i}_in"] = le
        out[f"c{i}_meta"] = np.array([nl, bm], dtype=np.int32)
        out[f"c{i}_sorted"] = sr.numpy()
        out[f"c{i}_block"] = be.numpy()
        out[f"c{i}_npad"] = npad.numpy()
    out["names"] = np.array([c[0] for c in cases])
    np.savez_compressed(HERE / "align.npz", **out)


def make_combine(ref):
    fm = ref["fm"]
    g = torch.Generator().manual_seed(3)
    t, k, h = 17, 10, 64
    rows = torch.randn(t * k, h, generator=g) * torch.logspace(-3, 3, k).repeat(t)[:, None]
    got = fm.combine_rank_order(rows, t, k)
    np.savez_compressed(HERE / "combine.npz", rows=rows.numpy(), out=got.numpy(), t=t, k=k)


def make_moe_ref(ref):
    R = ref["reference_torch"]
    affine_ref = ref["affine_ref"]
    lay = BASELINE_LAYOUT
    T, E, K, layer = 4, 512, 10, 0
    x_bits = synth.activations(SEED, T, lay.hidden)
    rw_bits = synth.router_weight(SEED, E, lay.hidden, layer)
    sg_bits = synth.shared_gate_weight(SEED, lay.hidden, layer)
    sh_rec = synth.expert_record(lay, SEED, layer, E)          # the shared expert is record index E
    cache = {}

    def deq_record(rec):
        outs = []
        for (q, s, b) in synth.split_record(lay, rec):
            outs.append(affine_ref.dequant(torch.from_numpy(q.view(np.int32)), t_bf16(s), t_bf16(b), 4, lay.gs))
        return tuple(outs)

    def expert(L, e):
        if e not in cache:
            cache[e] = deq_record(synth.expert_record(lay, SEED, L, e))
        return cache[e]

    x = torch.from_numpy(synth.bf16_bits_to_f32(x_bits))
    rw = torch.from_numpy(synth.bf16_bits_to_f32(rw_bits))
    sg = torch.from_numpy(synth.bf16_bits_to_f32(sg_bits))
    shg, shu, shd = deq_record(sh_rec)
    with torch.no_grad():
        out, ti = R.moe_ref(x, rw, K, expert, layer, shg, shu, shd, sg)
    np.savez_compressed(HERE / "moe_ref.npz", out=out.numpy().astype(np.float32), ids=ti.numpy().astype(np.int32),
                        seed=SEED, layer=layer, T=T, E=E, K=K, hidden=lay.hidden, inter=lay.inter,
                        inputs_sha=sha(x_bits, rw_bits, sg_bits, sh_rec, synth.expert_record(lay, SEED, layer, 0)))


def make_decode_ref(ref):
    tm = ref["test_moe"]
    affine_ref = ref["affine_ref"]
    lay = REFERENCE_LAYOUT
    n_exp, R = 12, 2
    recs = [synth.expert_record(lay, SEED + 1, 0, e) for e in range(n_exp)]
    deqs = []
    for rec in recs:
        deqs.append([affine_ref.dequant(torch.from_numpy(q.view(np.int32)), t_bf16(s), t_bf16(b), 4, lay.gs)
                     for (q, s, b) in synth.split_record(lay, rec)])
    rng = np.random.default_rng(9)
    x_bits = synth.activations(SEED + 1, R, lay.hidden)
    ids = np.stack([rng.permutation(n_exp)[:10] for _ in range(R)]).astype(np.int32)
    w = rng.dirichlet(np.ones(10), size=R).astype(np.float32)
    x = torch.from_numpy(synth.bf16_bits_to_f32(x_bits)).to(torch.bfloat16)
    out = tm._reference(x, torch.from_numpy(ids), torch.from_numpy(w), deqs)
    np.savez_compressed(HERE / "decode_ref.npz", out=out.numpy(), ids=ids, w=w, x_bits=x_bits,
                        n_exp=n_exp, seed=SEED + 1, inputs_sha=sha(*recs))


def make_fused_ref(ref):
    tf = ref["test_fused"]
    lay = REFERENCE_LAYOUT
    n_exp, T, R = 6, 8, 12
    recs = [synth.expert_record(lay, SEED + 2, 0, e) for e in range(n_exp)]
    pieces = []
    for rec in recs:
        pieces.append(tuple((torch.from_numpy(q.view(np.int32)), t_bf16(s), t_bf16(b))
                            for (q, s, b) in synth.split_record(lay, rec)))
    rng = np.random.default_rng(13)
    x_bits = synth.activations(SEED + 2, T, lay.hidden)
    expert = rng.integers(0, n_exp, R).astype(np.int32)
    token = (np.arange(R) // 3).astype(np.int32)
    weight = (rng.random(R) + 0.1).astype(np.float32)
    w = dict(x=torch.from_numpy(synth.bf16_bits_to_f32(x_bits)).to(torch.bfloat16), expert=torch.from_numpy(expert),
             token=torch.from_numpy(token), weight=torch.from_numpy(weight), pieces=pieces)
    rows = list(range(R))
    exact = tf._reference(w, rows, torch.float64)
    bf16p = tf._reference(w, rows, torch.float32, bf16_path=True)
    swap = tf._reference(w, rows, torch.float64, swap=True)
    np.savez_compressed(HERE / "fused_ref.npz", exact=exact.numpy().astype(np.float32),
                        bf16_path=bf16p.numpy().astype(np.float32), swap=swap.numpy().astype(np.float32),
                        x_bits=x_bits, expert=expert, token=token, weight=weight, n_exp=n_exp, seed=SEED + 2,
                        inputs_sha=sha(*recs))


def make_sweep_plan(ref):
    plan = ref["sweep"].plan_sweep
    rng = np.random.default_rng(SEED + 77)
    cases = [(0, 0.5, 32), (40, 1.0, 32), (40, 0.0, 32), (1000, 0.3, 7), (1000, 0.7, 1), (20480, 0.4, 32)]
    out = {"n_cases": len(cases)}
    for c, (r, frac, gs) in enumerate(cases):
        ids = rng.integers(0, 512, r).astype(np.int32) if c != 5 else (rng.zipf(1.1, r) % 512).astype(np.int32)
        res = rng.random(512) < frac
        p = plan(ids, res, gs)
        out[f"ids_{c}"], out[f"res_{c}"], out[f"gs_{c}"], out[f"order_{c}"] = ids, res, gs, p.order
        out[f"groups_{c}"] = np.array([[g.row_lo, g.row_hi, int(g.resident), g.experts.size] for g in p.groups],
                                      dtype=np.int64).reshape(-1, 4)
        out[f"experts_{c}"] = (np.concatenate([g.experts for g in p.groups]) if p.groups
                               else np.zeros(0, np.int32))
    np.savez_compressed(HERE / "sweep_plan.npz", **out)


def make_experts_bin(ref):
    import shutil
    import subprocess
    import tempfile
    refp = ref["path"]
    sys.path.insert(0, str(refp / "tests" / "t0"))
    from synth_ckpt import write_synth_checkpoint  # noqa: E402
    dst = HERE / "experts_bin"
    dst.mkdir(exist_ok=True)
    with tempfile.TemporaryDirectory() as td:
        model, out = Path(td) / "model", Path(td) / "out"
        exp = write_synth_checkpoint(model, layers=2, experts=16, hidden=64, ff=64)
        subprocess.run([sys.executable, str(refp / "tools" / "repack_experts.py"), "--model", str(model), "--out",
                        str(out), "--allow-buffered", "--expect-record", "0", "--max-mbps", "0"], check=True,
                       capture_output=True)
        shutil.copy(out / "experts.bin", dst / "experts.bin")
        shutil.copy(out / "experts.manifest.json", dst / "experts.manifest.json")
    names = [f"{p}.{k}" for p in ("gate_proj", "up_proj", "down_proj") for k in ("weight", "scales", "biases")]
    t = exp["tensors"]
    pieces = [[[hashlib.sha256(np.ascontiguousarray(t[f"language_model.model.layers.{L}.mlp.switch_mlp.{n}"][e])
                               .tobytes()).hexdigest() for n in names] for e in range(16)] for L in range(2)]
    (dst / "pieces.json").write_text(json.dumps({"hidden": 64, "inter": 64, "gs": 64, "sha256": pieces}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of a slotstream-spark checkout")
    ap.add_argument("--only", default=None, help="comma-separated fixture makers to run (e.g. make_sweep_plan)")
    a = ap.parse_args()
    refp = Path(a.reference).resolve()
    sys.path.insert(0, str(refp))
    sys.path.insert(0, str(refp / "tests" / "t0"))
    sys.path.insert(0, str(refp / "tests" / "gates"))
    from slotstream_spark.kernels import affine_ref, moe_align  # noqa: E402
    from slotstream_spark.kernels import fused_moe_affine as fm  # noqa: E402
    from slotstream_spark.model import reference_torch  # noqa: E402
    from slotstream_spark.engine import sweep  # noqa: E402
    import test_topk_stable  # noqa: E402
    import test_moe_gemv_affine  # noqa: E402
    import test_fused_moe_affine  # noqa: E402
    ref = dict(affine_ref=affine_ref, moe_align=moe_align, fm=fm, reference_torch=reference_torch,
               test_topk=test_topk_stable, test_moe=test_moe_gemv_affine, test_fused=test_fused_moe_affine, sweep=sweep, path=refp)
    torch.set_num_threads(8)
    makers = (make_affine, make_topk, make_align, make_combine, make_moe_ref, make_decode_ref, make_fused_ref,
              make_sweep_plan, make_experts_bin)
    only = None if a.only is None else set(a.only.split(","))
    for f in makers:
        if only is not None and f.__name__ not in only:
            continue
        f(ref)
        print("wrote", f.__name__)


if __name__ == "__main__":
    main()
