"""moe_align kernel: bit-exact against the reference's golden outputs and the oracle (GPU)."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def _align(le, nl, bm, emap=None):
    from slotstream_b200.kernels.moe_align import moe_align
    t = torch.from_numpy(np.ascontiguousarray(le, dtype=np.int32)).cuda()
    em = None if emap is None else torch.from_numpy(np.ascontiguousarray(emap, dtype=np.int32)).cuda()
    sr, be, npad = moe_align(t, nl, bm, expert_map=em)
    torch.cuda.synchronize()
    return sr.cpu().numpy(), be.cpu().numpy(), npad.cpu().numpy()


def test_align_matches_reference_golden():
    g = np.load(GOLDEN / "align.npz")
    for i, name in enumerate(g["names"]):
        nl, bm = (int(v) for v in g[f"c{i}_meta"])
        sr, be, npad = _align(g[f"c{i}_in"], nl, bm)
        assert np.array_equal(sr, g[f"c{i}_sorted"]), name
        assert np.array_equal(be, g[f"c{i}_block"]), name
        assert np.array_equal(npad, g[f"c{i}_npad"]), name


@pytest.mark.parametrize("r,nl,bm", [(327680, 512, 128), (81920, 512, 64), (40960, 32, 64), (100003, 1280, 16)])
def test_align_large_vs_oracle(r, nl, bm):
    rng = np.random.default_rng(r)
    le = np.minimum(rng.zipf(1.3, r) - 1, nl + 5).astype(np.int32)     # skewed, some out of range
    le[rng.random(r) < 0.05] = -1
    sr, be, npad = _align(le, nl, bm)
    rs, rb, rn = O.moe_align(le, nl, bm)
    assert np.array_equal(npad, rn)
    assert np.array_equal(sr, rs)
    assert np.array_equal(be, rb)


@pytest.mark.parametrize("n", [20000, 70000])   # one CTA; a cluster of CTAs (32768 rows and more)
def test_align_with_expert_map_equals_gather_then_align(n):
    rng = np.random.default_rng(1)
    ids = rng.integers(-2, 514, n).astype(np.int32)
    emap = np.full(512, -1, dtype=np.int32)
    group = rng.permutation(512)[:32]
    emap[group] = np.arange(32)
    local = np.where((ids >= 0) & (ids < 512), emap[np.clip(ids, 0, 511)], -1).astype(np.int32)
    got = _align(ids, 32, 64, emap)
    ref = O.moe_align(local, 32, 64)
    for a, b in zip(got, ref):
        assert np.array_equal(a, b)


def test_align_is_deterministic():
    rng = np.random.default_rng(2)
    le = rng.integers(0, 512, 81920).astype(np.int32)
    a = _align(le, 512, 128)
    b = _align(le, 512, 128)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)
