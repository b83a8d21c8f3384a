"""Expert-parallel exchange protocol on CPU: two gloo ranks drive slotstream_b200.ep.ep_forward with
oracle-backed compute; the routed sums must equal the one-rank layer (exact mode bit for bit, default mode to
fp32 reassociation), for strided and contiguous expert placement and skewed routing."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ep_cpu_ops import CpuOps, bits_to_bf16, single_rank_reference
from oracle import ep_oracle as EO
from slotstream_b200 import synth
from slotstream_b200.records import RecordLayout

LAY = RecordLayout(128, 64, 64)
E, K, T = 16, 4, 12


def _world(seed):
    recs = [synth.expert_record(LAY, seed, 0, e) for e in range(E)]
    shared = synth.expert_record(LAY, seed, 0, E)
    rw = synth.router_weight(seed, E, LAY.hidden, 0)
    sg = synth.shared_gate_weight(seed, LAY.hidden, 0)
    return recs, shared, rw, sg


def _tokens(rank, counts=None):
    return synth.activations(70 + rank, T if counts is None else counts[rank], LAY.hidden)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir, strided, exact, zipf, mb=1, bf16=False, counts=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from slotstream_b200.ep import ep_forward
        recs, shared, rw, sg = _world(5)
        bias = synth.zipf_bias(E) * 4 if zipf else None
        ops = CpuOps(LAY, recs, shared, rw, sg, K, E, world, rank, strided=strided, bias=bias)
        y = ep_forward(ops, bits_to_bf16(_tokens(rank, counts)), K, world, exact=exact, micro_batches=mb,
                       partials_bf16=bf16)
        np.save(os.path.join(out_dir, f"routed{rank}.npy"), ops.routed.numpy())
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y.view(torch.int16).numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("strided,exact,zipf,mb", [(True, True, False, 1), (False, True, True, 1), (True, False, True, 1),
                                                   (True, True, True, 2), (False, False, False, 3)])
def test_ep_exchange_matches_single_rank(tmp_path, strided, exact, zipf, mb):
    """mb > 1: the tokens split into micro-batches with overlapped exchanges; the sums stay the same."""
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path), strided, exact, zipf, mb), nprocs=world,
                       join=True, start_method="spawn")
    recs, shared, rw, sg = _world(5)
    bias = synth.zipf_bias(E) * 4 if zipf else None
    for rank in range(world):
        got = np.load(tmp_path / f"routed{rank}.npy")
        ref = single_rank_reference(LAY, recs, shared, rw, sg, K, _tokens(rank), bias=bias)
        if exact:
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        else:
            np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)


def test_plan_orders_rows_by_destination_then_token():
    rng = np.random.default_rng(3)
    ids = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K)).astype(np.float32)
    dc, st, sm, ts, te = EO.plan(ids, w, E, 4, True)
    assert dc[:, 0].sum() == len(st) and dc[:, 1].sum() == T * K
    off = np.concatenate([[0], np.cumsum(dc[:, 0])])
    for d in range(4):
        toks = st[off[d]:off[d + 1]]
        assert np.all(np.diff(toks) > 0)
        for r, t in zip(range(off[d], off[d + 1]), toks):
            assert ts[t, d] == r
            mine = [j for j in range(K) if ids[t, j] % 4 == d]
            assert sm[r, 2 * K + 1] == len(mine)
            assert [sm[r, j] for j in mine] == [ids[t, j] // 4 for j in mine]
    assert np.all((ts >= 0) == (te >= 0))


def test_ep_exchange_with_bf16_partials(tmp_path):
    """Default mode with the partial sums rounded to bf16 for the return: routed within the partials' rounding
    (relative L2 under 2^-8) of the one-rank layer."""
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path), True, False, True, 2, True),
                       nprocs=world, join=True, start_method="spawn")
    recs, shared, rw, sg = _world(5)
    for rank in range(world):
        got = np.load(tmp_path / f"routed{rank}.npy").astype(np.float64)
        ref = single_rank_reference(LAY, recs, shared, rw, sg, K, _tokens(rank), bias=synth.zipf_bias(E) * 4)
        ref = ref.astype(np.float64)
        assert np.linalg.norm(got - ref) <= 2.0 ** -8 * np.linalg.norm(ref)
        assert not np.array_equal(got, ref)   # the rounding did happen


@pytest.mark.parametrize("exact", [True, False])
def test_ep_exchange_with_uneven_and_empty_ranks(tmp_path, exact):
    """Four ranks holding 0, 2, 12 and 5 tokens with micro_batches = 3: every rank posts the same collectives (the
    part count does not depend on the token count), empty parts exchange zero rows, and each rank's sums equal the
    one-rank layer on its own tokens."""
    world, counts = 4, (0, 2, 12, 5)
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path), True, exact, True, 3, False, counts),
                       nprocs=world, join=True, start_method="spawn")
    recs, shared, rw, sg = _world(5)
    for rank in range(world):
        got = np.load(tmp_path / f"routed{rank}.npy")
        assert got.shape == (counts[rank], LAY.hidden)
        if counts[rank] == 0:
            continue
        ref = single_rank_reference(LAY, recs, shared, rw, sg, K, _tokens(rank, counts), bias=synth.zipf_bias(E) * 4)
        if exact:
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        else:
            np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)


class _CorruptOps(CpuOps):
    """Rank 0's plan claims more entries for rank 1 than its rows can carry."""

    def plan(self, ids, w):
        p = super().plan(ids, w)
        if self.rank == 0:
            p.dest_count[1, 1] = p.dest_count[1, 0] * self.k + 5
        return p


def _corrupt_main(rank, world, port, out_dir):
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=8))
    outcome = "returned"
    try:
        from slotstream_b200.ep import ExchangeError, ep_forward
        recs, shared, rw, sg = _world(5)
        ops = _CorruptOps(LAY, recs, shared, rw, sg, K, E, world, rank, strided=True)
        try:
            ep_forward(ops, bits_to_bf16(_tokens(rank)), K, world)
        except ExchangeError:
            outcome = "inconsistent counts"
        except RuntimeError:
            outcome = "collective failed"
    finally:
        with open(os.path.join(out_dir, f"outcome{rank}"), "w") as f:
            f.write(outcome)
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_corrupt_counts_end_every_rank_with_an_error(tmp_path):
    """One rank sends a count vector that cannot be right: the rank receiving it raises before posting the dispatch,
    and the sender's next collective ends with the process group's timeout -- every rank stops with an error, none
    hangs and none computes on the bad sizes."""
    world = 2
    mp.start_processes(_corrupt_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    outcomes = [(tmp_path / f"outcome{r}").read_text() for r in range(world)]
    assert outcomes[1] == "inconsistent counts"
    assert outcomes[0] in ("inconsistent counts", "collective failed")


def test_balanced_labels_even_out_the_ranks():
    """balanced_labels: a permutation of the experts whose strided placement gives every rank about the same
    routing count (Zipf-skewed counts), where the plain strided placement of the original ids does not."""
    import numpy as np
    from slotstream_b200.ep import balanced_labels, owned_experts
    rng = np.random.default_rng(0)
    counts = np.bincount((rng.zipf(1.3, 40000) - 1) % 512, minlength=512)
    for g in (2, 4, 8):
        label, expert = balanced_labels(counts, g)
        assert sorted(label.tolist()) == list(range(512)) and np.array_equal(label[expert], np.arange(512))
        per_rank = [counts[expert[owned_experts(r, 512, g, True)]].sum() for r in range(g)]
        strided = [counts[owned_experts(r, 512, g, True)].sum() for r in range(g)]
        assert max(per_rank) <= max(strided)
        assert max(per_rank) - min(per_rank) <= counts.max()   # within one expert of even
