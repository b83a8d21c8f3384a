"""Expert-parallel prefill kernels on the GPU.

* the plan kernel against the oracle restatement, bit for bit (G = 2, 4, 8; strided and contiguous placement);
* G ranks emulated on one GPU (the all-to-alls done by concatenation): the exact-mode layer output equals the
  one-GPU fused layer bit for bit, the default mode within fp32 reassociation;
* two real ranks over NCCL when two GPUs are visible (skipped otherwise).
"""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch

from gpu_helpers import bf16_tensor, record
from oracle import ep_oracle as EO
from slotstream_b200 import synth
from slotstream_b200.records import BASELINE_LAYOUT

pytestmark = pytest.mark.gpu
E, K = 512, 10


@pytest.mark.parametrize("T", [3000, 20000])   # one CTA; a cluster of CTAs (4096 tokens and more)
@pytest.mark.parametrize("G,strided", [(2, True), (4, False), (8, True), (8, False)])
def test_plan_matches_oracle(G, strided, T):
    from slotstream_b200 import _lib
    rng = np.random.default_rng(G)
    ids = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K)).astype(np.float32)
    ref = EO.plan(ids, w, E, G, strided)
    cap = T * min(G, K)
    dc = torch.empty((G, 2), dtype=torch.int32, device="cuda")
    st = torch.empty(cap, dtype=torch.int32, device="cuda")
    sm = torch.empty((cap, 2 * K + 2), dtype=torch.int32, device="cuda")
    ts = torch.empty((T, G), dtype=torch.int32, device="cuda")
    te = torch.empty((T, G), dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    P = _lib.ptr
    ids_d, w_d = torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda()   # held until the kernel has run
    _lib.check(_lib.lib().ssb_ep_plan(P(ids_d), P(w_d), T, K, E // G, G, int(strided), P(dc), P(st), P(sm), P(ts),
                                      P(te), P(err), _lib.stream()), "plan")
    torch.cuda.synchronize()
    n = int(ref[1].size)
    assert int(err.item()) == 0
    assert np.array_equal(dc.cpu().numpy(), ref[0])
    assert np.array_equal(st[:n].cpu().numpy(), ref[1])
    assert np.array_equal(sm[:n].cpu().numpy(), ref[2])
    assert np.array_equal(ts.cpu().numpy(), ref[3])
    assert np.array_equal(te.cpu().numpy(), ref[4])


@pytest.fixture(scope="module")
def world():
    lay = BASELINE_LAYOUT
    recs = torch.from_numpy(np.stack([record(lay, 0, 0, e) for e in range(E + 1)])).cuda()
    base = recs.data_ptr() + torch.arange(E + 1, dtype=torch.int64) * lay.record_bytes
    rw = bf16_tensor(synth.router_weight(0, E, lay.hidden, 0))
    sg = bf16_tensor(synth.shared_gate_weight(0, lay.hidden, 0))
    bias = torch.from_numpy(synth.zipf_bias(E)).cuda()
    return dict(lay=lay, recs=recs, base=base, rw=rw, sg=sg, bias=bias)


def _one_gpu(W, x):
    from slotstream_b200.kernels.fused_moe_affine import combine_rank_order
    from slotstream_b200.kernels.moe_layer import PrefillLayerBuffers, moe_layer_prefill
    lay = W["lay"]
    bufs = PrefillLayerBuffers(x.shape[0], K, lay.hidden, lay.inter, E)
    y = moe_layer_prefill(x, W["rw"], W["base"].cuda(), W["sg"], K, bufs, bias=W["bias"]).clone()
    routed = combine_rank_order(bufs.out_rows[:x.shape[0] * K], x.shape[0], K)
    torch.cuda.synchronize()
    assert int(bufs.err.item()) == 0
    return y, routed


def _emulated(W, xs, G, strided, exact):
    """Every rank's steps of ep_forward on one GPU, the all-to-alls done by slicing and concatenation."""
    from slotstream_b200.ep import CudaOps, _prefix, owned_experts
    ops = []
    for r in range(G):
        gp = W["base"][owned_experts(r, E, G, strided)].cuda()
        ops.append(CudaOps(W["rw"], W["sg"], gp, int(W["base"][E]), K, W["lay"].inter, G, strided, bias=W["bias"]))
    st = []
    for r in range(G):
        ids, w, shg = ops[r].route(xs[r])
        sh = ops[r].shared(xs[r], shg)
        plan = ops[r].plan(ids, w)
        dc = plan.dest_count.cpu().numpy()
        n = int(dc[:, 0].sum())   # the plan is sized for the worst case; ep_forward trims it the same way
        plan.send_token, plan.send_meta = plan.send_token[:n], plan.send_meta[:n]
        st.append(dict(ids=ids, sh=sh, plan=plan, send_x=ops[r].gather(xs[r], plan.send_token), dc=dc))

    def blocks(r, key, counts_col):   # rank r's send buffer split per destination
        off = _prefix(st[r]["dc"][:, counts_col].tolist())
        return [st[r][key][off[d]:off[d + 1]] for d in range(G)]

    for d in range(G):
        st[d]["recv_x"] = torch.cat([blocks(r, "send_x", 0)[d] for r in range(G)])
        st[d]["recv_meta"] = torch.cat([st[r]["plan"].send_meta[_prefix(st[r]["dc"][:, 0].tolist())[d]:
                                                                 _prefix(st[r]["dc"][:, 0].tolist())[d + 1]]
                                        for r in range(G)])
        rrows = [int(st[r]["dc"][d, 0]) for r in range(G)]
        rent = [int(st[r]["dc"][d, 1]) for r in range(G)]
        ent = ops[d].unpack(st[d]["recv_meta"], _prefix(rrows), _prefix(rent), sum(rent))
        out_rows = ops[d].experts(st[d]["recv_x"], ent)
        st[d]["ret_out"] = out_rows if exact else ops[d].combine_rows(out_rows, ent)
        st[d]["ret_off"] = _prefix(rent if exact else rrows)
    ys, routed = [], []
    for r in range(G):
        parts = [st[d]["ret_out"][st[d]["ret_off"][r]:st[d]["ret_off"][r + 1]] for d in range(G)]
        ret = torch.cat(parts)
        reo = _prefix(st[r]["dc"][:, 1].tolist())[:G] if exact else None
        ys.append(ops[r].combine(ret, st[r]["plan"], st[r]["ids"], reo, st[r]["sh"], exact))
        routed.append(ops[r].routed)
    torch.cuda.synchronize()
    assert all(int(o.err.item()) == 0 for o in ops)
    return ys, routed


@pytest.mark.parametrize("G,strided,exact", [(2, True, True), (4, False, True), (8, True, True), (4, True, False)])
def test_emulated_ranks_match_one_gpu(world, G, strided, exact):
    xs = [bf16_tensor(synth.activations(90 + r, 160, world["lay"].hidden)) for r in range(G)]
    ys, routed = _emulated(world, xs, G, strided, exact)
    for r in range(G):
        y1, routed1 = _one_gpu(world, xs[r])
        if exact:
            assert torch.equal(routed[r].view(torch.int32), routed1.view(torch.int32))
            assert torch.equal(ys[r], y1)
        else:
            torch.testing.assert_close(routed[r], routed1, rtol=1e-5, atol=1e-4)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world_size, port, out_dir, mb=1, bf16=False, tokens=300, zipf=True, exact=None):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world_size, device_id=torch.device("cuda", rank),
                            timeout=timedelta(seconds=120))
    try:
        from slotstream_b200.ep import CudaOps, ep_forward, owned_experts
        lay = BASELINE_LAYOUT
        recs = torch.from_numpy(np.stack([record(lay, 0, 0, e) for e in range(E + 1)])).cuda()
        base = recs.data_ptr() + torch.arange(E + 1, dtype=torch.int64) * lay.record_bytes
        W = dict(lay=lay, recs=recs, base=base, rw=bf16_tensor(synth.router_weight(0, E, lay.hidden, 0)),
                 sg=bf16_tensor(synth.shared_gate_weight(0, lay.hidden, 0)),
                 bias=torch.from_numpy(synth.zipf_bias(E)).cuda() if zipf else None)
        x = bf16_tensor(synth.activations(90 + rank, tokens, lay.hidden, tag=tokens))
        ops = CudaOps(W["rw"], W["sg"], base[owned_experts(rank, E, world_size, True)].cuda(), int(base[E]), K,
                      lay.inter, world_size, True, bias=W["bias"])
        exact = (not bf16) if exact is None else exact
        y = ep_forward(ops, x, K, world_size, exact=exact, micro_batches=mb, partials_bf16=bf16)
        y1, routed1 = _one_gpu(W, x)
        torch.cuda.synchronize()
        d, r = (y.float() - y1.float()), y1.float()
        if exact:
            ok = bool(torch.equal(y, y1)) and bool(torch.equal(ops.routed.view(torch.int32), routed1.view(torch.int32)))
        elif bf16:   # partial sums rounded to bf16 on the return: within the layer tolerance of one GPU
            ok = bool(d.norm() <= 5e-3 * r.norm()) and bool(d.abs().max() <= 2e-2 * r.abs().max())
        else:        # fp32 partial sums: the one-GPU rank-order sum reassociated per destination
            dr = ops.routed - routed1
            ok = bool(dr.norm() <= 1e-5 * routed1.norm()) and bool(d.norm() <= 1e-3 * r.norm())
        ok = ok and int(ops.err.item()) == 0
        with open(os.path.join(out_dir, f"ok{rank}"), "w") as f:
            f.write("1" if ok else f"0 rel {float(d.norm() / r.norm()):.3e} max {float(d.abs().max()):.3e}")
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _spawn(tmp_path, n, **kw):
    import torch.multiprocessing as mp
    args = (n, _free_port(), str(tmp_path), kw.get("mb", 1), kw.get("bf16", False), kw.get("tokens", 300),
            kw.get("zipf", True), kw.get("exact"))
    mp.start_processes(_nccl_rank, args=args, nprocs=n, join=True, start_method="spawn")
    for r in range(n):
        assert (tmp_path / f"ok{r}").read_text() == "1", (r, (tmp_path / f"ok{r}").read_text())


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("mb,bf16", [(1, False), (2, False), (1, True)])
def test_two_ranks_over_nccl_match_one_gpu(tmp_path, mb, bf16):
    """mb = 2: micro-batched exchange, the expert GEMMs of one part overlapping the transfers of the other;
    bf16: partial sums returned in bf16, compared within the layer tolerance."""
    _spawn(tmp_path, 2, mb=mb, bf16=bf16)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs four GPUs")
@pytest.mark.parametrize("zipf", [True, False])
@pytest.mark.parametrize("mode", ["exact", "fp32", "bf16"])
def test_all_ranks_over_nccl_32k_tokens_match_one_gpu(tmp_path, zipf, mode):
    """Every visible GPU a rank (4 or 8), 32,768 tokens per rank, Zipf-skewed and uniform routing: each rank's
    expert-parallel output against the one-GPU layer on the same tokens -- bit for bit in exact mode, within fp32
    reassociation with fp32 partial sums, within the layer tolerance with bf16 partial sums."""
    n = 8 if torch.cuda.device_count() >= 8 else 4
    _spawn(tmp_path, n, tokens=32768, zipf=zipf, bf16=mode == "bf16", exact=mode == "exact")
