"""Benchmark of the B200 MoE hot path; prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload prefill|decode|slotpool|sweep] [--impl reference]

Workloads (synthetic data with the distributions BASELINE.json names):
* ``decode``  (configs[1]): one decode step = 48 stacked config[0] MoE layers at batch b (default 1), Zipf(1.1)
  routing, all 48 x 512 expert records resident in HBM, the step captured in one CUDA graph. Each layer reads
  its own resident N(0,1) hidden state (the attention / hyper-connection segments between MoE layers, which
  renormalise the residual stream in the real model, are not part of this path).
* ``prefill`` (configs[2]/[3]): one step = one config[0] layer over a chunk of tokens per GPU.
* ``sweep``   (configs[2] with a partly resident layer): the prefill layer when only the hottest half of its
  records sit in HBM; the rest are staged per 32-expert group from pinned host memory beside the compute.
* ``slotpool``: one step = one fresh token through 48 layers whose routed experts stream through an
  HBM slot pool of 1 GiB chunks holding 70% of the records (misses copied from pinned host memory on a side
  stream); metric = MoE-path ms per token. The default run reports it as the ``slotpool`` sub-measurement.

Timing: W untimed warm-up steps, then K steps, each bracketed by CUDA events on the launching stream with an
L2 flush (256 MiB write) before it, barrier + synchronize on both sides, max over ranks. The JSON line carries
``roofline`` (dominant launch vs MEASURED_PEAKS.json), ``cpu_baseline`` (oracle port on the host cores, rank 0,
N=1), ``e2e`` (host buffers through the public API), ``gpu_launches`` and ``clocks``.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "slotstream-spark_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "MoE-layer tokens/s (decode b=1 HBM GB/s; prefill TFLOPS) at 1/2/4/8 B200"
L2_FLUSH_BYTES = 256 << 20
# DRAM bytes (read + write) per launch of the dominant kernel: constants measured by ncu (dram__bytes_read.sum +
# dram__bytes_write.sum, one replay pass) on earlier runs of these same workloads, not in this run
TRAFFIC_BYTES = {
    "prefill_gate_up_32768": 1_853_983_744 + 349_953_280,   # one gate_up launch of the 32,768-token layer
    "prefill_gate_up_8192": 654_045_440 + 88_479_744,       # one gate_up launch of the 8,192-token layer
    "decode_fused_b1": 21_684_736,                          # one fused b = 1 decode layer launch
}
TRAFFIC_SOURCE = "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch, measured on an earlier run of " \
                 "this workload (a constant of this file, not measured in this run)"


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.samples = []
        self.proc = None
        self.t_on = self.t_off = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "20", "-i", str(self.dev)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        threading.Thread(target=self._read, daemon=True).start()
        # nvidia-smi takes a moment to start: wait for its first sample so that the timed region is covered
        t0 = time.monotonic()
        while not self.samples and time.monotonic() - t0 < 5.0 and self.proc.poll() is None:
            time.sleep(0.01)

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.monotonic(), [v.strip() for v in line.split(",")]))

    def mark_on(self):
        self.t_on = time.monotonic()

    def mark_off(self):
        self.t_off = time.monotonic()

    def stop(self):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        inside = [s for t, s in self.samples if self.t_on is not None and self.t_on <= t <= (self.t_off or t)]
        # a timed region shorter than the sampling period: the samples within 0.2 s of it (GPU still busy)
        near = [s for t, s in self.samples
                if self.t_on is not None and self.t_on - 0.2 <= t <= (self.t_off or t) + 0.2]
        use = inside if inside else (near if near else [s for _, s in self.samples])
        sm = [float(s[1]) for s in use if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in use if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in use for i in range(4) if len(s) > 5 + i and s[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(use), "samples_in_timed_region": len(inside),
                "samples_within_0.2s": len(near)}


# ------------------------------------------------------------------ distributed plumbing
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()


def max_over_ranks(v, world):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def timed_steps(run, k, flush_buf, world, clocks=None):
    """Per-step CUDA-event times (ms) on the current stream, L2 flushed before every step."""
    st = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(k)]
    barrier(world)
    if clocks:
        clocks.mark_on()
    for a, b in evs:
        flush_buf.zero_()
        a.record(st)
        run()
        b.record(st)
    barrier(world)
    if clocks:
        clocks.mark_off()
    return [a.elapsed_time(b) for a, b in evs]


def pipelined_steps(x_dev, graphs, y_dev, x_host, k, world):
    """ms per step of k steps over two buffer sets: step i copies x_host[i % 2] into x_dev[i % 2] on an H2D
    stream, replays graphs[i % 2] on the current stream and copies y_dev[i % 2] out on a D2H stream; a buffer
    set is reused only after its previous step's compute (for x) and D2H (for y) finished. Timed from an event
    before the first copy to the last D2H, on the device."""
    comp = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    y_host = [torch.empty(y.shape, dtype=y.dtype).pin_memory() for y in y_dev]
    ev = lambda: torch.cuda.Event()  # noqa: E731
    ev_in, ev_c, ev_out = [ev() for _ in range(k)], [ev() for _ in range(k)], [ev() for _ in range(k)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    t0.record(comp)
    h2d.wait_event(t0)
    for i in range(k):
        b = i % 2
        if i >= 2:
            h2d.wait_event(ev_c[i - 2])          # x_dev[b] is free once step i-2 computed
        with torch.cuda.stream(h2d):
            x_dev[b].copy_(x_host[b], non_blocking=True)
        ev_in[i].record(h2d)
        comp.wait_event(ev_in[i])
        if i >= 2:
            comp.wait_event(ev_out[i - 2])       # y_dev[b] is free once step i-2's D2H finished
        graphs[b].replay()
        ev_c[i].record(comp)
        d2h.wait_event(ev_c[i])
        with torch.cuda.stream(d2h):
            y_host[b].copy_(y_dev[b], non_blocking=True)
        ev_out[i].record(d2h)
    comp.wait_event(ev_out[k - 1])
    t1.record(comp)
    barrier(world)
    return t0.elapsed_time(t1) / k


# ------------------------------------------------------------------ CPU leg (cpu_baseline + parity of this run)
def cpu_leg_prefill(LAY, recs, router_w, sh_gate_w, bias, x, y_dev, ids_dev, passes):
    """The reference's CPU path (oracle/cpu_baseline.py) over this run's own prefill chunk: the records, router
    and tokens copied back from the GPU, `passes` timed passes over the whole chunk (0: one untimed pass), and the
    GPU layer output of the timed step compared with the CPU result on the same bytes."""
    from oracle.cpu_baseline import CpuLayer, parity, time_prefill_chunks
    L = CpuLayer.from_tensors(LAY, recs.cpu(), router_w.cpu(), sh_gate_w.cpu(), None if bias is None else bias.cpu())
    rec, y_cpu, ids_cpu = time_prefill_chunks(L, x.cpu(), n_chunks=max(1, passes))
    par = parity(y_dev.cpu(), ids_dev.cpu(), y_cpu, ids_cpu)
    par["reference"] = "CPU path of the reference (oracle/cpu_baseline.py) on the same records and tokens"
    return (rec if passes else None), par


def cpu_leg_decode(LAY, W, x0, y0, ids0, seconds):
    """Decode layer 0 of this run on the CPU (its 512 records and shared record copied back): parity of the GPU
    layer-0 output for the b tokens of the timed step, and, when seconds > 0, the CPU decode rate."""
    from oracle.cpu_baseline import CpuLayer, decode_token_layer, parity, time_decode
    E = 512
    recs = torch.cat([W["recs"][:E], W["shared"][:1]]).cpu()
    L = CpuLayer.from_tensors(LAY, recs, W["router_w"][0].cpu(), W["sh_gate_w"][0].cpu(), W["bias"].cpu())
    ys, ids = [], []
    with torch.no_grad():
        for t in range(x0.shape[0]):
            y, i = decode_token_layer(L, x0[t:t + 1].cpu().float())
            ys.append(y)
            ids.append(i)
    par = parity(y0.cpu(), ids0.cpu(), torch.cat(ys), torch.cat(ids))
    par["reference"] = "CPU path of the reference (oracle/cpu_baseline.py), layer 0 of this run's step"
    return (time_decode(L, seconds=seconds) if seconds > 0 else None), par


# ------------------------------------------------------------------ decode workload
def decode_world(args, rank):
    """Resident records (layers x 512 routed + one shared per layer), router weights and slot tables."""
    from slotstream_b200 import synth
    from slotstream_b200.records import BASELINE_LAYOUT as LAY, MAP_LAYERS
    NL, E = args.layers, 512
    dev = torch.device("cuda")
    rb = LAY.record_bytes
    seed = 1000 + rank
    recs = torch.empty((NL * E, rb), dtype=torch.uint8, device=dev)
    synth.fill_records_device(LAY, recs, seed)
    shared = torch.empty((NL, rb), dtype=torch.uint8, device=dev)
    synth.fill_records_device(LAY, shared, seed + 7)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    router_w = (torch.randn(NL, E, LAY.hidden, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    sh_gate_w = (torch.randn(NL, LAY.hidden, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    bias = torch.from_numpy(synth.zipf_bias(E)).to(dev)
    map_t = torch.full((MAP_LAYERS * E,), -1, dtype=torch.int32, device=dev)
    map_t[:NL * E] = torch.arange(NL * E, dtype=torch.int32, device=dev)
    slot_ptr = recs.data_ptr() + torch.arange(NL * E, dtype=torch.int64, device=dev) * rb
    return dict(recs=recs, shared=shared, router_w=router_w, sh_gate_w=sh_gate_w, bias=bias, map_t=map_t,
                slot_ptr=slot_ptr, gen=g)


def bench_decode(args, world, rank, batch=None, W=None, cpu_seconds=None):
    from slotstream_b200.kernels.moe_layer import DecodeLayerBuffers, decode_layers, moe_layer_decode
    from slotstream_b200.records import BASELINE_LAYOUT as LAY
    NL, E, K = args.layers, 512, 10
    b = batch or args.batch
    dev = torch.device("cuda")
    rb = LAY.record_bytes
    W = W or decode_world(args, rank)
    recs, shared, router_w, sh_gate_w = W["recs"], W["shared"], W["router_w"], W["sh_gate_w"]
    bias, map_t, slot_ptr, g = W["bias"], W["map_t"], W["slot_ptr"], W["gen"]
    x = torch.randn(NL, b, LAY.hidden, device=dev, generator=g).to(torch.bfloat16)
    bufs = [DecodeLayerBuffers(b, K, LAY.hidden, LAY.inter, E, dev) for _ in range(NL)]
    prefetch = args.decode_prefetch
    side = torch.cuda.Stream() if prefetch else None

    def step():
        # every layer's MoE launch (with --decode-prefetch a side stream prefetches the next layer's router weight
        # and shared record into L2)
        decode_layers(x, router_w, sh_gate_w, shared, map_t, slot_ptr, K, bufs, bias=bias, prefetch_next=prefetch,
                      side=side)

    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    torch.cuda.synchronize()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        flush.zero_()
        graph.replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    times = timed_steps(graph.replay, args.steps, flush, world, clocks)
    clocks.stop()
    ms = max_over_ranks(sum(times) / len(times), world)

    # bytes per step from the routing the step actually produced (unique experts per layer)
    uniq = [int(torch.unique(bf.ids).numel()) for bf in bufs]
    per_layer_fixed = rb + E * LAY.hidden * 2 + LAY.hidden * 2 + b * LAY.hidden * 2 * 2
    step_bytes = sum(u * rb for u in uniq) + NL * per_layer_fixed
    errs = sum(int(bf.err.item()) for bf in bufs)

    # dominant launch, timed per layer outside the graph after an L2 flush: at b <= 2 the whole layer is one
    # cooperative launch (moe_decode_fused); above, the gate_up + down pair of moe_decode_layer
    from slotstream_b200 import _lib
    from slotstream_b200.kernels.moe_layer import FUSED_MAX_ROWS
    fused = b <= FUSED_MAX_ROWS
    st = torch.cuda.current_stream()
    lt = []
    for l in range(NL):
        moe_layer_decode(x[l], router_w[l], l, map_t, slot_ptr, shared[l], sh_gate_w[l], K, bufs[l], bias=bias)
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        if fused:
            moe_layer_decode(x[l], router_w[l], l, map_t, slot_ptr, shared[l], sh_gate_w[l], K, bufs[l], bias=bias)
        else:
            rc = _lib.lib().ssb_moe_decode_layer(
                _lib.ptr(x[l]), _lib.ptr(bufs[l].ids), _lib.ptr(bufs[l].w), b, K, LAY.hidden, LAY.inter, l,
                _lib.ptr(map_t), map_t.numel(), _lib.ptr(slot_ptr), slot_ptr.numel(), shared[l].data_ptr(),
                _lib.ptr(bufs[l].sh_gate), _lib.ptr(bufs[l].bases), _lib.ptr(bufs[l].h), _lib.ptr(bufs[l].o),
                _lib.ptr(bufs[l].out), _lib.ptr(bufs[l].y), 0, _lib.ptr(bufs[l].err), _lib.stream())
            _lib.check(rc, "moe_decode_layer")
        e1.record(st)
        torch.cuda.synchronize()
        lt.append(e0.elapsed_time(e1))
    launch_ms = sum(lt) / len(lt)
    if fused:
        launch_bytes = step_bytes / NL
        kname = "moe_decode_fused (whole layer: router, select, gate_up, down, combine)"
    else:
        launch_bytes = (sum(u * rb for u in uniq) + NL * (rb + b * LAY.hidden * 2 * 2)) / NL
        kname = "moe_decode_layer (grouped gate_up + down + rank_sum)"
    pk = peaks()
    # the roofline figure is the layer's time inside the timed 48-layer graph (step time / layers); the launch timed
    # alone after an L2 flush (cold caches, no neighbour overlap) is reported beside it
    layer_ms = ms / NL
    achieved = launch_bytes / (layer_ms * 1e-3) / 1e9
    roofline = {"bound": "hbm", "kernel": kname, "achieved": round(achieved, 1),
                "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                "peak_source": pk["source"] + " (copy)", "timing": "per layer inside the timed graph (step / layers)",
                "traffic": TRAFFIC_BYTES["decode_fused_b1"] if (fused and b == 1) else None,
                "traffic_source": TRAFFIC_SOURCE,
                "bytes_per_launch": int(launch_bytes), "layer_us": round(layer_ms * 1e3, 2),
                "isolated_launch_us": round(launch_ms * 1e3, 2),
                "isolated_launch_gbs": round(launch_bytes / (launch_ms * 1e-3) / 1e9, 1)}

    # e2e: host inputs (pinned) -> device, graph step, outputs -> host, all inside the timed region
    x_host = x.cpu().pin_memory()
    y_host = torch.empty((NL, b, LAY.hidden), dtype=torch.bfloat16).pin_memory()
    y_dev = torch.stack([bf.y for bf in bufs])

    def e2e_step():
        x.copy_(x_host, non_blocking=True)
        graph.replay()
        y_host.copy_(torch.stack([bf.y for bf in bufs]), non_blocking=True)

    for _ in range(2):
        e2e_step()
    e2e_times = timed_steps(e2e_step, args.steps, flush, world)
    e2e_ms = max_over_ranks(sum(e2e_times) / len(e2e_times), world)
    del y_dev

    value = world * b / (ms * 1e-3)
    res = {
        "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"decode_step_{NL}layer_b{b}", "layers": NL, "batch": b, "hidden": LAY.hidden,
                   "inter": LAY.inter, "experts": E, "topk": K, "shared_experts": 1, "routing": "zipf_s1.1",
                   "weights": "affine4_gs64 resident in HBM (48x512 records)", "cuda_graph": True,
                   "next_layer_l2_prefetch": prefetch,
                   "l2": "flushed before every step (256 MiB write)", "parallelism": f"replicas{world}"},
        "hbm_gbs_per_step": round(step_bytes / (ms * 1e-3) / 1e9, 1),
        "bytes_per_step": int(step_bytes), "unique_experts_per_layer_mean": round(sum(uniq) / NL, 2),
        "roofline": roofline,
        "e2e": {"value": round(world * b / (e2e_ms * 1e-3), 2), "unit": "tokens/s",
                "h2d_bytes_per_step": int(x.numel() * 2), "d2h_bytes_per_step": int(y_host.numel() * 2)},
        "gpu_launches": (1 if b <= FUSED_MAX_ROWS else 5) * NL * args.steps,
        "clocks": clocks.summary(),
        "device_errors": errs,
    }
    if cpu_seconds is not None:
        cb, par = cpu_leg_decode(LAY, W, x[0], bufs[0].y, bufs[0].ids, cpu_seconds)
        res["parity"] = par
        if cb is not None:
            res["cpu_baseline"] = cb
    return res


# ------------------------------------------------------------------ slot-pool streaming decode
def bench_slotpool(args, world, rank):
    """48-layer b=1 decode whose routed experts stream through an HBM slot pool of 1 GiB chunks holding 70% of
    the 48 x 512 records (random initial slot table, CLOCK replacement); every step is a fresh token with uniform
    routing, so about 30% of the experts it needs are absent and are copied from pinned host records on a side
    stream while the layer waits on an event. Metric: MoE-path time per token."""
    from slotstream_b200 import synth
    from slotstream_b200.kernels.moe_layer import DecodeLayerBuffers
    from slotstream_b200.records import BASELINE_LAYOUT as LAY
    from slotstream_b200.slot_pool import SlotPool, decode_layer_streaming, host_table
    NL, E, K = args.layers, 512, 10
    dev = torch.device("cuda")
    rb = LAY.record_bytes
    seed = 4000 + rank
    # host store: 512 distinct pinned records, expert e of every layer reads record e
    store_dev = torch.empty((E, rb), dtype=torch.uint8, device=dev)
    synth.fill_records_device(LAY, store_dev, seed)
    store = torch.empty((E, rb), dtype=torch.uint8).pin_memory()
    store.copy_(store_dev)
    del store_dev
    shared = torch.empty((NL, rb), dtype=torch.uint8, device=dev)
    synth.fill_records_device(LAY, shared, seed + 7)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    router_w = (torch.randn(NL, E, LAY.hidden, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    sh_gate_w = (torch.randn(NL, LAY.hidden, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    n_tok = args.warmup + 2 * args.steps + 4
    xs = torch.randn(n_tok, NL, 1, LAY.hidden, device=dev, generator=g).to(torch.bfloat16)
    table = host_table(store.data_ptr(), rb, NL, E, per_layer=False)
    capacity = int(round(args.pool_fraction * NL * E))
    pool = SlotPool(rb, NL, E, chunk_bytes=1 << 30)
    pool.resize(capacity)
    copy = torch.cuda.Stream()
    # random initial slot table: a random 70% of the (layer, expert) pairs, filled in random order
    rng = np.random.default_rng(seed)
    pick = rng.permutation(NL * E)[:capacity]
    for l in range(NL):
        ex = pick[pick // E == l] % E
        if ex.size:
            pool.ensure(l, ex, table, copy, torch.cuda.current_stream())
    pool.release()
    torch.cuda.synchronize()
    bufs = [DecodeLayerBuffers(1, K, LAY.hidden, LAY.inter, E, dev) for _ in range(NL)]
    ids_host = torch.empty((1, K), dtype=torch.int32).pin_memory()
    tok = [0]
    launches = [0]

    def step():
        t = tok[0] % n_tok
        tok[0] += 1
        for l in range(NL):
            _, st_ = decode_layer_streaming(pool, table, xs[t, l], router_w[l], l, shared[l], sh_gate_w[l], K, bufs[l],
                                            copy_stream=copy, ids_host=ids_host)
            launches[0] += 4 + (1 if st_[1] else 0)

    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    h0, m0, b0 = pool.counters()
    launches[0] = 0
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    times = timed_steps(step, args.steps, flush, world, clocks)
    clocks.stop()
    h1, m1, b1 = pool.counters()
    n_launch = launches[0]
    ms = max_over_ranks(sum(times) / len(times), world)
    errs = sum(int(bf.err.item()) for bf in bufs)
    miss_frac = (m1 - m0) / max(1, (h1 - h0) + (m1 - m0))
    h2d_per_step = (b1 - b0) / args.steps

    # the copy engine's own H2D rate for record-sized pinned copies (the bound of this workload)
    dst = torch.empty((64, rb), dtype=torch.uint8, device=dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(copy):
        for rep in range(2):
            e0.record(copy)
            for i in range(64):
                dst[i].copy_(store[(7 * i + rep) % E], non_blocking=True)
            e1.record(copy)
    torch.cuda.synchronize()
    h2d_gbs = 64 * rb / (e0.elapsed_time(e1) * 1e-3) / 1e9
    del dst
    achieved = h2d_per_step / (ms * 1e-3) / 1e9

    # e2e: the token's hidden states from pinned host memory and the layers' outputs back, inside the step
    n_e2e = max(3, args.steps // 4)
    tok0 = tok[0]
    x_host = xs[tok0:tok0 + n_e2e].cpu().pin_memory()   # tokens no step has used yet
    y_host = torch.empty((NL, 1, LAY.hidden), dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        t = tok[0]
        xs[t].copy_(x_host[t - tok0], non_blocking=True)
        step()
        y_host.copy_(torch.stack([bf.y for bf in bufs]), non_blocking=True)

    e2e_times = timed_steps(e2e_step, n_e2e, flush, world)
    e2e_ms = max_over_ranks(sum(e2e_times) / len(e2e_times), world)
    res = {
        "metric": "MoE-path time per token (slot-pool streaming decode)", "value": round(ms, 4), "unit": "ms/token",
        "higher_is_better": False, "tokens_per_s": round(1e3 / ms, 2), "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": f"slotpool_decode_{NL}layer_b1", "layers": NL, "batch": 1, "experts": E, "topk": K,
                   "routing": "uniform (fresh token every step)", "pool_slots": capacity,
                   "pool_fraction_of_records": args.pool_fraction, "chunk_bytes": 1 << 30,
                   "pool_chunks": pool.chunks, "host_store": "512 pinned records shared by the layers",
                   "l2": "flushed before every step (256 MiB write)", "cuda_graph": False},
        "miss_fraction": round(miss_frac, 4), "misses_per_layer": round((m1 - m0) / (args.steps * NL), 3),
        "h2d_bytes_per_step": int(h2d_per_step),
        "roofline": {"bound": "h2d", "kernel": "host-to-device record copies (copy engine)",
                     "achieved": round(achieved, 2), "peak": round(h2d_gbs, 2), "unit": "GB/s",
                     "frac": round(achieved / h2d_gbs, 4), "peak_source": "measured in this run: 64 pinned "
                     "record copies back to back on the copy stream", "traffic": None},
        "e2e": {"value": round(e2e_ms, 4), "unit": "ms/token", "h2d_bytes_per_step": int(h2d_per_step + x_host[0].numel() * 2),
                "d2h_bytes_per_step": int(y_host.numel() * 2 + NL * K * 4)},
        "gpu_launches": n_launch,
        "clocks": clocks.summary(),
        "device_errors": errs,
    }
    pool.close()
    return res


# ------------------------------------------------------------------ prefill workload (configs[2], configs[3] per GPU)
FLOP_PER_TOKEN = 10 * 6_291_456 + 6_291_456 + 2 * 2048 * 512 + 4096   # routed + shared + router + shared gate
# kernels of one prefill layer step: router GEMM, shared-gate logits, select, align, row positions, row permute,
# gate_up GEMM, down GEMM, combine (the position reset before the permute is a memset, not a kernel)
PREFILL_LAUNCHES = 9


def bench_prefill(args, world, rank, cpu_passes=None):
    from slotstream_b200 import _lib, synth
    from slotstream_b200.kernels.moe_layer import PrefillLayerBuffers, moe_layer_prefill
    from slotstream_b200.records import BASELINE_LAYOUT as LAY
    E, K, T = 512, 10, args.tokens
    dev = torch.device("cuda")
    rb = LAY.record_bytes
    seed = 2000 + rank
    recs = torch.empty((E + 1, rb), dtype=torch.uint8, device=dev)
    synth.fill_records_device(LAY, recs, seed)
    group_ptr = recs.data_ptr() + torch.arange(E + 1, dtype=torch.int64, device=dev) * rb
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    router_w = (torch.randn(E, LAY.hidden, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    sh_gate_w = (torch.randn(LAY.hidden, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    bias = torch.from_numpy(synth.zipf_bias(E)).to(dev) if args.routing == "zipf" else None
    x = torch.randn(T, LAY.hidden, device=dev, generator=g).to(torch.bfloat16)
    bufs = PrefillLayerBuffers(T, K, LAY.hidden, LAY.inter, E, dev)

    def step():
        moe_layer_prefill(x, router_w, group_ptr, sh_gate_w, K, bufs, bias=bias)

    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    torch.cuda.synchronize()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        flush.zero_()
        graph.replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    times = timed_steps(graph.replay, args.steps, flush, world, clocks)
    clocks.stop()
    ms = max_over_ranks(sum(times) / len(times), world)
    errs = int(bufs.err.item())
    counts = torch.bincount(bufs.ids.reshape(-1).long(), minlength=E)
    n_padded = int(bufs.num_padded.item())

    # dominant launches, timed alone on the aligned rows the step produced (L2 flushed before each)
    st = torch.cuda.current_stream()
    L = _lib.lib()

    def timed(fn, reps=3):
        out = []
        for _ in range(reps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            fn()
            e1.record(st)
            torch.cuda.synchronize()
            out.append(e0.elapsed_time(e1))
        return sum(out) / len(out)

    sr, be, npd = bufs.sorted_rows, bufs.block_expert, bufs.num_padded
    # the two grouped GEMMs exactly as the layer launches them (rows permuted into expert order by the step)
    gu_ms = timed(lambda: _lib.check(L.ssb_sorted_gate_up(
        _lib.ptr(bufs.x_sorted), LAY.hidden, LAY.inter, _lib.ptr(bufs.row_token), bufs.rows, _lib.ptr(sr),
        _lib.ptr(be), _lib.ptr(npd), sr.numel(), _lib.ptr(group_ptr), E + 1, E, _lib.ptr(bufs.h), None,
        _lib.stream()), "gate_up"))
    dn_ms = timed(lambda: _lib.check(L.ssb_sorted_down(
        _lib.ptr(bufs.h), bufs.rows, LAY.hidden, LAY.inter, _lib.ptr(bufs.row_weight), _lib.ptr(sr), _lib.ptr(be),
        _lib.ptr(npd), sr.numel(), _lib.ptr(group_ptr), E + 1, E, _lib.ptr(bufs.out_rows), None, _lib.stream()),
        "down"))
    gu_flop = 2.0 * bufs.rows * 2 * LAY.inter * LAY.hidden
    dn_flop = 2.0 * bufs.rows * LAY.inter * LAY.hidden
    pk = peaks()
    gu_tf = gu_flop / (gu_ms * 1e-3) / 1e12
    roofline = {"bound": "tensor", "kernel": "fused_moe gate_up (k_gate_up_wide: tcgen05 M128xN256 grouped GEMM, "
                                              "256 x (128 gate + 128 up) tiles, SwiGLU epilogue)",
                "achieved": round(gu_tf, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": round(gu_tf / pk["bf16_tflops"], 4), "peak_source": pk["source"] + " (burst)",
                "traffic": TRAFFIC_BYTES.get(f"prefill_gate_up_{T}") if args.routing == "zipf" else None,
                "traffic_source": TRAFFIC_SOURCE,
                "flop_per_launch": gu_flop, "launch_ms": round(gu_ms, 4),
                "padded_rows": n_padded, "rows": bufs.rows,
                "down": {"achieved": round(dn_flop / (dn_ms * 1e-3) / 1e12, 1), "launch_ms": round(dn_ms, 4)}}

    # e2e through the public API with host buffers: x H2D, the layer, y D2H
    x_host = x.cpu().pin_memory()
    y_host = torch.empty((T, LAY.hidden), dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        x.copy_(x_host, non_blocking=True)
        graph.replay()
        y_host.copy_(bufs.y, non_blocking=True)

    for _ in range(2):
        e2e_step()
    e2e_times = timed_steps(e2e_step, args.steps, flush, world)
    e2e_serial_ms = max_over_ranks(sum(e2e_times) / len(e2e_times), world)

    # the same, double-buffered as a serving loop runs it: step i's x H2D and y D2H go on two copy streams, so
    # they overlap the compute of steps i-1 and i+1 (every step still copies its own x in and its y out)
    bufs2 = PrefillLayerBuffers(T, K, LAY.hidden, LAY.inter, E, dev)
    x2 = torch.empty_like(x)
    x2.copy_(x)
    moe_layer_prefill(x2, router_w, group_ptr, sh_gate_w, K, bufs2, bias=bias)
    torch.cuda.synchronize()
    graph2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph2):
        moe_layer_prefill(x2, router_w, group_ptr, sh_gate_w, K, bufs2, bias=bias)
    torch.cuda.synchronize()
    pipe_args = ([x, x2], [graph, graph2], [bufs.y, bufs2.y], [x_host, x.cpu().pin_memory()])
    pipelined_steps(*pipe_args, 4, world)   # warm-up of the two-stream schedule
    e2e_ms = max_over_ranks(pipelined_steps(*pipe_args, args.steps, world), world)
    del graph2, bufs2, x2

    value = world * T / (ms * 1e-3)
    res = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"prefill_layer_{T}tok_per_gpu", "tokens_per_gpu": T, "hidden": LAY.hidden,
                   "inter": LAY.inter, "experts": E, "topk": K, "shared_experts": 1, "routing": f"{args.routing}"
                   + ("_s1.1" if args.routing == "zipf" else ""), "weights": "affine4_gs64 resident in HBM",
                   "cuda_graph": True, "l2": "flushed before every step (256 MiB write); inputs > L2",
                   "parallelism": f"replicas{world}" if world > 1 else "single"},
        "tflops": round(world * T * FLOP_PER_TOKEN / (ms * 1e-3) / 1e12, 1),
        "flop_per_token": FLOP_PER_TOKEN,
        "expert_rows": {"max": int(counts.max()), "zero_experts": int((counts == 0).sum()), "padded": n_padded},
        "roofline": roofline,
        "e2e": {"value": round(world * T / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": int(x.numel() * 2), "d2h_bytes_per_step": int(y_host.numel() * 2),
                "ms_per_step": round(e2e_ms, 4),
                "schedule": "double-buffered: each step's x H2D and y D2H on copy streams beside the neighbouring "
                            "steps' compute",
                "serial": {"value": round(world * T / (e2e_serial_ms * 1e-3), 1), "ms_per_step": round(e2e_serial_ms, 4),
                           "schedule": "H2D, layer, D2H one after the other on one stream"}},
        "gpu_launches": PREFILL_LAUNCHES * args.steps,
        "clocks": clocks.summary(),
        "device_errors": errs,
    }
    if cpu_passes is not None:
        cb, par = cpu_leg_prefill(LAY, recs, router_w, sh_gate_w, bias, x, bufs.y, bufs.ids, cpu_passes)
        res["parity"] = par
        if cb is not None:
            res["cpu_baseline"] = cb
    return res


# ------------------------------------------------------------------ prefill sweep with a partly resident layer
def bench_sweep(args, world, rank):
    """The prefill layer when only part of its 512 records sit in HBM (the prefill MoE sweep): the resident share is
    the hottest experts of the chunk's routing (what a pool filled from the routing frequencies holds), the other
    records are staged per 32-expert group from pinned host memory on a copy stream while earlier groups compute.
    The bound is the slower of the all-resident layer and the staged bytes over the measured pinned H2D bandwidth."""
    from slotstream_b200 import _lib, synth
    from slotstream_b200.kernels.moe_layer import PrefillLayerBuffers, moe_layer_prefill
    from slotstream_b200.records import BASELINE_LAYOUT as LAY
    from slotstream_b200.sweep import PrefillSweep
    E, K, T = 512, 10, args.tokens
    dev = torch.device("cuda")
    rb = LAY.record_bytes
    seed = 2000 + rank
    recs = torch.empty((E + 1, rb), dtype=torch.uint8, device=dev)
    synth.fill_records_device(LAY, recs, seed)
    host = recs.cpu().pin_memory()
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    router_w = (torch.randn(E, LAY.hidden, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    sh_gate_w = (torch.randn(LAY.hidden, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    bias = torch.from_numpy(synth.zipf_bias(E)).to(dev) if args.routing == "zipf" else None
    x = torch.randn(T, LAY.hidden, device=dev, generator=g).to(torch.bfloat16)
    group_ptr = recs.data_ptr() + torch.arange(E + 1, dtype=torch.int64, device=dev) * rb
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    # the all-resident layer: the result the sweep must equal bit for bit, and the compute-side bound (eager, as the
    # sweep runs)
    full = PrefillLayerBuffers(T, K, LAY.hidden, LAY.inter, E, dev)

    def resident_step():
        moe_layer_prefill(x, router_w, group_ptr, sh_gate_w, K, full, bias=bias)

    for _ in range(args.warmup):
        resident_step()
    torch.cuda.synchronize()
    full_ms = max_over_ranks(sum(timed_steps(resident_step, args.steps, flush, world)) / args.steps, world)
    counts = torch.bincount(full.ids.reshape(-1).long(), minlength=E).cpu().numpy()
    n_used = int((counts > 0).sum())               # experts the chunk routes to (Zipf routing leaves many idle)
    n_res = int(round(args.resident_fraction * n_used))
    hottest = np.lexsort((np.arange(E), -counts))[:n_res]
    res_ptr = {int(e): recs.data_ptr() + int(e) * rb for e in hottest}
    shared_ptr = recs.data_ptr() + E * rb
    host_base = host.data_ptr()
    sw = PrefillSweep(LAY.hidden, LAY.inter, K, T, rb)

    def step():
        sw.layer(x, router_w, sh_gate_w, shared_ptr, res_ptr, lambda e: host_base + e * rb, bias=bias)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    bit_equal = bool(torch.equal(sw.bufs.y.view(torch.int16), full.y.view(torch.int16)))
    ids_equal = bool(torch.equal(sw.bufs.ids, full.ids))
    s0 = sw.stats.as_dict()
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    times = timed_steps(step, args.steps, flush, world, clocks)
    clocks.stop()
    ms = max_over_ranks(sum(times) / len(times), world)
    s1 = sw.stats.as_dict()
    per = {key: (s1[key] - s0[key]) / args.steps for key in s1}
    staged_bytes = per["bytes_staged"]
    groups = len(sw.last_plan.groups) + 1

    # the staging link's own bandwidth: one pinned 1 GiB host-to-device copy on this box, timed with events
    probe_h = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    probe_d = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
    probe_d.copy_(probe_h, non_blocking=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    probe_d.copy_(probe_h, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    h2d_gbs = (1 << 30) / (e0.elapsed_time(e1) * 1e-3) / 1e9
    del probe_h, probe_d
    achieved = staged_bytes / (ms * 1e-3) / 1e9
    bound_ms = max(full_ms, staged_bytes / (h2d_gbs * 1e9) * 1e3)

    x_host = x.cpu().pin_memory()
    y_host = torch.empty((T, LAY.hidden), dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        x.copy_(x_host, non_blocking=True)
        step()
        y_host.copy_(sw.bufs.y, non_blocking=True)

    for _ in range(2):
        e2e_step()
    e2e_ms = max_over_ranks(sum(timed_steps(e2e_step, args.steps, flush, world)) / args.steps, world)
    return {
        "metric": METRIC, "value": round(world * T / (ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"prefill_sweep_{T}tok_resident{n_res}of{n_used}used", "tokens_per_gpu": T,
                   "resident_records": n_res, "experts_with_rows": n_used, "staged_per_step": per["records_staged"],
                   "resident_choice": "the hottest experts of the chunk's routing", "routing": args.routing,
                   "group_size": sw.group_size, "staging_groups": sw.staging_groups, "inflight": sw.inflight,
                   "l2": "flushed before every step (256 MiB write); inputs > L2", "cuda_graph": False},
        "all_resident_ms": round(full_ms, 4),
        "bound_ms": round(bound_ms, 4),
        "roofline": {"bound": "h2d" if bound_ms > full_ms else "tensor",
                     "kernel": "staging copies (pinned host -> HBM) overlapped with the grouped GEMMs",
                     "achieved": round(achieved, 1), "peak": round(h2d_gbs, 1), "unit": "GB/s",
                     "frac": round(achieved / h2d_gbs, 4),
                     "peak_source": "measured in this run: one pinned 1 GiB host-to-device copy",
                     "staged_bytes_per_step": int(staged_bytes), "frac_of_bound": round(bound_ms / ms, 4),
                     "traffic": None},
        "parity": {"bit_equal_to_all_resident": bit_equal, "ids_equal": ids_equal},
        "stats_per_step": per,
        "e2e": {"value": round(world * T / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": int(x.numel() * 2 + staged_bytes), "d2h_bytes_per_step": int(y_host.numel() * 2),
                "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": (3 + 1 + 1 + 2 * groups + 1) * args.steps,   # route, align, permute, 2 per group, combine
        "clocks": clocks.summary(),
        "device_errors": int(sw.bufs.err.item()) + int(full.err.item()),
    }


# ------------------------------------------------------------------ expert-parallel prefill (configs[3], N > 1)
def pipelined_eager(x_dev, run, x_host, y_host, k, world):
    """ms per step of k eager steps over two buffer sets, as ``pipelined_steps`` but with ``run(b) -> y`` (a layer
    call that may synchronise the host, like the expert-parallel exchange) instead of a graph replay: step i's x
    H2D goes on a copy stream ahead of its compute and its y D2H on another, overlapping the neighbouring steps.
    ``y_host``: two pinned output buffers allocated by the caller beforehand (a pinned allocation inside the timed
    loop would cost tens of milliseconds and synchronise the device)."""
    comp = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev = lambda: torch.cuda.Event()  # noqa: E731
    ev_in, ev_c, ev_out = [ev() for _ in range(k + 1)], [ev() for _ in range(k)], [ev() for _ in range(k)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    t0.record(comp)
    h2d.wait_event(t0)

    def copy_in(i):
        if i >= 2:
            h2d.wait_event(ev_c[i - 2])          # x_dev[b] is free once step i-2 computed
        with torch.cuda.stream(h2d):
            x_dev[i % 2].copy_(x_host[i % 2], non_blocking=True)
        ev_in[i].record(h2d)

    copy_in(0)
    for i in range(k):
        b = i % 2
        if i + 1 < k:
            copy_in(i + 1)                        # the next step's input crosses while this one computes
        comp.wait_event(ev_in[i])
        y = run(b)
        ev_c[i].record(comp)
        if i >= 2:
            d2h.wait_event(ev_out[i - 2])
        d2h.wait_event(ev_c[i])
        with torch.cuda.stream(d2h):
            y_host[b].copy_(y, non_blocking=True)
            y.record_stream(d2h)
        ev_out[i].record(d2h)
    comp.wait_event(ev_out[k - 1])
    t1.record(comp)
    barrier(world)
    return t0.elapsed_time(t1) / k


def bench_prefill_ep(args, world, rank):
    from slotstream_b200 import synth
    from slotstream_b200.ep import CudaOps, balanced_labels, ep_forward, owned_experts
    from slotstream_b200.kernels.moe_layer import PrefillLayerBuffers, moe_layer_prefill
    from slotstream_b200.records import BASELINE_LAYOUT as LAY
    E, K, T = 512, 10, args.tokens
    dev = torch.device("cuda")
    rb = LAY.record_bytes
    owned = owned_experts(rank, E, world, strided=True)
    # every rank generates the same 513 records (same seed) and owns the strided share of them; the others stay
    # so that each rank can run the one-GPU layer on its own tokens for the parity check below
    recs = torch.empty((E + 1, rb), dtype=torch.uint8, device=dev)
    synth.fill_records_device(LAY, recs, 3000)
    base = recs.data_ptr() + torch.arange(E + 1, dtype=torch.int64, device=dev) * rb
    group_ptr = base[torch.tensor(owned, device=dev)].contiguous()
    g = torch.Generator(device=dev)
    g.manual_seed(2000)                       # router and shared gate replicated: same on every rank
    router_w = (torch.randn(E, LAY.hidden, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    sh_gate_w = (torch.randn(LAY.hidden, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    bias = torch.from_numpy(synth.zipf_bias(E)).to(dev) if args.routing == "zipf" else None
    g.manual_seed(2100 + rank)                # each rank its own tokens
    x = torch.randn(T, LAY.hidden, device=dev, generator=g).to(torch.bfloat16)
    ep_router_w, ep_bias = router_w, bias
    if args.placement == "balanced":
        # expert placement from measured routing counts (summed over the ranks, so every rank derives the same
        # labels): relabel the experts so that the strided placement of the labels evens out the ranks' rows
        logits = x.float() @ router_w.float().t()
        if bias is not None:
            logits += bias
        cnt = torch.bincount(logits.topk(K, dim=1).indices.reshape(-1), minlength=E).to(torch.int64)
        del logits
        if world > 1:
            torch.distributed.all_reduce(cnt)
        label, expert = balanced_labels(cnt.cpu().numpy(), world)
        expert_t = torch.from_numpy(expert).to(dev)
        ep_router_w = router_w[expert_t].contiguous()
        ep_bias = bias[expert_t].contiguous() if bias is not None else None
        group_ptr = base[expert_t[torch.tensor(owned, device=dev)]].contiguous()
    ops = CudaOps(ep_router_w, sh_gate_w, group_ptr, int(base[E]), K, LAY.inter, world, strided=True, bias=ep_bias,
                  sm_reserve=args.sm_reserve)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def measure(partials, phases_out=None):
        def step():
            return ep_forward(ops, x, K, world, micro_batches=args.micro_batches, partials_bf16=partials == "bf16")
        for _ in range(args.warmup):
            flush.zero_()
            step()
        torch.cuda.synchronize()
        clocks = ClockSampler(torch.cuda.current_device())
        clocks.start()
        times = timed_steps(step, args.steps, flush, world, clocks)
        clocks.stop()
        ms = max_over_ranks(sum(times) / len(times), world)
        # one more step, instrumented: phase times (max over ranks) and this rank's received rows
        ph = []
        barrier(world)
        flush.zero_()
        y = ep_forward(ops, x, K, world, micro_batches=args.micro_batches, partials_bf16=partials == "bf16",
                       phases=ph)
        torch.cuda.synchronize()
        evs = [(n, e) for n, *e in ph if n != "rows"]
        rows = [r for r in ph if r[0] == "rows"][0]
        phase_ms = {}
        for (n0, e0), (n1, e1) in zip(evs, evs[1:]):
            phase_ms[n1] = max_over_ranks(e0[0].elapsed_time(e1[0]), world)
        step_ms = max_over_ranks(evs[0][1][0].elapsed_time(evs[-1][1][0]), world)
        load = torch.tensor([rows[1], rows[2]], dtype=torch.float64, device=dev)
        if world > 1:
            allv = [torch.empty_like(load) for _ in range(world)]
            torch.distributed.all_gather(allv, load)
        else:
            allv = [load]
        recv_rows = [int(v[0].item()) for v in allv]
        recv_ent = [int(v[1].item()) for v in allv]
        return ms, y.clone(), clocks.summary(), {
            "ms": {k: round(v, 4) for k, v in phase_ms.items()}, "instrumented_step_ms": round(step_ms, 4),
            "received_rows_per_rank": {"min": min(recv_rows), "max": max(recv_rows)},
            "received_entries_per_rank": {"min": min(recv_ent), "max": max(recv_ent), "mean": sum(recv_ent) / world},
            "note": "CUDA events on the launching stream at the phase borders of one extra step, max over ranks; "
                    "the shared expert runs on a side stream inside these phases"}

    def parity_vs_one_gpu(y_ep):
        """This rank's tokens through the one-GPU layer (all 513 records on this rank): the EP output must match it
        within the layer tolerance (fp32 partial sums differ from the one-GPU rank-order sum by reassociation)."""
        bufs = PrefillLayerBuffers(T, K, LAY.hidden, LAY.inter, E, dev)
        y1 = moe_layer_prefill(x, router_w, base, sh_gate_w, K, bufs, bias=bias)
        torch.cuda.synchronize()
        d = (y_ep.double() - y1.double())
        stats = torch.tensor([float(d.norm() / y1.double().norm()), float(d.abs().max()),
                              float((y_ep.view(torch.int16) != y1.view(torch.int16)).double().mean())],
                             dtype=torch.float64, device=dev)
        if world > 1:
            torch.distributed.all_reduce(stats, op=torch.distributed.ReduceOp.MAX)
        del bufs
        return {"rel_l2": round(float(stats[0]), 7), "max_abs": round(float(stats[1]), 5),
                "bf16_outputs_differing_frac": round(float(stats[2]), 6),
                "reference": "the one-GPU layer (moe_layer_prefill, all records resident) on each rank's own tokens; "
                             "max over ranks", "bar": "rel_l2 <= 1e-2"}

    ms, y_ep, clocks, phases = measure(args.partials)
    value = world * T / (ms * 1e-3)
    errs = int(ops.err.item())
    parity = parity_vs_one_gpu(y_ep)
    alt = None
    if not args.no_partials_alt:
        other = "bf16" if args.partials == "fp32" else "fp32"
        ms2, y2, clocks2, phases2 = measure(other)
        alt = {"partials": other, "value": round(world * T / (ms2 * 1e-3), 1), "ms_per_step": round(ms2, 4),
               "phases": phases2, "parity": parity_vs_one_gpu(y2), "clocks": clocks2}

    # e2e: this rank's tokens from pinned host memory, the layer, y back to the host, double-buffered like N=1
    x2 = x.clone()
    x_host = [x.cpu().pin_memory(), x2.cpu().pin_memory()]

    def run(b):
        return ep_forward(ops, (x, x2)[b], K, world, micro_batches=args.micro_batches,
                          partials_bf16=args.partials == "bf16")

    y_host = [torch.empty((T, LAY.hidden), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    pipelined_eager([x, x2], run, x_host, y_host, 2, world)   # warm-up of the two-stream schedule
    e2e_ms = max_over_ranks(pipelined_eager([x, x2], run, x_host, y_host, args.steps, world), world)
    pk = peaks()
    tf = T * FLOP_PER_TOKEN / (ms * 1e-3) / 1e12      # per GPU: each rank's share of the layer's FLOPs
    roofline = {"bound": "tensor", "kernel": "whole expert-parallel layer step per GPU (FLOPs of its tokens)",
                "achieved": round(tf, 1), "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s",
                "frac": round(tf / pk["bf16_tflops_sustained"], 4), "peak_source": pk["source"] + " (sustained)",
                "traffic": None}
    # route (router GEMM, shared-gate logits, select) 3 + shared expert (align + 4) 5 + per part: plan, gather,
    # unpack, experts (align + 4), partial sums, combine = 10
    launches = 8 + 10 * args.micro_batches
    res = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"ep_prefill_layer_{T}tok_per_gpu", "tokens_per_gpu": T, "hidden": LAY.hidden,
                   "inter": LAY.inter, "experts": E, "experts_per_gpu": len(owned),
                   "placement": ("balanced: experts relabelled from this chunk's routing counts, strided over the "
                                 "labels" if args.placement == "balanced" else "strided (e % G)"),
                   "topk": K, "shared_experts": 1, "routing": "zipf_s1.1" if args.routing == "zipf" else "uniform",
                   "exchange": f"NCCL all-to-all-v (dispatch rows + metadata, {args.partials} partial sums back)",
                   "partials": args.partials, "micro_batches": args.micro_batches, "gemm_sm_reserve": args.sm_reserve,
                   "l2": "flushed before every step (256 MiB write); inputs > L2", "parallelism": f"ep{world}"},
        "tflops_per_gpu": round(tf, 1), "roofline": roofline, "phases": phases, "parity": parity,
        "e2e": {"value": round(world * T / (e2e_ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": world * T * LAY.hidden * 2, "d2h_bytes_per_step": world * T * LAY.hidden * 2,
                "schedule": "double-buffered on every rank: each step's x H2D and y D2H on copy streams beside the "
                            "neighbouring steps' compute (bytes summed over the ranks)"},
        "gpu_launches": launches * args.steps, "clocks": clocks, "device_errors": errs,
    }
    if alt is not None:
        res["partials_alt"] = alt
    return res


# ------------------------------------------------------------------ main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", choices=["prefill", "decode", "slotpool", "sweep"], default="prefill")
    ap.add_argument("--pool-fraction", type=float, default=0.7,
                    help="slotpool: share of the layers x 512 records the HBM pool holds")
    ap.add_argument("--no-slotpool", action="store_true", help="skip the slot-pool sub-measurement at N=1")
    ap.add_argument("--resident-fraction", type=float, default=0.5,
                    help="sweep: share of the experts the chunk routes to whose records are resident in HBM (the "
                         "hottest; the rest are staged from pinned host memory)")
    ap.add_argument("--no-sweep", action="store_true", help="skip the partly resident sweep sub-measurement at N=1")
    ap.add_argument("--tokens", type=int, default=32768, help="prefill tokens per GPU")
    ap.add_argument("--routing", choices=["zipf", "uniform"], default="zipf")
    ap.add_argument("--batch", type=int, default=1, help="decode batch")
    ap.add_argument("--layers", type=int, default=48, help="decode layers per step (48 = configs[1])")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode sub-measurement at N=1")
    ap.add_argument("--decode-prefetch", action="store_true",
                    help="decode: side-stream L2 prefetch of the next layer's router weight and shared record "
                         "(measured slower; off by default)")
    ap.add_argument("--no-chunks", action="store_true", help="skip the 2K / 8K-token prefill sub-measurements")
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="decode CPU baseline sample length")
    ap.add_argument("--cpu-passes", type=int, default=2, help="prefill CPU baseline: timed passes over the chunk")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU leg (baseline and parity)")
    ap.add_argument("--replicas", action="store_true", help="N > 1: independent one-GPU layers instead of EP")
    ap.add_argument("--placement", choices=["balanced", "strided"], default="strided",
                    help="N > 1: expert placement (strided by id, or balanced from measured routing counts)")
    ap.add_argument("--micro-batches", type=int, default=1,
                    help="N > 1: token parts whose exchanges overlap the expert GEMMs of their neighbours")
    ap.add_argument("--partials", choices=["fp32", "bf16"], default="fp32",
                    help="N > 1: precision of the per-(token, destination) partial sums sent back (the line also "
                         "reports the other precision as a sub-measurement unless --no-partials-alt)")
    ap.add_argument("--no-partials-alt", action="store_true")
    ap.add_argument("--sm-reserve", type=int, default=0,
                    help="N > 1 with micro-batches: SMs the persistent GEMMs leave to the overlapped all-to-alls")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        # the reference's path is CPU-only: rank 0 alone runs it, other ranks exit without work
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps(reference_arm(args, int(os.environ.get("WORLD_SIZE", "1")))), flush=True)
        return
    world, rank, _ = dist_setup()
    cpu = rank == 0 and world == 1 and not args.no_cpu_baseline
    if args.workload == "decode":
        res = bench_decode(args, world, rank, cpu_seconds=args.cpu_seconds if cpu else None)
    elif args.workload == "slotpool":
        res = bench_slotpool(args, world, rank)
    elif args.workload == "sweep":
        res = bench_sweep(args, world, rank)
    elif world > 1 and not args.replicas:
        res = bench_prefill_ep(args, world, rank)
    else:
        res = bench_prefill(args, world, rank, cpu_passes=args.cpu_passes if cpu else None)
        torch.cuda.empty_cache()
        if world == 1 and not args.no_chunks:
            # configs[2] also names 2,048- and 8,192-token chunks: the same layer, measured the same way
            res["chunks"] = {}
            for tk in (2048, 8192, 32768):
                if tk == args.tokens:
                    continue
                a2 = argparse.Namespace(**vars(args))
                a2.tokens = tk
                c = bench_prefill(a2, world, rank, cpu_passes=0 if cpu else None)
                res["chunks"][str(tk)] = {k: c[k] for k in ("value", "unit", "ms_per_step", "tflops", "roofline",
                                                            "e2e", "clocks", "device_errors", "parity") if k in c}
                torch.cuda.empty_cache()
        if world == 1 and not args.no_decode:
            W = decode_world(args, rank)
            d = bench_decode(args, world, rank, 1, W, cpu_seconds=args.cpu_seconds if cpu else None)
            res["decode"] = {k: d[k] for k in ("value", "unit", "ms_per_step", "config", "hbm_gbs_per_step",
                                               "bytes_per_step", "roofline", "e2e", "clocks", "parity",
                                               "cpu_baseline") if k in d}
            # configs[1] also names batch 2 (speculative verify) and 16: same records, same step
            res["decode"]["other_batches"] = {}
            for bb in (2, 16):
                e = bench_decode(args, world, rank, bb, W, cpu_seconds=0 if cpu else None)
                res["decode"]["other_batches"][str(bb)] = {
                    "value": e["value"], "unit": e["unit"], "ms_per_step": e["ms_per_step"],
                    "hbm_gbs_per_step": e["hbm_gbs_per_step"], "bytes_per_step": e["bytes_per_step"],
                    "roofline_frac": e["roofline"]["frac"], "kernel": e["roofline"]["kernel"],
                    "parity": e.get("parity")}
            del W
            torch.cuda.empty_cache()
        if world == 1 and not args.no_slotpool:
            s = bench_slotpool(args, world, rank)
            res["slotpool"] = {k: s[k] for k in ("metric", "value", "unit", "tokens_per_s", "ms_per_step", "config",
                                                 "miss_fraction", "misses_per_layer", "h2d_bytes_per_step",
                                                 "roofline", "e2e", "gpu_launches", "clocks", "device_errors")}
            torch.cuda.empty_cache()
        if world == 1 and not args.no_sweep:
            s = bench_sweep(args, world, rank)
            res["sweep"] = {k: s[k] for k in ("value", "unit", "ms_per_step", "config", "all_resident_ms", "bound_ms",
                                              "roofline", "parity", "e2e", "gpu_launches", "clocks", "device_errors")}
            torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def reference_arm(args, world):
    """The reference's own CPU path for this workload (oracle/cpu_baseline.py, the torch restatement of moe_ref /
    affine_ref / stable top-k) on all host cores, on the GPU arm's config: prefill steps are whole chunks of
    args.tokens tokens (each routed expert dequantised once per chunk, as the GPU arm's layer reads each record once);
    decode steps are one token through 48 layers (dequantisation inside, as the reference's CPU branch)."""
    sys.path.insert(0, str(ROOT))
    from oracle.cpu_baseline import CpuLayer, decode_token_layer, host_info, prefill_chunk
    from slotstream_b200.records import BASELINE_LAYOUT as LAY
    threads = os.cpu_count()
    torch.set_num_threads(threads)
    layer = CpuLayer.from_seed(LAY, 0)
    if args.routing == "uniform":
        layer.bias = None
    g = torch.Generator().manual_seed(0)
    times = []
    with torch.no_grad():
        if args.workload == "decode":
            b = args.batch
            xs = torch.randn(args.steps + 1, b, LAY.hidden, generator=g).bfloat16().float()

            def step(i):
                for _ in range(args.layers):
                    for t in range(b):
                        decode_token_layer(layer, xs[i, t:t + 1])
            config = {"workload": f"decode_step_{args.layers}layer_b{b}", "layers": args.layers, "batch": b,
                      "hidden": LAY.hidden, "inter": LAY.inter, "experts": 512, "topk": 10, "routing": "zipf_s1.1"}
            units, dtype, sample = b, "f32", f"{args.layers} layers x {b} token(s) per step, dequantisation inside"
        else:
            x = torch.randn(args.tokens, LAY.hidden, generator=g).bfloat16().float()

            def step(i):
                prefill_chunk(layer, x)
            wl = (f"ep_prefill_layer_{args.tokens}tok_per_gpu" if world > 1 and not args.replicas
                  else f"prefill_layer_{args.tokens}tok_per_gpu")
            config = {"workload": wl, "tokens_per_gpu": args.tokens, "hidden": LAY.hidden, "inter": LAY.inter,
                      "experts": 512, "topk": 10, "shared_experts": 1,
                      "routing": args.routing + ("_s1.1" if args.routing == "zipf" else "")}
            units, dtype = args.tokens, "f32"
            sample = f"whole {args.tokens}-token chunks, each routed expert dequantised once per chunk"
        for i in range(min(args.warmup, 1)):
            step(i)
        for i in range(args.steps):
            t0 = time.perf_counter()
            step(i)
            times.append(time.perf_counter() - t0)
    ms = 1e3 * sum(times) / len(times)
    v = units / (ms * 1e-3)
    cb = {"value": v, "unit": "tokens/s", "kind": "port", "sample": sample, "steps_timed": len(times)}
    cb.update(host_info(threads))
    return {"metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
            "warmup": min(args.warmup, 1), "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": dtype, "data": "synthetic", "impl": "reference", "config": config,
            "cpu_baseline": cb, "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}}


if __name__ == "__main__":
    main()
