"""Benchmark of the B200 paged-decode attention (BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --vllm-e2e [--eager]

Workload (N = 1): BASELINE config 2 -- Qwen2.5-3B decode attention, B=8,
16 query / 2 KV heads, head_dim 128, block_size 32, context 2048, bf16, KV
pool 2x the needed blocks with scattered block tables.  A step is one
decode-attention call over the batch (one kernel launch).  Inputs rotate over
12 independent KV pools (403 MB > 3x the 126 MB L2) so HBM, not L2, is
measured.  The timed K steps run as CUDA-graph replays of the public API's
launch; time is taken with CUDA events on the launching stream.

With N > 1 (torchrun, one rank per GPU) every rank runs the same per-GPU
workload on its own requests (requests are independent: no data-path
collective), ``scaling`` is "weak" and ``value`` is the whole-job tokens/s
(N * B * K / max-over-ranks time).  The nested ``ragged`` object reports
BASELINE config 4 (B=64 Llama-3-8B shape, log-uniform lengths up to 131072)
sharded across the N ranks by length-balanced (LPT) request sharding.

``--impl reference`` times the reference's own CPU path of the algorithm
(flashdec/paged_reference.py's paged_decode_attention_ref, imported from the
reference installed under baseline/_ref; the numpy oracle restating it when
that install is absent) on the same workload, on all host cores, on rank 0
only.

``--vllm-e2e`` (opt-in, a few minutes, one GPU) times vLLM's own
``LLM.generate`` on the Qwen2.5-3B architecture with dummy weights, once with
vLLM's TRITON_ATTN backend and once with this package's CUSTOM backend, and
prints their decode step times and greedy-token agreement as one JSON line.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = ("paged decode attn p50 µs & HBM GB/s (% of peak), B8 ctx2048; "
          "tok/s at 1–8 GPUs")
C2 = dict(batch=8, hq=16, hkv=2, d=128, bs=32, ctx=2048, pool_factor=2)
NUM_POOLS = 12
E2E_STEPS = 2400  # end-to-end steps timed (a multiple of NUM_POOLS and of the four streams)


def _peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _traffic_from_profile(name):
    """Per-launch DRAM bytes recorded by an ncu capture (profiles/<name>.txt)."""
    p = REPO / "profiles" / f"{name}.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------
def build_c2_pools(torch, device, seed):
    cfg = C2
    b, hkv, d, bs = cfg["batch"], cfg["hkv"], cfg["d"], cfg["bs"]
    nblk = cfg["ctx"] // bs
    pool = cfg["pool_factor"] * b * nblk
    g = torch.Generator(device=device).manual_seed(seed)
    pools = []
    for _ in range(NUM_POOLS):
        k = torch.randn((pool, hkv, bs, d), device=device, dtype=torch.bfloat16, generator=g)
        v = torch.randn((pool, hkv, bs, d), device=device, dtype=torch.bfloat16, generator=g)
        perm = torch.randperm(pool, device=device, generator=g)[: b * nblk]
        bt = perm.reshape(b, nblk).to(torch.int32).contiguous()
        q = torch.randn((b, cfg["hq"], d), device=device, dtype=torch.bfloat16, generator=g)
        pools.append(dict(q=q, k=k, v=v, bt=bt))
    sl = torch.full((b,), cfg["ctx"], device=device, dtype=torch.int32)
    return pools, sl


def c2_bytes():
    from oracle.paged_attention import attention_bytes

    return attention_bytes([C2["ctx"]] * C2["batch"], C2["hq"], C2["hkv"], C2["d"], C2["bs"])


def ragged_requests(seed=4, batch=64):
    from tests.golden.cases import c4_lengths

    return c4_lengths(seed, batch)


# ---------------------------------------------------------------------------
# our implementation
# ---------------------------------------------------------------------------
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import flashdec_b200
    from flashdec_b200.sharding import lpt_partition
    from oracle.paged_attention import attention_bytes

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    # clocks are sampled over the whole run (warm-up, timed region and every
    # leg), so the record always has samples
    clocks = ClockSampler(torch.cuda.current_device()).__enter__()
    try:
        return _run_ours(args, rank, world, torch, dist, device, clocks)
    finally:
        clocks.__exit__(None, None, None)


def _run_ours(args, rank, world, torch, dist, device, clocks):
    import flashdec_b200

    pools, sl = build_c2_pools(torch, device, seed=1234 + rank)
    outs = [torch.empty_like(p["q"]) for p in pools]
    stream = torch.cuda.Stream(device)

    def step(i):
        p = pools[i % NUM_POOLS]
        flashdec_b200.paged_decode_attention_into(p["q"], p["k"], p["v"], p["bt"], sl,
                                                  outs[i % NUM_POOLS])

    # warm-up (also sizes the workspace and builds tensor maps)
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            step(i)
    stream.synchronize()

    # graph of G steps (rotating pools), replayed to cover exactly K steps
    G = min(args.steps, 1200)
    G -= G % NUM_POOLS if G >= NUM_POOLS else 0
    G = max(G, 1)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(G):
            step(i)
    reps, rem = divmod(args.steps, G)
    graph_rem = None
    if rem:
        graph_rem = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_rem, stream=stream):
            for i in range(rem):
                step(i)
    for _ in range(2):
        graph.replay()
    stream.synchronize()

    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        # the GPU is kept busy while the host enqueues the replays, so the
        # events time device work only
        torch.cuda._sleep(200000)
        start.record(stream)
        for _ in range(reps):
            graph.replay()
        if graph_rem is not None:
            graph_rem.replay()
        end.record(stream)
    stream.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    elapsed_ms = start.elapsed_time(end)
    t = torch.tensor([elapsed_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    ms_per_step = max_ms / args.steps

    # p50 of single launches (one-step graphs, GPU kept busy so host enqueue
    # time is not inside the events)
    single = []
    for i in range(NUM_POOLS):
        gi = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gi, stream=stream):
            step(i)
        single.append(gi)
    lat = []
    with torch.cuda.stream(stream):
        for r in range(240):
            torch.cuda._sleep(20000)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            single[r % NUM_POOLS].replay()
            e1.record(stream)
            lat.append((e0, e1))
    stream.synchronize()
    lat_us = sorted(a.elapsed_time(b) * 1000.0 for a, b in lat[40:])
    p50_us = lat_us[len(lat_us) // 2]

    # end to end through the public API: each step's q, block tables and
    # seq_lens sit in one pinned host arena (the way a serving host stages a
    # step's inputs) and cross in one H2D copy; paged_decode_attention_into
    # writes a preallocated output, which is read back by one D2H copy.
    # Consecutive steps rotate over four streams with their own device
    # buffers, so one step's copies overlap the other steps' kernels (a
    # step's H2D -> decode -> D2H chain is latency-bound at about 25 us on its
    # own); a step's three operations stay in order on its stream, and each
    # stream has its own decode workspace.  The step count does not depend on
    # --steps (E2E_STEPS), so start-up does not dominate; every step's output
    # lands in its own pinned buffer and all of them are checked afterwards.
    e2e = None
    if not args.kernel_only:
        e2e_steps = E2E_STEPS

        def seg(nbytes):
            return (nbytes + 255) // 256 * 256

        q_nb = pools[0]["q"].numel() * pools[0]["q"].element_size()
        bt_nb = pools[0]["bt"].numel() * pools[0]["bt"].element_size()
        sl_nb = sl.numel() * sl.element_size()
        arena_nb = seg(q_nb) + seg(bt_nb) + seg(sl_nb)

        def views(arena):
            o_bt, o_sl = seg(q_nb), seg(q_nb) + seg(bt_nb)
            return (arena[:q_nb].view(pools[0]["q"].dtype).view(pools[0]["q"].shape),
                    arena[o_bt:o_bt + bt_nb].view(pools[0]["bt"].dtype)
                    .view(pools[0]["bt"].shape),
                    arena[o_sl:o_sl + sl_nb].view(sl.dtype).view(sl.shape))

        harena = []
        for p in pools:
            h = torch.zeros(arena_nb, dtype=torch.uint8).pin_memory()
            hq_v, hbt_v, hsl_v = views(h)
            hq_v.copy_(p["q"].cpu())
            hbt_v.copy_(p["bt"].cpu())
            hsl_v.copy_(sl.cpu())
            harena.append(h)
        nbuf = 4
        e2e_streams = [torch.cuda.Stream(device) for _ in range(nbuf)]
        darenas = [torch.empty(arena_nb, dtype=torch.uint8, device=device) for _ in range(nbuf)]
        dviews = [views(x) for x in darenas]
        douts = [torch.empty_like(pools[0]["q"]) for _ in range(nbuf)]
        hout = torch.empty((e2e_steps,) + tuple(pools[0]["q"].shape),
                           dtype=pools[0]["q"].dtype).pin_memory()

        # per-step operands resolved before the timed loop (plain list reads
        # inside it)
        hout_rows = list(hout.unbind(0))
        kv = [(p["k"], p["v"]) for p in pools]
        decode_into = flashdec_b200.paged_decode_attention_into
        copy_async = flashdec_b200.copy_async  # one cudaMemcpyAsync per call, from C++
        set_stream = torch.cuda.set_stream

        # Steps are staged ahead: step i's stream and buffers are i mod nbuf,
        # and right after step i's D2H the same stream takes the H2D of step
        # i + nbuf (which reuses step i's buffers, in order on that stream).
        # So every step's inputs are in flight nbuf - 1 steps before its
        # kernel, and each step switches streams once.  (Issued in step order,
        # a D2H that waits for its kernel holds the next step's H2D behind it
        # in the copy queue and the steps run one after another: 15.7-18.3 us
        # per step against 12.9 us staged.)

        def e2e_run(n):
            for i in range(min(nbuf, n)):
                set_stream(e2e_streams[i])
                copy_async(darenas[i], harena[i % NUM_POOLS])
            for i in range(n):
                bb = i % nbuf
                set_stream(e2e_streams[bb])
                dq, dbt, dsl = dviews[bb]
                k, v = kv[i % NUM_POOLS]
                decode_into(dq, k, v, dbt, dsl, douts[bb])
                copy_async(hout_rows[i % e2e_steps], douts[bb])
                if i + nbuf < n:
                    copy_async(darenas[bb], harena[(i + nbuf) % NUM_POOLS])

        # Warm-up of 2 x E2E_STEPS untimed steps: a fresh process's first few
        # thousand steps of this loop run 15-17 us per step before settling at
        # about 13 (three consecutive 2400-step runs: 17.4, 15.7, 12.9 us), and
        # a serving loop lives in the settled state.
        with torch.cuda.stream(stream):
            e2e_run(2 * e2e_steps)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        with torch.cuda.stream(stream):
            e2e_run(e2e_steps)
        torch.cuda.synchronize()  # every step stream
        wall = time.perf_counter() - t0
        # every step's host output equals a device-resident decode of its pool
        expect = torch.stack([flashdec_b200.decode(pools[j]["q"], pools[j]["k"], pools[j]["v"],
                                                   pools[j]["bt"], sl).cpu()
                              for j in range(NUM_POOLS)])
        idx = torch.arange(e2e_steps) % NUM_POOLS
        if not torch.equal(hout, expect[idx]):
            bad = int((hout != expect[idx]).flatten(1).any(1).sum())
            raise RuntimeError(f"e2e: {bad} of {e2e_steps} steps differ from the device-resident "
                               "decode of their inputs")
        te = torch.tensor([wall * 1000.0], device=device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = float(te.item())
        e2e = {
            "value": world * C2["batch"] * e2e_steps / (e2e_ms / 1000.0),
            "unit": "tokens/s",
            "h2d_bytes_per_step": int(arena_nb),
            "d2h_bytes_per_step": int(douts[0].numel() * douts[0].element_size()),
            "steps": e2e_steps,
            "warmup_steps": 2 * e2e_steps,
            "us_per_step": e2e_ms * 1000.0 / e2e_steps,
            "api": "flashdec_b200.paged_decode_attention_into; q, block tables and seq_lens in one "
                   "pinned host arena, one H2D and one D2H copy per step (flashdec_b200.copy_async: "
                   "one cudaMemcpyAsync each); steps rotate over "
                   "four streams with their own device buffers and workspaces, each step's "
                   "inputs copied in three steps ahead of its kernel (after the D2H of the "
                   "step four back, on the same stream)",
            "check": f"all {e2e_steps} host outputs equal the device-resident decode of their inputs",
            "timing": "wall clock between device-wide synchronisations",
        }

    # ragged long-context batch, LPT-sharded over ranks
    ragged = None if args.kernel_only else run_ragged(torch, dist, device, rank, world, stream, args)
    extra = {}
    if world == 1 and not args.kernel_only:
        extra["c2_ctx1024"] = run_c2_ctx1024(torch, device, stream, args)
        extra["c3_rope_append"] = run_c3(torch, device, stream)
        extra["vllm_launcher"] = run_vllm_launcher(torch, device, stream)
        extra["c5_engine_step"] = run_c5(torch, device, args)
        extra["c5_layer_decode"] = run_c5_layer(torch, device, stream)
        # BASELINE config 1 is a CPU config (fp32, which the GPU path does not
        # take): the reference CPU path timed on it beside c2
        c1 = cpu_baseline_sample(args, seconds=float(os.environ.get("FD_C1_SECONDS", "3")),
                                 workload="c1")
        c1["workload"] = ("BASELINE c1: B4, 16q/2kv, D128, bs32, fp32, seq U[64,512], 128-block "
                          "permuted pool (CPU only)")
        extra["c1_cpu"] = c1

    if world > 1:
        dist.barrier()
    if rank != 0:
        return None
    nbytes = c2_bytes()
    peak, peak_kind = _peaks()
    achieved = nbytes / (ms_per_step / 1000.0) / 1e9
    # the CPU baseline is a rank-0, one-GPU figure: at N > 1 the GPUs are not
    # held for it
    cpu = None if (args.kernel_only or world > 1) else cpu_baseline_sample(args)
    return {
        "metric": METRIC,
        "value": world * C2["batch"] * args.steps / (max_ms / 1000.0),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "p50_us": p50_us,
        "hbm_gbs": achieved,
        "pct_of_peak": 100.0 * achieved / peak,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) q/k/v, scattered block tables)",
        "config": c2_config(world),
        "timing": "CUDA-graph replay of the public API launch, CUDA events on the launching "
                  "stream, max over ranks",
        "roofline": {
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "peak_kind": peak_kind,
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": _traffic_from_profile("wave_decode_c2_ctx2048"),
            "algorithmic_bytes_per_launch": nbytes,
            "kernel": "fd::wave_decode_kernel<bf16,128,0,1,cluster,plain>",
        },
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": args.steps,
        "ragged": ragged,
        **extra,
        "clocks": clocks.summary(),
    }


def run_ragged(torch, dist, device, rank, world, stream, args, batch=64):
    """B=64 Llama-3-8B attention shape (32q/8kv, D128,
    bs16) with log-uniform lengths in [512, 131072], LPT-sharded."""
    import flashdec_b200
    from flashdec_b200.sharding import lpt_partition
    from oracle.paged_attention import attention_bytes

    lens = ragged_requests(batch=batch)
    shards = lpt_partition(lens, world)
    mine = [lens[i] for i in shards[rank]]
    hq, hkv, d, bs = 32, 8, 128, 16
    nblk = [-(-n // bs) for n in mine]
    total = sum(nblk)
    g = torch.Generator(device=device).manual_seed(99 + rank)
    k = torch.randn((total + 1, hkv, bs, d), device=device, dtype=torch.bfloat16, generator=g)
    v = torch.randn_like(k)
    perm = torch.randperm(total + 1, device=device, generator=g)
    bt = torch.full((len(mine), max(nblk)), -1, device=device, dtype=torch.int32)
    pos = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[pos:pos + n].to(torch.int32)
        pos += n
    sl = torch.tensor(mine, device=device, dtype=torch.int32)
    q = torch.randn((len(mine), hq, d), device=device, dtype=torch.bfloat16, generator=g)
    out = torch.empty_like(q)
    with torch.cuda.stream(stream):
        for _ in range(3):
            flashdec_b200.paged_decode_attention_into(q, k, v, bt, sl, out)
    stream.synchronize()
    steps = max(5, min(args.steps // 200, 50))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        flashdec_b200.paged_decode_attention_into(q, k, v, bt, sl, out)
    graph.replay()
    stream.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
    stream.synchronize()
    ms = e0.elapsed_time(e1) / steps
    local_bytes = attention_bytes(mine, hq, hkv, d, bs)
    # per-rank time, requests and bytes (every rank's numbers, not rank 0's)
    mine_t = torch.tensor([ms, len(mine), local_bytes], device=device, dtype=torch.float64)
    if world > 1:
        every = torch.empty((world, 3), device=device, dtype=torch.float64)
        dist.all_gather_into_tensor(every, mine_t)
    else:
        every = mine_t.view(1, 3)
    every = every.cpu().tolist()
    rank_ms = [r[0] for r in every]
    max_ms = max(rank_ms)
    peak, _ = _peaks()
    rank_gbs = [r[2] / (r[0] / 1000.0) / 1e9 for r in every]
    res = {
        "workload": "BASELINE c4: B64 Llama-3-8B attention (32q/8kv, D128, bs16), seq log-uniform [512,131072]",
        "tokens_per_step": len(lens),
        "ms_per_step_max_rank": max_ms,
        "ms_per_step_mean_rank": sum(rank_ms) / world,
        "max_over_mean": max_ms / (sum(rank_ms) / world),
        "tokens_per_s": len(lens) / (max_ms / 1000.0),
        "rank_ms": rank_ms,
        "rank_requests": [int(r[1]) for r in every],
        "rank_hbm_gbs": rank_gbs,
        "rank_frac_of_peak": [g / peak for g in rank_gbs],
        "steps": steps,
        "scaling": "strong (fixed 64-request batch split across ranks, LPT by length)",
    }
    if world > 1:
        res["gather"] = _timed_gather(torch, dist, device, stream, out, shards, rank, world)
    return res


def _timed_gather(torch, dist, device, stream, out, shards, rank, world, reps=20):
    """NCCL all-gather of the ranks' [B_r, Hq, D] outputs to the global batch
    (flashdec_b200.sharding.gather_outputs), timed with CUDA events (max over
    ranks) and checked once: rank 0 compares an fp64 checksum of every
    shard's rows in the gathered batch with the checksum its owner computed
    locally."""
    from flashdec_b200.sharding import gather_outputs

    with torch.cuda.stream(stream):
        for _ in range(3):
            glob = gather_outputs(out, shards, rank)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            glob = gather_outputs(out, shards, rank)
        e1.record(stream)
    stream.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) * 1000.0 / reps], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    local = out.double().sum().view(1)
    sums = torch.empty(world, device=device, dtype=torch.float64)
    dist.all_gather_into_tensor(sums, local)
    ok = True
    if rank == 0:
        for r, idx in enumerate(shards):
            got = glob[torch.as_tensor(idx, device=device)].double().sum()
            ok = ok and bool(got == sums[r])
    flag = torch.tensor([0 if ok else 1], device=device, dtype=torch.int32)
    dist.all_reduce(flag, op=dist.ReduceOp.MAX)
    if int(flag.item()):
        raise RuntimeError("gathered outputs differ from the ranks' local outputs")
    rows = max(len(s) for s in shards)
    return {"us_max_rank": float(t.item()),
            "bytes_per_rank": rows * out.shape[1] * out.shape[2] * out.element_size(),
            "collective": "all_gather_into_tensor (NCCL), padded to the largest shard",
            "check": "fp64 checksum of every shard's gathered rows equals its owner's"}


def _graph_time_us(torch, stream, fn, reps, inner=1):
    """Mean device time of `fn` replayed as a CUDA graph of `inner` calls."""
    with torch.cuda.stream(stream):
        for _ in range(3):
            fn()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for _ in range(inner):
            fn()
    g.replay()
    stream.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        # the GPU is kept busy while the host enqueues the replays (as for the
        # c2 line), so the events time device work only
        torch.cuda._sleep(200000)
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
    stream.synchronize()
    return e0.elapsed_time(e1) * 1000.0 / (reps * inner)


def run_c2_ctx1024(torch, device, stream, args):
    """BASELINE config 2 at context 1024 (same shapes, 12 rotating pools)."""
    import flashdec_b200
    from oracle.paged_attention import attention_bytes

    saved = dict(C2)
    C2["ctx"] = 1024
    try:
        pools, sl = build_c2_pools(torch, device, seed=77)
    finally:
        C2.clear()
        C2.update(saved)
    outs = [torch.empty_like(p["q"]) for p in pools]
    state = {"i": 0}

    def step():
        i = state["i"] % NUM_POOLS
        state["i"] += 1
        p = pools[i]
        flashdec_b200.paged_decode_attention_into(p["q"], p["k"], p["v"], p["bt"], sl, outs[i])

    us = _graph_time_us(torch, stream, step, reps=max(10, min(args.steps // 120, 500)),
                        inner=NUM_POOLS * 10)
    nbytes = attention_bytes([1024] * C2["batch"], C2["hq"], C2["hkv"], C2["d"], C2["bs"])
    peak, _ = _peaks()
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"workload": "BASELINE c2 at context 1024 (B8, 16q/2kv, D128, bs32, bf16)",
            "us_per_step": us, "tokens_per_s": C2["batch"] / (us * 1e-6),
            "algorithmic_bytes": nbytes, "hbm_gbs": gbs, "frac_of_peak": gbs / peak}


def run_vllm_launcher(torch, device, stream, reps=200):
    """The reference's own headline configuration (its only published
    B8/ctx2048 number, benchmarks/results/vllm_qwen_attention_summary.md:24):
    the vLLM decode launcher (flashdec/kernels/paged_decode.py:728-919) at B8,
    context 2048, Qwen2.5-3B attention shape (16 q / 2 KV heads, head_dim
    128), vLLM's 16-token NHD cache [blocks, 2, 16, kv_heads, 128] with the
    fused current-token append (the step's K/V rows stored at slot_mapping
    and attended), CUDA-graph replay over rotating pools larger than L2."""
    from flashdec_b200.kernels.paged_decode import _vllm_paged_decode_attention_into
    from oracle.paged_attention import attention_bytes

    b, hq, hkv, d, bs, ctx = 8, 16, 2, 128, 16, 2048
    nblk = ctx // bs
    pool = 2 * b * nblk
    g = torch.Generator(device=device).manual_seed(55)
    pools = []
    for _ in range(NUM_POOLS):
        kv = torch.randn((pool, 2, bs, hkv, d), device=device, dtype=torch.bfloat16, generator=g)
        bt = torch.randperm(pool, device=device, generator=g)[: b * nblk].reshape(b, nblk)
        bt = bt.to(torch.int32).contiguous()
        # the current token (position ctx - 1) goes to its page's last slot
        slot = (bt[:, -1].to(torch.int64) * bs + (ctx - 1) % bs).contiguous()
        q = torch.randn((b, hq, d), device=device, dtype=torch.bfloat16, generator=g)
        k = torch.randn((b, hkv, d), device=device, dtype=torch.bfloat16, generator=g)
        v = torch.randn((b, hkv, d), device=device, dtype=torch.bfloat16, generator=g)
        pools.append((q, k, v, kv, bt, slot, torch.empty_like(q)))
    sl = torch.full((b,), ctx, device=device, dtype=torch.int32)
    # vLLM's split workspace (softmax_segm_*, 16 segments); the auto plan
    # merges inside the kernel and does not touch it
    acc = torch.empty((b, hq, 16, d), device=device, dtype=torch.float32)
    mx = torch.empty((b, hq, 16), device=device, dtype=torch.float32)
    sm = torch.empty((b, hq, 16), device=device, dtype=torch.float32)
    state = {"i": 0}

    def step():
        q, k, v, kv, bt, slot, out = pools[state["i"] % len(pools)]
        state["i"] += 1
        _vllm_paged_decode_attention_into(q, k, v, kv, bt, sl, out, slot, acc, mx, sm,
                                          num_reqs=b, num_q_heads=hq, num_kv_heads=hkv,
                                          head_dim=d, block_size=bs, sm_scale=d ** -0.5,
                                          num_splits=0)

    us = _graph_time_us(torch, stream, step, reps=max(10, reps // 12), inner=NUM_POOLS * 10)
    # K/V read once per KV head (the cache holds ctx - 1 tokens, the current
    # one comes from the call), plus the appended rows read and stored
    nbytes = attention_bytes([ctx] * b, hq, hkv, d, bs) + 2 * b * hkv * d * 2 * 2
    peak, _ = _peaks()
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"workload": "vLLM launcher (reference headline config): B8 ctx2048, 16q/2kv, D128, "
                        "16-token NHD 5-D cache, fused current-token append, graph replay",
            "us_per_step": us, "tokens_per_s": b / (us * 1e-6), "algorithmic_bytes": nbytes,
            "hbm_gbs": gbs, "frac_of_peak": gbs / peak,
            "traffic": _traffic_from_profile("wave_decode_vllm_b8_ctx2048"),
            "reference_published_us": 38.528,
            "reference_published": "RTX 5070, benchmarks/results/vllm_qwen_attention_summary.md:24"}


def run_c3(torch, device, stream, cpu_seconds=2.0, api_reps=200):
    """fused RoPE + KV append of 64 tokens (16 q heads,
    2 KV heads, D128, theta 1e6) into distinct slots of a 4096 x 32 pool."""
    import numpy as np

    import flashdec_b200
    from flashdec_b200._fused_rope_kv_append import _fused_rope_kv_append_trusted

    g = torch.Generator(device=device).manual_seed(33)
    n, hq, hkv, d, nb, bs = 64, 16, 2, 128, 4096, 32
    q = torch.randn((n, hq, d), device=device, dtype=torch.bfloat16, generator=g)
    k = torch.randn((n, hkv, d), device=device, dtype=torch.bfloat16, generator=g)
    v = torch.randn((n, hkv, d), device=device, dtype=torch.bfloat16, generator=g)
    kc = torch.zeros((nb, hkv, bs, d), device=device, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(nb * bs, device=device, generator=g)[:n]
    bid = (slots // bs).to(torch.int64)
    off = (slots % bs).to(torch.int64)
    pos = torch.randint(0, 32768, (n,), device=device, generator=g, dtype=torch.int64)
    q_out = torch.empty_like(q)

    def step():
        _fused_rope_kv_append_trusted(q, k, v, kc, vc, bid, off, pos, rotary_dim=d, base=1e6,
                                      q_out=q_out)

    us = _graph_time_us(torch, stream, step, reps=200, inner=50)
    # end to end through the public API (value checks synchronise, as in the reference)
    e0 = time.perf_counter()
    for _ in range(api_reps):
        flashdec_b200.fused_rope_kv_append(q, k, v, kc, vc, bid, off, pos, rotary_dim=d,
                                           base=1e6)
    torch.cuda.synchronize()
    api_us = (time.perf_counter() - e0) * 1e6 / api_reps if api_reps else None
    nbytes = 2 * n * hq * d * 2 + 2 * n * hkv * d * 2 + 2 * n * hkv * d * 2 + 3 * n * 8
    # CPU reference on the same inputs: the oracle's RoPE of Q and K (a
    # restatement of flashdec/rope.py:26-85) and in-place slot writes
    from oracle.rope import apply_rope as apply_rope_ref

    qh, kh, vh = (t.float().cpu().numpy() for t in (q, k, v))
    kch = np.zeros((nb, hkv, bs, d), np.float32)
    vch = np.zeros_like(kch)
    bh, oh, ph = bid.cpu().numpy(), off.cpu().numpy(), pos.cpu().numpy()
    t0 = time.perf_counter()
    cpu_reps = 0
    while time.perf_counter() - t0 < cpu_seconds:
        apply_rope_ref(qh, ph, d, 1e6, "bfloat16")
        k_rot = apply_rope_ref(kh, ph, d, 1e6, "bfloat16")
        kch[bh, :, oh, :] = k_rot
        vch[bh, :, oh, :] = vh
        cpu_reps += 1
    cpu_us = (time.perf_counter() - t0) * 1e6 / cpu_reps if cpu_reps else None
    return {"workload": "BASELINE c3: fused RoPE + KV append, 64 tokens, 16q/2kv, D128, "
                        "theta 1e6, distinct slots in a 4096x32 pool",
            "us_per_call_device": us, "us_per_call_public_api": api_us,
            "algorithmic_bytes": nbytes,
            "note": "latency-bound (0.13 MB): a roofline fraction is not meaningful here",
            "cpu_reference_us": cpu_us, "cpu_reference": "numpy oracle: RoPE of q and k + "
            "in-place slot writes, 1 thread"}


def run_c5(torch, device, args, num_layers=36, num_requests=16, prefix_tokens=4096):
    """full transactional DecodeEngine step over 36 layers
    of the Qwen2.5-3B attention shape; 16 requests share a refcounted
    4096-token prefix plus private tails U[0, 1024]; RoPE + append then paged
    decode per layer; one token committed per step."""
    import numpy as np

    from flashdec_b200 import DecodeEngine, PagedKVCache
    from oracle.paged_attention import attention_bytes

    hq, hkv, d, bs = 16, 2, 128, 32
    rng = np.random.default_rng(55)
    tails = [int(x) for x in rng.integers(0, 1025, size=num_requests)]
    steps = max(3, min(args.steps // 6000, 20))
    prefix_blocks = prefix_tokens // bs
    max_blocks = prefix_blocks + sum((t + steps + 40) // bs + 2 for t in tails) + 16
    cache = PagedKVCache(num_layers, hkv, d, bs, max_blocks, dtype=torch.bfloat16,
                         device=device, prefix_cache_capacity_blocks=prefix_blocks)
    eng = DecodeEngine(cache, append_backend="fused_cuda")
    g = torch.Generator(device=device).manual_seed(5)
    shape = (num_layers, prefix_blocks, hkv, bs, d)
    eng.register_prefix("sys", torch.randn(shape, device=device, dtype=torch.bfloat16, generator=g),
                        torch.randn(shape, device=device, dtype=torch.bfloat16, generator=g))
    ids = list(range(num_requests))
    for r in ids:
        eng.add_request(r)
    eng.admit()
    for r in ids:
        cache.attach_prefix(r, "sys")
    # private tails, written through cache transactions (not timed)
    kv = torch.randn((num_requests, hkv, d), device=device, dtype=torch.bfloat16, generator=g)
    for t in range(max(tails)):
        rows = [r for r in ids if tails[r] > t]
        tx = cache.begin_token(rows)
        for layer in range(num_layers):
            cache.write_token_layer(tx, layer, kv[: len(rows)], kv[: len(rows)])
        cache.commit_token(tx)
    q = torch.randn((num_layers, num_requests, hq, d), device=device, dtype=torch.bfloat16,
                    generator=g)
    k = torch.randn((num_layers, num_requests, hkv, d), device=device, dtype=torch.bfloat16,
                    generator=g)
    v = torch.randn_like(k)

    # per-layer operands as separate tensors, the way a model hands each
    # layer's projections to the engine
    qs, ks, vs = list(q.unbind(0)), list(k.unbind(0)), list(v.unbind(0))

    def engine_step():
        tx = eng.begin_step(ids)
        for layer in range(num_layers):
            eng.step_layer(tx, layer, qs[layer], ks[layer], vs[layer], rotary_dim=d, base=1e6)
        return eng.commit_step(tx)

    for _ in range(2):
        engine_step()
    torch.cuda.synchronize()
    lens0 = [cache.request_state(r)["seq_len"] for r in ids]
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for _ in range(steps):
        engine_step()
    e1.record()
    torch.cuda.synchronize()
    wall_us = (time.perf_counter() - t0) * 1e6 / steps
    dev_us = e0.elapsed_time(e1) * 1000.0 / steps
    logical = attention_bytes([n + 1 for n in lens0], hq, hkv, d, bs) * num_layers
    unique = (prefix_tokens + sum(n - prefix_tokens for n in lens0)) * hkv * d * 4 * num_layers
    return {"workload": "BASELINE c5: DecodeEngine begin_step / 36 x step_layer / commit_step, "
                        "16 requests sharing a 4096-token prefix + tails U[0,1024], Qwen2.5-3B "
                        "attention shape, fused RoPE+append then paged decode per layer",
            "steps": steps, "us_per_step_wall": wall_us, "us_per_step_device_span": dev_us,
            "tokens_per_s": num_requests / (wall_us * 1e-6),
            "us_per_layer_wall": wall_us / num_layers,
            "gpu_launches_per_step": num_layers,  # one fused RoPE + append + decode per layer
            "logical_kv_bytes_per_step": logical, "unique_kv_bytes_per_step": unique,
            "note": "host-driven (Python engine per layer, no graph capture); one launch per "
                    "layer (RoPE + K/V store + decode)"}


def run_c5_layer(torch, device, stream, reps=300, num_requests=16, prefix_tokens=4096):
    """One attention layer of the c5 shape through the plain decode: 16
    requests whose block tables share the same 128 prefix pages, then private
    tails U[1, 1025] tokens (the lengths of the engine leg's first step);
    back-to-back paged_decode_attention_into launches, CUDA events."""
    import numpy as np

    import flashdec_b200
    from oracle.paged_attention import attention_bytes

    hq, hkv, d, bs = 16, 2, 128, 32
    rng = np.random.default_rng(55)
    tails = [int(x) + 1 for x in rng.integers(0, 1025, size=num_requests)]
    pre = prefix_tokens // bs
    rows, nxt = [], pre
    for t in tails:
        n = -(-t // bs)
        rows.append(list(range(pre)) + list(range(nxt, nxt + n)))
        nxt += n
    width = max(len(r) for r in rows)
    bt_h = torch.full((num_requests, width), -1, dtype=torch.int32)
    for i, r in enumerate(rows):
        bt_h[i, :len(r)] = torch.tensor(r, dtype=torch.int32)
    bt = bt_h.to(device)
    lens = [prefix_tokens + t for t in tails]
    sl = torch.tensor(lens, dtype=torch.int32, device=device)
    g = torch.Generator(device=device).manual_seed(7)
    k = torch.randn((nxt, hkv, bs, d), device=device, dtype=torch.bfloat16, generator=g)
    v = torch.randn_like(k)
    q = torch.randn((num_requests, hq, d), device=device, dtype=torch.bfloat16, generator=g)
    out = torch.empty_like(q)
    with torch.cuda.stream(stream):
        for _ in range(20):
            flashdec_b200.paged_decode_attention_into(q, k, v, bt, sl, out)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            flashdec_b200.paged_decode_attention_into(q, k, v, bt, sl, out)
        e1.record(stream)
    stream.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / reps
    # the same layer through the cascade (shared pages read once per KV head);
    # median of three timed rounds (a process's first round is slower)
    from flashdec_b200 import _native

    cg = _native.CascadeGroups([list(range(num_requests))], [pre], num_requests, bs, device)

    def cascade():
        _native.cascade_decode(q, k, v, bt, sl, out, cg, sm_scale=d ** -0.5, block_size=bs,
                               num_seqs=num_requests)

    # The eager call costs more host time than the GPU needs for it, so the
    # device time comes from a CUDA graph of 100 calls (the call forks its
    # second stream and joins it back, so it captures); the host time of an
    # eager call is reported beside it.
    with torch.cuda.stream(stream):
        for _ in range(20):
            cascade()
    stream.synchronize()
    t0 = time.perf_counter()
    with torch.cuda.stream(stream):
        for _ in range(reps):
            cascade()
    host_us = (time.perf_counter() - t0) * 1e6 / reps
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(100):
            cascade()
    rounds = []
    with torch.cuda.stream(stream):
        for _ in range(4):
            c0 = torch.cuda.Event(enable_timing=True)
            c1 = torch.cuda.Event(enable_timing=True)
            c0.record(stream)
            graph.replay()
            c1.record(stream)
            stream.synchronize()
            rounds.append(c0.elapsed_time(c1) * 1000.0 / 100)
    del graph
    casc_us = sorted(rounds[1:])[1]
    logical = attention_bytes(lens, hq, hkv, d, bs)
    unique = nxt * hkv * bs * d * 2 * 2
    return {"workload": "c5 shape, one layer, plain decode: 16 requests sharing a 4096-token "
                        "prefix (same pages) + tails U[1,1025]",
            "us_per_call": us, "launches": reps, "logical_kv_bytes": logical,
            "unique_kv_bytes": unique, "cascade_us_per_call": casc_us,
            "cascade_rounds_us": rounds, "cascade_host_us_per_eager_call": host_us,
            "note": "plain: the shared prefix pages are L2 hits after the first reader; bound by "
                    "per-SM ingest of the logical bytes, not HBM. cascade: shared pages read once "
                    "per KV head; device time from graph replay, the eager call is host-bound"}


def run_sweep(torch, device, stream):
    """Decode latency over batch x context for the Qwen attention shape
    (16q/2kv, D128, bs32, bf16), graph replay over rotating pools of at least
    400 MB where the shape allows; one JSON line per point."""
    from oracle.paged_attention import attention_bytes

    import flashdec_b200

    hq, hkv, d, bs = 16, 2, 128, 32
    peak, _ = _peaks()
    points = []
    for batch in (1, 2, 4, 8, 16, 32, 64, 128):
        for ctx in (1024, 4096, 16384):
            if batch * ctx > 128 * 16384:
                continue
            nblk = ctx // bs
            g = torch.Generator(device=device).manual_seed(batch * 7 + ctx)
            per_pool = 2 * batch * nblk * hkv * bs * d * 2 * 2
            npools = max(2, min(12, math.ceil(400e6 / per_pool)))
            pools = []
            for _ in range(npools):
                k = torch.randn((batch * nblk, hkv, bs, d), device=device, dtype=torch.bfloat16,
                                generator=g)
                v = torch.randn_like(k)
                bt = torch.randperm(batch * nblk, device=device, generator=g).reshape(
                    batch, nblk).to(torch.int32)
                q = torch.randn((batch, hq, d), device=device, dtype=torch.bfloat16, generator=g)
                pools.append((q, k, v, bt, torch.empty_like(q)))
            sl = torch.full((batch,), ctx, device=device, dtype=torch.int32)
            state = {"i": 0}

            def step():
                q, k, v, bt, o = pools[state["i"] % len(pools)]
                state["i"] += 1
                flashdec_b200.paged_decode_attention_into(q, k, v, bt, sl, o)

            us = _graph_time_us(torch, stream, step, reps=20,
                                inner=len(pools) * max(1, 24 // len(pools)))
            nbytes = attention_bytes([ctx] * batch, hq, hkv, d, bs)
            gbs = nbytes / (us * 1e-6) / 1e9
            points.append({"batch": batch, "context": ctx, "us_per_step": round(us, 3),
                           "hbm_gbs": round(gbs, 1), "frac_of_peak": round(gbs / peak, 4),
                           "pools": npools})
            del pools
            torch.cuda.empty_cache()
    return points


# ---------------------------------------------------------------------------
# CPU reference (the numpy oracle restating flashdec/paged_reference.py)
# ---------------------------------------------------------------------------
def _cpu_workload(seed=7, cfg=None):
    import numpy as np

    from tests.golden.cases import _normal

    cfg = cfg or C2
    rng = np.random.default_rng(seed)
    b, hq, hkv, d, bs, ctx = cfg["batch"], cfg["hq"], cfg["hkv"], cfg["d"], cfg["bs"], cfg["ctx"]
    nblk = ctx // bs
    pool = cfg["pool_factor"] * b * nblk
    q = _normal(rng, (b, hq, d), "bfloat16")
    k = _normal(rng, (pool, hkv, bs, d), "bfloat16")
    v = _normal(rng, (pool, hkv, bs, d), "bfloat16")
    bt = rng.permutation(pool)[: b * nblk].reshape(b, nblk).astype(np.int32)
    sl = np.full((b,), ctx, np.int32)
    return q, k, v, bt, sl


def _c1_workload(seed=11):
    """B=4, 16q/2kv, D128, bs32, fp32, seq U[64,512], a
    seeded permutation of a 128-block pool, sm_scale 128^-0.5."""
    import numpy as np

    rng = np.random.default_rng(seed)
    b, hq, hkv, d, bs, nb = 4, 16, 2, 128, 32, 128
    sl = rng.integers(64, 513, size=b).astype(np.int32)
    maxblk = nb // b
    bt = rng.permutation(nb)[: b * maxblk].reshape(b, maxblk).astype(np.int32)
    q = rng.standard_normal((b, hq, d)).astype(np.float32)
    k = rng.standard_normal((nb, hkv, bs, d)).astype(np.float32)
    v = rng.standard_normal((nb, hkv, bs, d)).astype(np.float32)
    return q, k, v, bt, sl


# ---------------------------------------------------------------------------
# CPU side.  The timed CPU path is the reference's own PyTorch
# paged_decode_attention_ref (flashdec/paged_reference.py:19-125) from the
# reference install under baseline/_ref when it is there ("reference"), else
# the numpy oracle restating it ("port").  Sequences run one per task on a
# process pool with one worker per host core (each worker limited to one
# thread); the pool is started with "spawn" (fresh interpreters), which is
# safe after CUDA is initialised.  Each worker builds the seeded workload
# itself.
# ---------------------------------------------------------------------------
REF_DIR = REPO / "baseline" / "_ref"
_POOL_WORK = None
_POOL_FN = None


def _reference_available():
    return (REF_DIR / "flashdec" / "paged_reference.py").exists()


def _pool_init(kind, workload):
    global _POOL_WORK, _POOL_FN
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(limits=1)  # one core per worker
    except Exception:
        pass
    arrays = _c1_workload() if workload == "c1" else _cpu_workload()
    if kind == "reference":
        import torch

        torch.set_num_threads(1)
        sys.path.insert(0, str(REF_DIR))
        # the repository's own ``flashdec`` (an alias of flashdec_b200) must
        # not stand in for the reference: drop it if anything imported it
        for name in [m for m in sys.modules if m == "flashdec" or m.startswith("flashdec.")]:
            del sys.modules[name]
        import flashdec.paged_reference as ref_mod
        from flashdec.paged_reference import paged_decode_attention_ref

        if not Path(ref_mod.__file__).resolve().is_relative_to(REF_DIR.resolve()):
            raise RuntimeError(f"reference arm imported {ref_mod.__file__}, not the reference")

        q, k, v, bt, sl = arrays
        dt = torch.float32 if workload == "c1" else torch.bfloat16
        _POOL_WORK = (torch.from_numpy(q).to(dt), torch.from_numpy(k).to(dt),
                      torch.from_numpy(v).to(dt), torch.from_numpy(bt), torch.from_numpy(sl))
        _POOL_FN = paged_decode_attention_ref
    else:
        from oracle import paged_decode_attention_ref

        _POOL_WORK = arrays
        dtype = "float32" if workload == "c1" else "bfloat16"
        _POOL_FN = lambda q, k, v, bt, sl: paged_decode_attention_ref(q, k, v, bt, sl, dtype=dtype)


def _pool_seq(i):
    q, k, v, bt, sl = _POOL_WORK
    i %= q.shape[0]
    _POOL_FN(q[i:i + 1], k, v, bt[i:i + 1], sl[i:i + 1])
    return i


def _cpu_pool(workload="c2"):
    import multiprocessing as mp

    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    n = max(1, min(n, 64))
    kind = "reference" if _reference_available() else "port"
    pool = mp.get_context("spawn").Pool(n, initializer=_pool_init, initargs=(kind, workload))
    pool.map(_pool_seq, range(n))  # start-up (imports, workload) outside the timing
    return pool, n, kind


def _pool_sequences(pool, n, seconds):
    """Run sequences on the pool for about `seconds`; (sequences, elapsed)."""
    done = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        chunk = 4 * n
        pool.map(_pool_seq, range(done, done + chunk))
        done += chunk
    return done, time.perf_counter() - t0


_KIND_TEXT = {
    "reference": "the reference's own PyTorch paged_decode_attention_ref "
                 "(flashdec/paged_reference.py:19-125, installed under baseline/_ref)",
    "port": "the numpy oracle restating flashdec/paged_reference.py:19-125 (no reference "
            "install under baseline/_ref)",
}


def cpu_baseline_sample(args, seconds=None, workload="c2"):
    """Time the CPU path on a bounded sample of the workload's sequences on
    all host cores."""
    seconds = seconds if seconds is not None else float(os.environ.get("FD_CPU_SECONDS", "10"))
    pool, n, kind = _cpu_pool(workload)
    try:
        n_seq, dt = _pool_sequences(pool, n, seconds)
    finally:
        pool.close()
        pool.join()
    what = ("c1 (B4, 16q/2kv, D128, bs32, fp32, seq U[64,512])" if workload == "c1"
            else "c2 (ctx 2048, 16q/2kv, D128, bf16)")
    return {
        "value": n_seq / dt,
        "unit": "tokens/s",
        "cores": n,
        "kind": kind,
        "sample": f"{n_seq} sequences of the {what} workload in {dt:.1f} s on {n} worker "
                  f"processes (one core each), {_KIND_TEXT[kind]}",
    }


def c2_config(world):
    """The `config` both arms report (same keys and values)."""
    return {
        "workload": "BASELINE c2: Qwen2.5-3B-shape paged decode attention, B8 ctx2048",
        "batch_per_gpu": C2["batch"], "q_heads": C2["hq"], "kv_heads": C2["hkv"],
        "head_dim": C2["d"], "block_size": C2["bs"], "context": C2["ctx"],
        "kv_pool_blocks": C2["pool_factor"] * C2["batch"] * C2["ctx"] // C2["bs"],
        "l2": f"inputs rotate over {NUM_POOLS} KV pools ({NUM_POOLS * 2 * 2 * C2['batch'] * C2['ctx'] * C2['hkv'] * C2['d'] * 2 * C2['pool_factor'] // 2**20} MiB) > 3x L2",
        "parallelism": f"request-sharded x{world} (no data-path collective)",
    }


def run_reference(args, rank, world):
    if rank != 0:
        return None
    # A step is one c2 batch (8 sequences) on the host cores; the sample is
    # sized by time, not by --steps, so that the rate is not dominated by
    # start-up (at least FD_REF_SECONDS, default 10 s).
    budget = float(os.environ.get("FD_REF_SECONDS", "10"))
    pool, n, kind = _cpu_pool("c2")
    try:
        n_seq, dt = _pool_sequences(pool, n, budget)
    finally:
        pool.close()
        pool.join()
    steps = max(1, n_seq // C2["batch"])
    value = n_seq / dt
    return {
        "metric": METRIC,
        "impl": "reference",
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1000.0 * dt / steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) q/k/v, scattered block tables)",
        "config": c2_config(world),
        "cpu_baseline": {
            "value": value, "unit": "tokens/s", "cores": n, "kind": kind,
            "sample": f"{n_seq} c2 sequences ({steps} batches of 8) in {dt:.1f} s on {n} worker "
                      f"processes (one core each): {_KIND_TEXT[kind]}",
        },
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


# Qwen2.5-3B's architecture (public model config); weights are vLLM's dummy
# initialisation, so no checkpoint is needed
QWEN25_3B = {
    "architectures": ["Qwen2ForCausalLM"], "model_type": "qwen2", "hidden_size": 2048,
    "intermediate_size": 11008, "num_hidden_layers": 36, "num_attention_heads": 16,
    "num_key_value_heads": 2, "max_position_embeddings": 32768, "rope_theta": 1000000.0,
    "rms_norm_eps": 1e-06, "vocab_size": 151936, "tie_word_embeddings": True,
    "torch_dtype": "bfloat16", "hidden_act": "silu", "use_sliding_window": False,
    "max_window_layers": 36, "bos_token_id": 151643, "eos_token_id": 151643,
}
VLLM_E2E = dict(batch=8, prompt=2048, decode=128)


def run_vllm_e2e(eager):
    """Opt-in (--vllm-e2e): vLLM ``LLM.generate`` on the Qwen2.5-3B
    architecture (dummy weights), B8 prompts of 2048 tokens, 128 greedy decode
    tokens each, once with vLLM's TRITON_ATTN backend and once with this
    package's CUSTOM backend, each in its own process.  Decode throughput is
    the difference between a 129-token and a 1-token generation of the same
    prompts (so prefill is taken out)."""
    import tempfile

    res = {}
    with tempfile.TemporaryDirectory() as tmp:
        model = Path(tmp) / "model"
        model.mkdir()
        (model / "config.json").write_text(json.dumps(QWEN25_3B))
        for backend in ("TRITON_ATTN", "CUSTOM"):
            out = Path(tmp) / f"{backend}.json"
            cmd = [sys.executable, str(Path(__file__).resolve()), "--vllm-e2e-worker", backend,
                   str(out), str(model)] + (["--eager"] if eager else [])
            subprocess.run(cmd, cwd=REPO, check=True, timeout=1800)
            res[backend] = json.loads(out.read_text())
    t, c = res["TRITON_ATTN"], res["CUSTOM"]
    tt, ct = t.pop("tokens"), c.pop("tokens")
    first, prefix = greedy_agreement(tt, ct)
    return {"vllm_e2e": "Qwen2.5-3B architecture, dummy weights, B8 x 2048-token prompts, 128 greedy "
                        "decode tokens, vLLM LLM.generate",
            "cuda_graphs": not eager, "triton_attn": t, "custom": c,
            "decode_speedup": t["decode_ms_per_step"] / c["decode_ms_per_step"],
            "greedy_first_token_agreement": first,
            "greedy_common_prefix_mean": prefix}


def greedy_agreement(ref_tokens, our_tokens):
    """Greedy token sequences of two backends on the same prompts -> (share
    of sequences whose first token agrees, mean share of each sequence equal
    up to its first difference).  bf16 attention rounding can flip a near-tie,
    after which a greedy sequence diverges, so the common prefix, not the
    count of equal positions, is the measure."""
    if len(ref_tokens) != len(our_tokens) or not ref_tokens:
        raise ValueError("need the same, non-zero number of sequences from both backends")
    first = sum(bool(a) and bool(b) and a[0] == b[0]
                for a, b in zip(ref_tokens, our_tokens)) / len(ref_tokens)
    prefix = []
    for a, b in zip(ref_tokens, our_tokens):
        n = next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), min(len(a), len(b)))
        prefix.append(n / max(len(a), len(b), 1))
    return first, sum(prefix) / len(prefix)


def _vllm_e2e_worker(backend, out_path, model_dir, eager):
    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")  # engine core in-process
    import numpy as np

    calls = {"n": 0}
    if backend == "CUSTOM":
        import flashdec_b200.vllm_backend as vb
        from flashdec_b200 import vllm_plugin

        vllm_plugin.register()
        orig = vb._vllm_paged_decode_attention_into

        def counted(*a, **k):
            calls["n"] += 1
            return orig(*a, **k)

        vb._vllm_paged_decode_attention_into = counted
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt

    cfg = VLLM_E2E
    llm = LLM(model=model_dir, load_format="dummy", skip_tokenizer_init=True, dtype="bfloat16",
              max_model_len=cfg["prompt"] + cfg["decode"] + 64, gpu_memory_utilization=0.5,
              attention_backend=backend, seed=0, enforce_eager=eager,
              max_num_seqs=cfg["batch"])
    rng = np.random.default_rng(0)
    prompts = [TokensPrompt(prompt_token_ids=[int(x) for x in rng.integers(100, 150000, cfg["prompt"])])
               for _ in range(cfg["batch"])]

    tokens = []

    def timed(n):
        sp = SamplingParams(max_tokens=n, temperature=0.0, ignore_eos=True, detokenize=False)
        t0 = time.perf_counter()
        outs = llm.generate(prompts, sp, use_tqdm=False)
        dt = time.perf_counter() - t0
        assert all(len(o.outputs[0].token_ids) == n for o in outs)
        tokens[:] = [list(o.outputs[0].token_ids) for o in outs]
        return dt

    timed(4)  # warm-up
    t1 = min(timed(1) for _ in range(3))
    tn = min(timed(cfg["decode"] + 1) for _ in range(3))
    step_ms = (tn - t1) * 1000.0 / cfg["decode"]
    Path(out_path).write_text(json.dumps({
        "backend": backend, "prefill_s": t1, "generate_s": tn, "decode_ms_per_step": step_ms,
        "decode_tokens_per_s": cfg["batch"] / (step_ms / 1000.0),
        "flashdec_launcher_calls": calls["n"], "tokens": tokens}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=120000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--sweep", action="store_true",
                    help="print decode latency over batch x context (Qwen shape), one JSON "
                         "line per point, and exit")
    ap.add_argument("--kernel-only", nargs="?", const="c2", default=None,
                    choices=["c2", "c3", "c4", "c5", "vllm"],
                    help="time only one device-resident workload (no e2e or CPU legs): c2 "
                         "(default), c3 (fused RoPE + append), c4 (16 requests of the ragged "
                         "batch, 1.5 GB of KV), c5 (one layer of the c5 shape, plain decode) or "
                         "vllm (the vLLM launcher at B8 ctx2048 with the fused append); "
                         "the small cases used for ncu captures")
    ap.add_argument("--vllm-e2e", action="store_true",
                    help="opt-in: vLLM LLM.generate decode throughput on the Qwen2.5-3B "
                         "architecture (dummy weights), TRITON_ATTN against CUSTOM; minutes")
    ap.add_argument("--eager", action="store_true", help="with --vllm-e2e: no CUDA graphs")
    ap.add_argument("--vllm-e2e-worker", nargs=3, default=None, help=argparse.SUPPRESS)
    args = ap.parse_args()
    if args.vllm_e2e_worker:
        _vllm_e2e_worker(*args.vllm_e2e_worker, eager=args.eager)
        return
    if args.vllm_e2e:
        print(json.dumps(run_vllm_e2e(args.eager)), flush=True)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    if args.sweep:
        import torch

        device = torch.device("cuda", 0)
        torch.cuda.set_device(device)
        for point in run_sweep(torch, device, torch.cuda.Stream(device)):
            print(json.dumps({"sweep": "qwen-shape decode", **point}), flush=True)
        return
    if args.kernel_only in ("c3", "c4", "c5", "vllm"):
        import torch

        device = torch.device("cuda", 0)
        torch.cuda.set_device(device)
        stream = torch.cuda.Stream(device)
        if args.kernel_only == "c3":
            res = run_c3(torch, device, stream, cpu_seconds=0.0, api_reps=0)
        elif args.kernel_only == "c5":
            res = run_c5_layer(torch, device, stream, reps=min(args.steps, 300))
        elif args.kernel_only == "vllm":
            res = run_vllm_launcher(torch, device, stream, reps=min(args.steps, 200))
        else:
            res = run_ragged(torch, None, device, 0, 1, stream, args, batch=16)
        print(json.dumps({"kernel_only": args.kernel_only, **res}), flush=True)
        return
    import torch
    import torch.distributed as dist

    if world > 1:
        from datetime import timedelta

        # rank 0 prints exactly one JSON line on stdout.  NCCL's communicator
        # lines (INIT: ranks, devices, transports; teardown) are wanted in the
        # log, and NCCL writes them to the process's stdout: under torchrun
        # file descriptor 1 points at stderr for the whole run, and the JSON
        # line goes to a duplicate of the real stdout taken first.
        # (the image presets NCCL_DEBUG=VERSION, which prints no INIT lines)
        if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
        sys.stdout.flush()
        json_fd = os.dup(1)
        os.dup2(2, 1)
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    else:
        json_fd = None
    try:
        res = run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
    if res is not None:
        if json_fd is None:
            print(json.dumps(res), flush=True)
        else:
            sys.stdout.flush()
            os.write(json_fd, (json.dumps(res) + "\n").encode())
    if json_fd is not None:
        os.close(json_fd)


if __name__ == "__main__":
    main()
