"""Benchmark of the B200 paged decode attention (HELM's long-context decode hot path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload ("config 2"): isolated paged decode
attention, bf16, batch 4, 32 query heads / 8 KV heads (GQA 4), head_dim 128,
32768 tokens per sequence in 16-token pages placed by a seeded random
permutation of a 16384-page pool (1 GiB of K/V), Q/K/V ~ N(0,1), no mask.
A STEP is one decode-attention call over the whole batch; the K/V cache is
resident state in HBM (as in decode), the per-step inputs are q, the page
table and the lengths.  512 MiB of K/V are read per step, so every step
streams more than the 126 MB L2 (no flush needed).

Prints one JSON line (rank 0).  `value` is achieved algorithmic HBM GB/s of
the whole call (bytes of K/V + q + O + LSE + page table per step / device
time).  With N GPUs (torchrun) the same call is split by sequence: every rank
holds a page-aligned 1/N of each sequence's tokens in its own HBM, computes
fp32 partial states, and one peer-memory kernel per call exchanges and merges
them over NVLink (strong scaling; time = max over ranks).  The line also
carries `model_decode`: decode tok/s of BASELINE configs[3] (Qwen3-14B,
131072-token context, batch 1) tensor-parallel over the same N GPUs.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GRAPH_STEPS = 10   # decode calls per captured graph in the device-timed loop
METRIC = ("decode tok/s at 32k/128k ctx; paged-attn achieved HBM GB/s vs 8 TB/s peak")
B, HQ, HKV, D, P, T, POOL = 4, 32, 8, 128, 16, 32768, 16384
KV_BYTES = B * T * HKV * D * 2 * 2
ALG_BYTES = KV_BYTES + B * HQ * D * 2 * 2 + B * HQ * 4 + B * (T // P) * 4 + B * 4
WORKLOAD = ("config2: isolated paged decode attention, bf16, B=4, 32q/8kv heads, D=128, "
            "T=32768/seq, 16-token pages, randperm placement in a 16384-page pool")


def _set_shape(seq_len: int, pool_pages: int) -> None:
    """Shrinks the workload for profiling runs; the defaults are config 2."""
    global T, POOL, KV_BYTES, ALG_BYTES, WORKLOAD
    if seq_len == T and pool_pages == POOL:
        return
    if seq_len % P or pool_pages < B * seq_len // P:
        raise SystemExit("--seq-len must be a multiple of 16 and fit the pool")
    T, POOL = seq_len, pool_pages
    KV_BYTES = B * T * HKV * D * 2 * 2
    ALG_BYTES = KV_BYTES + B * HQ * D * 2 * 2 + B * HQ * 4 + B * (T // P) * 4 + B * 4
    WORKLOAD = WORKLOAD.replace("T=32768", f"T={T}").replace("16384-page", f"{POOL}-page") + \
        " (reduced profiling case)"


def _peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6.65 TB/s"


def make_inputs(seed: int = 0):
    """Draw order: permutation, K pool, V pool, q (torch CPU generator, seed 0)."""
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(POOL, generator=g)
    k = torch.randn(POOL, HKV, P, D, generator=g).to(torch.bfloat16)
    v = torch.randn(POOL, HKV, P, D, generator=g).to(torch.bfloat16)
    q = torch.randn(B, HQ, D, generator=g).to(torch.bfloat16)
    pool = torch.stack([k, v], dim=1)  # [POOL, 2, HKV, P, D]
    page_table = perm[:B * (T // P)].view(B, T // P).to(torch.int32)
    kv_lens = torch.full((B,), T, dtype=torch.int32)
    return q, pool, page_table, kv_lens


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.dev), "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        with open(self.file.name) as f:
            rows = [r.strip().split(", ") for r in f if r.strip()]
        os.unlink(self.file.name)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
            except ValueError:
                continue
            for n, flag in zip(names, r[5:9]):
                if flag.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "samples": len(sm), "reasons": sorted(reasons)}


def cpu_baseline(q, pool, page_table, kv_lens, budget_s: float = 12.0, steps: int | None = None):
    """The oracle port (oracle/paged_attention.c) over the full config-2 workload,
    all host threads; repeated until `budget_s` elapsed (or `steps` times)."""
    import oracle
    threads = os.cpu_count() or 1
    nump, used = oracle.dense_page_lists(kv_lens.numpy(), P, page_table.shape[1])
    bits = pool.view(torch.int16).numpy().view(np.uint16)
    qf = q.float().numpy()
    pt = page_table.numpy()

    def once():
        return oracle.paged_attention(qf, bits, oracle.DT_BF16, pt, nump, used,
                                      num_kv_heads=HKV, page_size=P, scale=D ** -0.5,
                                      threads=threads)
    once()  # warm (page faults, thread start-up)
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        once()
        times.append(time.perf_counter() - t0)
        if steps is not None and len(times) >= steps:
            break
        if steps is None and time.perf_counter() - t_start > budget_s:
            break
    per = statistics.median(times)
    cpu = "unknown"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    cpu = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"value": ALG_BYTES / per / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"full config-2 workload (4x32768 tokens, 512 MiB K/V) per call, "
                      f"median of {len(times)} calls, {per * 1e3:.1f} ms/call, CPU: {cpu}",
            "times": times}


def _config() -> dict:
    """The workload, printed identically by both arms."""
    return {"workload": WORKLOAD, "kv_bytes_per_step": KV_BYTES,
            "algorithmic_bytes_per_step": ALG_BYTES,
            "l2": "inputs larger than L2 (512 MiB K/V streamed per step), no flush"}


def run_reference(args, rank: int):
    if rank != 0:
        return
    q, pool, pt, kl = make_inputs(0)
    for _ in range(args.warmup):
        cpu_baseline(q, pool, pt, kl, steps=1)
    res = cpu_baseline(q, pool, pt, kl, steps=args.steps)
    per = sum(res["times"]) / len(res["times"])
    line = {"metric": METRIC, "value": res["value"], "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "impl": "reference", "config": _config(),
            "parallelism": f"host threads ({res['cores']}) of one node, rank 0 only",
            "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": res["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _split_inputs(rank: int, world: int, dev: torch.device):
    """Rank `rank`'s share of the config-2 call split by sequence: tokens
    [a, b) of every sequence (page-aligned, split_ranges), in a pool of its own
    (the shard's pages at random slots), drawn on the device.  q is the same
    on every rank."""
    from helm_b200.runtime.seq_parallel import split_ranges
    a, b = split_ranges(T, P, world)[rank]
    npg = (b - a) // P
    slots = B * npg + 64
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    pool = torch.randn(slots, 2, HKV, P, D, generator=g, device=dev).to(torch.bfloat16)
    pt = torch.randperm(slots, generator=g, device=dev)[:B * npg].view(B, npg).to(torch.int32)
    kl = torch.full((B,), b - a, dtype=torch.int32, device=dev)
    q = torch.randn(B, HQ, D, generator=torch.Generator().manual_seed(0)).to(torch.bfloat16)
    return q, pool, pt, kl, b - a


def _raise_on_status(status: int, world: int, dev: torch.device) -> None:
    """Raises on every rank when any rank's device status word reports an error
    (so that no rank goes on to a collective the failed one will not join)."""
    t = torch.tensor([status], dtype=torch.int64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    if int(t.item()) != 0:
        raise RuntimeError(f"device status {status} on this rank, {int(t.item())} on some rank")


def _timed(fn, steps: int, world: int, dev: torch.device, stream, clocks_soak: bool):
    """Device time of `steps` calls of fn (CUDA events on `stream`, barrier and
    synchronize on both sides), max over ranks; optional nvidia-smi sampling."""
    def barrier():
        if world > 1:
            torch.distributed.barrier()
    barrier()
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = None
    n_soak = 0
    if clocks_soak:
        # keep the GPU under the same load for ~0.6 s so that nvidia-smi sees it; the
        # count of soak calls is agreed by all ranks (a call may hold a collective, so
        # every rank must make the same number of them)
        t0 = time.perf_counter()
        fn(5)
        torch.cuda.synchronize(dev)
        per = max(time.perf_counter() - t0, 1e-4)
        t = torch.tensor([min(2000, int(0.6 / per) + 1)], dtype=torch.int64, device=dev)
        if world > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        n_soak = int(t.item())
        barrier()
    with ClockSampler(dev.index) as sampler:
        for _ in range(n_soak):
            fn(5)
        torch.cuda.synchronize(dev)
        ev0.record(stream)
        fn(steps)
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    clocks = sampler.summary()
    barrier()
    mine = ev0.elapsed_time(ev1)
    t = torch.tensor([mine], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item()), mine, clocks


def run_b200(args, rank: int, world: int, dev: torch.device):
    """Config 2 on `world` GPUs.  N = 1: the whole call on one GPU.  N > 1: the
    same call split by sequence -- every rank streams its token range of all
    four sequences from its own HBM into fp32 partial states, and one
    peer-memory kernel per call exchanges and merges them over NVLink, so
    every rank ends with the full output (strong scaling, total work fixed)."""
    from helm_b200 import _capi
    stream = torch.cuda.current_stream(dev)
    if world == 1:
        q, pool, pt, kl = make_inputs(0)
        qd, pd, ptd, kld = q.to(dev), pool.to(dev), pt.to(dev), kl.to(dev)
        t_rank = T
    else:
        q, pd, ptd, kld, t_rank = _split_inputs(rank, world, dev)
        qd = q.to(dev)
        pt = ptd.cpu()
        kl = kld.cpu()
    out = torch.empty(B, HQ, D, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(B, HQ, dtype=torch.float32, device=dev)
    px = None
    if world > 1:
        from helm_b200.runtime.seq_parallel import PeerExchange
        px = PeerExchange(B * HQ, D, dev)
        part = torch.empty(B * HQ * (D + 1), dtype=torch.float32, device=dev)
        o_part, lse_part = part[:B * HQ * D].view(B, HQ, D), part[B * HQ * D:].view(B, HQ)

    def step(qx=None, ptx=None, klx=None, outx=None, lsex=None):
        qx = qd if qx is None else qx
        ptx = ptd if ptx is None else ptx
        klx = kld if klx is None else klx
        outx = out if outx is None else outx
        lsex = lse if lsex is None else lsex
        if px is None:
            _capi.paged_decode_attention(qx, pd, ptx, klx, num_kv_heads=HKV, page_size=P,
                                         scale=D ** -0.5, out=outx, lse=lsex,
                                         max_kv_len_hint=t_rank)
            return
        _capi.paged_decode_attention(qx, pd, ptx, klx, num_kv_heads=HKV, page_size=P,
                                     scale=D ** -0.5, out=o_part, lse=lse_part,
                                     max_kv_len_hint=t_rank)
        px.merge(o_part.view(B * HQ, D), lse_part.view(B * HQ), outx.view(B * HQ, D),
                 lsex.view(B * HQ))

    try:
        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize(dev)
        if _capi.device_status(dev) != 0:
            raise RuntimeError("device status reported an error during warm-up")
        # decode calls as a captured decode loop runs them: GRAPH_STEPS consecutive
        # calls in one CUDA graph (each the decode kernel plus its PDL-dependent
        # merge kernel, or at N > 1 the peer exchange-merge; with decode overlap,
        # the next call's decode kernel is placed while the previous one finishes
        # -- its inputs are not written there)
        gsteps = max(d for d in range(1, GRAPH_STEPS + 1) if args.steps % d == 0)
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side), _capi.decode_overlap():
            with torch.cuda.graph(graph, stream=side):
                for _ in range(gsteps):
                    step()
        stream.wait_stream(side)
        graph.replay()
        torch.cuda.synchronize(dev)

        def replays(n_steps):
            for _ in range(max(1, n_steps // gsteps)):
                graph.replay()

        elapsed_ms, mine_ms, clocks = _timed(replays, args.steps, world, dev, stream, True)
        value = ALG_BYTES * args.steps / (elapsed_ms / 1e3) / 1e9

        # ---- end to end through the public API, host buffers ---------------------
        # per step: one pinned H2D copy of the packed inputs (q, page table,
        # lengths) and one D2H copy of the packed results (O, LSE)
        n_q, n_pt, n_kl = qd.numel() * 2, ptd.numel() * 4, kld.numel() * 4
        n_in = n_q + n_pt + n_kl
        host_in = torch.empty(n_in, dtype=torch.uint8).pin_memory()
        host_in[:n_q].view(torch.bfloat16).copy_(q.reshape(-1))
        host_in[n_q:n_q + n_pt].view(torch.int32).copy_(pt.reshape(-1))
        host_in[n_q + n_pt:].view(torch.int32).copy_(kl.reshape(-1))
        dev_in = torch.empty(n_in, dtype=torch.uint8, device=dev)
        q_in = dev_in[:n_q].view(torch.bfloat16).view(B, HQ, D)
        pt_in = dev_in[n_q:n_q + n_pt].view(torch.int32).view(ptd.shape)
        kl_in = dev_in[n_q + n_pt:].view(torch.int32)
        n_o, n_l = out.numel() * 2, lse.numel() * 4
        dev_res = torch.empty(n_o + n_l, dtype=torch.uint8, device=dev)
        out_res = dev_res[:n_o].view(torch.bfloat16).view(B, HQ, D)
        lse_res = dev_res[n_o:].view(torch.float32).view(B, HQ)
        host_res = torch.empty(n_o + n_l, dtype=torch.uint8).pin_memory()

        def e2e(n_steps):
            for _ in range(n_steps):
                dev_in.copy_(host_in, non_blocking=True)
                step(q_in, pt_in, kl_in, out_res, lse_res)
                host_res.copy_(dev_res, non_blocking=True)

        e2e(3)
        e2e_ms, _, _ = _timed(e2e, args.steps, world, dev, stream, False)
        e2e_value = ALG_BYTES * args.steps / (e2e_ms / 1e3) / 1e9
        # the end-to-end result must equal the device-resident one
        torch.cuda.synchronize(dev)
        if not torch.equal(host_res[:n_o].view(torch.bfloat16).view(B, HQ, D).to(dev), out):
            raise RuntimeError("end-to-end output differs from the device-resident output")
        del graph
        status = _capi.device_status(dev)
    finally:
        if px is not None:
            px.close()
    _raise_on_status(status, world, dev)

    model = None
    if not args.no_model_block:
        model = _model_block(_tp_decode("config4", args, rank, world, dev, steps=32,
                                        warmup=3), world)

    if rank != 0:
        return
    peak, peak_src = _peaks()
    avg_launch_ms = mine_ms / args.steps   # this rank, kernels of one call
    rank_bytes = ALG_BYTES if world == 1 else \
        (B * t_rank * HKV * D * 2 * 2 + B * HQ * D * 2 + B * HQ * (D + 1) * 4 + ptd.numel() * 4
         + B * 4)
    achieved = rank_bytes / (avg_launch_ms / 1e3) / 1e9
    traffic = None
    tpath = os.path.join(REPO, "profiles", "paged_decode_config2_traffic.json")
    if world == 1 and os.path.exists(tpath):
        with open(tpath) as f:
            traffic = json.load(f).get("dram_bytes_per_launch")
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": _config(),
        "parallelism": ("one GPU" if world == 1 else
                        f"sequence split x{world}: {t_rank} tokens of each sequence per GPU, "
                        "fp32 (O, LSE) exchanged and merged over NVLink by one peer-memory "
                        "kernel per call"),
        "decode_attention_calls_per_s": 1e3 / (elapsed_ms / args.steps),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "kernel": ("paged_decode_kernel + merge_split_pairs_kernel (PDL dependent)"
                                if world == 1 else
                                "paged_decode_kernel (fp32 partial) + seq_exchange_merge_kernel")
                               + "; achieved = this GPU's algorithmic bytes / time of the "
                                 "whole step",
                     "peak_source": peak_src,
                     "clock_note": "clocks sampled over a 0.6 s soak at the same load "
                                   "immediately before and during the timed region"},
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": n_in,
                "d2h_bytes_per_step": n_o + n_l,
                "note": "one packed pinned H2D copy (q, page table, lengths) and one packed "
                        "D2H copy (O, LSE) per call, eager launches through the C-ABI wrapper"},
        "gpu_launches": 2 * args.steps,
        "execution": f"value: CUDA graphs of {gsteps} consecutive decode calls (decode "
                     "overlap on), replayed",
        "clocks": clocks,
    }
    if model is not None:
        line["model_decode"] = model
    if world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline(q, pool, pt, kl)
        line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
    print(json.dumps(line), flush=True)


def run_seqsplit(args, rank: int, world: int, dev: torch.device):
    """Decode attention of BASELINE configs[3] at 131072 tokens (Qwen3-14B heads:
    40 q / 8 KV, D=128, 16-token pages, B=1), the sequence split over `world`
    GPUs: every rank streams its own page range from its own HBM, the fp32
    partial states are all-gathered over NCCL and merged.  Total work is
    fixed (strong scaling); time = max over ranks; value = algorithmic bytes of
    the whole attention / time."""
    from helm_b200.runtime.seq_parallel import SeqSplitAttention, split_ranges
    from helm_b200 import _capi
    Bq, Hq, Hkv, Dh, Pg, Tt = 1, 40, 8, 128, 16, 131072
    kv_bytes = Bq * Tt * Hkv * Dh * 2 * 2
    alg = kv_bytes + Bq * Hq * Dh * 2 * 2 + Bq * Hq * 4 + Bq * (Tt // Pg) * 4
    a, b = split_ranges(Tt, Pg, world)[rank]
    npg = -(-(b - a) // Pg)
    g = torch.Generator().manual_seed(1000 + rank)
    pool = torch.randn(npg + 8, 2, Hkv, Pg, Dh, generator=g).to(torch.bfloat16).to(dev)
    pt = torch.randperm(npg + 8, generator=g)[:npg].view(1, npg).to(torch.int32).to(dev)
    kl = torch.tensor([b - a], dtype=torch.int32, device=dev)
    q = torch.randn(Bq, Hq, Dh, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16).to(dev)
    sp = SeqSplitAttention(exchange=args.exchange)

    def step():
        return sp.decode(q, pool, pt, kl, num_kv_heads=Hkv, page_size=Pg, scale=Dh ** -0.5,
                         max_kv_len_hint=b - a)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    # the decode step (kernel, NCCL all-gather, merge) is replayed as one CUDA
    # graph: no host work between steps
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side), _capi.decode_overlap():
        step()
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(graph, stream=side):
            step()
    torch.cuda.current_stream(dev).wait_stream(side)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(dev)
    with ClockSampler(dev.index) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item()) / args.steps
    del graph  # graphs holding NCCL calls go before the process group
    sp.close()
    if _capi.device_status(dev) != 0:
        raise RuntimeError("device status reported an error")
    if rank == 0:
        line = {"metric": METRIC, "value": alg / (ms / 1e3) / 1e9, "unit": "GB/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic",
                "config": {"workload": "seqsplit128k: configs[3] attention, B=1, 40q/8kv, D=128, "
                                       "T=131072, 16-token pages, split over the GPUs, fp32 "
                                       "(O, LSE) exchanged and merged "
                                       + ("by one peer-memory kernel over NVLink"
                                          if args.exchange == "p2p" else
                                          "by NCCL all-gather + merge kernel"),
                           "exchange": args.exchange if world > 1 else "none (1 GPU)",
                           "tokens_per_gpu": b - a, "algorithmic_bytes_per_step": alg,
                           "attention_calls_per_s_one_layer": 1e3 / ms,
                           "parallelism": f"sequence split x{world}",
                           "execution": "CUDA graph replay of the whole step"},
                "gpu_launches": args.steps * (1 if world == 1 else 2),
                "clocks": clocks.summary()}
        print(json.dumps(line), flush=True)


MODEL_WORKLOADS = {
    # Qwen3-0.6B, 512-token prompt, 64 greedy steps, 64-token pages,
    # kv-offload on at the reference's default watermark (no page is evicted at 576 tokens)
    "config1": dict(arch="qwen3-0.6b", batch=1, prompt=512, steps=64, page=64, cold=0.0),
    # Qwen3-8B, 4096-token prompt, 256 steps, the oldest 75% of the
    # prompt's pages held in pinned host memory and staged per layer inside the step
    "config3": dict(arch="qwen3-8b", batch=1, prompt=4096, steps=256, page=64, cold=0.75),
}


TP_WORKLOADS = {
    # Qwen3-14B at 131072 tokens of context, B=1; KV heads and weights
    # sharded over the GPUs (tensor parallel), decode tok/s at N = 1, 2, 4, 8
    "config4": dict(name="qwen3-14b", dtype=torch.bfloat16, batch=1, context=131072, steps=128,
                    arch=dict(hidden=5120, layers=40, q_heads=40, kv_heads=8, head_dim=128,
                              intermediate=17408, vocab=151936, qk_norm=True, theta=1e6)),
    # Llama-2-13B fp16, B=16 x 2048-token contexts, MHA heads sharded
    "config5": dict(name="llama2-13b", dtype=torch.float16, batch=16, context=2048, steps=256,
                    arch=dict(hidden=5120, layers=40, q_heads=40, kv_heads=40, head_dim=128,
                              intermediate=13824, vocab=32000, qk_norm=False, theta=1e4)),
}


def _tp_decode(name: str, args, rank: int, world: int, dev: torch.device, steps: int,
               warmup: int, seq: bool = False, profile_step: bool = False) -> dict:
    """Decode tok/s of a tensor-parallel model over `world` GPUs (BASELINE
    configs[3] / configs[4]).  Random-init weights drawn per shard; the
    context's K/V pages are filled with N(0,1) values (prefill is not part of
    the decode metric and a 131072-token prefill is not timed here).  Total
    work is fixed as N grows (strong scaling); time = max over ranks.  Returns
    the measurements (every rank)."""
    from helm_b200 import _capi
    from helm_b200.runtime.seq_decode import SeqSplitDecodeModel
    from helm_b200.runtime.tp_decode import TPDecodeModel, synthetic_shard
    w = TP_WORKLOADS[name]
    K, W = steps, max(warmup, 3)
    Bq, ctx, arch = w["batch"], w["context"], w["arch"]
    e2e_steps = min(K, 32)
    if seq:   # the whole model on every rank (same seed), K/V split by token range
        shard = synthetic_shard(arch, 0, 1, w["dtype"], dev)
        tp = SeqSplitDecodeModel(shard, batch=Bq, context_len=ctx,
                                 max_new=3 + W + K + e2e_steps + 16, page_size=16)
    else:
        # --shard-of N on one GPU: rank 0's shard of an N-way split, run without the
        # exchange (per-rank kernel shapes of N GPUs, for profiling on one GPU)
        n_split = getattr(args, "shard_of", 0) or world
        shard = synthetic_shard(arch, rank if n_split == world else 0, n_split, w["dtype"], dev)
        tp = TPDecodeModel(shard, batch=Bq, max_len=ctx + 3 + W + K + e2e_steps + 16,
                           page_size=16)
    try:
        tp.fill_kv(ctx)
        for _ in range(3):
            tp.step()
        tp.capture()
        for _ in range(W):
            tp.replay()
        torch.cuda.synchronize(dev)

        def replays(n):
            for _ in range(n):
                tp.replay()
        ms_total, _, clocks = _timed(replays, K, world, dev, torch.cuda.current_stream(dev),
                                     False)
        ms = ms_total / K
        # end to end: every step's tokens read back to pinned host memory (streaming)
        host_tok = torch.empty(Bq, 1, dtype=torch.long).pin_memory()
        if world > 1:
            torch.distributed.barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            tp.replay()
            host_tok.copy_(tp.ids, non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()
        e2e_ms = (time.perf_counter() - t0) * 1e3 / e2e_steps
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        if world > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t[0])
        if profile_step:   # one eager step for `ncu --profile-from-start off`
            torch.cuda.synchronize(dev)
            torch.cuda.profiler.start()
            tp.step()
            torch.cuda.synchronize(dev)
            torch.cuda.profiler.stop()
        status = _capi.device_status(dev)
        # bytes this rank reads per step: its weight shard + its KV heads at the mean context
        wbytes = sum(x.numel() for lw in shard.layers for x in
                     (lw.wqkv, lw.wo, lw.wg, lw.wu, lw.wd)) * shard.embed.element_size()
        wbytes += shard.lm_head.numel() * shard.lm_head.element_size() + Bq * arch["hidden"] * 2
        mean_ctx = ctx + 3 + W + K / 2
        if seq:   # this rank's token range (the last rank also holds the new tokens)
            a, b = tp.range
            mean_ctx = (b - a) + ((3 + W + K / 2) if tp.tail else 0)
        kv_bytes = len(shard.layers) * Bq * mean_ctx * 2 * shard.hkv * shard.head_dim * 2
        n_layers = len(shard.layers)
    finally:
        tp.close()
        del tp, shard
        torch.cuda.empty_cache()
    _raise_on_status(status, world, dev)
    hbm, peak_src = _peaks()
    step_bytes = wbytes + kv_bytes
    achieved = step_bytes / (ms / 1e3) / 1e9
    return dict(w=w, K=K, W=W, Bq=Bq, ctx=ctx, ms=ms, e2e_ms=e2e_ms, clocks=clocks,
                wbytes=wbytes, kv_bytes=kv_bytes, step_bytes=step_bytes, achieved=achieved,
                hbm=hbm, peak_src=peak_src, n_layers=n_layers,
                tok_s=Bq / (ms / 1e3), roofline_tok_s=Bq / (step_bytes / (hbm * 1e9)),
                workload=(f"{name}: {w['name']} random-init, batch {Bq}, {ctx}-token context "
                          f"(K/V filled synthetically), greedy decode, 16-token pages, " + (
                              f"K/V sequence-split x{world} (token ranges), weights replicated"
                              if seq else
                              f"tensor parallel x{world} (KV heads, q/k/v/gate/up rows, "
                              f"o/down columns, lm_head vocab)")))


def run_tp(args, rank: int, world: int, dev: torch.device):
    w = TP_WORKLOADS[args.workload]
    seq = args.kv_split == "sequence"
    r = _tp_decode(args.workload, args, rank, world, dev,
                   args.steps if args.steps_given else w["steps"], args.warmup, seq=seq,
                   profile_step=args.profile_step)
    if rank != 0:
        return
    K, Bq = r["K"], r["Bq"]
    line = {"metric": METRIC, "value": r["tok_s"], "unit": "tok/s", "n_gpus": world,
            "steps": K, "warmup": r["W"], "ms_per_step": r["ms"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16" if w["dtype"] == torch.bfloat16 else "fp16",
            "data": "synthetic (random-init weight shards, N(0,1) K/V context)",
            "config": {"workload": r["workload"],
                       "execution": ("one CUDA graph replay per step; per layer the partial "
                                     "attention states (O, LSE) of the ranks are exchanged and "
                                     "merged over NVLink by one peer-memory kernel" if seq else
                                     "one CUDA graph replay per step; row-parallel projections "
                                     "all-reduce over NVLink inside the GEMV kernel; greedy pick "
                                     "by one NCCL all-gather"),
                       "l2": "weights + K/V per step exceed L2",
                       "parallelism": f"seq{world}" if seq else f"tp{world}"},
            "roofline": {"bound": "hbm", "achieved": r["achieved"], "peak": r["hbm"],
                         "unit": "GB/s", "frac": r["achieved"] / r["hbm"], "traffic": None,
                         "bytes_per_step_per_gpu": r["step_bytes"],
                         "weight_bytes_per_gpu": r["wbytes"],
                         "kv_bytes_per_step_per_gpu": r["kv_bytes"],
                         "roofline_tok_s": r["roofline_tok_s"], "peak_source": r["peak_src"]},
            "e2e": {"value": Bq / (r["e2e_ms"] / 1e3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": Bq * 8,
                    "note": "graph replay + per-step copy of the new tokens to pinned host "
                            "memory and a host sync (token streaming)"},
            "gpu_launches": ((8 if seq and world > 1 else 7) * r["n_layers"] + 1) * K,
            "clocks": r["clocks"]}
    print(json.dumps(line), flush=True)


def _model_block(r: dict, world: int) -> dict:
    """The config-4 decode summary carried in the default bench line."""
    return {"metric": "decode tok/s", "workload": r["workload"], "n_gpus": world,
            "tok_s": r["tok_s"], "ms_per_step": r["ms"], "steps": r["K"],
            "roofline_tok_s_per_gpu_bytes": r["roofline_tok_s"],
            "roofline_frac": r["achieved"] / r["hbm"], "achieved_gbs_per_gpu": r["achieved"],
            "bytes_per_step_per_gpu": r["step_bytes"],
            "e2e_tok_s": r["Bq"] / (r["e2e_ms"] / 1e3), "clocks": r["clocks"]}


GEMV_SHAPES = {  # one Qwen3-14B layer at batch 1: (rows, input width, SwiGLU)
    "qkv": (7168, 5120, False), "o": (5120, 5120, False), "gateup": (17408, 5120, True),
    "down": (5120, 17408, False),
    # the same layer's per-rank shapes under 8-way tensor parallelism
    "qkv_tp8": (896, 5120, False), "o_tp8": (5120, 640, False),
    "gateup_tp8": (2176, 5120, True), "down_tp8": (5120, 2176, False),
}


def run_gemv(args, rank: int, world: int, dev: torch.device):
    """Weight-streaming rate of helm_decode_gemv on the projection shapes of one
    Qwen3-14B layer (batch 1; RMSNorm fused on q/k/v and gate/up).  Each shape
    runs as CUDA graphs of 20 calls; value = weight bytes / time over all of
    them.  --gemv-shape restricts the run to one shape (eager calls only), the
    form used for an ncu capture."""
    from helm_b200 import _capi
    if world > 1:
        return _run_allreduce_gemv(args, rank, world, dev)
    tp8 = args.gemv_set == "tp8"
    shapes = [args.gemv_shape] if args.gemv_shape else \
        [n for n in GEMV_SHAPES if n.endswith("_tp8") == tp8]
    per, tot_bytes, tot_us = {}, 0, 0.0
    for name in shapes:
        N, K, glu = GEMV_SHAPES[name]
        g = torch.Generator(device=dev).manual_seed(0)
        # distinct weight copies in turn, so that consecutive calls stream more than L2
        nbytes = N * K * 2 * (2 if glu else 1)
        copies = min(20, max(1, -(-(256 << 20) // nbytes)))
        ws = [(torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
              for _ in range(copies)]
        w2s = [(torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
               if glu else None for _ in range(copies)]
        x = torch.randn(1, K, device=dev, generator=g).to(torch.bfloat16)
        nw = torch.ones(K, device=dev, dtype=torch.bfloat16) \
            if name.startswith(("qkv", "gateup")) else None
        y = torch.empty(1, N, device=dev, dtype=torch.bfloat16)
        turn = [0]

        def fn():
            i = turn[0] % copies
            turn[0] += 1
            _capi.decode_gemv(x, ws[i], out=y, norm_w=nw, w2=w2s[i])
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize(dev)
        if args.gemv_shape:
            for _ in range(args.steps):
                fn()
            torch.cuda.synchronize(dev)
            continue
        gr = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.cuda.graph(gr, stream=side):
            for _ in range(20):
                fn()
        torch.cuda.current_stream(dev).wait_stream(side)
        gr.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(1, args.steps // 20)
        e0.record()
        for _ in range(reps):
            gr.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) * 1e3 / (20 * reps)
        per[name] = {"rows": N, "k": K, "swiglu": glu, "us": us, "gbs": nbytes / us / 1e3}
        tot_bytes += nbytes
        tot_us += us
        del ws, w2s
    if rank != 0 or args.gemv_shape:
        return
    hbm, peak_src = _peaks()
    value = tot_bytes / tot_us / 1e3
    print(json.dumps({"metric": "decode GEMV weight-streaming rate (Qwen3-14B layer, batch 1)",
                      "value": value, "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
                      "warmup": args.warmup, "ms_per_step": tot_us / 1e3,
                      "higher_is_better": True, "scaling": "none", "vs_baseline": None,
                      "dtype": "bf16", "data": "synthetic",
                      "config": {"workload": "gemv: the four projections of one Qwen3-14B layer"
                                             + (" (per-rank shapes of 8-way tensor parallelism)"
                                                if tp8 else "")
                                             + "; consecutive calls use distinct weight copies "
                                               "(more than L2 per 20 calls)",
                                 "shapes": per},
                      "roofline": {"bound": "hbm", "achieved": value, "peak": hbm, "unit": "GB/s",
                                   "frac": value / hbm, "traffic": None,
                                   "peak_source": peak_src},
                      "gpu_launches": 20 * max(1, args.steps // 20) * len(per)}), flush=True)


def _run_allreduce_gemv(args, rank: int, world: int, dev: torch.device):
    """The row-parallel projections of one Qwen3-14B layer under `world`-way
    tensor parallelism (o_proj 5120 x 5120/N, down_proj 5120 x 17408/N, batch 1,
    residual fused): helm_decode_gemv_allreduce against the same GEMV without
    the exchange, each as CUDA graphs of 20 calls on rotating weight copies;
    time = max over ranks.  The difference is what the all-reduce costs."""
    from helm_b200 import _capi
    from helm_b200.runtime.tp_decode import _PeerBuffers
    shapes = {"o": (5120, 5120 // world), "down": (5120, 17408 // world)}
    peers = _PeerBuffers(_capi.decode_gemv_allreduce_bytes(5120, 1, world), dev, None, rank,
                         world)
    res = {}
    try:
        for name, (N, K) in shapes.items():
            g = torch.Generator(device=dev).manual_seed(rank)
            copies = min(20, max(1, -(-(256 << 20) // (N * K * 2))))
            ws = [(torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
                  for _ in range(copies)]
            x = torch.randn(1, K, device=dev, generator=g).to(torch.bfloat16)
            y = torch.zeros(1, N, device=dev, dtype=torch.bfloat16)
            for kind in ("plain", "allreduce"):
                def call(i, kind=kind):
                    if kind == "plain":
                        _capi.decode_gemv(x, ws[i % copies], out=y, residual=y)
                    else:
                        _capi.decode_gemv_allreduce(peers.ptrs, rank, x, ws[i % copies], out=y,
                                                    residual=y)
                for i in range(4):
                    call(i)
                torch.cuda.synchronize(dev)
                torch.distributed.barrier()
                gr = torch.cuda.CUDAGraph()
                side = torch.cuda.Stream(dev)
                side.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(side), torch.cuda.graph(gr, stream=side):
                    for i in range(20):
                        call(i)
                torch.cuda.current_stream(dev).wait_stream(side)
                gr.replay()
                reps = max(1, args.steps // 20)

                def replays(n, gr=gr, reps=reps):
                    for _ in range(reps):
                        gr.replay()
                ms, _, _ = _timed(replays, 1, world, dev, torch.cuda.current_stream(dev), False)
                res.setdefault(name, {"rows": N, "k": K})[kind + "_us"] = ms * 1e3 / (20 * reps)
                del gr
            res[name]["allreduce_cost_us"] = res[name]["allreduce_us"] - res[name]["plain_us"]
            del ws
        status = _capi.device_status(dev)
    finally:
        peers.close()
    if status != 0:
        raise RuntimeError(f"device status {status}")
    if rank == 0:
        print(json.dumps({"metric": "row-parallel GEMV with in-kernel all-reduce", "unit": "us",
                          "n_gpus": world, "higher_is_better": False, "shapes": res}), flush=True)


PREFILL = dict(Hq=40, Hkv=8, D=128, P=64, S=512)  # configs[3] (Qwen3-14B), one 512-token chunk


def run_prefill(args, rank: int, world: int, dev: torch.device):
    """Chunk-prefill attention of configs[3]: one layer's 512-query chunk over
    --seq-len cached tokens (default 131072, the prompt's last chunk), HELM's
    chunk-causal mask in bf16.  Times helm_paged_prefill_attention (pages read
    in place) and, beside it, the path it replaces: gather_kv to dense K/V +
    torch SDPA with the mask.  value = attention TFLOP/s of the native kernel
    (4 * S * Hq * T * D per call, every key of every row computed, as the
    reference's masked branch does).  Timed: the tcgen05 kernel (the default;
    HELM_B200_PREFILL_KERNEL=mma selects the mma.sync one) as
    _prefill_dense_pages calls it for HELM's chunk mask, which it recognises
    as chunk-causal (value); beside it the same kernel reading the mask, the
    mma.sync kernel and the gather + SDPA path."""
    import torch.nn.functional as F

    from helm_b200 import _capi
    c = PREFILL
    Tk = args.seq_len if args.seq_len_given else 131072
    S, Hq, Hkv, D, Pg = c["S"], c["Hq"], c["Hkv"], c["D"], c["P"]
    pages = Tk // Pg
    g = torch.Generator(device=dev).manual_seed(0)
    pool = torch.randn(pages + 8, 2, Hkv, Pg, D, device=dev, generator=g).to(torch.bfloat16)
    table = torch.randperm(pages + 8, device=dev, generator=g)[:pages].view(1, pages).to(torch.int32)
    lens = torch.tensor([Tk], dtype=torch.int32, device=dev)
    q = torch.randn(1, S, Hq, D, device=dev, generator=g).to(torch.bfloat16).transpose(1, 2)
    past = Tk - S
    i = torch.arange(S, device=dev).view(S, 1)
    j = torch.arange(Tk, device=dev).view(1, Tk)
    mask = torch.where(j <= past + i, 0.0, torch.finfo(torch.bfloat16).min)
    mask = mask.to(torch.bfloat16).view(1, 1, S, Tk)
    scale = D ** -0.5

    def native():
        return _capi.paged_prefill_attention(q, pool, table, lens, num_kv_heads=Hkv, page_size=Pg,
                                             scale=scale, max_kv_len=Tk, mask=mask)

    def gathered():
        k, v = _capi.gather_kv(pool, table, lens, Tk, num_kv_heads=Hkv, page_size=Pg)
        return F.scaled_dot_product_attention(q, k, v, attn_mask=mask, scale=scale,
                                              enable_gqa=True)

    def timed(fn, n):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / n

    def native_causal():  # HELM's chunk mask as _prefill_dense_pages passes it
        return _capi.paged_prefill_attention(q, pool, table, lens, num_kv_heads=Hkv, page_size=Pg,
                                             scale=scale, max_kv_len=Tk, causal=True)

    steps = args.steps if args.steps_given else 10
    a = native_causal().float()
    b = gathered().float()
    diff = float((a - b).abs().max())
    diff_mask = float((native().float() - b).abs().max())
    ms = timed(native_causal, steps)
    ms_mask = timed(native, max(1, steps // 2))
    # a left-padded prompt: HELM's padding mask as a first visible key
    pad = Tk // 32
    starts = torch.tensor([pad], dtype=torch.int32, device=dev)

    def native_padded():
        return _capi.paged_prefill_attention(q, pool, table, lens, num_kv_heads=Hkv, page_size=Pg,
                                             scale=scale, max_kv_len=Tk, causal=True,
                                             kv_starts=starts)
    ms_pad = timed(native_padded, max(1, steps // 2))
    ms_ref = timed(gathered, max(1, steps // 2))
    prev = os.environ.get("HELM_B200_PREFILL_KERNEL")
    try:   # the other kernels, for comparison
        os.environ["HELM_B200_PREFILL_KERNEL"] = "mma"
        ms_mma = timed(native_causal, max(1, steps // 2))
        os.environ["HELM_B200_PREFILL_KERNEL"] = "tc1"
        ms_tc1 = timed(native_causal, max(1, steps // 2))
        diff_tc1 = float((native_causal().float() - b).abs().max())
    finally:
        if prev is None:
            del os.environ["HELM_B200_PREFILL_KERNEL"]
        else:
            os.environ["HELM_B200_PREFILL_KERNEL"] = prev
    if rank != 0:
        return
    flop = 4.0 * S * Hq * Tk * D
    tflops = flop / (ms * 1e-3) / 1e12
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            peak, src = float(json.load(f)["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops)"
    except (OSError, KeyError, ValueError):
        peak, src = 1590.0, "fallback 1.59 PFLOP/s"
    print(json.dumps({"metric": "chunk-prefill attention TFLOP/s (configs[3] chunk, one layer)",
                      "value": tflops, "unit": "TFLOP/s", "n_gpus": 1, "steps": steps,
                      "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                      "scaling": "none", "vs_baseline": None, "dtype": "bf16",
                      "data": "synthetic",
                      "config": {"workload": f"prefill: 1 x {S} queries x {Hq}/{Hkv} heads over "
                                             f"{Tk} cached tokens, page {Pg}, HELM chunk mask",
                                 "kernel": {"mma": "mma.sync", "tc1": "tcgen05, one query "
                                            "tile per CTA"}.get(
                                     os.environ.get("HELM_B200_PREFILL_KERNEL"),
                                     "tcgen05, two query tiles per CTA"),
                                 "one_tile_tcgen05_kernel_ms": ms_tc1,
                                 "max_abs_diff_one_tile_vs_gather_sdpa": diff_tc1,
                                 "mask": "recognised as chunk-causal (causal limit, no mask reads)",
                                 "ms_with_mask_read": ms_mask,
                                 "left_padded_ms": ms_pad,
                                 "left_padded_note": f"first {pad} keys padded, given as a key "
                                                     "start (no mask reads)",
                                 "gather_sdpa_ms": ms_ref, "speedup_vs_gather_sdpa": ms_ref / ms,
                                 "mma_sync_kernel_ms": ms_mma,
                                 "max_abs_diff_vs_gather_sdpa": diff,
                                 "max_abs_diff_mask_read_vs_gather_sdpa": diff_mask},
                      "roofline": {"bound": "tensor", "achieved": tflops, "peak": peak,
                                   "unit": "TFLOP/s", "frac": tflops / peak, "traffic": None,
                                   "peak_source": src},
                      "gpu_launches": 2 * steps}), flush=True)


def _h2d_gbs(dev: torch.device, nbytes: int = 1 << 30) -> float:
    """Pinned host -> device copy bandwidth (best of 5), the link roofline."""
    h = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    d = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    best = 0.0
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        d.copy_(h, non_blocking=True)
        e1.record()
        e1.synchronize()
        best = max(best, nbytes / (e0.elapsed_time(e1) / 1e3) / 1e9)
    del h, d
    return best


def _time_cold_copies(gd, dev: torch.device, reps: int = 3) -> float:
    """Milliseconds the copy engine needs for one step's cold-page copies
    alone (the same per-layer copy lists the captured step issues, on an idle
    GPU, best of `reps`)."""
    from helm_b200 import _capi
    ctx = gd.ctx
    s = torch.cuda.Stream(dev)
    best = float("inf")
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record(s)
        for plan in ctx.cold_plan:
            for host_pool, srcs, dsts in plan:
                _capi.copy_pages(ctx.pool.storage, host_pool.storage, dsts, srcs, dev, stream=s)
        e1.record(s)
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    return best


def run_model(args, rank: int, world: int, dev: torch.device):
    """Decode tok/s of a whole model: random-init
    weights, random prompt, greedy decode through KVOffloadManager + GraphDecoder
    (every decode step one CUDA graph replay).  Timed: exactly K decode steps
    (steps 1..K of one generate call) with CUDA events, host bookkeeping and
    any re-capture included.  Every rank runs its own replica (weak scaling)."""
    from helm_b200.runtime.graph_decode import GraphDecoder
    from helm_b200.runtime.kv_cache import get_paging_stats, reset_paging_stats
    from helm_b200.runtime.kv_offload import KVOffloadConfig, KVOffloadManager
    from helm_b200.synthetic import build_model, make_config
    from helm_b200 import _capi
    w = MODEL_WORKLOADS[args.workload]
    K = args.steps if args.steps_given else w["steps"]
    cfg = make_config(w["arch"])
    model = build_model(cfg, seed=0, std=0.02, dtype=torch.bfloat16, device=dev)
    model.eval()
    Bq, S = w["batch"], w["prompt"]
    prompt = torch.randint(0, cfg.vocab_size, (Bq, S), generator=torch.Generator().manual_seed(0))
    prompt = prompt.pin_memory()
    L, Hkv, Dh = cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim
    tok_bytes = 2 * Hkv * Dh * 2                       # K+V of one token of one layer
    wm = None
    if w["cold"] > 0:     # keep the newest (1 - cold) of the prompt's pages on the GPU
        wm = int((1 - w["cold"]) * S * tok_bytes * L)
    kcfg = KVOffloadConfig.from_model(model, page_size=w["page"], gpu_watermark_bytes=wm)
    mgr = KVOffloadManager(model, kcfg)
    gd = GraphDecoder(model, mgr, max_len=S + K + 1, fused=args.stage == "fused")
    try:
        for _ in range(max(args.warmup, 3)):
            gd.generate(prompt.to(dev, non_blocking=True), 4)
        torch.cuda.synchronize(dev)
        if world > 1:
            torch.distributed.barrier()
        reset_paging_stats()
        with ClockSampler(dev.index) as clocks:
            t0 = time.perf_counter()
            toks = gd.generate(prompt.to(dev, non_blocking=True), K + 1)
            toks_host = toks.cpu()
            wall = time.perf_counter() - t0
        ms = gd.decode_ms() / K
        stats = get_paging_stats()
        h2d_step = gd.h2d_bytes / K
        plan_ms = (gd.plan_seconds - gd.plan_wait_seconds) * 1e3 / K
        wait_ms = gd.plan_wait_seconds * 1e3 / K
        captures = gd.captures
        prefetch = None
        if w["cold"] > 0:
            # the two bounds of a step with cold pages, measured: the step's copies alone
            # on the copy engine, and the same decode with every page resident in HBM
            copy_ms = _time_cold_copies(gd, dev)
            mgr.restore()
            mgr = KVOffloadManager(model, KVOffloadConfig.from_model(
                model, page_size=w["page"], gpu_watermark_bytes=1 << 50))
            gd_hot = GraphDecoder(model, mgr, max_len=S + K + 1, fused=args.stage == "fused")
            gd_hot.generate(prompt.to(dev, non_blocking=True), 4)
            gd_hot.generate(prompt.to(dev, non_blocking=True), K + 1)
            hot_ms = gd_hot.decode_ms() / K
            prefetch = {"copy_alone_ms_per_step": copy_ms, "all_resident_ms_per_step": hot_ms,
                        "h2d_gbs_copy_alone": h2d_step / (copy_ms / 1e3) / 1e9,
                        "overlap": ms / max(copy_ms, hot_ms),
                        "note": "overlap = step time / max(copies alone, all-resident step); "
                                "1.0 = the slower of the two fully hides the other"}
    finally:
        mgr.restore()
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    if _capi.device_status(dev) != 0:
        raise RuntimeError("device status reported an error")
    if rank != 0:
        return
    n_params = sum(p.numel() for p in model.parameters())
    embed = model.get_input_embeddings().weight
    tied = model.get_output_embeddings().weight.data_ptr() == embed.data_ptr()
    # every weight is read once per step; an untied input embedding only by its B rows
    weight_bytes = (n_params - (0 if tied else embed.numel())) * 2
    mean_ctx = S + (K + 1) / 2
    kv_step = L * Bq * mean_ctx * tok_bytes
    step_bytes = weight_bytes + kv_step
    hbm, peak_src = _peaks()
    link = _h2d_gbs(dev)
    achieved = step_bytes / (ms / 1e3) / 1e9
    t_floor = max(step_bytes / (hbm * 1e9), h2d_step / (link * 1e9)) * 1e3
    line = {"metric": METRIC, "value": world * Bq / (ms / 1e3), "unit": "tok/s",
            "n_gpus": world, "steps": K, "warmup": max(args.warmup, 3), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (random-init weights, uniform random prompt)",
            "config": {"workload": f"{args.workload}: {w['arch']} random-init bf16, batch {Bq}, "
                                   f"{S}-token prompt, {K} greedy decode steps, "
                                   f"{w['page']}-token pages, "
                                   f"{int(w['cold'] * 100)}% of prompt pages host-resident",
                       "execution": "one CUDA graph replay per decode step (re-captured when "
                                    "the cold page set changes)",
                       "stage": ("FusedDecodeStage: 7 launches per layer (fused RMSNorm/SwiGLU/"
                                 "residual GEMVs, fused append, paged attention)"
                                 if args.stage == "fused" else
                                 "HF modules with the patched attention forward"),
                       "l2": "weights + KV per step exceed L2",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": None,
                         "bytes_per_step": step_bytes, "weight_bytes": weight_bytes,
                         "kv_bytes_per_step_mean": kv_step,
                         "h2d_bytes_per_step": h2d_step, "h2d_link_gbs_measured": link,
                         "h2d_gbs_achieved": h2d_step / (ms / 1e3) / 1e9,
                         "h2d_frac_of_link": h2d_step / (ms / 1e3) / 1e9 / link,
                         "step_floor_ms": t_floor, "frac_of_floor": t_floor / ms,
                         "peak_source": peak_src},
            "e2e": {"value": Bq * (K + 1) / wall, "unit": "tok/s",
                    "h2d_bytes_per_step": prompt.numel() * 8 / (K + 1),
                    "d2h_bytes_per_step": toks_host.numel() * 8 / (K + 1),
                    "note": "one generate() call from a pinned host prompt to host tokens, "
                            "prefill and graph captures included"},
            "prefetch": prefetch,
            "host_plan_ms_per_step": plan_ms,
            "host_wait_ms_per_step": wait_ms,   # the host ahead of the GPU: waits on uploads
            "graph_captures": captures,
            "paging": stats,
            # this library's kernels per step: per layer append + attention (+ merge) and,
            # with the fused stage, four GEMVs; plus the lm_head GEMV
            "gpu_launches": (7 * L + 1 if args.stage == "fused" else 3 * L) * K,
            "clocks": clocks.summary()}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=["config2", "seqsplit128k", "gemv", "prefill"]
                    + sorted(MODEL_WORKLOADS) + sorted(TP_WORKLOADS),
                    default="config2",
                    help="config2 (default, BASELINE configs[1]); the 128k-token attention of "
                         "configs[3] split across the GPUs (strong scaling); or whole-model "
                         "decode tok/s of configs[0] (config1) / configs[2] (config3)")
    ap.add_argument("--gemv-set", choices=["full", "tp8"], default="full",
                    help="gemv workload: the layer's shapes on one GPU, or one rank's under "
                         "8-way tensor parallelism")
    ap.add_argument("--gemv-shape", choices=sorted(GEMV_SHAPES), default=None,
                    help="gemv workload: run one shape with eager calls (for an ncu capture)")
    ap.add_argument("--profile-step", action="store_true",
                    help="config4/config5: also run one eager step between "
                         "cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    ap.add_argument("--stage", choices=["fused", "hf"], default="fused",
                    help="config1/config3: decode step as FusedDecodeStage or as HF modules")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="seqsplit128k: how partial states cross GPUs")
    ap.add_argument("--kv-split", choices=["head", "sequence"], default="head",
                    help="config4/config5 over N GPUs: tensor parallel with KV heads sharded "
                         "(head), or the whole model on every rank with the K/V split by "
                         "token range and partial states merged over NVLink (sequence)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--shard-of", type=int, default=0,
                    help="config4/config5 on one GPU: run rank 0's shard of an N-way tensor-"
                         "parallel split without the exchange (per-rank shapes, profiling)")
    ap.add_argument("--no-model-block", action="store_true",
                    help="default workload: skip the config-4 model-decode block")
    ap.add_argument("--seq-len", type=int, default=T,
                    help="tokens per sequence (profiling a smaller case only; for the "
                         "prefill workload, the cached tokens, default 131072)")
    ap.add_argument("--pool-pages", type=int, default=POOL,
                    help="page-pool slots (profiling a smaller case only)")
    args = ap.parse_args()
    args.steps_given = args.steps is not None
    args.seq_len_given = args.seq_len != T
    if args.steps is None:
        args.steps = 50
    _set_shape(args.seq_len, args.pool_pages)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=120),
                                             device_id=dev)
    try:
        if args.workload == "seqsplit128k":
            run_seqsplit(args, rank, world, dev)
        elif args.workload in MODEL_WORKLOADS:
            run_model(args, rank, world, dev)
        elif args.workload in TP_WORKLOADS:
            run_tp(args, rank, world, dev)
        elif args.workload == "gemv":
            run_gemv(args, rank, world, dev)
        elif args.workload == "prefill":
            run_prefill(args, rank, world, dev)
        else:
            run_b200(args, rank, world, dev)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
