#!/usr/bin/env python
"""Benchmark of the B200 paged-MHA forward (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl fgw_b200|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Headline workload (the one the reference's headline MFU is quoted on):
B2 H8 Q4096 KV2048 BF16 D128, 128-token pages with a shuffled block table, non-causal, N(0,1)
synthetic data. A step is one forward call over that batch. With N GPUs every rank runs its own
batch of 2 (weak scaling: per-GPU work fixed, global batch 2N), with no collective on the data path.
The L2 (126 MB) is flushed with a 256 MiB write before every timed step, since the step's inputs
(50 MB) would otherwise stay cached.

Also measured in the same line (``decode``): BASELINE config 5, B256 H32 Q1 KV log-uniform in
[1024, 32768], BF16 D128, 64-token pages scattered in a shared pool (~38 GB of K+V), sharded by head
across the N ranks (strong scaling: whole-box microseconds per call, max over ranks).

And (``gather``): the paged-cache gather pre-pass on the same config-5 pool — both K and V of every
request packed densely (live lengths rounded up to whole pages, the layout of FGW's gather experiment),
HBM-bound; the ``attend_after_gather`` field times the decode attention over the packed copy.

``--impl reference`` times the reference algorithm on the host cores instead: FGW's CPU FP32
reference restated in NumPy (``oracle/``; the reference itself is Python on an Ascend stack and cannot
run here), on the same headline workload, rank 0 only.
"""
import argparse
import contextlib
import json
import math
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "µs/call + % roofline (TC TFLOP/s long-Q, HBM GB/s decode) at 1/2/4/8 B200"
LONGQ = dict(batch=2, sq=4096, heads=8, dim=128, page=128, kv=2048)
DECODE = dict(batch=256, sq=1, heads=32, dim=128, page=64, kv_lo=1024, kv_hi=32768)
ASCEND_V7_TFLOPS = 237.4  # FGW's published figure: v7 persistent28, B2H8 Q4096 KV2048, Ascend 950PR
FLUSH_BYTES = 256 << 20


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["fgw_b200", "reference"], default="fgw_b200")
    p.add_argument("--no-decode", action="store_true", help="skip the config-5 decode measurement")
    p.add_argument("--no-gather", action="store_true", help="skip the gather pre-pass measurement")
    p.add_argument("--sweep-splits", default=None, metavar="JSON",
                   help="run the config-3 split sweep instead, write its rows to JSON and print a summary line")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--path", choices=["auto", "decode", "tensor"], default="auto")
    p.add_argument("--splits", type=int, default=None, help="force num_splits for the headline workload")
    p.add_argument("--tensor-kernel", choices=["auto", "pairs", "single", "halves"], default="auto",
                   help="tcgen05 kernel of the long-query workloads")
    p.add_argument("--task-assignment", choices=["strided", "contiguous", "tail"], default=None,
                   help="schedule of the long-query workloads (default: the library's choice)")
    p.add_argument("--only", choices=["longq", "decode", "d256"], default=None,
                   help="measure one workload (profiling): config 2, config 5, or config 2's shape at D = 256")
    p.add_argument("--decode-batch", type=int, default=DECODE["batch"],
                   help="requests in the decode workload (smaller values make profiling captures small)")
    return p.parse_args(argv)


# ----------------------------------------------------------------------------------------------- setup
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def init_dist(world, local):
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def _reduce_over_ranks(value, world, op):
    if world == 1:
        return value
    import torch.distributed as dist
    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=op)
    return float(t.item())


def max_over_ranks(value, world):
    import torch.distributed as dist
    return _reduce_over_ranks(value, world, dist.ReduceOp.MAX if world > 1 else None)


def sum_over_ranks(value, world):
    import torch.distributed as dist
    return _reduce_over_ranks(value, world, dist.ReduceOp.SUM if world > 1 else None)


def head_shard(heads, rank, world):
    """Decode is sharded by heads: rank r holds heads [r*H/N, (r+1)*H/N) of every page (H divisible by N)."""
    if heads % world:
        raise ValueError(f"{heads} heads do not split evenly over {world} ranks")
    per = heads // world
    return rank * per, per


@contextlib.contextmanager
def local_host_memory(device):
    """Pinned host buffers made inside this block land on the GPU's own NUMA node: the process runs on the CPUs
    NVML reports as closest to the GPU while they are allocated (the pages are placed where they are first
    touched), and its CPU affinity is restored afterwards. Host-to-device copies from a remote node cross the
    inter-socket link, which several ranks then share. Does nothing where NVML or the affinity call is missing."""
    saved = None
    try:
        import pynvml
        pynvml.nvmlInit()
        try:
            prop = torch.cuda.get_device_properties(device)
            bus = f"{prop.pci_domain_id:08x}:{prop.pci_bus_id:02x}:{prop.pci_device_id:02x}.0"
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            words = pynvml.nvmlDeviceGetCpuAffinity(handle, ((os.cpu_count() or 64) + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        cpus = {64 * w + bit for w, word in enumerate(words) for bit in range(64) if (word >> bit) & 1}
        current = os.sched_getaffinity(0)
        if cpus & current:
            saved = current
            os.sched_setaffinity(0, cpus & current)
    except Exception:  # no NVML, no such device, or no affinity control: allocate where we are
        saved = None
    try:
        yield
    finally:
        if saved is not None:
            os.sched_setaffinity(0, saved)


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return data["hbm_gbs"], data["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------------------------------------- inputs
def longq_inputs(seed, device, sq=None, **shape):
    """Config 2's inputs (``shape`` overrides batch / heads / dim / kv / page; ``pool_pages`` draws the table from
    a larger pool, as config 1's 16 of 64 pages)."""
    c = dict(LONGQ, sq=sq or LONGQ["sq"], **{k: v for k, v in shape.items() if k != "pool_pages"})
    width = c["kv"] // c["page"]
    gen = torch.Generator().manual_seed(seed)
    pool_pages = shape.get("pool_pages", c["batch"] * width)
    table = torch.randperm(pool_pages, generator=gen)[: c["batch"] * width].reshape(c["batch"], width).to(torch.int32)
    lengths = torch.full((c["batch"],), c["kv"], dtype=torch.int32)
    pool_rows = pool_pages * c["page"]
    gdev = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(c["batch"], c["sq"], c["heads"], c["dim"], generator=gdev, device=device).to(torch.bfloat16)
    k = torch.randn(pool_rows, c["heads"], c["dim"], generator=gdev, device=device).to(torch.bfloat16)
    v = torch.randn(pool_rows, c["heads"], c["dim"], generator=gdev, device=device).to(torch.bfloat16)
    return {"q": q, "k": k, "v": v, "table": table.to(device), "lengths": lengths.to(device),
            "host_lengths": lengths.tolist(), "width": width, "page": c["page"], "causal": False}


def decode_lengths(seed, batch):
    c = DECODE
    rng = np.random.default_rng(seed)
    logs = rng.uniform(math.log(c["kv_lo"]), math.log(c["kv_hi"]), size=batch)
    return np.minimum(np.floor(np.exp(logs)).astype(np.int64), c["kv_hi"])


def decode_inputs(seed, rank, world, device, batch):
    """Config 5, head-sharded: this rank holds heads [rank*H/N, (rank+1)*H/N) of every page."""
    c = dict(DECODE, batch=batch)
    lengths = decode_lengths(seed, batch)
    pages_per = (lengths + c["page"] - 1) // c["page"]
    width = int(pages_per.max())
    total_pages = int(pages_per.sum())
    rng = np.random.default_rng(seed + 1)
    perm = rng.permutation(total_pages + 8)[:total_pages]  # pages scattered over a slightly larger pool
    table = np.zeros((c["batch"], width), dtype=np.int32)
    start = 0
    for b, n in enumerate(pages_per):
        table[b, :n] = perm[start:start + n]
        start += n
    pool_rows = (total_pages + 8) * c["page"]
    _, heads = head_shard(c["heads"], rank, world)
    gdev = torch.Generator(device=device).manual_seed(seed + 17 * rank)
    q = torch.randn(c["batch"], 1, heads, c["dim"], generator=gdev, device=device).to(torch.bfloat16)
    k = torch.empty(pool_rows, heads, c["dim"], dtype=torch.bfloat16, device=device)
    v = torch.empty_like(k)
    chunk = 1 << 20
    for t in (k, v):
        flat = t.view(-1)
        for i in range(0, flat.numel(), chunk * 64):
            n = min(chunk * 64, flat.numel() - i)
            flat[i:i + n] = torch.randn(n, generator=gdev, device=device, dtype=torch.float32).to(torch.bfloat16)
    return {"q": q, "k": k, "v": v, "table": torch.from_numpy(table).to(device),
            "lengths": torch.from_numpy(lengths.astype(np.int32)).to(device), "host_lengths": lengths.tolist(),
            "width": width, "page": c["page"], "causal": False, "heads": heads}


# --------------------------------------------------------------------------------------------- helpers
class ClockSampler:
    """nvidia-smi clock/throttle sampling while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.device_index = device_index
        self.proc = None
        self.file = None

    def __enter__(self):
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader",
                 "-lms", "200"], stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.file.flush()

    def summary(self):
        rows = []
        try:
            text = pathlib.Path(self.file.name).read_text()
        finally:
            os.unlink(self.file.name)
        for line in text.splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1].split()[0]), float(parts[2].split()[0]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        loaded = [r for r in rows if r[0] > 500] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, flag in enumerate(r[2]) if flag.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def timed_steps(step_fns, steps, warmup, flush, stream):
    """Run warmup + steps; per step, flush L2 (untimed) then time each stage with events.

    step_fns: list of (name, fn) run in order each step. Returns {name: [ms per step]} and total list.
    """
    for _ in range(warmup):
        for _, fn in step_fns:
            fn()
    torch.cuda.synchronize()
    per = {name: [] for name, _ in step_fns}
    totals = []
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(len(step_fns) + 1)] for _ in range(steps)]
    for i in range(steps):
        if flush is not None:
            flush.zero_()
        ev = events[i]
        ev[0].record(stream)
        for j, (_, fn) in enumerate(step_fns):
            fn()
            ev[j + 1].record(stream)
    torch.cuda.synchronize()
    for i in range(steps):
        ev = events[i]
        for j, (name, _) in enumerate(step_fns):
            per[name].append(ev[j].elapsed_time(ev[j + 1]))
        totals.append(ev[0].elapsed_time(ev[-1]))
    return per, totals


def flops_of(inp, sq, heads, dim):
    from fgw_b200.operators.mha.work import useful_flops  # the reference's FLOP policy (bench_mha_mfu.py:63-66)
    return useful_flops(inp["host_lengths"], sq, heads, dim, inp["causal"])


def bytes_of(inp, batch, sq, heads, dim):
    from fgw_b200.operators.mha.work import algorithmic_bytes
    return algorithmic_bytes(inp["host_lengths"], batch, sq, heads, dim, inp["width"], 2)


# ------------------------------------------------------------------------------------------ our kernels
def run_longq(args, rank, world, device, stream):
    from fgw_b200.operators.mha.current import build_kernel, mha_paged_decode
    c = LONGQ
    inp = longq_inputs(1000 + rank, device)
    kernel = build_kernel(c["batch"], c["sq"], c["heads"], c["dim"], inp["k"].shape[0], inp["width"], c["page"],
                          False, "bfloat16", device.index, num_splits=args.splits,
                          full_kv_cache=True, path=args.path, tensor_kernel=args.tensor_kernel,
                          task_assignment=args.task_assignment)
    ws = kernel.new_workspace(device)
    out = torch.empty_like(inp["q"])
    a = (inp["q"], inp["k"], inp["v"], inp["table"], inp["lengths"])
    fns = [("plan", lambda: kernel.plan_kernel(*a, ws)), ("attend", lambda: kernel.attend_kernel(*a, ws, out))]
    if kernel.num_splits > 1:
        fns.append(("merge", lambda: kernel.merge_only(*a, ws, out)))
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=device)
    flops = flops_of(inp, c["sq"], c["heads"], c["dim"])
    barrier(world)
    torch.cuda.synchronize()
    per, totals = timed_steps(fns, args.steps, args.warmup, flush, stream)
    torch.cuda.synchronize()
    barrier(world)
    eager_step_ms = sum(totals) / len(totals)
    attend_ms = sum(per["attend"]) / len(per["attend"])

    # The same step captured once as a CUDA graph and replayed: no host launch gaps between the planning
    # and attention launches. This is the step time `value` reports.
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _, fn in fns:
            fn()
    torch.cuda.current_stream(device).wait_stream(side)
    with torch.cuda.graph(graph):
        for _, fn in fns:
            fn()
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(device.index) as clocks:
        _, graph_totals = timed_steps([("step", graph.replay)], args.steps, args.warmup, flush, stream)
        torch.cuda.synchronize()
        barrier(world)
    step_ms = sum(graph_totals) / len(graph_totals)

    # The reference's own protocol (bench_mha_mfu.py:221-247): median of 51 CUDA-event samples after 20
    # warm-ups, with a warm L2 and with the L2 flushed before every sample. Outside the K timed steps above.
    protocol = {}
    for name, fl in (("warm_l2", None), ("flushed_l2", flush)):
        _, samples = timed_steps([("step", graph.replay)], 51, 20, fl, stream)
        protocol[name + "_us_median"] = statistics.median(samples) * 1e3

    # End to end through the public API: pinned host inputs -> device -> forward -> host output, every step.
    with local_host_memory(device):
        host = {k: inp[k].cpu().pin_memory() for k in ("q", "k", "v", "table", "lengths")}
        host_out = torch.empty(inp["q"].shape, dtype=inp["q"].dtype, pin_memory=True)
        host_outs = [torch.empty(inp["q"].shape, dtype=inp["q"].dtype, pin_memory=True) for _ in range(2)]
    dev_bufs = {k: torch.empty_like(inp[k]) for k in host}

    def forward(bufs, out_buf):
        return mha_paged_decode(bufs["q"], bufs["k"], bufs["v"], bufs["table"], bufs["lengths"], c["page"], False,
                                num_splits=args.splits, path=args.path, cache_lengths=inp["host_lengths"], out=out_buf,
                                tensor_kernel=args.tensor_kernel, task_assignment=args.task_assignment)

    def e2e_step():
        for key in host:
            dev_bufs[key].copy_(host[key], non_blocking=True)
        host_out.copy_(forward(dev_bufs, None), non_blocking=True)

    e2e_steps = max(3, args.steps // 2)
    _, e2e_totals = timed_steps([("e2e", e2e_step)], e2e_steps, 2, flush, stream)
    e2e_serial_ms = statistics.median(e2e_totals)
    # The same steps as a serving loop runs them: double-buffered inputs and outputs on three streams, so step
    # i + 1's upload overlaps step i's forward and download (the two copy directions use different engines).
    sets = [{k: torch.empty_like(inp[k]) for k in host} for _ in range(2)]
    outs = [torch.empty_like(inp["q"]) for _ in range(2)]
    s_up, s_comp, s_down = (torch.cuda.Stream(device) for _ in range(3))
    uploaded, computed, downloaded = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))

    def pipelined(n):
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for st in (s_up, s_comp, s_down):
            st.wait_event(start)
        for i in range(n):
            b = i % 2
            with torch.cuda.stream(s_up):
                if i >= 2:
                    s_up.wait_event(computed[b])  # step i - 2 has finished reading this input set
                for key in host:
                    sets[b][key].copy_(host[key], non_blocking=True)
                uploaded[b].record(s_up)
            with torch.cuda.stream(s_comp):
                s_comp.wait_event(uploaded[b])
                if i >= 2:
                    s_comp.wait_event(downloaded[b])  # step i - 2's output has reached the host
                forward(sets[b], outs[b])
                computed[b].record(s_comp)
            with torch.cuda.stream(s_down):
                s_down.wait_event(computed[b])
                host_outs[b].copy_(outs[b], non_blocking=True)
                downloaded[b].record(s_down)
        for b in range(min(n, 2)):
            stream.wait_event(downloaded[b])
        end.record(stream)
        torch.cuda.synchronize()
        return start.elapsed_time(end) / n

    pipelined(4)
    e2e_ms = pipelined(max(e2e_steps, 10))
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = host_out.numel() * host_out.element_size()
    # parity spot check of the benchmarked output (first request, first 256 query rows), PyTorch FP32
    ok = check_longq(inp, out)
    del graph
    return {"kernel": kernel, "inp": inp, "flops": flops, "step_ms": step_ms, "attend_ms": attend_ms,
            "eager_step_ms": eager_step_ms, "protocol": protocol, "e2e_serial_ms": e2e_serial_ms,
            "per": per, "e2e_ms": e2e_ms, "h2d": h2d, "d2h": d2h, "clocks": clocks.summary(), "parity": ok,
            "launches_per_step": len(fns)}


def run_longq_shape(args, rank, world, device, stream, seed, sq, steps=None, **shape):
    """One more long-query (or config-1) shape: plan + attend per step with the L2 flushed, per-stage events; and the
    same step replayed as a CUDA graph (what a serving loop that captures its launches pays per call)."""
    from fgw_b200.operators.mha.current import build_kernel
    c = dict(LONGQ, sq=sq, **{k: v for k, v in shape.items() if k != "pool_pages"})
    inp = longq_inputs(seed + rank, device, sq=sq, **shape)
    kernel = build_kernel(c["batch"], sq, c["heads"], c["dim"], inp["k"].shape[0], inp["width"], c["page"],
                          False, "bfloat16", device.index, num_splits=args.splits, full_kv_cache=True, path=args.path,
                          tensor_kernel=args.tensor_kernel)
    ws = kernel.new_workspace(device)
    out = torch.empty_like(inp["q"])
    a = (inp["q"], inp["k"], inp["v"], inp["table"], inp["lengths"])
    fns = [("plan", lambda: kernel.plan_kernel(*a, ws)), ("attend", lambda: kernel.attend_kernel(*a, ws, out))]
    if kernel.num_splits > 1:
        fns.append(("merge", lambda: kernel.merge_only(*a, ws, out)))
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=device)
    barrier(world)
    torch.cuda.synchronize()
    steps = steps or max(3, args.steps // 4)
    # per-stage events (plan, attend[, merge]) for the attend kernel's roofline
    per, _ = timed_steps(fns, steps, 3, flush, stream)
    # the call itself (the launch callable: plan + attend, split partials merged in place on the decode path),
    # eager and replayed as a CUDA graph (captured as the headline's is), L2 flushed before each
    call = [("call", lambda: kernel(*a, out=out, workspace=ws))]
    # launches of one call: plan + attend, plus the merge launch of a split tensor-path call
    per_call = 2 + (1 if kernel.num_splits > 1 and kernel.execution_path != "sm100_decode" else 0)
    _, totals = timed_steps(call, steps, 3, flush, stream)
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        call[0][1]()
    torch.cuda.current_stream(device).wait_stream(side)
    with torch.cuda.graph(graph):
        call[0][1]()
    torch.cuda.synchronize()
    _, graph_ms = timed_steps([("step", graph.replay)], steps, 3, flush, stream)
    torch.cuda.synchronize()
    del graph
    barrier(world)
    ok = check_longq(inp, out)
    return {"flops": flops_of(inp, sq, c["heads"], c["dim"]),
            "bytes": bytes_of(inp, c["batch"], sq, c["heads"], c["dim"]),
            "step_ms": sum(totals) / len(totals), "graph_ms": statistics.median(graph_ms),
            "attend_ms": sum(per["attend"]) / len(per["attend"]), "parity": ok,
            "launches": (len(fns) + 2 * per_call) * steps, "num_splits": kernel.num_splits,
            "task_assignment": kernel.task_assignment, "execution_path": kernel.execution_path}


def run_longq_32k(args, rank, world, device, stream):
    """Config 2's second size (Q = 32768, KV 2048)."""
    return run_longq_shape(args, rank, world, device, stream, 2000, 32768)


def torch_reference(q, keys, values, scale):
    """Plain PyTorch FP32 attention of query rows q [R, H, D] over keys/values [N, H, D] (all visible)."""
    s = torch.einsum("rhd,nhd->hrn", q.float(), keys.float()) * scale
    return torch.einsum("hrn,nhd->rhd", torch.softmax(s, dim=-1), values.float())


def live_rows(table_row, length, page, device):
    """Pool rows of a request's first `length` tokens, in logical order."""
    pages = table_row[: (length + page - 1) // page].long()
    return (pages[:, None] * page + torch.arange(page, device=device)[None, :]).reshape(-1)[:length]


def check_longq(inp, out):
    """Spot check of the benchmarked output (first request, first 256 query rows) against a PyTorch FP32
    reference of the same attention."""
    rows = min(256, out.shape[1])
    idx = live_rows(inp["table"][0], inp["host_lengths"][0], inp["page"], out.device)
    want = torch_reference(inp["q"][0, :rows], inp["k"][idx], inp["v"][idx], inp["q"].shape[-1] ** -0.5)
    err = float((out[0, :rows].float() - want).abs().max())
    return {"rows_checked": rows, "max_abs_err": err, "pass": bool(err <= 2e-2), "reference": "torch fp32"}


def run_decode(args, rank, world, device, stream):
    from fgw_b200.operators.mha.current import build_kernel
    c = dict(DECODE, batch=args.decode_batch)
    inp = decode_inputs(4242, rank, world, device, args.decode_batch)
    heads = inp["heads"]
    kernel = build_kernel(c["batch"], 1, heads, c["dim"], inp["k"].shape[0], inp["width"], c["page"], False,
                          "bfloat16", device.index, cache_lengths=tuple(inp["host_lengths"]), path="decode")
    ws = kernel.new_workspace(device)
    out = torch.empty_like(inp["q"])
    a = (inp["q"], inp["k"], inp["v"], inp["table"], inp["lengths"])
    fns = [("plan", lambda: kernel.plan_kernel(*a, ws)), ("attend", lambda: kernel.attend_kernel(*a, ws, out))]
    if kernel.num_splits > 1:
        fns.append(("merge", lambda: kernel.merge_only(*a, ws, out)))
    barrier(world)
    torch.cuda.synchronize()
    steps = max(5, args.steps // 2)
    per, totals = timed_steps(fns, steps, max(3, args.warmup // 2), None, stream)
    torch.cuda.synchronize()
    barrier(world)
    step_ms = sum(totals) / len(totals)
    attend_ms = sum(per["attend"]) / len(per["attend"])
    nbytes = bytes_of(inp, c["batch"], 1, heads, c["dim"])
    # parity spot check: 4 requests of this shard against a PyTorch FP32 reference
    idx = [0, 1, 2, 3]
    err = 0.0
    for b in idx:
        rows = live_rows(inp["table"][b], inp["host_lengths"][b], c["page"], device)
        want = torch_reference(inp["q"][b], inp["k"][rows], inp["v"][rows], c["dim"] ** -0.5)
        err = max(err, float((out[b].float() - want).abs().max()))
    return {"kernel": kernel, "step_ms": step_ms, "attend_ms": attend_ms, "bytes": nbytes, "per": per,
            "parity": {"requests_checked": len(idx), "max_abs_err": err, "pass": bool(err <= 2e-2),
                       "reference": "torch fp32"},
            "launches_per_step": len(fns), "steps": steps, "inp": inp, "out": out}


def run_decode_serving(args, dc, rank, world, device, stream):
    """Config 5 as a serving loop runs it: every step the cache lengths grow by one token (each request appends
    one), the step's query rows and lengths are uploaded from pinned host memory, the forward goes through the
    product API (mha_paged_decode_sharded: this rank's heads) with the host copy of the new lengths, and the
    output is read back. The launcher is cached per shape and split count, so new lengths cost no rebuild;
    ``host_us_per_call`` is the host time the API call itself takes (median), the rest is device time."""
    from fgw_b200.operators.mha.sharded import mha_paged_decode_sharded
    inp = dc["inp"]
    steps = max(10, args.steps)
    base = np.asarray(inp["host_lengths"], dtype=np.int32)  # the cache_seqlens dtype, kept on the host as well
    with local_host_memory(device):
        host_q = inp["q"].cpu().pin_memory()
        host_len = torch.empty(base.shape[0], dtype=torch.int32).pin_memory()
        host_out = torch.empty(inp["q"].shape, dtype=inp["q"].dtype).pin_memory()
    dev_q, dev_len = torch.empty_like(inp["q"]), torch.empty_like(inp["lengths"])
    out = torch.empty_like(inp["q"])
    schedule = [np.maximum(base - (steps + 3 - i), 1) for i in range(steps + 3)]  # grows to the config's lengths
    host_us, events = [], []
    for i, lengths in enumerate(schedule):
        host_len.numpy()[:] = lengths
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        dev_q.copy_(host_q, non_blocking=True)
        dev_len.copy_(host_len, non_blocking=True)
        t0 = time.perf_counter()
        mha_paged_decode_sharded(dev_q, inp["k"], inp["v"], inp["table"], dev_len, inp["page"], shard="heads",
                                 cache_lengths=lengths, out=out)
        host_us.append((time.perf_counter() - t0) * 1e6)
        host_out.copy_(out, non_blocking=True)
        e1.record(stream)
        events.append((e0, e1))
    torch.cuda.synchronize()
    step_ms = [a.elapsed_time(b) for a, b in events][3:]  # the first three are warm-up
    live = [int(x.sum()) for x in schedule[3:]]
    nbytes = statistics.mean(live) * inp["heads"] * DECODE["dim"] * 2 * 2
    return {"step_ms": statistics.median(step_ms), "host_us": statistics.median(host_us[3:]),
            "host_us_max": max(host_us[3:]), "bytes": nbytes, "steps": steps,
            "h2d": host_q.numel() * host_q.element_size() + host_len.numel() * 4,
            "d2h": host_out.numel() * host_out.element_size()}


def run_longq_strong(args, rank, world, device, stream):
    """Config 2 strong-scaled: the one B2 H8 call sharded by head over the ranks through the product API
    (mha_paged_decode_sharded), each rank H/N heads of both requests; timed without and with the gathered output
    (one all-gather). Eager steps with the L2 flushed, device time per rank, max over ranks."""
    from fgw_b200.operators.mha.sharded import head_shard, mha_paged_decode_sharded
    c = LONGQ
    first, count = head_shard(c["heads"], rank, world)
    inp = longq_inputs(1000, device)  # the same call on every rank: rank r keeps its heads
    heads = slice(first, first + count)
    q = inp["q"][:, :, heads].contiguous()
    k, v = inp["k"][:, heads].contiguous(), inp["v"][:, heads].contiguous()
    a = (q, k, v, inp["table"], inp["lengths"], c["page"])
    kw = dict(shard="heads", cache_lengths=inp["host_lengths"], tensor_kernel=args.tensor_kernel)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=device)
    result = {}
    for name, gather in (("local", False), ("gathered", True)):
        fn = (lambda g=gather: mha_paged_decode_sharded(*a, gather=g, **kw))
        barrier(world)
        per, totals = timed_steps([(name, fn)], max(5, args.steps // 2), 3, flush, stream)
        barrier(world)
        result[name + "_ms"] = statistics.median(totals)
    out = mha_paged_decode_sharded(*a, gather=True, **kw)
    torch.cuda.synchronize()
    ok = check_longq(inp, out)  # the assembled output against a PyTorch FP32 reference
    flops = flops_of(inp, c["sq"], c["heads"], c["dim"])
    return {**result, "flops": flops, "parity": ok, "heads_per_rank": count,
            "launches": 2 * 2 * max(5, args.steps // 2)}  # plan + attend per call, both variants


def run_gather(args, dc, device, stream):
    """Paged-cache gather of K and V over the config-5 pool into packed dense buffers, then the decode attention
    over the packed copy (identity page table, original lengths), against the direct decode's output."""
    from fgw_b200.operators.mha.current import build_kernel
    from fgw_b200.operators.mha.paged_cache_gather import packed_layout, paged_cache_gather
    c = dict(DECODE, batch=args.decode_batch)
    inp = dc["inp"]
    heads, page, dim = inp["heads"], c["page"], c["dim"]
    offsets, rows, table = packed_layout(inp["host_lengths"], page, inp["width"])
    cu = torch.tensor(offsets, dtype=torch.int32, device=device)
    dense_table = torch.tensor(table, dtype=torch.int32, device=device)
    pool_pages = inp["k"].shape[0] // page
    dense = {n: torch.empty((rows, heads, dim), dtype=torch.bfloat16, device=device) for n in ("k", "v")}
    caches = {n: inp[n].view(pool_pages, page, heads, dim) for n in ("k", "v")}
    fns = [(f"gather_{n}", (lambda n=n: paged_cache_gather(dense[n][:offsets[-1]], caches[n], inp["table"], cu)))
           for n in ("k", "v")]
    steps = max(5, args.steps // 2)
    per, totals = timed_steps(fns, steps, max(3, args.warmup // 2), None, stream)
    gather_ms = sum(totals) / len(totals)
    nbytes = 2 * 2 * offsets[-1] * heads * dim * 2  # K and V, each read once and written once
    # exactness: the packed rows of a few requests equal their pool pages
    exact = True
    for b in (0, 1, len(offsets) - 2):
        n_pages = (offsets[b + 1] - offsets[b]) // page
        ids = inp["table"][b, :n_pages].long()
        for n in ("k", "v"):
            want = caches[n][ids].reshape(-1, heads, dim)
            exact = exact and torch.equal(dense[n][offsets[b]:offsets[b + 1]].view(torch.int16), want.view(torch.int16))
    kernel = build_kernel(c["batch"], 1, heads, dim, rows, inp["width"], page, False, "bfloat16", device.index,
                          cache_lengths=tuple(inp["host_lengths"]), path="decode")
    ws = kernel.new_workspace(device)
    out = torch.empty_like(inp["q"])
    a = (inp["q"], dense["k"], dense["v"], dense_table, inp["lengths"])
    afns = [("plan", lambda: kernel.plan_kernel(*a, ws)), ("attend", lambda: kernel.attend_kernel(*a, ws, out))]
    if kernel.num_splits > 1:
        afns.append(("merge", lambda: kernel.merge_only(*a, ws, out)))
    _, atotals = timed_steps(afns, steps, max(3, args.warmup // 2), None, stream)
    torch.cuda.synchronize()
    same = bool(torch.equal(out.view(torch.int16), dc["out"].view(torch.int16)))
    del dense
    return {"gather_ms": gather_ms, "bytes": nbytes, "per": per, "exact": bool(exact),
            "attend_after_gather_ms": sum(atotals) / len(atotals), "same_output_as_direct": same,
            "packed_rows": offsets[-1], "launches": (len(fns) + len(afns)) * steps}


def host_cores():
    """Physical cores of this host (logical CPUs when the count of physical ones is unknown)."""
    try:
        import psutil
        count = psutil.cpu_count(logical=False)
    except Exception:
        count = None
    return count or os.cpu_count() or 1


def use_all_host_cores():
    """Lets NumPy's BLAS use every physical core, whatever OMP_NUM_THREADS torchrun set (it sets 1), and
    returns the thread count the BLAS pools now have."""
    cores = host_cores()
    try:
        from threadpoolctl import threadpool_info, threadpool_limits
        threadpool_limits(limits=cores, user_api="blas")
        counts = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        if counts:
            return max(counts)
    except Exception:
        pass
    return cores


def headline_config(world):
    """Workload description of the headline line, shared by both arms so the driver can match them."""
    c = LONGQ
    return {"workload": "longq_b2h8_q4096_kv2048_bf16_d128_page128", "global_batch": c["batch"] * world,
            "seq_len": c["sq"], "kv_len": c["kv"], "heads": c["heads"], "head_dim": c["dim"], "page": c["page"],
            "parallelism": f"batch-shard x{world}",
            "l2": "flushed (256 MiB write) before every timed step"}


def cpu_longq_sample(budget_s=12.0):
    """Times the NumPy oracle on the headline workload, growing the sample until ~budget_s of work."""
    from oracle import paged_attention_chunked, useful_flops
    cores = use_all_host_cores()
    c = LONGQ
    width = c["kv"] // c["page"]
    rng = np.random.default_rng(5)
    table = rng.permutation(c["batch"] * width).reshape(c["batch"], width).astype(np.int32)
    pool = c["batch"] * width * c["page"]
    k = rng.standard_normal((pool, c["heads"], c["dim"]), dtype=np.float32)
    v = rng.standard_normal((pool, c["heads"], c["dim"]), dtype=np.float32)
    rows, heads = 256, 1
    elapsed, flops, calls = 0.0, 0, 0
    while True:
        q = rng.standard_normal((1, rows, heads, c["dim"]), dtype=np.float32)
        t0 = time.perf_counter()
        paged_attention_chunked(q, k[:, :heads], v[:, :heads], table[:1], np.array([c["kv"]]), c["page"], False)
        dt = time.perf_counter() - t0
        elapsed += dt
        flops += useful_flops([c["kv"]], rows, heads, c["dim"], False)
        calls += 1
        if elapsed >= budget_s or calls >= 64:
            break
        if dt < budget_s / 8:
            if rows < c["sq"]:
                rows *= 2
            elif heads < c["heads"]:
                heads *= 2
    value = flops / elapsed / 1e12
    return {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{calls} oracle calls on slices of config 2 (last: 1 request, {rows} query rows, {heads} heads,"
                      f" KV 2048), {elapsed:.1f} s of CPU work, NumPy FP32 restatement of FGW's reference()"}


# ---------------------------------------------------------------------------------------- reference arm
# split counts: the B200 model's candidates (general_split_cost_model.B200_SPLITS), each up to the KV tiles;
# beyond config 3's grid, one request and head over a 128K-token cache (where 64 / 128 splits pay off)
SWEEP = dict(shapes=((1, 1), (2, 8)), dtypes=("float16", "bfloat16"), queries=(1, 4, 16, 64, 512),
             kvs=(512, 2048, 8192, 32768), dim=128, page=128, long=((1, 1, 131072, (1, 4)),))


def run_split_sweep(args, device, stream):
    """Config 3: every (B, H) x dtype x Q x KV of the reference's split sweep, full caches, page 128, N(0,1)
    data; for each candidate split count up to the KV tiles, the median of 5 timings of 20 calls replayed from a
    CUDA graph (plan + attend + merge; warm L2, as the reference's scan). Rows in the split-model fitter's format."""
    from fgw_b200.operators.mha.current import build_kernel
    from fgw_b200.operators.mha.general_split_cost_model import B200_SPLITS
    c = SWEEP
    rows = []
    grid = [(b, h, kv, c["queries"]) for (b, h) in c["shapes"] for kv in c["kvs"]] + list(c["long"])
    for (b, h, kv, queries) in grid:
        width = kv // c["page"]
        g = torch.Generator(device=device).manual_seed(31 + b + kv)
        pool = b * width
        table = torch.randperm(pool, device=device, generator=g)[:pool].reshape(b, width).int()
        lengths = torch.full((b,), kv, dtype=torch.int32, device=device)
        kf = torch.randn(pool * c["page"], h, c["dim"], device=device, generator=g)
        vf = torch.randn(pool * c["page"], h, c["dim"], device=device, generator=g)
        for dtype in c["dtypes"]:
            tdtype = getattr(torch, dtype)
            k, v = kf.to(tdtype), vf.to(tdtype)
            for sq in queries:
                q = torch.randn(b, sq, h, c["dim"], device=device, generator=g).to(tdtype)
                # FP16 takes the general route (the default FP16 route accepts no explicit split count)
                mode = "general" if dtype == "float16" else "stable"
                auto = build_kernel(b, sq, h, c["dim"], pool * c["page"], width, c["page"], False, dtype,
                                    device.index, full_kv_cache=True, cache_lengths=(kv,) * b, cube_mode=mode)
                median = {}
                for splits in B200_SPLITS:
                    # the route's explicit num_splits where it takes the count, else the B200 measurement
                    # hook (64 / 128, and 32 on the BF16 route, are candidates of the B200 model only)
                    kernel = None
                    for how in (dict(num_splits=splits), dict(_b200_splits=splits)):
                        try:
                            kernel = build_kernel(b, sq, h, c["dim"], pool * c["page"], width, c["page"], False,
                                                  dtype, device.index, full_kv_cache=True, cube_mode=mode, **how)
                            break
                        except ValueError:
                            continue
                    if kernel is None:
                        continue  # more splits than KV tiles
                    ws = kernel.new_workspace(device)
                    out = torch.empty_like(q)
                    a = (q, k, v, table, lengths)
                    for _ in range(3):
                        kernel(*a, out=out, workspace=ws)
                    torch.cuda.synchronize()
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph):
                        for _ in range(20):
                            kernel(*a, out=out, workspace=ws)
                    times = []
                    for _ in range(6):
                        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        e0.record(stream)
                        graph.replay()
                        e1.record(stream)
                        torch.cuda.synchronize()
                        times.append(e0.elapsed_time(e1) * 1e3 / 20)
                    median[str(splits)] = statistics.median(times[1:])
                    del graph
                if not median:
                    continue
                best = min(median, key=median.get)
                rows.append({"case": f"B{b}H{h}_Q{sq}_KV{kv}", "key": f"B{b}H{h}_Q{sq}_KV{kv}_{dtype}",
                             "B": b, "Q": sq, "H": h, "D": c["dim"], "dtype": dtype, "page_size": c["page"],
                             "table_width": width, "lengths": [kv] * b, "median_us": median,
                             "auto_num_splits": auto.num_splits, "split_policy": auto.split_policy,
                             "best_num_splits": int(best),
                             "auto_relative_to_best": median.get(str(auto.num_splits), float("nan"))
                             / median[best]})
    return rows


def reference_arm(args, rank, world):
    if rank != 0:
        return 0
    from oracle import paged_attention_chunked, useful_flops
    cores = use_all_host_cores()
    c = LONGQ
    width = c["kv"] // c["page"]
    rng = np.random.default_rng(5)
    table = rng.permutation(c["batch"] * width).reshape(c["batch"], width).astype(np.int32)
    pool = c["batch"] * width * c["page"]
    k = rng.standard_normal((pool, c["heads"], c["dim"]), dtype=np.float32)
    v = rng.standard_normal((pool, c["heads"], c["dim"]), dtype=np.float32)
    q_full = rng.standard_normal((c["batch"], c["sq"], c["heads"], c["dim"]), dtype=np.float32)
    lengths = np.full(c["batch"], c["kv"])
    # size the per-step sample so the whole run stays within a few minutes
    rows = c["sq"]
    t0 = time.perf_counter()
    paged_attention_chunked(q_full[:, :128], k, v, table, lengths, c["page"], False)
    per_row = (time.perf_counter() - t0) / 128
    budget = 150.0 / max(1, args.steps + args.warmup)
    if per_row * rows > budget:
        rows = max(128, int(budget / per_row) // 128 * 128)
    q = q_full[:, :rows]
    flops = useful_flops(lengths.tolist(), rows, c["heads"], c["dim"], False)
    for _ in range(args.warmup):
        paged_attention_chunked(q, k, v, table, lengths, c["page"], False)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        paged_attention_chunked(q, k, v, table, lengths, c["page"], False)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * sum(times) / len(times)
    value = flops / (ms * 1e-3) / 1e12
    sample = (f"{rows} of 4096 query rows per request (B2 H8 KV2048 D128), FP32 NumPy restatement of FGW's CPU "
              f"reference, BLAS on {cores} threads (every physical core of the host)")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": headline_config(world),
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------------------------- main
def main(argv=None):
    args = parse_args(argv)
    rank, world, local = dist_env()
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    init_dist(world, local)
    device = torch.device("cuda", local)
    stream = torch.cuda.current_stream(device)
    if args.sweep_splits:
        rows = run_split_sweep(args, device, stream)
        pathlib.Path(args.sweep_splits).write_text(json.dumps({"rows": rows, "gpu": torch.cuda.get_device_name(device),
                                                               "source_precision_us": 0.001}, indent=1) + "\n")
        # shapes whose auto choice is a split count the route only takes from auto are not measurable (NaN)
        ratios = [r["auto_relative_to_best"] for r in rows if r["auto_relative_to_best"] == r["auto_relative_to_best"]]
        print(json.dumps({"sweep": "config3_split_sweep", "cases": len(rows),
                          "auto_within_2pct": sum(x <= 1.02 for x in ratios),
                          "auto_geomean_relative_to_best": math.exp(sum(math.log(x) for x in ratios) / len(ratios)),
                          "auto_max_relative_to_best": max(ratios), "rows_file": args.sweep_splits}), flush=True)
        return 0
    hbm_peak, tc_peak, peak_kind = measured_peaks()
    line = {"metric": METRIC, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "dtype": "bf16", "data": "synthetic"}
    lq = None
    if args.only in (None, "longq"):
        lq = run_longq(args, rank, world, device, stream)
        c = LONGQ
        step_ms = max_over_ranks(lq["step_ms"], world)
        attend_ms = max_over_ranks(lq["attend_ms"], world)
        e2e_ms = max_over_ranks(lq["e2e_ms"], world)
        total_flops = sum_over_ranks(lq["flops"], world)
        achieved = lq["flops"] / (lq["attend_ms"] * 1e-3) / 1e12
        traffic = None
        prof = ROOT / "profiles" / "traffic_per_launch.json"
        if prof.exists():
            traffic = json.loads(prof.read_text()).get("longq_attend")
        k = lq["kernel"]
        line.update({
            "value": total_flops / (step_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": step_ms,
            "us_per_call": step_ms * 1e3,
            "vs_baseline": (total_flops / (step_ms * 1e-3) / 1e12 / world) / ASCEND_V7_TFLOPS,
            "config": headline_config(world),
            "kernel": {"num_splits": k.num_splits, "execution_path": k.execution_path,
                       "compute_grid": k.compute_grid, "task_assignment": k.task_assignment},
            "vs_baseline_source": "published: 237.4 TFLOP/s, FGW v7 persistent28 on Ascend 950PR (per GPU)",
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": tc_peak, "unit": "TFLOP/s",
                         "frac": achieved / tc_peak, "traffic": traffic,
                         "kernel": "attend (" + k.execution_path + ")", "peak_source": f"{peak_kind} bf16_tflops"},
            "e2e": {"value": total_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": lq["h2d"], "d2h_bytes_per_step": lq["d2h"], "ms_per_step": e2e_ms,
                    "how": "mha_paged_decode each step with its inputs uploaded from pinned host memory and its "
                           "output downloaded; steps pipelined on three streams with double buffers (upload of "
                           "step i+1 overlaps forward + download of step i)",
                    "serial_ms_per_step": max_over_ranks(lq["e2e_serial_ms"], world)},
            "clocks": lq["clocks"], "parity": lq["parity"],
            "gpu_launches": lq["launches_per_step"] * args.steps,
            "stage_ms": {n: statistics.mean(v) for n, v in lq["per"].items()},
            "eager_step_ms": max_over_ranks(lq["eager_step_ms"], world),
            "reference_protocol": {
                "what": "median of 51 CUDA-graph steps after 20 warm-ups (FGW bench_mha_mfu.py), max over ranks",
                **{k: max_over_ranks(v / 1e3, world) * 1e3 for k, v in lq["protocol"].items()},
                "warm_l2_tflops": total_flops / (max_over_ranks(lq["protocol"]["warm_l2_us_median"] / 1e3, world)
                                                 * 1e-3) / 1e12},
            "step_timing": "CUDA-graph replay of plan+attend(+merge), L2 flushed before each step; stage_ms and "
                           "roofline from per-launch events of the same step run eagerly",
        })
    if args.only is None:
        lq32 = run_longq_32k(args, rank, world, device, stream)
        attend_ms = max_over_ranks(lq32["attend_ms"], world)
        step_ms32 = max_over_ranks(lq32["step_ms"], world)
        achieved = lq32["flops"] / (lq32["attend_ms"] * 1e-3) / 1e12
        line["longq_q32768"] = {
            "workload": "longq_b2h8_q32768_kv2048_bf16_d128_page128", "scaling": "weak",
            "us_per_call": step_ms32 * 1e3, "graph_us_per_call": max_over_ranks(lq32["graph_ms"], world) * 1e3,
            "unit": "TFLOP/s",
            "value": sum_over_ranks(lq32["flops"], world) / (step_ms32 * 1e-3) / 1e12,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": tc_peak, "unit": "TFLOP/s",
                         "frac": achieved / tc_peak, "kernel": "attend", "peak_source": f"{peak_kind} bf16_tflops"},
            "num_splits": lq32["num_splits"], "task_assignment": lq32["task_assignment"],
            "l2": "flushed (256 MiB write) before every step; eager plan + attend, per-stage events",
            "parity": lq32["parity"], "gpu_launches": lq32["launches"]}
        line["gpu_launches"] = line.get("gpu_launches", 0) + lq32["launches"]
    if args.only in (None, "d256"):
        # more shapes of BASELINE's configurations, weak-scaled like the headline (every rank its own call)
        extra = [
            ("config1", "decode_b1h1_q1_kv2048_bf16_d128_page128_16of64", "hbm",
             dict(seed=3000, sq=1, steps=max(10, args.steps), batch=1, heads=1, pool_pages=64), 32.9),
            ("b1h1_q32768", "longq_b1h1_q32768_kv2048_bf16_d128_page128", "tensor",
             dict(seed=3100, sq=32768, batch=1, heads=1), 175.0),
            ("longq_d256", "longq_b2h8_q4096_kv2048_bf16_d256_page128", "tensor",
             dict(seed=3200, sq=4096, dim=256), None),
        ]
        if args.only == "d256":
            extra = extra[2:]
        for key, workload, bound, shape, published in extra:
            r = run_longq_shape(args, rank, world, device, stream, **shape)
            ms = max_over_ranks(r["step_ms"], world)
            graph_ms = max_over_ranks(r["graph_ms"], world)
            if bound == "tensor":
                achieved = r["flops"] / (r["attend_ms"] * 1e-3) / 1e12
                roof = {"bound": "tensor", "achieved": achieved, "peak": tc_peak, "unit": "TFLOP/s",
                        "frac": achieved / tc_peak, "kernel": "attend (" + r["execution_path"] + ")",
                        "peak_source": f"{peak_kind} bf16_tflops"}
                value, unit = sum_over_ranks(r["flops"], world) / (ms * 1e-3) / 1e12, "TFLOP/s"
            else:
                achieved = r["bytes"] / (r["attend_ms"] * 1e-3) / 1e9
                roof = {"bound": "hbm (launch-bound in practice)", "achieved": achieved, "peak": hbm_peak,
                        "unit": "GB/s", "frac": achieved / hbm_peak, "kernel": "attend (" + r["execution_path"] + ")",
                        "peak_source": f"{peak_kind} hbm_gbs"}
                value, unit = sum_over_ranks(r["bytes"], world) / (ms * 1e-3) / 1e9, "GB/s"
            line[key] = {"workload": workload, "scaling": "weak", "us_per_call": ms * 1e3,
                         "graph_us_per_call": graph_ms * 1e3, "value": value, "unit": unit, "roofline": roof,
                         "num_splits": r["num_splits"], "task_assignment": r["task_assignment"],
                         "l2": "flushed (256 MiB write) before every step; us_per_call = the launch callable "
                               "eager, graph_us_per_call = the same call replayed as a CUDA graph; roofline from "
                               "per-stage events of plan + attend",
                         "parity": r["parity"], "gpu_launches": r["launches"]}
            if published is not None:
                line[key]["published_ascend_us"] = published
            line["gpu_launches"] = line.get("gpu_launches", 0) + r["launches"]
        if lq is None:
            d = line["longq_d256"]
            line.update({"value": d["value"], "unit": d["unit"], "ms_per_step": d["us_per_call"] / 1e3,
                         "vs_baseline": None, "config": {"workload": d["workload"]}, "roofline": d["roofline"]})
    if args.only is None:
        st = run_longq_strong(args, rank, world, device, stream)
        local_ms = max_over_ranks(st["local_ms"], world)
        gathered_ms = max_over_ranks(st["gathered_ms"], world)
        line["longq_strong"] = {
            "workload": "longq_b2h8_q4096_kv2048_bf16_d128_page128", "scaling": "strong",
            "parallelism": f"head-shard x{world} ({st['heads_per_rank']} heads per GPU)",
            "us_per_call": local_ms * 1e3, "unit": "TFLOP/s", "value": st["flops"] / (local_ms * 1e-3) / 1e12,
            "gathered_us_per_call": gathered_ms * 1e3,
            "gathered_value": st["flops"] / (gathered_ms * 1e-3) / 1e12,
            "how": "mha_paged_decode_sharded per rank (eager, L2 flushed, median step, max over ranks); gathered = "
                   "plus one all-gather assembling O[B,Sq,H,D] on every rank",
            "parity": st["parity"], "gpu_launches": st["launches"]}
        line["gpu_launches"] = line.get("gpu_launches", 0) + st["launches"]
    if not args.no_decode and args.only in (None, "decode"):
        dc = run_decode(args, rank, world, device, stream)
        step_ms = max_over_ranks(dc["step_ms"], world)
        attend_ms = max_over_ranks(dc["attend_ms"], world)
        total_bytes = sum_over_ranks(dc["bytes"], world)
        args_batch = args.decode_batch
        achieved = dc["bytes"] / (dc["attend_ms"] * 1e-3) / 1e9
        k = dc["kernel"]
        decode = {"workload": f"decode_b{args.decode_batch}h32_q1_kvlogu1024_32768_bf16_d128_page64",
                  "scaling": "strong",
                  "parallelism": f"head-shard x{world}", "us_per_call": step_ms * 1e3,
                  "value": total_bytes / (step_ms * 1e-3) / 1e9, "unit": "GB/s",
                  "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                               "frac": achieved / hbm_peak, "kernel": "attend (" + k.execution_path + ")",
                               "peak_source": f"{peak_kind} hbm_gbs"},
                  "num_splits": k.num_splits, "parity": dc["parity"],
                  "gpu_launches": dc["launches_per_step"] * dc["steps"],
                  "stage_ms": {n: statistics.mean(v) for n, v in dc["per"].items()}}
        sv = run_decode_serving(args, dc, rank, world, device, stream)
        sv_ms = max_over_ranks(sv["step_ms"], world)
        decode["serving"] = {
            "how": "lengths grow by one token per step; per step: H2D of Q and lengths from pinned memory, "
                   "mha_paged_decode_sharded with the host lengths, D2H of O; device time per step (median, max "
                   "over ranks); host_us_per_call = host time of the API call",
            "ms_per_step": sv_ms, "value": sum_over_ranks(sv["bytes"], world) / (sv_ms * 1e-3) / 1e9, "unit": "GB/s",
            "host_us_per_call": max_over_ranks(sv["host_us"], world),
            "host_us_per_call_max": max_over_ranks(sv["host_us_max"], world),
            "h2d_bytes_per_step": sv["h2d"], "d2h_bytes_per_step": sv["d2h"], "steps": sv["steps"],
            "gpu_launches": 2 * sv["steps"]}
        decode["gpu_launches"] += 2 * sv["steps"]
        line["decode"] = decode
        line["gpu_launches"] = line.get("gpu_launches", 0) + decode["gpu_launches"]
        if not args.no_gather:
            gt = run_gather(args, dc, device, stream)
            g_ms = max_over_ranks(gt["gather_ms"], world)
            achieved = gt["bytes"] / (gt["gather_ms"] * 1e-3) / 1e9
            g_traffic = None
            prof = ROOT / "profiles" / "traffic_per_launch.json"
            if prof.exists():
                ratio = json.loads(prof.read_text()).get("gather_traffic_per_algorithmic_byte")
                if ratio:
                    g_traffic = ratio * gt["bytes"] / 2  # one launch (one cache) of this rank
            line["gather"] = {
                "workload": f"paged_cache_gather_k_and_v_of_{decode['workload']}", "scaling": "strong",
                "us_per_call": g_ms * 1e3, "value": sum_over_ranks(gt["bytes"], world) / (g_ms * 1e-3) / 1e9,
                "unit": "GB/s", "packed_rows_per_rank": gt["packed_rows"],
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                             "frac": achieved / hbm_peak, "kernel": "gather_kernel (two launches: K, V)",
                             "traffic": g_traffic, "traffic_unit": "bytes per launch",
                             "peak_source": f"{peak_kind} hbm_gbs"},
                "exact_rows": gt["exact"],
                "attend_after_gather_us": max_over_ranks(gt["attend_after_gather_ms"], world) * 1e3,
                "gather_plus_attend_us": (g_ms + max_over_ranks(gt["attend_after_gather_ms"], world)) * 1e3,
                "direct_attend_us": step_ms * 1e3,
                "same_output_as_direct": gt["same_output_as_direct"],
                "gpu_launches": gt["launches"]}
            line["gpu_launches"] += gt["launches"]
        del dc
        if lq is None:
            line.update({"value": decode["value"], "unit": "GB/s", "ms_per_step": step_ms, "vs_baseline": None,
                         "config": {"workload": decode["workload"]}, "roofline": decode["roofline"]})
    if rank == 0 and world == 1 and args.only is None and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_longq_sample()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
