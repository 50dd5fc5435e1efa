"""Benchmark of the DSA sparse-attention decode path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl {ours,reference}]

Workload (BASELINE cfg2, synthetic, seeded): per GPU one decode batch of
T=64 query tokens, 16 heads, contexts U[1024, 65536], page size 64, shuffled
page tables, 2048 distinct top-k positions per token (-1 padded), bf16
~N(0,1) queries, ~N(0,0.25) latent cache (about 2.3 GB per GPU).  A step is
one call of the operator over the batch.  Under torchrun each rank runs its
own batch (request sharding, no collective on the data path; weak scaling).

Metric: query tokens per second, whole job (all ranks); also reported as
achieved HBM GB/s of the attention kernel against MEASURED_PEAKS.json.
L2 is flushed (256 MiB write, then a 256 MiB read) before every timed step; each step is timed
with CUDA events on the launching stream and summed, max over ranks.

--impl reference times the reference's own CPU implementation of the path
on the host cores instead: its golden PyTorch function `run`
(solution/triton/indexer_kernel.py:436-497), imported unmodified from the
copy in baseline/_ref (placed there by baseline/install_reference.py), on the
same cfg2 batch with all host threads; rank 0 only (the number is one host's,
not per GPU).  Without baseline/_ref the CPU port of `run` in oracle/ is timed
instead and the line says so.

The default line also carries a "cfg4" object (indexer + top-k + attention
step of BASELINE cfg4 on this GPU) and, under torchrun with N >= 2, a "cfg3"
object (128 heads sharded over the N GPUs, gather fused into the epilogues,
with the NCCL all-gather variant and a parity flag against a local 128-head
computation).
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "DSA decode query-tokens/sec (whole job); achieved HBM GB/s vs B200 peak"
UNIT = "query_tokens/s"
# dram__bytes_read.sum + dram__bytes_write.sum of one dsa_attention_kernel launch
# captured on the small case of this workload (`--tokens 8`: 19,134,464 B read +
# 512 B written for 19,218,944 algorithmic bytes); traffic grows with the rows
# gathered, so a full launch is scaled by its algorithmic bytes
ATTN_TRAFFIC_PER_ALG_BYTE = (19_134_464 + 512) / 19_218_944
WORKLOAD = ("cfg2 batched decode: T=64 tokens/GPU, 16 heads, ckv512+kpe64 bf16, page 64, "
            "ctx U[1024,65536], topk 2048 (-1 padded), shuffled page tables")


L2_NOTE = ("flushed before every step, untimed: 256 MiB written, then 256 MiB of another buffer "
           "read, so no input is L2-resident and the write-back of the flush's own dirty lines "
           "is not charged to the step")


class L2Flush:
    """Evicts the 126 MB L2 between timed steps: a 256 MiB write (the usual
    flush) followed by a 256 MiB read, which pushes the dirty lines of the
    write out before the timed region instead of inside it."""

    def __init__(self, device):
        self.w = torch.empty(256 << 20, dtype=torch.uint8, device=device)
        self.r = torch.ones(64 << 20, dtype=torch.float32, device=device)
        self.acc = torch.empty((), dtype=torch.float32, device=device)

    def __call__(self, i=0):
        self.w.fill_(i & 0xFF)
        torch.sum(self.r, dim=0, out=self.acc)


def bind_to_gpu_numa(device_index: int) -> str:
    """Run this process on the CPUs of the NUMA node the GPU's PCIe link
    attaches to (read from sysfs through the GPU's PCI bus id), so that pinned
    host buffers allocated afterwards are local to that link.  Returns a short
    description for the JSON line; leaves the affinity alone when the topology
    cannot be read."""
    try:
        pr = torch.cuda.get_device_properties(device_index)
        bdf = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bdf}/numa_node") as f:
            node = int(f.read().strip())
        if node < 0:
            return f"gpu {bdf}: no NUMA node reported, affinity unchanged"
        with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
            spec = f.read().strip()
        cpus = set()
        for part in spec.split(","):
            a, _, b = part.partition("-")
            cpus.update(range(int(a), int(b or a) + 1))
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return f"gpu {bdf}: node {node} CPUs not available, affinity unchanged"
        os.sched_setaffinity(0, cpus)
        return f"gpu {bdf} on NUMA node {node}: process bound to its {len(cpus)} CPUs"
    except (OSError, ValueError, AttributeError) as e:
        return f"affinity unchanged ({type(e).__name__})"


def graph_timed_steps(fn, steps, flush, side, stream, per_graph=50):
    """Device time (ms) of each of `steps` calls of fn(), run as CUDA-graph
    nodes: every captured step is flush(), a start event, fn(), an end event
    (events recorded as graph nodes); the graph holds min(per_graph, steps)
    steps and is replayed until `steps` have run."""
    n = min(per_graph, steps)
    starts = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(n)]
    ends = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(n)]
    side.wait_stream(stream)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        fn()  # first-call set-up outside the capture
        with torch.cuda.graph(g, stream=side):
            for j in range(n):
                flush(j)
                starts[j].record(side)
                fn()
                ends[j].record(side)
    stream.wait_stream(side)
    torch.cuda.synchronize()
    times = []
    while len(times) < steps:
        g.replay()
        torch.cuda.synchronize()
        times += [starts[j].elapsed_time(ends[j]) for j in range(min(n, steps - len(times)))]
    return times


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks + throttle reasons sampled during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return self
        # the timed region starts only once the sampler is producing samples
        t0 = time.time()
        while time.time() - t0 < 10 and os.path.getsize(self.path) == 0:
            time.sleep(0.02)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 7:
                try:
                    rows.append((float(f[0]), float(f[1]), f[3:7]))
                except ValueError:
                    pass
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v == "Active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def dist_setup(n):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n and world != 1:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}")
    return rank, world, local


def reference_run_fn():
    """The reference golden function `run` (solution/triton/indexer_kernel.py:
    436-497) from the unmodified copy in baseline/_ref, or (None, reason).
    The module uses `math` without importing it (:490), so `math` is added to
    its namespace; its file is not changed."""
    path = os.path.join(ROOT, "baseline", "_ref", "solution", "triton", "indexer_kernel.py")
    if not os.path.isfile(path):
        return None, "baseline/_ref is missing (baseline/install_reference.py was not run)"
    try:
        spec = importlib.util.spec_from_file_location("_ref_indexer_kernel", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    except Exception as e:  # noqa: BLE001  (e.g. triton missing on the host)
        return None, f"cannot import the reference: {type(e).__name__}: {e}"
    mod.math = math
    return mod.run, None


def measure_reference_gpu(qn, qp, ckv, kpe, idx, scale, out, lse, flush, side, stream, steps):
    """The reference's own GPU operators on this batch: the Triton `kernel`
    (solution/triton/kernel.py:138-182) and `kernel_splitk` with SPLIT_K=16
    (:496-567), imported unmodified from baseline/_ref, each captured in CUDA
    graphs and timed exactly like this library's operator (graph nodes, L2
    flushed before every step).  Also the largest difference of their results
    from this library's (out, lse) on the full batch.  Returns a dict, or
    {"unavailable": why}."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isfile(os.path.join(ref, "solution", "triton", "kernel.py")):
        return {"unavailable": "baseline/_ref is missing (baseline/install_reference.py was not run)"}
    try:
        if ref not in sys.path:
            sys.path.insert(0, ref)
        import solution.triton.kernel as rk  # namespace package of the unmodified checkout
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"cannot import the reference kernels: {type(e).__name__}: {e}"}
    T = idx.shape[0]
    res = {"source": "baseline/_ref solution/triton/kernel.py (unmodified), CUDA graphs, L2 flushed per step",
           "steps": steps}
    variants = (("kernel", lambda: rk.kernel(qn, qp, ckv, kpe, idx, scale)),
                ("kernel_splitk16", lambda: rk.kernel_splitk(qn, qp, ckv, kpe, idx, scale, SPLIT_K=16)))
    for name, fn in variants:
        try:
            with torch.cuda.stream(side):
                ro, rl = fn()  # compiles the Triton kernel outside any capture
            torch.cuda.synchronize()
            ms = statistics.median(graph_timed_steps(fn, steps, flush, side, stream))
            d_out = (ro.float() - out.float()).abs()
            fin = torch.isfinite(rl) & torch.isfinite(lse)
            res[name] = {"ms_per_step": ms, "value": T / (ms / 1e3), "unit": UNIT,
                         "max_abs_diff_out_vs_ours": float(torch.nan_to_num(d_out, nan=float("inf")).max()),
                         "max_abs_diff_lse_vs_ours": float((rl - lse).abs()[fin].max()) if fin.any() else 0.0}
        except Exception as e:  # noqa: BLE001
            res[name] = {"unavailable": f"{type(e).__name__}: {e}"}
    return res


def reference_cpu_run(qn, qp, ckv, kpe, idx, scale, max_calls, budget_s=60.0, warmup=1):
    """Time the reference `run` on the host cores (torch CPU, all threads) on
    the full batch: one call = every token of the batch over the whole cache,
    which `run` first upcasts to fp32 (indexer_kernel.py:458-459), exactly as
    the reference evaluates it.  Times up to max_calls calls, stopping once
    budget_s is spent (at least one).  Returns None when the reference is not
    available, else a dict (tokens/s, cores, sample, calls)."""
    run, why = reference_run_fn()
    if run is None:
        return {"unavailable": why}
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    h = [t.detach().cpu() for t in (qn, qp, ckv, kpe, idx)]
    for _ in range(warmup):
        run(*h, scale)
    times, t_all = [], time.perf_counter()
    while len(times) < max(1, max_calls):
        t0 = time.perf_counter()
        run(*h, scale)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > budget_s:
            break
    T = idx.shape[0]
    med = statistics.median(times)
    return {"value": T / med, "unit": UNIT, "cores": cores, "kind": "reference",
            "sample": f"reference run() (baseline/_ref, torch CPU, {torch.get_num_threads()} threads) "
                      f"on the full batch of {T} tokens and its whole cache, median of "
                      f"{len(times)} call(s) after {warmup} warm-up",
            "calls": len(times), "s_per_call": med}


def cpu_baseline_run(qn, qp, ckv, kpe, idx, scale, reps=3):
    """The reference algorithm (CPU port in oracle/) on the rows of the same
    batch: the selected rows are compacted into a small host cache so the
    work per token is identical.  Returns (tokens/s, cores, sample)."""
    from oracle import oracle as O

    def out_bits(t):
        return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
    valid = idx >= 0
    uniq, inv = torch.unique(idx[valid].long(), return_inverse=True)
    sidx = torch.full_like(idx, -1)
    sidx[valid] = inv.to(torch.int32)
    npg = (uniq.numel() + 63) // 64

    def compact(cache, d):
        flat = cache.reshape(-1, d)[uniq]
        pad = torch.zeros((npg * 64 - uniq.numel(), d), dtype=cache.dtype, device=cache.device)
        return out_bits(torch.cat([flat, pad]).reshape(npg, 64, d))

    args = (out_bits(qn), out_bits(qp), compact(ckv, 512), compact(kpe, 64), sidx.cpu().numpy())
    cores = os.cpu_count() or 1
    O.dsa_attention(*args, scale, nthreads=cores)  # warm-up
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        O.dsa_attention(*args, scale, nthreads=cores)
        times.append(time.perf_counter() - t0)
    T = idx.shape[0]
    return T / statistics.median(times), cores, (
        f"full batch of {T} tokens (selected rows compacted to host), median of {reps}")


def run_reference_arm(args):
    rank, world, local = dist_setup(args.gpus)
    if rank != 0:
        return
    from flashinfer_repo_b200.bench_inputs import make_cfg2_device
    dev = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    qn, qp, ckv, kpe, idx, scale = make_cfg2_device(seed=0, device=dev)
    T = int(idx.shape[0])
    ref = reference_cpu_run(qn, qp, ckv, kpe, idx, scale, max_calls=args.steps, budget_s=90.0,
                            warmup=min(args.warmup, 1))
    if "unavailable" not in ref:
        v, cb, dtype = ref["value"], ref, "f32"
        steps = ref["calls"]
        note = ("reference arm: the reference's own golden CPU function run() "
                "(solution/triton/indexer_kernel.py:436-497), unmodified, from baseline/_ref, "
                "on all host threads; one step = one run() call on the whole batch; timed calls "
                "capped by a 90 s budget (steps = calls actually timed)")
    else:  # no reference copy on this machine: the CPU port of run()
        vals = []
        for i in range(args.warmup + min(args.steps, 10)):
            v, cores, sample = cpu_baseline_run(qn, qp, ckv, kpe, idx, scale, reps=1)
            if i >= args.warmup:
                vals.append(v)
        v = statistics.median(vals)
        steps, dtype = len(vals), "f64"
        cb = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}
        note = f"reference arm: {ref['unavailable']}; timed the CPU port of run() (oracle/) instead"
    cb = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
        "steps": steps, "steps_requested": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * T / v,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype,
        "data": "synthetic (seeded, BASELINE cfg2 shapes and distributions)",
        "config": {"workload": WORKLOAD, "tokens_per_gpu": T,
                   "parallelism": f"request-shard x{args.gpus} (reference arm: rank 0's host only)",
                   "l2": "not applicable (host CPU)", "launch": "host CPU, torch",
                   "note": note},
        "cpu_baseline": cb,
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def copy_bandwidth(dev, nbytes=64 << 20, reps=5):
    """Pinned host<->device copy bandwidth (GB/s) of this machine, measured
    with CUDA events: the context for the e2e number."""
    h = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    d = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    out = {}
    for name, fn in (("h2d_gbs", lambda: d.copy_(h, non_blocking=True)),
                     ("d2h_gbs", lambda: h.copy_(d, non_blocking=True))):
        fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            ts.append(a.elapsed_time(b))
        out[name] = nbytes / (min(ts) / 1e3) / 1e9
    return out


def copy_floor_ms(dev, uploads, downloads, steps=200):
    """Per-step time of the e2e pipeline's own copies alone (its pinned and
    device buffers, the same copy calls), the upload on one stream and the
    downloads on another at once, no kernels: the directions contend on the
    host link, so this, not either bandwidth alone, is the floor the e2e
    pipeline can reach on this machine.  uploads / downloads: per buffer set,
    a list of (dst, src) pairs."""
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    st = torch.cuda.current_stream(dev)
    nb = len(uploads)
    res = []
    for _ in range(2):  # the first round warms the copy path
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        up.wait_stream(st)
        down.wait_stream(st)
        for i in range(steps):
            with torch.cuda.stream(up):
                for dst, src in uploads[i % nb]:
                    dst.copy_(src, non_blocking=True)
            with torch.cuda.stream(down):
                for dst, src in downloads[i % nb]:
                    dst.copy_(src, non_blocking=True)
        st.wait_stream(up)
        st.wait_stream(down)
        e1.record(st)
        e1.synchronize()
        res.append(e0.elapsed_time(e1) / steps)
    return res[-1]


def run_ours(args):
    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    all_cpus = os.sched_getaffinity(0)
    numa = bind_to_gpu_numa(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    from flashinfer_repo_b200 import kernel, read_device_error
    from flashinfer_repo_b200.bench_inputs import attention_bytes, make_cfg2_device

    qn, qp, ckv, kpe, idx, scale = make_cfg2_device(seed=1000 + rank, device=dev, T=args.tokens)
    T = idx.shape[0]
    alg_bytes = attention_bytes(idx)
    flush = L2Flush(dev)
    out = torch.empty((T, 16, 512), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((T, 16), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    for _ in range(args.warmup):
        flush(1)
        kernel(qn, qp, ckv, kpe, idx, scale, output=out, lse=lse)
    torch.cuda.synchronize()
    if read_device_error(dev):
        raise SystemExit("device error flag set during warm-up")

    # ---- device-resident timing (value + roofline).  Steps run as CUDA-graph
    # nodes: each captured step is the untimed L2 flush, a start event, the
    # operator call (attention grid + merge grid), an end event; one graph
    # holds up to 50 steps and is replayed until K steps have run.  A step's
    # time is its event interval on the device, so neither Python nor a graph
    # launch per step is counted, as inside a decode step captured whole.
    side = torch.cuda.Stream(dev)

    def op():
        kernel(qn, qp, ckv, kpe, idx, scale, output=out, lse=lse)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        step_ms = graph_timed_steps(op, args.steps, flush, side, stream)
        if dist:
            dist.barrier()
    total_ms = sum(step_ms)
    clocks = clk.summary()

    # ---- the dominant kernel alone (roofline): the attention grid without the
    # merge grid (profiling option attention_grids=1), captured and timed the same way
    from flashinfer_repo_b200 import options
    with options(attention_grids=1):
        with torch.cuda.stream(side):
            op()
        attn_ms = graph_timed_steps(op, min(args.steps, 200), flush, side, stream)
    attn_kernel_ms = statistics.mean(attn_ms)
    kernel(qn, qp, ckv, kpe, idx, scale, output=out, lse=lse)  # leave complete results

    # ---- end to end through the public API with host buffers: every step
    # uploads its queries and indices from pinned host memory, runs the
    # operator and downloads output + LSE.  Three streams form a pipeline
    # (upload of step i+1 and download of step i-1 under the compute of step
    # i); four buffer sets, ordered by events.  Steps
    # alternate between two independent batches (two 2.1 GB caches), so the
    # rows gathered by consecutive steps (2 x 151 MB) do not fit in L2.
    NB = 4
    qn2, qp2, ckv2, kpe2, idx2, _ = make_cfg2_device(seed=5000 + rank, device=dev, T=args.tokens)
    batches = [(qn, qp, ckv, kpe, idx), (qn2, qp2, ckv2, kpe2, idx2)]
    # a step's inputs sit in one pinned staging buffer (q_nope | q_pe | indices,
    # 256-byte aligned parts), uploaded with one copy into a device buffer whose
    # typed views are the operator's arguments
    def layout(ts):
        offs, o = [], 0
        for t in ts:
            offs.append(o)
            o += (t.numel() * t.element_size() + 255) // 256 * 256
        return offs, o

    def views(buf, ts, offs):
        return tuple(buf[o:o + t.numel() * t.element_size()].view(t.dtype).view(t.shape)
                     for t, o in zip(ts, offs))
    host_in = []
    for b_ in batches:
        ts = (b_[0], b_[1], b_[4])
        offs, nbytes = layout(ts)
        hb = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
        for t, v in zip(ts, views(hb, ts, offs)):
            v.copy_(t.cpu())
        host_in.append((hb, ts, offs))
    host = [host_in[b_ % 2][0] for b_ in range(NB)]
    dstage = [torch.empty(h.numel(), dtype=torch.uint8, device=dev) for h in host]
    dbuf = [views(dstage[b_], host_in[b_ % 2][1], host_in[b_ % 2][2]) for b_ in range(NB)]
    # a step's results likewise: output and LSE are typed views of one device
    # buffer, downloaded with one copy into one pinned buffer
    res_ts = (out, lse)
    res_offs, res_bytes = layout(res_ts)
    h_res = [torch.empty(res_bytes, dtype=torch.uint8).pin_memory() for _ in range(NB)]
    d_res = [torch.empty(res_bytes, dtype=torch.uint8, device=dev) for _ in range(NB)]
    h_out, h_lse = zip(*[views(h, res_ts, res_offs) for h in h_res])
    d_out, d_lse = zip(*[views(d, res_ts, res_offs) for d in d_res])
    h2d = host[0].numel()
    d2h = h_out[0].numel() * 2 + h_lse[0].numel() * 4
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def part_up(b_):
        dstage[b_].copy_(host[b_], non_blocking=True)

    def part_comp(b_):
        cb = batches[b_ % 2]
        kernel(dbuf[b_][0], dbuf[b_][1], cb[2], cb[3], dbuf[b_][2], scale, output=d_out[b_],
               lse=d_lse[b_])

    def part_down(b_):
        h_res[b_].copy_(d_res[b_], non_blocking=True)
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(stream)
    g_parts = []
    with torch.cuda.stream(cap):
        for b_ in range(NB):  # first-call set-up outside the captures
            part_up(b_)
            part_comp(b_)
            part_down(b_)
        torch.cuda.synchronize()
        for b_ in range(NB):  # per-buffer graphs of each part (variant A)
            trio = []
            for fn in (part_up, part_comp, part_down):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=cap):
                    fn(b_)
                trio.append(g)
            g_parts.append(trio)
    torch.cuda.synchronize()
    # Two ways to drive the same pipeline, both timed, the faster reported:
    # A) the host replays each step's three per-buffer graphs on the three
    #    streams (host launch work per step, copies and kernels overlap freely);
    # B) G steps captured once as one multi-stream CUDA graph (the streams are
    #    branches, the events edges), one launch per G steps, so a slow host
    #    cannot pace the steps.
    G = 40
    up_done = [torch.cuda.Event() for _ in range(NB)]
    comp_done = [torch.cuda.Event() for _ in range(NB)]
    down_done = [torch.cuda.Event() for _ in range(NB)]

    def e2e_steps_a(n):
        for i in range(n):
            b_ = i % NB
            if i >= NB:
                up.wait_event(comp_done[b_])
            with torch.cuda.stream(up):
                g_parts[b_][0].replay()
            up_done[b_].record(up)
            stream.wait_event(up_done[b_])
            if i >= NB:
                stream.wait_event(down_done[b_])
            g_parts[b_][1].replay()
            comp_done[b_].record(stream)
            down.wait_event(comp_done[b_])
            with torch.cuda.stream(down):
                g_parts[b_][2].replay()
            down_done[b_].record(down)

    e2e_steps_a(max(args.warmup, NB))
    torch.cuda.synchronize()
    a_start, a_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a_start.record(stream)
    up.wait_event(a_start)
    down.wait_event(a_start)
    e2e_steps_a(args.steps)
    a_end.record(down)
    torch.cuda.synchronize()
    e2e_a = a_start.elapsed_time(a_end)

    def e2e_steps(n):
        for i in range(n):
            b_ = i % NB
            if i >= NB:
                up.wait_event(comp_done[b_])       # inputs of step i-NB consumed
            with torch.cuda.stream(up):
                part_up(b_)
            up_done[b_].record(up)
            cap.wait_event(up_done[b_])
            if i >= NB:
                cap.wait_event(down_done[b_])     # outputs of step i-NB downloaded
            with torch.cuda.stream(cap):
                part_comp(b_)
            comp_done[b_].record(cap)
            down.wait_event(comp_done[b_])
            with torch.cuda.stream(down):
                part_down(b_)
            down_done[b_].record(down)
        cap.wait_stream(up)
        cap.wait_stream(down)

    pipe = torch.cuda.CUDAGraph()
    cap.wait_stream(stream)
    with torch.cuda.graph(pipe, stream=cap):
        up.wait_stream(cap)
        down.wait_stream(cap)
        e2e_steps(G)
    torch.cuda.synchronize()
    for _ in range(max(1, args.warmup // G + 1)):
        pipe.replay()
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = (args.steps + G - 1) // G
    e_start.record(stream)
    for _ in range(reps):
        pipe.replay()
    e_end.record(stream)
    torch.cuda.synchronize()
    e2e_b = e_start.elapsed_time(e_end) * args.steps / (reps * G)
    e2e_total = min(e2e_a, e2e_b)
    last = (args.steps - 1) % NB
    ok = torch.equal(h_out[last].to(dev), d_out[last])
    if read_device_error(dev) or not ok:
        raise SystemExit("device error flag set, or downloaded output differs, during the timed steps")

    # max over ranks
    t = torch.tensor([total_ms, e2e_total], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, e2e_total = t.tolist()
    value = world * T * args.steps / (total_ms / 1e3)
    e2e_value = world * T * args.steps / (e2e_total / 1e3)
    avg_kernel_ms = attn_kernel_ms
    achieved = alg_bytes / (avg_kernel_ms / 1e3) / 1e9
    peak, peak_kind = peaks()

    copies = copy_bandwidth(dev)
    floor_ms = copy_floor_ms(dev, [[(dstage[b_], host[b_])] for b_ in range(NB)],
                             [[(h_res[b_], d_res[b_])] for b_ in range(NB)])
    cfg4 = None if args.skip_extras else measure_cfg4(dev, rank, min(args.steps, 20), args.warmup, 128)
    cfg3 = (measure_cfg3(dev, world, rank, min(args.steps, 20), args.warmup, dist)
            if world > 1 and not args.skip_extras else None)

    ref_gpu = None
    if world == 1 and not args.skip_extras:
        with torch.cuda.stream(side):
            kernel(qn, qp, ckv, kpe, idx, scale, output=out, lse=lse)
        torch.cuda.synchronize()
        ref_gpu = measure_reference_gpu(qn, qp, ckv, kpe, idx, scale, out, lse, flush, side, stream,
                                        min(args.steps, 50))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not args.skip_extras:
        os.sched_setaffinity(0, all_cpus)  # the CPU baseline uses every host core
        ref = reference_cpu_run(qn, qp, ckv, kpe, idx, scale, max_calls=3, budget_s=30.0)
        v, cores, sample = cpu_baseline_run(qn, qp, ckv, kpe, idx, scale)
        port = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample,
                "note": "the fp64 C port of run() in oracle/, selected rows compacted"}
        if "unavailable" in ref:
            cpu = dict(port, note=port["note"] + "; reference unavailable: " + ref["unavailable"])
        else:
            cpu = {k: ref[k] for k in ("value", "unit", "cores", "kind", "sample")}
            cpu["port"] = port

    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded, BASELINE cfg2 shapes and distributions)",
            "config": {"workload": WORKLOAD, "tokens_per_gpu": T, "parallelism": f"request-shard x{world}",
                       "l2": L2_NOTE,
                       "launch": "value: steps as nodes of a CUDA graph (50 per graph), each step timed by its own event pair on the device; e2e: the public API with host copies",
                       "alg_bytes_per_step_per_gpu": alg_bytes},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": round(ATTN_TRAFFIC_PER_ALG_BYTE * alg_bytes),
                         "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum of the T=8 capture, scaled by algorithmic bytes)",
                         "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
                         "kernel": "dsa_attention_kernel", "avg_kernel_ms": avg_kernel_ms,
                         "step_ms_incl_merge_grid": statistics.mean(step_ms),
                         "step_frac": alg_bytes / (statistics.mean(step_ms) / 1e3) / 1e9 / peak},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_total / args.steps,
                    "host_numa": numa,
                    "host_driven_ms_per_step": e2e_a / args.steps,
                    "one_graph_ms_per_step": e2e_b / args.steps,
                    "pcie_floor_ms_per_step": h2d / (copies["h2d_gbs"] * 1e9) * 1e3,
                    "copy_floor_ms_per_step": floor_ms,
                    "copy_bandwidth_gbs": copies,
                    "note": "kernel() with pinned host buffers: per step the upload of q_nope, "
                            "q_pe and sparse_indices (one staging buffer, one copy), the operator, "
                            "and the download of output + "
                            "LSE (one buffer, one copy), pipelined over upload/compute/download streams (4 buffer sets), driven "
                            "by the host per step or as 40 steps in one multi-stream CUDA graph (the "
                            "faster is the value), alternating two batches (inputs "
                            "larger than L2); pcie_floor = upload bytes at the pinned host-to-device "
                            "bandwidth measured on this machine (copy_bandwidth_gbs); copy_floor = the "
                            "same per-step upload and download run alone on two streams at once, "
                            "measured here (the directions contend on the host link)"},
            "gpu_launches": 2 * args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "cfg4": cfg4,
            "cfg3": cfg3,
            "reference_gpu": ref_gpu,
        }), flush=True)
    if dist:
        dist.destroy_process_group()


def measure_cfg4(dev, rank, steps, warmup, requests):
    """BASELINE cfg4 on this GPU: one DSA decode step = FP8 indexer over
    `requests` requests x 32768 tokens -> exact top-2048 -> 16-head sparse MLA
    attention on the selected slots.  Each stage is one CUDA graph; the three
    replays of a step run behind an untimed L2 flush and a GPU sleep, so the
    events see device time only.  Returns per-stage times and rooflines."""
    from flashinfer_repo_b200 import indexer as IX
    from flashinfer_repo_b200 import kernel
    from flashinfer_repo_b200.bench_inputs import attention_bytes, indexer_bytes, make_cfg4_device
    d = make_cfg4_device(seed=2000 + rank, device=dev, T=requests)
    T = d["seq_lens"].numel()
    flush = L2Flush(dev)
    stream = torch.cuda.current_stream(dev)
    scores = torch.empty((T, d["block_table"].shape[1] * 64), dtype=torch.float32, device=dev)
    out = torch.empty((T, 16, 512), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((T, 16), dtype=torch.float32, device=dev)
    box = {}

    def k_indexer():
        IX.indexer_scores(d["q8"], d["k8"], d["scale"], d["w"], d["seq_lens"], d["block_table"], out=scores)

    def k_topk():  # position order: the attention operator does not need score order
        box["slots"] = IX.topk_select(scores, d["seq_lens"], d["block_table"], 2048, order="position")[1]

    def k_attention():
        kernel(d["q_nope"], d["q_pe"], d["ckv"], d["kpe"], box["slots"], d["sm_scale"], output=out, lse=lse)
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    graphs = []
    with torch.cuda.stream(side):
        for fn in (k_indexer, k_topk, k_attention):
            fn()
        torch.cuda.synchronize()
        for fn in (k_indexer, k_topk, k_attention):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                fn()
            graphs.append(g)
    stream.wait_stream(side)
    slots = box["slots"]
    for _ in range(warmup):
        flush(1)
        for g in graphs:
            g.replay()
    torch.cuda.synchronize()
    parts = np.zeros(3)
    with ClockSampler(dev.index) as clk:
        for i in range(steps):
            flush(i)
            torch.cuda._sleep(100_000)
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            ev[0].record(stream)
            for j, g in enumerate(graphs):
                g.replay()
                ev[j + 1].record(stream)
            ev[3].synchronize()
            parts += [ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]), ev[2].elapsed_time(ev[3])]
    parts /= steps
    # the whole step as one CUDA graph (indexer -> top-k -> attention, as a
    # serving loop would capture it), timed the same way
    from flashinfer_repo_b200.pipeline import DecodeStepGraph
    step = DecodeStepGraph(d["q8"], d["k8"], d["scale"], d["w"], d["seq_lens"], d["block_table"],
                           d["q_nope"], d["q_pe"], d["ckv"], d["kpe"], d["sm_scale"])
    one = []
    for i in range(warmup + steps):
        flush(i)
        torch.cuda._sleep(100_000)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        step.replay()
        e1.record(stream)
        e1.synchronize()
        if i >= warmup:
            one.append(e0.elapsed_time(e1))
    total = statistics.median(one)
    ib = indexer_bytes(d["seq_lens"])
    ab = attention_bytes(slots)
    peak, kind = peaks()
    res = {
        "workload": f"cfg4: T={T} requests, ctx 32768, FP8 indexer 64x128, top-2048, 16-head MLA",
        "steps": steps, "value": T / (total / 1e3), "unit": UNIT, "ms_per_step": total,
        "step": "one CUDA graph of the whole step (pipeline.DecodeStepGraph), median",
        "ms_per_step_stage_sum": float(parts.sum()),
        "kernels_ms": {"indexer": parts[0], "topk": parts[1], "attention": parts[2]},
        "indexer_roofline": {"bound": "hbm", "kernel": "dsa_indexer_kernel", "alg_bytes": ib,
                             "achieved": ib / (parts[0] / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                             "frac": ib / (parts[0] / 1e3) / 1e9 / peak,
                             "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({kind})"},
        "attention_roofline": {"alg_bytes": ab, "achieved": ab / (parts[2] / 1e3) / 1e9, "unit": "GB/s",
                               "frac": ab / (parts[2] / 1e3) / 1e9 / peak},
        "gpu_launches_per_step": 4,  # indexer, top-k, attention, merge
        "clocks": clk.summary(),
    }
    del d, scores, out, lse, box, graphs, step
    torch.cuda.empty_cache()
    return res


def run_cfg4(args):
    """BASELINE cfg4 alone (see measure_cfg4)."""
    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    r = measure_cfg4(dev, rank, args.steps, args.warmup, args.requests)
    print(json.dumps({
        "metric": "DSA decode step (indexer + top-k + attention) query-tokens/sec", "value": r["value"],
        "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp8+bf16", "data": "synthetic (seeded, BASELINE cfg4 shapes and distributions)",
        "config": {"workload": r["workload"], "l2": L2_NOTE},
        "kernels_ms": r["kernels_ms"],
        "roofline": dict(r["indexer_roofline"], traffic=None),
        "attention_roofline": r["attention_roofline"],
        "gpu_launches": 4 * args.steps, "clocks": r["clocks"],
    }), flush=True)


def measure_cfg3(dev, world, rank, steps, warmup, dist):
    """BASELINE cfg3 over the `world` GPUs of this job: T=8 tokens, 128 heads,
    context 131072, clustered top-k, latent cache replicated on every GPU;
    heads sharded 128/N per rank.  Timed, max over ranks: the fused step (each
    rank's epilogues store its heads into every rank's output over NVLink, then
    the cross-GPU barrier at the end of its last grid), the NCCL all-gather
    step (16k-head kernel, pack, all_gather_into_tensor, unpack) and the
    per-rank kernel alone.  Before each timed step the ranks meet in a device-
    side barrier, so that host-side skew between the processes is not timed.  Parity:
    both gathered results are compared with a 128-head computation on this GPU
    (same inputs), flags ANDed over ranks."""
    from flashinfer_repo_b200 import kernel
    from flashinfer_repo_b200.bench_inputs import attention_bytes, make_cfg3_device
    from flashinfer_repo_b200.parallel import PeerHeadShardedAttention, head_sharded_attention
    qn, qp, ckv, kpe, idx, scale = make_cfg3_device(seed=3000, device=dev)  # same on every rank
    T, H = qn.shape[:2]
    h = H // world
    sl = slice(h * rank, h * (rank + 1))
    stream = torch.cuda.current_stream(dev)
    flush = L2Flush(dev)
    peer = PeerHeadShardedAttention(T, H, dev) if world > 1 else None

    def step():
        if world > 1:
            return peer(qn, qp, ckv, kpe, idx, scale)
        return kernel(qn, qp, ckv, kpe, idx, scale)

    def step_allgather():
        return head_sharded_attention(qn, qp, ckv, kpe, idx, scale)
    # parity first (fresh results of both paths against the local 128-head call)
    full_out, full_lse = kernel(qn, qp, ckv, kpe, idx, scale)
    fo, fl = step()
    go, gl = step_allgather()
    torch.cuda.synchronize()
    parity = torch.tensor([
        int(torch.equal(fo, full_out) and torch.equal(fl, full_lse)),
        int(torch.equal(go, full_out) and torch.equal(gl, full_lse))], dtype=torch.int64, device=dev)
    maxdiff = torch.tensor([(fo.float() - full_out.float()).abs().max().item(),
                            (go.float() - full_out.float()).abs().max().item()],
                           dtype=torch.float64, device=dev)
    for _ in range(warmup):
        step()
        if world > 1:
            step_allgather()
    torch.cuda.synchronize()
    k_ms, s_ms, g_ms = [], [], []
    for i in range(steps):
        if world > 1:  # the all-gather variant, for comparison (same L2 state)
            flush(i)
            dist.barrier()
            torch.cuda.synchronize()
            torch.cuda._sleep(2_000_000)  # ~1 ms of GPU work covers the host enqueue
            peer.barrier()  # ranks leave together on the device: host skew is not timed
            g0 = torch.cuda.Event(enable_timing=True)
            g1 = torch.cuda.Event(enable_timing=True)
            g0.record(stream)
            step_allgather()
            g1.record(stream)
            g1.synchronize()
            g_ms.append(g0.elapsed_time(g1))
        flush(i)
        e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        e[0].record(stream)
        kernel(qn[:, sl], qp[:, sl], ckv, kpe, idx, scale)
        e[1].record(stream)
        flush(i)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        torch.cuda._sleep(2_000_000)  # ~1 ms: the GPU stays busy while the host enqueues the step
        if world > 1:
            peer.barrier()  # ranks leave together on the device: host skew is not timed
        e[2].record(stream)
        step()
        e3 = torch.cuda.Event(enable_timing=True)
        e3.record(stream)
        e3.synchronize()
        k_ms.append(e[0].elapsed_time(e[1]))
        s_ms.append(e[2].elapsed_time(e3))
    t = torch.tensor([statistics.median(k_ms), statistics.median(s_ms),
                      statistics.median(g_ms) if g_ms else 0.0], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(parity, op=dist.ReduceOp.MIN)
        dist.all_reduce(maxdiff, op=dist.ReduceOp.MAX)
        dist.barrier()
        peer.close()
    kms, sms, gms = t.tolist()
    peak, _ = peaks()
    ab = attention_bytes(idx) * (h // 16)  # the 16-head operator's bytes per head group
    return {
        "workload": "cfg3: T=8, 128 heads, ctx 131072, clustered top-2048",
        "parallelism": f"heads {h}/rank x {world}" + (
            ", outputs stored into every rank's buffer by the epilogues, barrier inside the operator"
            if world > 1 else ""),
        "scaling": "strong", "steps": steps,
        "value": T / (sms / 1e3), "unit": UNIT,
        "ms_per_step_fused_gather": sms, "ms_per_step_nccl_allgather": gms if world > 1 else None,
        "kernel_ms_per_rank": kms,
        "parity_vs_local_128_heads": {"fused_bitwise_equal": bool(parity[0].item()),
                                      "nccl_bitwise_equal": bool(parity[1].item()),
                                      "fused_max_abs_diff": maxdiff[0].item(),
                                      "nccl_max_abs_diff": maxdiff[1].item()},
        "roofline": {"bound": "hbm", "kernel": "dsa_attention_kernel",
                     "achieved": ab / (kms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": ab / (kms / 1e3) / 1e9 / peak,
                     "note": "algorithmic bytes per rank = 16-head operator bytes x head groups"},
        "gpu_launches_per_step": 2,  # attention + merge grid (the barrier runs inside the last grid)
    }


def run_cfg3(args):
    """BASELINE cfg3 alone (see measure_cfg3); strong scaling, the job is fixed."""
    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import torch.distributed as dist
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    r = measure_cfg3(dev, world, rank, args.steps, args.warmup, dist)
    if rank == 0:
        print(json.dumps({
            "metric": "DSA decode query-tokens/sec, 128 heads (head-sharded)", "value": r["value"],
            "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": r["ms_per_step_fused_gather"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded, BASELINE cfg3 shapes and distributions)",
            "config": {"workload": r["workload"], "parallelism": r["parallelism"], "l2": L2_NOTE},
            "cfg3": r, "roofline": dict(r["roofline"], traffic=None),
            "gpu_launches": args.steps * r["gpu_launches_per_step"],
        }), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_cfg5(args):
    """BASELINE cfg5 chunked prefill: one sequence per GPU, 4096 query tokens
    at the end of a 65536-token context, causal top-2048 each, 16 heads.
    The 72 MiB latent cache is mostly L2-resident, so both the HBM-formula
    bandwidth and the tensor throughput are reported."""
    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    all_cpus = os.sched_getaffinity(0)
    numa = bind_to_gpu_numa(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    from flashinfer_repo_b200 import kernel
    from flashinfer_repo_b200.bench_inputs import attention_bytes, attention_flops, make_prefill_device
    qn, qp, ckv, kpe, idx, scale = make_prefill_device(seed=5000 + rank, device=dev,
                                                       queries=args.queries)
    T = idx.shape[0]
    out = torch.empty((T, 16, 512), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((T, 16), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    flush = L2Flush(dev)
    for _ in range(args.warmup):
        kernel(qn, qp, ckv, kpe, idx, scale, output=out, lse=lse)
    torch.cuda.synchronize()
    ms = []
    if dist:
        dist.barrier()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            flush(i)
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            kernel(qn, qp, ckv, kpe, idx, scale, output=out, lse=lse)
            s1.record(stream)
            s1.synchronize()
            ms.append(s0.elapsed_time(s1))
    t = torch.tensor([statistics.median(ms)], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    kms = t.item()
    peak, kind = peaks()
    pk = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {"bf16_tflops": 1590.0}
    ab, fl = attention_bytes(idx), attention_flops(idx)
    if rank == 0:
        print(json.dumps({
            "metric": "DSA chunked-prefill query-tokens/sec (whole job)", "value": world * T / (kms / 1e3),
            "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": kms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded, BASELINE cfg5 shapes and distributions)",
            "config": {"workload": f"cfg5: {T} queries/GPU, ctx 65536, causal top-2048, 16 heads",
                       "attention_kernel": args.attention_kernel,
                       "l2": L2_NOTE + "; the 72 MiB cache is re-read from L2 within a step"},
            "roofline": {"bound": "hbm (per-token formula)", "achieved": ab / (kms / 1e3) / 1e9, "peak": peak,
                         "unit": "GB/s", "frac": ab / (kms / 1e3) / 1e9 / peak, "traffic": None},
            "tensor": {"achieved_tflops": fl / (kms / 1e3) / 1e12, "peak_tflops": pk["bf16_tflops"],
                       "frac": fl / (kms / 1e3) / 1e12 / pk["bf16_tflops"]},
            "gpu_launches": 2 * args.steps, "clocks": clk.summary(),
        }), flush=True)
    if dist:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="cfg2", choices=["cfg2", "cfg3", "cfg4", "cfg5"],
                    help="cfg2 = headline batched decode; cfg4 = indexer + top-k + attention")
    ap.add_argument("--requests", type=int, default=128, help="cfg4 requests per GPU (default 128)")
    ap.add_argument("--tokens", type=int, default=64,
                    help="cfg2 query tokens per GPU (default 64, the headline; smaller only for profiling)")
    ap.add_argument("--skip-extras", action="store_true",
                    help="omit the cfg4/cfg3 sub-objects and the CPU baseline (profiling runs)")
    ap.add_argument("--queries", type=int, default=4096, help="cfg5 query tokens per GPU (default 4096)")
    ap.add_argument("--attention-kernel", type=int, default=0, choices=[0, 1, 2],
                    help="library option attention_kernel: 0 default, 1 mma.sync, 2 tcgen05")
    args = ap.parse_args()
    if args.attention_kernel and args.impl == "ours":
        from flashinfer_repo_b200 import set_options
        set_options(attention_kernel=args.attention_kernel)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference_arm(args)
    elif args.workload == "cfg4":
        run_cfg4(args)
    elif args.workload == "cfg3":
        run_cfg3(args)
    elif args.workload == "cfg5":
        run_cfg5(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
