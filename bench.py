"""Benchmark of the dense-contraction hot path on B200 (one JSON line on rank 0).

Metric: "GEMM TFLOP/s & GEMV HBM GB/s per B200, % roofline, at 1/2/4/8 GPUs".

Headline workload -- BASELINE config 2, decode GEMV ``x[1,8192] @ W[8192,8192]^T`` bf16,
strong-scaled: a *step* is one product over the whole 8192 x 8192 weight (128 MiB).
  * N = 1: one ``rk_gemv`` launch per step.
  * N > 1: the weight is split by rows, rank r holding rows [r*8192/N, (r+1)*8192/N); a
    step is one ``rk_gemv_allgather`` launch per rank, which streams the rank's block and
    stores its slice of the output into every rank's full ``out[1, 8192]`` over NVLink, so
    the output all-gather is inside the timed step.
Steps rotate over several weight sets (more than 2 x 126 MB of L2 per rank) so every step
streams its weight from HBM; ``value`` = the bytes of all steps (the whole weight plus x and
out per step) / the device time of the timed region (max over ranks).

``e2e``: the same step through the public API -- ``radeon_kernels.gemv`` at N = 1,
``radeon_kernels.distributed.ShardedGemv(..., gather=True)`` at N > 1 -- with the step's
activation copied host->device from pinned memory and the full result copied back every
step, the steps captured into a CUDA graph.

``suite``: the other BASELINE configs measured in the same run (GEMM TFLOP/s with the
tcgen05 kernels, FFN-down GEMV at M = 1/4/16, the decode neighbours), each with its
roofline fraction; at N > 1 config 5 runs with B split into N column blocks, compute-only
and with the fused all-gather, next to the NCCL all-gather it replaces.

``--impl reference`` times the reference's own path for the same workload on the host
CPU cores (``oracle/reference_path.py``: ``torch.mm`` as in providers/torch_fallback.py /
ops/gemv/reference.py), rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "radeon-kernels_b200"))
sys.path.insert(0, str(REPO))

METRIC = "GEMM TFLOP/s & GEMV HBM GB/s per B200, % roofline, at 1/2/4/8 GPUs"
DATA = "synthetic (seeded torch.Generator, BASELINE config 2 distributions: x~N(0,1), W~N(0,1/8192))"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
ROTATE = 4  # weight matrices cycled through by the headline loop


def load_peaks() -> tuple[dict, str]:
    path = REPO / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return data, "measured"
    except (OSError, json.JSONDecodeError):
        return dict(FALLBACK_PEAKS), "fallback"


def load_traffic() -> dict:
    path = REPO / "profiles" / "traffic.json"
    try:
        return json.loads(path.read_text())
    except (OSError, json.JSONDecodeError):
        return {}


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""

    FIELDS = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self._thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL,
                text=True,
            )
            self._thread = threading.Thread(target=self._drain, daemon=True)
            self._thread.start()
        except OSError:
            self.proc = None
        return self

    def _drain(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self._thread is not None:
                self._thread.join(timeout=2)

    def summary(self) -> dict:
        sm, sm_max, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                sm_max = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": sm_max,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# ------------------------------------------------------------------------ distributed
class Dist:
    def __init__(self, n_gpus: int):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.n_gpus = n_gpus
        self.pg = None

    def init(self, backend: str = "nccl"):
        import datetime

        import torch
        import torch.distributed as dist

        if self.world > 1:
            if backend == "nccl":
                torch.cuda.set_device(self.local_rank)
            dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=120))
            self.pg = dist.group.WORLD

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier()

    def max(self, value: float) -> float:
        if self.world == 1:
            return value
        import torch
        import torch.distributed as dist

        t = torch.tensor([value], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()


# ------------------------------------------------------------------------ workloads
def seeded(shape, seed, dist, dtype, device="cuda"):
    import torch

    gen = torch.Generator(device=device).manual_seed(seed)
    if dist == "uniform":
        x = torch.rand(shape, generator=gen, device=device) * 2 - 1
    elif dist == "uniform16":
        x = (torch.rand(shape, generator=gen, device=device) * 2 - 1) / 16
    elif dist == "normal64":
        x = torch.randn(shape, generator=gen, device=device) / 64
    elif dist == "normal":
        x = torch.randn(shape, generator=gen, device=device)
    else:  # "normal/<fan_in>"
        x = torch.randn(shape, generator=gen, device=device) / float(dist.split("/")[1]) ** 0.5
    return x.to({"bf16": torch.bfloat16, "fp16": torch.float16}[dtype])


def gemv_bytes(m, n, k):
    return (n * k + m * k + m * n) * 2


def time_loop(fn, steps: int, stream) -> float:
    """Total device milliseconds of `steps` calls on `stream` (events on that stream)."""

    import torch

    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(steps):
        fn(i)
    stop.record(stream)
    stop.synchronize()
    return start.elapsed_time(stop)


L2_BYTES = 126 * 1024 * 1024
DRAM_INTERFACE_GBS = 8161.3  # ncu: 2048 B per DRAM cycle at 3.985 GHz (B200)
HEAD_M, HEAD_N, HEAD_K = 1, 8192, 8192


def rotation(block_bytes: int) -> int:
    """Weight sets a rank cycles through: at least ROTATE, and more than 2 x L2 in total."""

    return max(ROTATE, -(-2 * L2_BYTES // block_bytes) + 1)


def headline_config(world: int) -> dict:
    """The workload description both arms print (the driver compares them)."""

    return {
        "workload": "gemv-decode-bf16-m1-n8192-k8192 (BASELINE config 2), x @ W^T over the whole "
        "8192 x 8192 weight per step; N > 1: weight rows split over the N GPUs, output all-gathered "
        "inside the step",
        "m": HEAD_M,
        "n": HEAD_N,
        "k": HEAD_K,
        "n_per_gpu": HEAD_N // world,
        "l2": "inputs larger than L2: weight sets rotated per step, > 2 x 126 MB per GPU",
        "parallelism": "single GPU" if world == 1 else f"weight-row shards x{world} + fused NVLink all-gather",
    }


def capture_graph(step, count: int, stream, offset: int = 0):
    """CUDA graph of `count` calls step(offset + i), captured on a side stream."""

    import torch

    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    cap.wait_stream(stream)
    with torch.cuda.stream(cap):
        with torch.cuda.graph(graph, stream=cap):
            for i in range(count):
                step(offset + i)
    stream.wait_stream(cap)
    torch.cuda.synchronize()
    return graph


class ExactReplay:
    """Runs exactly `steps` calls of `step` as replays of (at most) two captured graphs."""

    def __init__(self, step, steps: int, stream, block: int = 40):
        self.block = max(1, min(block, steps))
        self.full = steps // self.block
        self.main = capture_graph(step, self.block, stream)
        rest = steps - self.full * self.block
        self.tail = capture_graph(step, rest, stream, offset=self.full * self.block) if rest else None

    def __call__(self, _i=0):
        for _ in range(self.full):
            self.main.replay()
        if self.tail is not None:
            self.tail.replay()

    def release(self):
        self.main = self.tail = None


def timed_region(run, dist: Dist, stream) -> tuple[float, float]:
    """(max-over-ranks ms, this rank's ms) of one call of run(), barrier + sync on both sides."""

    import torch

    dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    run()
    stop.record(stream)
    stop.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    local = start.elapsed_time(stop)
    return dist.max(local), local


def sharded_weights(dist: Dist, dtype: str = "bf16"):
    rows = HEAD_N // dist.world
    count = rotation(rows * HEAD_K * 2)
    return [seeded((rows, HEAD_K), 100 + 17 * dist.rank + r, "normal/8192", dtype) for r in range(count)]


def headline(args, dist: Dist, ext, peaks, peak_kind):
    """Config 2 decode GEMV, kernel-only, inputs resident; CUDA graphs of the launch loop.

    N = 1: ``rk_gemv`` over the full weight.  N > 1: ``rk_gemv_allgather`` over this rank's
    row block (the fused all-gather), exactly ``--steps`` launches per rank; the plain
    ``rk_gemv`` of the block alone is timed too, so the exchange's share is visible.
    """

    import torch

    m, k = HEAD_M, HEAD_K
    rows = HEAD_N // dist.world
    weights = sharded_weights(dist)
    x = seeded((m, k), 1, "normal", "bf16")
    stream = torch.cuda.current_stream()
    local_out = torch.empty(m, rows, dtype=x.dtype, device="cuda")

    def compute_only(i):
        ext.gemv_out(x, weights[i % len(weights)], local_out, 0)

    exchange = None
    if dist.world > 1:
        from radeon_kernels.distributed.peer import PeerExchange, fused_path_available

        if not fused_path_available(x):
            raise RuntimeError("bench: the fused all-gather needs every rank on its own NVLink-connected GPU")
        exchange = PeerExchange((m, HEAD_N), x.dtype)

        def step(i):
            ext.gemv_allgather(x, weights[i % len(weights)], exchange.output, exchange.out_ptrs,
                               exchange.ctl_ptrs, exchange.rank, exchange.timeout_ns)
    else:
        step = compute_only

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    if exchange is not None:
        # The gathered output equals the single-GPU kernel's on the concatenated weight blocks.
        local = ext.gemv_out(x, weights[(max(args.warmup, 3) - 1) % len(weights)],
                             torch.empty(m, rows, dtype=x.dtype, device="cuda"), 2)
        mine = exchange.output[:, dist.rank * rows:(dist.rank + 1) * rows]
        if not torch.equal(mine.view(torch.int16), local.view(torch.int16)):
            raise RuntimeError("bench: the fused all-gather output differs from the local GEMV")

    steps = args.steps
    runner = ExactReplay(step, steps, stream)
    runner()  # warm replay
    torch.cuda.synchronize()
    ms, ms_local = timed_region(runner, dist, stream)
    runner.release()
    per_launch_s = ms_local / 1e3 / steps

    compute = None
    if exchange is not None:
        plain = ExactReplay(compute_only, steps, stream)
        plain()
        torch.cuda.synchronize()
        c_ms, _ = timed_region(plain, dist, stream)
        plain.release()
        compute = {"us_per_step": round(c_ms * 1e3 / steps, 3),
                   "what": "rk_gemv over the rank's row block alone (no exchange), same rotation"}

    # Context for the roofline: one launch with nothing before it to overlap, so the L2
    # prefetch each CTA issues before its dependency wait hides nothing.  The L2 flush
    # (two 256 MiB writes, ~80 us of device time) is still running when the events and the
    # launch are enqueued, so no host launch latency falls between the events.
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    isolated = []
    for i in range(21):
        flush.zero_()
        flush.zero_()
        isolated.append(time_loop(lambda j: compute_only(i), 1, stream))
    del flush
    torch.cuda.synchronize()

    bytes_step = gemv_bytes(m, HEAD_N, k)  # the whole logical problem, per step
    # Per-rank algorithmic HBM bytes of one launch: the weight block and x read, the full
    # output written into this rank's memory (its own block and every peer's).
    rank_bytes = (rows * k + m * k + m * HEAD_N) * 2
    value = bytes_step * steps / (ms / 1e3) / 1e9
    achieved = rank_bytes / per_launch_s / 1e9
    result = {
        "value": value,
        "ms_per_step": ms / steps,
        "steps": steps,
        "roofline": {
            "bound": "hbm",
            "achieved": round(achieved, 1),
            "peak": peaks["hbm_gbs"],
            "unit": "GB/s",
            "frac": round(achieved / peaks["hbm_gbs"], 4),
            "peak_source": peak_kind,
            "kernel": "gemv_stream_kernel" + ("<PEER> (rk_gemv_allgather)" if exchange is not None else " (rk_gemv)"),
            "bytes_per_launch": rank_bytes,
            "isolated_launch": {
                "us": round(statistics.median(isolated) * 1e3, 2),
                "gbs": round(gemv_bytes(m, rows, k) / (statistics.median(isolated) / 1e3) / 1e9, 1),
                "what": "rk_gemv of the rank's weight block alone, L2 flushed before it, median of 21",
            },
            "dram_interface": {
                "gbs": DRAM_INTERFACE_GBS,
                "frac": round(achieved / DRAM_INTERFACE_GBS, 4),
                "what": "ncu dram__bytes.sum.peak_sustained (2048 B/cycle) x dram__cycles_elapsed.avg.per_second "
                        "(3.985 GHz) on B200; the measured peak above is a copy (reads and writes)",
            },
        },
        "bytes_per_step": bytes_step,
        "weight_sets_per_rank": len(weights),
        "launch": f"CUDA graphs replayed for exactly {steps} launches per rank (blocks of {runner.block})",
    }
    if compute is not None:
        result["compute_only"] = compute
        result["exchange_us_per_step"] = round(ms * 1e3 / steps - compute["us_per_step"], 3)
    if exchange is not None:
        exchange.close()
    return result


E2E_GRAPH_STEPS = 64  # independent steps captured in one CUDA graph (multiple of ROTATE and E2E_COPY_GROUP)
E2E_COPY_GROUP = 8  # N = 1: input copies issued per group, a group ahead of the kernels that read them


def e2e(args, dist: Dist):
    """The same GEMV through the public API with host buffers, copies inside the region.

    Every step copies its activation host->device from pinned memory, calls the public API
    (validation, dispatch, pack winner) and copies the full result back into pinned memory.
    N = 1: ``radeon_kernels.gemv``; the reported value comes from a CUDA graph captured from
    those calls: 64 independent steps, each with its own H2D copy and its own D2H copy.  The
    H2D copies run on a forked copy stream in groups of 8, which it works through in order, so
    a group's copies run while the kernels of the group before it run; one join precedes the
    group's first kernel.  Each D2H runs on
    a second stream right after its kernel.  A join in front of every kernel measured 2.7-3 us
    more per step (the kernel then cannot start early on its predecessor's tail).
    ``eager_serial`` is the same step issued eagerly with copy, kernel and copy serialised on
    one stream (the per-call latency).  N > 1: ``ShardedGemv(..., gather=True)`` (the fused
    all-gather kernel) in the same graph of 64 steps, in groups no larger than the number of
    exchange buffers: a gathered output buffer is rewritten by the next call on it, so its
    copy must finish first, and one join per group covers that too.
    """

    if dist.world > 1:
        return e2e_sharded(args, dist)

    import torch

    import radeon_kernels as rk

    m, n, k = HEAD_M, HEAD_N, HEAD_K
    weights = [seeded((n, k), 100 + r, "normal/8192", "bf16") for r in range(ROTATE)]
    bytes_step = gemv_bytes(m, n, k)
    stream = torch.cuda.current_stream()

    def rate(ms, steps):
        return round(bytes_step * steps / (ms / 1e3) / 1e9, 1)

    # Eager, serialised: copy in, GEMV, copy out, one stream.
    x_host = seeded((m, k), 1, "normal", "bf16", device="cpu").pin_memory()
    out_host = torch.empty((m, n), dtype=torch.bfloat16).pin_memory()
    x_dev = torch.empty((m, k), dtype=torch.bfloat16, device="cuda")

    def step(i):
        x_dev.copy_(x_host, non_blocking=True)
        out_host.copy_(rk.gemv(x_dev, weights[i % ROTATE]), non_blocking=True)

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    selected = rk.get_last_dispatch()["selected"]
    eager_steps = max(args.e2e_steps // 4, 10)
    dist.barrier()
    torch.cuda.synchronize()
    eager_ms = dist.max(time_loop(step, eager_steps, stream))
    dist.barrier()
    eager = {"value": rate(eager_ms, eager_steps), "ms_per_step": round(eager_ms / eager_steps, 5)}
    result = {"unit": "GB/s", "h2d_bytes_per_step": m * k * 2, "d2h_bytes_per_step": m * n * 2}

    G = E2E_GRAPH_STEPS
    xs_host = seeded((G, m, k), 2, "normal", "bf16", device="cpu").pin_memory()
    outs_host = torch.empty((G, m, n), dtype=torch.bfloat16).pin_memory()
    xs_dev = torch.empty((G, m, k), dtype=torch.bfloat16, device="cuda")
    h2d = torch.cuda.Stream()
    d2h = torch.cuda.Stream()
    cap = torch.cuda.Stream()
    kept = []

    def graph_body():
        here = torch.cuda.current_stream()
        h2d.wait_stream(here)
        d2h.wait_stream(here)
        ready = []
        with torch.cuda.stream(h2d):
            # Every step's input is copied separately; a group's copies complete on one event.
            for g0 in range(0, G, E2E_COPY_GROUP):
                for i in range(g0, g0 + E2E_COPY_GROUP):
                    xs_dev[i].copy_(xs_host[i], non_blocking=True)
                ready.append(torch.cuda.Event())
                ready[-1].record(h2d)
        for i in range(G):
            if i % E2E_COPY_GROUP == 0:
                here.wait_event(ready[i // E2E_COPY_GROUP])
            y = rk.gemv(xs_dev[i], weights[i % ROTATE])
            kept.append(y)
            done = torch.cuda.Event()
            done.record(here)
            d2h.wait_event(done)
            with torch.cuda.stream(d2h):
                outs_host[i].copy_(y, non_blocking=True)
        here.wait_stream(h2d)
        here.wait_stream(d2h)

    cap.wait_stream(stream)
    with torch.cuda.stream(cap):
        graph_body()  # eager warm-up: dispatch decisions and tensor maps are cached
    torch.cuda.synchronize()
    kept.clear()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=cap):
        graph_body()
    stream.wait_stream(cap)
    torch.cuda.synchronize()
    outs_host.zero_()
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    # The graph's results are the eager API's results, bit for bit.
    check = all(torch.equal(outs_host[i], rk.gemv(xs_dev[i], weights[i % ROTATE]).cpu()) for i in range(G))
    if not check:
        raise RuntimeError("e2e: graph-replayed rk.gemv results differ from eager calls")
    replays = max(args.e2e_steps // G, 10)
    dist.barrier()
    torch.cuda.synchronize()
    ms = dist.max(time_loop(lambda i: graph.replay(), replays, stream))
    dist.barrier()
    del graph
    steps = replays * G
    result.update({
        "value": rate(ms, steps),
        "ms_per_step": round(ms / steps, 5),
        "path": (f"CUDA graph of {G} captured steps: pinned H2D copy per step (forked copy stream, "
                 f"groups of {E2E_COPY_GROUP} issued a group ahead), "
                 f"radeon_kernels.gemv -> {selected}, pinned D2H copy (second stream); "
                 "outputs checked equal to eager calls"),
        "eager_serial": eager,
    })
    return result


def e2e_sharded(args, dist: Dist):
    """N > 1: per step a pinned H2D copy of x, ``ShardedGemv(gather=True)`` (the fused
    all-gather kernel) and a pinned D2H copy of the full output, 16 steps captured into one
    CUDA graph and replayed.  As at N = 1 the input copies run ahead on a copy stream and each
    output copy runs on a second stream right after its kernel; the operators rotate over the
    weight sets, each with its own exchange buffer, and a step's kernel waits for the output
    copy of the step that last used its buffer (the fused call rewrites it)."""

    import torch

    from radeon_kernels.distributed import ShardedGemv

    m, n, k = HEAD_M, HEAD_N, HEAD_K
    weights = sharded_weights(dist)
    operators = [ShardedGemv(w, n_total=n) for w in weights]
    R = len(operators)
    stream = torch.cuda.current_stream()
    G = E2E_GRAPH_STEPS
    xs_host = seeded((G, m, k), 2, "normal", "bf16", device="cpu").pin_memory()
    outs_host = torch.empty((G, m, n), dtype=torch.bfloat16).pin_memory()
    xs_dev = torch.empty((G, m, k), dtype=torch.bfloat16, device="cuda")
    h2d, d2h, cap = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()

    for i in range(max(args.warmup, 3, R)):
        operators[i % R](xs_dev[i % G], gather=True)  # first call of each operator: collective set-up
    torch.cuda.synchronize()

    # Steps in groups of at most R (one exchange buffer per operator): a group's inputs are
    # copied in while the group before it runs, and before its first kernel one join on its
    # inputs and one on the output copy that frees the last buffer it reuses (the copy stream
    # works in order, so that covers the group's other buffers too).
    gsz = min(E2E_COPY_GROUP, R)
    groups = [range(g0, min(g0 + gsz, G)) for g0 in range(0, G, gsz)]

    def graph_body():
        here = torch.cuda.current_stream()
        h2d.wait_stream(here)
        d2h.wait_stream(here)
        ready, copied = [], []
        with torch.cuda.stream(h2d):
            for grp in groups:
                for i in grp:
                    xs_dev[i].copy_(xs_host[i], non_blocking=True)
                ready.append(torch.cuda.Event())
                ready[-1].record(h2d)
        for gi, grp in enumerate(groups):
            here.wait_event(ready[gi])
            if grp.stop - 1 - R >= 0:
                here.wait_event(copied[grp.stop - 1 - R])  # every buffer of this group copied out
            for i in grp:
                y = operators[i % R](xs_dev[i], gather=True)
                done = torch.cuda.Event()
                done.record(here)
                d2h.wait_event(done)
                with torch.cuda.stream(d2h):
                    outs_host[i].copy_(y, non_blocking=True)
                    copied.append(torch.cuda.Event())
                    copied[-1].record(d2h)
        here.wait_stream(h2d)
        here.wait_stream(d2h)

    cap.wait_stream(stream)
    with torch.cuda.stream(cap):
        graph_body()  # eager run of the same body
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=cap):
        graph_body()
    stream.wait_stream(cap)
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    # Spot check: the replayed outputs equal the rank-local product on this rank's block.
    rows = n // dist.world
    from radeon_kernels import _native

    ext = _native.extension()
    for i in (0, G - 1):
        local = ext.gemv_out(xs_dev[i], weights[i % R], torch.empty(m, rows, dtype=torch.bfloat16, device="cuda"), 2)
        if not torch.equal(outs_host[i][:, dist.rank * rows:(dist.rank + 1) * rows], local.cpu()):
            raise RuntimeError("e2e: gathered output differs from the local block product")
    replays = max(args.e2e_steps // G, 10)
    ms, _ = timed_region(lambda: [graph.replay() for _ in range(replays)], dist, stream)
    del graph
    for op in operators:
        op.close()
    steps = replays * G
    return {
        "unit": "GB/s",
        "h2d_bytes_per_step": m * k * 2,
        "d2h_bytes_per_step": m * n * 2,
        "value": round(gemv_bytes(m, n, k) * steps / (ms / 1e3) / 1e9, 1),
        "ms_per_step": round(ms / steps, 5),
        "path": (f"CUDA graph of {G} captured steps: pinned H2D copy per step (forked copy stream, "
                 f"groups of {gsz} issued a group ahead), "
                 "radeon_kernels.distributed.ShardedGemv(gather=True) -> rk_gemv_allgather, pinned D2H "
                 "copy of the full output (second stream); outputs spot-checked against the local block"),
    }


def suite(args, dist: Dist, ext, peaks):
    """The other BASELINE configs (kernel-only, events on the launching stream)."""

    import torch

    results = {}
    stream = torch.cuda.current_stream()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    wanted = re.compile(args.suite_filter).search if args.suite_filter else (lambda name: True)

    def gemm_case(name, m, n, k, dtype, dist_name, seed, iters, scaling="replica", graph=False):
        if not wanted(name):
            return
        a = seeded((m, k), seed, dist_name, dtype)
        b = seeded((k, n), seed + 1, dist_name, dtype)
        c = torch.empty(m, n, dtype=a.dtype, device="cuda")
        for _ in range(2):
            ext.gemm_out(a, b, c, 0)
        torch.cuda.synchronize()
        if graph:
            # Small problems: launch-latency bound; measured as a CUDA graph of 20
            # back-to-back launches (inputs stay L2-resident, as they do in a model).
            g = torch.cuda.CUDAGraph()
            cap = torch.cuda.Stream()
            cap.wait_stream(stream)
            with torch.cuda.stream(cap):
                with torch.cuda.graph(g, stream=cap):
                    for _ in range(20):
                        ext.gemm_out(a, b, c, 0)
            stream.wait_stream(cap)
            torch.cuda.synchronize()
            g.replay()
            torch.cuda.synchronize()
            times = [time_loop(lambda i: g.replay(), 1, stream) / 20 for _ in range(iters)]
            lib_times = []
            del g
        else:
            # Interleaved with the same product through torch.mm (cuBLAS), a reference point for
            # the shape (not part of this library): both see the same clock and power state.
            times, lib_times = [], []
            torch.mm(a, b, out=c)
            for _ in range(iters):
                flush.zero_()  # L2 flush between timed launches
                times.append(time_loop(lambda i: ext.gemm_out(a, b, c, 0), 1, stream))
                flush.zero_()
                lib_times.append(time_loop(lambda i: torch.mm(a, b, out=c), 1, stream))
        dist.barrier()
        ms = dist.max(statistics.median(times))
        flops = 2.0 * m * n * k
        achieved = flops / (ms / 1e3) / 1e12
        results[name] = {
            "unit": "TFLOP/s",
            "value": round(achieved * dist.world, 1),
            "per_gpu": round(achieved, 1),
            "ms": round(ms, 4),
            "roofline_frac": round(achieved / peaks["bf16_tflops"], 4),
            "scaling": scaling,
            "shape": [m, n, k],
            "dtype": dtype,
            "timing": "CUDA graph of 20 launches, L2-warm" if graph else "single launch, L2 flushed",
        }
        if not graph:
            lib_ms = statistics.median(lib_times)
            results[name]["torch_mm_cublas_tflops"] = round(flops / (lib_ms / 1e3) / 1e12, 1)
        del a, b, c

    def gemv_case(name, m, n, k, dtype, seed, iters):
        if not wanted(name):
            return
        ws = [seeded((n, k), seed + r, f"normal/{k}", dtype) for r in range(ROTATE)]
        x = seeded((m, k), seed, "normal", dtype)
        out = torch.empty(m, n, dtype=x.dtype, device="cuda")
        for i in range(3):
            ext.gemv_out(x, ws[i % ROTATE], out, 0)
        torch.cuda.synchronize()
        # Same launch discipline as the headline: a CUDA graph of 40 launches over the
        # rotated weights, replayed.
        g = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream()
        cap.wait_stream(stream)
        with torch.cuda.stream(cap):
            with torch.cuda.graph(g, stream=cap):
                for i in range(40):
                    ext.gemv_out(x, ws[i % ROTATE], out, 0)
        stream.wait_stream(cap)
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        reps = max(1, iters // 40)
        ms = time_loop(lambda i: g.replay(), reps, stream) / (reps * 40)
        del g
        dist.barrier()
        ms = dist.max(ms)
        gbs = gemv_bytes(m, n, k) / (ms / 1e3) / 1e9
        results[name] = {
            "unit": "GB/s",
            "value": round(gbs * dist.world, 1),
            "per_gpu": round(gbs, 1),
            "us": round(ms * 1e3, 2),
            "roofline_frac": round(gbs / peaks["hbm_gbs"], 4),
            "scaling": "weak",
        }
        del ws

    def neighbour_case(name, op, tokens, hidden, dtype, seed):
        """silu_mul / rms_norm / add_rms_norm and their backward passes: HBM streams (bytes
        each launch must move: every input read once, every output written once)."""

        if not wanted(name):
            return
        elems = tokens * hidden
        streams = {
            "silu_mul": 3, "rms_norm": 2, "add_rms_norm": 4,
            "silu_mul_backward": 5,  # dy, gate, up -> grad_gate, grad_up
            "rms_norm_backward": 3,  # dy, x -> grad_x (+ weight in, grad_weight out)
            "add_rms_norm_backward": 5,  # dy, residual_out, d(residual_out) -> grad_x, grad_residual
        }[op]
        vectors = {"silu_mul": 0, "silu_mul_backward": 0, "rms_norm_backward": 2, "add_rms_norm_backward": 2}.get(op, 1)
        per_set = streams * elems * 2 + vectors * hidden * 2
        # Enough rotated input sets that a replay cycle touches > 2 x L2 (decode-sized cases
        # stay L2-resident whatever: they are launch-latency bound and reported as such).
        sets = max(2, min(64, -(-300_000_000 // per_set)))
        gen = torch.Generator(device="cuda").manual_seed(seed)
        tdt = {"bf16": torch.bfloat16, "fp16": torch.float16}[dtype]
        a = [torch.randn((tokens, hidden), generator=gen, device="cuda").to(tdt) for _ in range(sets)]
        b = [torch.randn((tokens, hidden), generator=gen, device="cuda").to(tdt) for _ in range(sets)]
        w = (1 + 0.1 * torch.randn((hidden,), generator=gen, device="cuda")).to(tdt)
        c = [torch.randn((tokens, hidden), generator=gen, device="cuda").to(tdt) for _ in range(sets)] if op in (
            "silu_mul_backward", "add_rms_norm_backward") else None
        if op == "silu_mul":
            step = lambda i: ext.silu_mul(a[i % sets], b[i % sets])  # noqa: E731
        elif op == "rms_norm":
            step = lambda i: ext.rms_norm(a[i % sets], w, 1e-6)  # noqa: E731
        elif op == "add_rms_norm":
            step = lambda i: ext.add_rms_norm(a[i % sets], b[i % sets], w, 1e-6)  # noqa: E731
        elif op == "silu_mul_backward":
            step = lambda i: ext.silu_mul_backward(a[i % sets], b[i % sets], c[i % sets])  # noqa: E731
        elif op == "rms_norm_backward":
            step = lambda i: ext.rms_norm_backward(a[i % sets], b[i % sets], w, 1e-6, True)  # noqa: E731
        else:
            step = lambda i: ext.add_rms_norm_backward(a[i % sets], c[i % sets], b[i % sets], w, 1e-6, True)  # noqa: E731
        for i in range(3):
            step(i)
        torch.cuda.synchronize()
        launches = max(20, sets)
        g = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream()
        cap.wait_stream(stream)
        with torch.cuda.stream(cap):
            with torch.cuda.graph(g, stream=cap):
                for i in range(launches):
                    step(i)
        stream.wait_stream(cap)
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        reps = 10
        ms = time_loop(lambda i: g.replay(), reps, stream) / (reps * launches)
        del g
        dist.barrier()
        ms = dist.max(ms)
        gbs = per_set / (ms / 1e3) / 1e9
        results[name] = {
            "unit": "GB/s",
            "value": round(gbs * dist.world, 1),
            "per_gpu": round(gbs, 1),
            "us": round(ms * 1e3, 2),
            "roofline_frac": round(gbs / peaks["hbm_gbs"], 4),
            "scaling": "replica",
            "shape": [tokens, hidden],
            "dtype": dtype,
            "timing": f"CUDA graph of {launches} launches over {sets} input sets"
            + (" (L2-resident: launch-latency bound)" if per_set * sets < 256_000_000 else ""),
        }
        del a, b, c

    def paged_case(name, batch, hq, hkv, ctx, d, bs, dtype, seed):
        """Paged decode attention: bytes = the K/V cache positions every sequence reads."""

        if not wanted(name):
            return
        tdt = {"bf16": torch.bfloat16, "fp16": torch.float16}[dtype]
        maxb = -(-ctx // bs)
        kv_bytes = batch * ctx * hkv * d * 2 * 2
        io_bytes = 2 * batch * hq * d * 2
        sets = max(2, min(32, -(-300_000_000 // kv_bytes)))
        gen = torch.Generator(device="cuda").manual_seed(seed)
        cases = []
        for _ in range(sets):
            nb = batch * maxb
            q = torch.randn((batch, hq, d), generator=gen, device="cuda").to(tdt)
            k = torch.randn((nb, bs, hkv, d), generator=gen, device="cuda").to(tdt)
            v = torch.randn((nb, bs, hkv, d), generator=gen, device="cuda").to(tdt)
            tables = torch.randperm(nb, generator=gen, device="cuda").view(batch, maxb).to(torch.int32)
            lens = torch.full((batch,), ctx, dtype=torch.int32, device="cuda")
            cases.append((q, k, v, tables, lens))
        scale = d ** -0.5
        step = lambda i: ext.paged_attention_decode(*cases[i % sets], scale)  # noqa: E731
        launches = max(20, sets)
        from radeon_kernels import _native

        lib = _native.library()

        def time_path(path):
            # The kernel choice is read when a call is launched, so a graph captured under a
            # path keeps that kernel.
            lib.rk_paged_attention_set_path(path)
            try:
                for i in range(3):
                    step(i)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                cap = torch.cuda.Stream()
                cap.wait_stream(stream)
                with torch.cuda.stream(cap):
                    with torch.cuda.graph(g, stream=cap):
                        for i in range(launches):
                            step(i)
                stream.wait_stream(cap)
                torch.cuda.synchronize()
                g.replay()
                torch.cuda.synchronize()
                reps = 10
                t = time_loop(lambda i: g.replay(), reps, stream) / (reps * launches)
                del g
            finally:
                lib.rk_paged_attention_set_path(0)
            dist.barrier()
            return dist.max(t)

        ms = time_path(0)
        ms_cuda_cores = time_path(1)
        tc_auto = d in (64, 128) and hq // hkv <= 16 and bs in (8, 16, 32, 64, 128) and not (hq == hkv and d == 64)
        gbs = (kv_bytes + io_bytes) / (ms / 1e3) / 1e9
        results[name] = {
            "unit": "GB/s",
            "value": round(gbs * dist.world, 1),
            "per_gpu": round(gbs, 1),
            "us": round(ms * 1e3, 2),
            "roofline_frac": round(gbs / peaks["hbm_gbs"], 4),
            "scaling": "replica",
            "shape": {"batch": batch, "query_heads": hq, "kv_heads": hkv, "context": ctx, "head_dim": d, "block_size": bs},
            "kernel": "tcgen05" if tc_auto else "cuda cores",
            "cuda_cores_us": round(ms_cuda_cores * 1e3, 2),
            "dtype": dtype,
            "timing": f"CUDA graph of {launches} launches over {sets} caches"
            + (" (L2-resident: latency bound)" if kv_bytes * sets < 256_000_000 else ""),
        }
        del cases

    def ffn_swiglu_case(name, m, n, k, dtype, iters):
        """Fused FFN-up + SwiGLU: both products (2 x 2MNK FLOP) and the epilogue, one kernel."""

        if not wanted(name):
            return
        gen = torch.Generator(device="cuda").manual_seed(3)
        tdt = {"bf16": torch.bfloat16, "fp16": torch.float16}[dtype]
        a = (torch.randn((m, k), generator=gen, device="cuda") / 64).to(tdt)
        b = (torch.randn((k, 2 * n), generator=gen, device="cuda") / 64).to(tdt)
        for _ in range(2):
            ext.gemm_swiglu(a, b, 0)
        torch.cuda.synchronize()
        times = []
        for _ in range(iters):
            flush.zero_()  # L2 flush between timed launches
            times.append(time_loop(lambda i: ext.gemm_swiglu(a, b, 0), 1, stream))
        dist.barrier()
        ms = dist.max(statistics.median(times))
        achieved = 2.0 * m * (2 * n) * k / (ms / 1e3) / 1e12
        results[name] = {
            "unit": "TFLOP/s",
            "value": round(achieved * dist.world, 1),
            "per_gpu": round(achieved, 1),
            "ms": round(ms, 4),
            "roofline_frac": round(achieved / peaks["bf16_tflops"], 4),
            "scaling": "replica",
            "shape": [m, n, k],
            "dtype": dtype,
            "timing": "single launch, L2 flushed; FLOP of both gate and up products",
        }
        del a, b

    def sdpa_case(name, b, hq, hkv, seq, d, causal, dtype, seed):
        """Prefill self-attention: FLOP counted as the reference's benchmark counts them
        (4 * batch * heads * head_dim * attended pairs, benchmarks/sdpa/benchmark.py:164-167).
        torch's scaled_dot_product_attention -- the reference's own fallback on a GPU
        (ops/sdpa/reference.py:39-57) -- is timed on the same inputs for comparison."""

        if not wanted(name):
            return
        import torch.nn.functional as F

        tdt = {"bf16": torch.bfloat16, "fp16": torch.float16}[dtype]
        per_set = (b * hq * seq * d + 2 * b * hkv * seq * d + b * hq * seq * d) * 2
        sets = max(2, min(32, -(-300_000_000 // per_set)))
        gen = torch.Generator(device="cuda").manual_seed(seed)
        draw = lambda shape: (torch.rand(shape, generator=gen, device="cuda") * 0.25 - 0.125).to(tdt)  # noqa: E731
        qkv = [(draw((b, hq, seq, d)), draw((b, hkv, seq, d)), draw((b, hkv, seq, d))) for _ in range(sets)]
        scale = d ** -0.5

        def graph_time(step):
            for i in range(3):
                step(i)
            torch.cuda.synchronize()
            launches = max(20, sets)
            g = torch.cuda.CUDAGraph()
            cap = torch.cuda.Stream()
            cap.wait_stream(stream)
            with torch.cuda.stream(cap):
                with torch.cuda.graph(g, stream=cap):
                    for i in range(launches):
                        step(i)
            stream.wait_stream(cap)
            torch.cuda.synchronize()
            g.replay()
            torch.cuda.synchronize()
            reps = 10
            ms = time_loop(lambda i: g.replay(), reps, stream) / (reps * launches)
            del g
            return ms

        ms = graph_time(lambda i: ext.sdpa(*qkv[i % sets], causal, scale))
        torch_ms = graph_time(lambda i: F.scaled_dot_product_attention(
            *qkv[i % sets], is_causal=causal, scale=scale, enable_gqa=hq != hkv))
        dist.barrier()
        ms = dist.max(ms)
        pairs = seq * (seq + 1) // 2 if causal else seq * seq
        tflops = 4.0 * b * hq * d * pairs / (ms / 1e3) / 1e12
        results[name] = {
            "unit": "TFLOP/s",
            "value": round(tflops * dist.world, 2),
            "per_gpu": round(tflops, 2),
            "us": round(ms * 1e3, 2),
            "torch_sdpa_us": round(torch_ms * 1e3, 2),
            "roofline_frac": round(tflops / peaks["bf16_tflops"], 4),
            "scaling": "replica",
            "shape": {"batch": b, "query_heads": hq, "kv_heads": hkv, "sequence": seq, "head_dim": d, "causal": causal},
            "dtype": dtype,
            "timing": f"CUDA graph over {sets} input sets (small cases: launch and latency bound)",
        }
        del qkv

    def c5_sharded_case(name, iters):
        """BASELINE config 5 with B split into N column blocks (strong scaling): the local
        product alone, the fused all-gather kernel (rk_gemm_allgather: every tile stored into
        every rank's C over NVLink while the next tile accumulates), and the NCCL form it
        replaces (local product, all_gather_into_tensor, rk_gather_column_blocks)."""

        if not wanted(name):
            return
        import torch.distributed as tdist

        from radeon_kernels.distributed.peer import PeerExchange

        M, N, K = 16384, 57344, 8192
        nb = N // g
        a = seeded((M, K), 4, "uniform16", "bf16")
        b = seeded((K, nb), 5 + dist.rank, "uniform16", "bf16")
        c_local = torch.empty(M, nb, dtype=a.dtype, device="cuda")
        exchange = PeerExchange((M, N), a.dtype)
        staged = torch.empty(g * M, nb, dtype=a.dtype, device="cuda")
        full = torch.empty(M, N, dtype=a.dtype, device="cuda")

        def compute():
            ext.gemm_out(a, b, c_local, 0)

        def fused():
            ext.gemm_allgather(a, b, exchange.output, exchange.out_ptrs, exchange.ctl_ptrs,
                               exchange.rank, exchange.timeout_ns)

        def nccl():
            ext.gemm_out(a, b, c_local, 0)
            tdist.all_gather_into_tensor(staged, c_local)
            ext.gather_column_blocks(staged.view(g, M, nb), full)

        def measure(fn):
            fn()
            torch.cuda.synchronize()
            times = []
            for _ in range(iters):
                flush.zero_()  # L2 flush between timed launches
                dist.barrier()
                times.append(time_loop(lambda i: fn(), 1, stream))
            dist.barrier()
            return dist.max(statistics.median(times))

        ms_compute = measure(compute)
        cool_down()
        ms_fused = measure(fused)
        cool_down()
        ms_nccl = measure(nccl)
        flops = 2.0 * M * N * K
        received = (g - 1) * M * nb * 2  # bytes of C each GPU receives from its peers
        # Roofline of the fused kernel: the slower of the tensor work at the sustained GEMM
        # peak and the bytes every GPU must receive at the measured 770 GB/s peer bandwidth.
        t_tensor = flops / g / (peaks["bf16_tflops_sustained"] * 1e12)
        t_link = received / 770e9
        target_ms = max(t_tensor, t_link) * 1e3
        results[name] = {
            "unit": "TFLOP/s",
            "value": round(flops / (ms_fused / 1e3) / 1e12, 1),
            "compute_only": {"ms": round(ms_compute, 4), "value": round(flops / (ms_compute / 1e3) / 1e12, 1),
                             "per_gpu": round(flops / g / (ms_compute / 1e3) / 1e12, 1),
                             "roofline_frac": round(flops / g / (ms_compute / 1e3) / 1e12 / peaks["bf16_tflops"], 4)},
            "with_gather_fused": {"ms": round(ms_fused, 4), "value": round(flops / (ms_fused / 1e3) / 1e12, 1),
                                  "gather_ms": round(ms_fused - ms_compute, 4),
                                  "nvlink_recv_gbs_per_gpu": round(received / (ms_fused / 1e3) / 1e9, 1),
                                  "vs_compute_only": round(ms_compute / ms_fused, 4)},
            "with_gather_nccl": {"ms": round(ms_nccl, 4), "value": round(flops / (ms_nccl / 1e3) / 1e12, 1),
                                 "gather_ms": round(ms_nccl - ms_compute, 4)},
            "roofline": {"bound": "nvlink" if t_link > t_tensor else "tensor", "target_ms": round(target_ms, 4),
                         "frac": round(target_ms / ms_fused, 4),
                         "basis": "max(2MNK/G / sustained bf16 peak, received bytes / 770 GB/s per GPU)"},
            "scaling": "strong",
            "shape": [M, N, K],
            "n_per_gpu": nb,
            "dtype": "bf16",
            "timing": "single call, L2 flushed, median of %d, max over ranks" % iters,
        }
        exchange.close()
        del a, b, c_local, staged, full, exchange

    def cool_down():
        # Let the power/clock state recover between long GEMM cases so one case's
        # power capping does not leak into the next measurement.
        torch.cuda.synchronize()
        time.sleep(1.0)

    g = dist.world
    # Config 1 first: a 7-10 us launch-bound case is sensitive to the clock state that the
    # heavier cases below leave behind.
    gemm_case("c1_gemm_1024_bf16", 1024, 1024, 1024, "bf16", "uniform", 0, 10, graph=True)
    for m in (1, 4, 16):
        gemv_case(f"c2_gemv_decode_bf16_m{m}", m, 8192, 8192, "bf16", 1, 400)
    for m in (1, 4, 16):
        gemv_case(f"c3_gemv_ffn_down_fp16_m{m}", m, 4096, 14336, "fp16", 2, 400)
    # Decode neighbours, the reference's workload cases (benchmarks/workloads/*.yaml).
    neighbour_case("swiglu_decode_h11008_bf16", "silu_mul", 1, 11008, "bf16", 50)
    neighbour_case("swiglu_prefill_t1024_h11008_bf16", "silu_mul", 1024, 11008, "bf16", 51)
    neighbour_case("swiglu_prefill_t512_h28672_bf16", "silu_mul", 512, 28672, "bf16", 52)
    neighbour_case("add_rms_norm_decode_h4096_bf16", "add_rms_norm", 1, 4096, "bf16", 53)
    neighbour_case("add_rms_norm_prefill_t2048_h4096_bf16", "add_rms_norm", 2048, 4096, "bf16", 54)
    neighbour_case("add_rms_norm_prefill_t1024_h8192_bf16", "add_rms_norm", 1024, 8192, "bf16", 55)
    neighbour_case("rms_norm_prefill_t2048_h4096_bf16", "rms_norm", 2048, 4096, "bf16", 56)
    neighbour_case("swiglu_backward_t1024_h11008_bf16", "silu_mul_backward", 1024, 11008, "bf16", 57)
    neighbour_case("rms_norm_backward_t2048_h4096_bf16", "rms_norm_backward", 2048, 4096, "bf16", 58)
    neighbour_case("add_rms_norm_backward_t2048_h4096_bf16", "add_rms_norm_backward", 2048, 4096, "bf16", 59)
    neighbour_case("rms_norm_backward_decode_h4096_bf16", "rms_norm_backward", 1, 4096, "bf16", 60)
    # Paged decode attention, the reference's workload cases (paged_attention_decode-1.0.yaml).
    paged_case("paged_b1_gqa32x8_c4096_d128_bf16", 1, 32, 8, 4096, 128, 16, "bf16", 60)
    paged_case("paged_b8_gqa32x8_c1024_d128_bf16", 8, 32, 8, 1024, 128, 16, "bf16", 61)
    paged_case("paged_b16_gqa32x8_c2048_d128_bf16", 16, 32, 8, 2048, 128, 16, "bf16", 62)
    paged_case("paged_b4_mha16_c2048_d64_bf16", 4, 16, 16, 2048, 64, 32, "bf16", 63)
    paged_case("paged_b4_gqa32x8_c1024_d256_bf16", 4, 32, 8, 1024, 256, 16, "bf16", 64)
    # Larger batches: HBM-bound (about 0.5 GB of cache per call).
    paged_case("paged_b64_gqa32x8_c2048_d128_bf16", 64, 32, 8, 2048, 128, 16, "bf16", 65)
    paged_case("paged_b8_mha32_c4096_d128_bf16", 8, 32, 32, 4096, 128, 16, "bf16", 66)
    # Prefill attention, the reference's workload cases (benchmarks/workloads/sdpa-1.0.yaml),
    # plus one long-sequence case that is tensor-core rather than latency bound.
    sdpa_case("sdpa_b1_mha16_s128_d64_causal_bf16", 1, 16, 16, 128, 64, True, "bf16", 70)
    sdpa_case("sdpa_b1_gqa32x8_s512_d128_causal_bf16", 1, 32, 8, 512, 128, True, "bf16", 71)
    sdpa_case("sdpa_b4_gqa32x8_s128_d128_causal_bf16", 4, 32, 8, 128, 128, True, "bf16", 72)
    sdpa_case("sdpa_b1_mha16_s256_d64_full_bf16", 1, 16, 16, 256, 64, False, "bf16", 73)
    sdpa_case("sdpa_b2_gqa16x4_s256_d256_causal_bf16", 2, 16, 4, 256, 256, True, "bf16", 74)
    sdpa_case("sdpa_b4_gqa32x8_s4096_d128_causal_bf16", 4, 32, 8, 4096, 128, True, "bf16", 75)
    cool_down()
    gemm_case("c4_gemm_ffn_up_fp16", 4096, 14336, 4096, "fp16", "normal64", 3, 10)
    cool_down()
    ffn_swiglu_case("c4_ffn_up_swiglu_fused_fp16", 4096, 14336, 4096, "fp16", 10)
    cool_down()
    if not args.quick:
        gemm_case("gemm_8192_bf16", 8192, 8192, 8192, "bf16", "uniform16", 7, 5)
        cool_down()
    if g == 1:
        gemm_case("c5_gemm_large_bf16_shard1", 16384, 57344, 8192, "bf16", "uniform16", 4, 3, scaling="strong")
    else:
        c5_sharded_case(f"c5_gemm_large_bf16_shard{g}", 3)
    del flush
    return results


def cpu_baseline(seconds: float) -> dict:
    """The reference's CPU path (torch.mm on host tensors), bounded sample of config 2."""

    import torch

    from oracle import reference_path

    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    gen = torch.Generator().manual_seed(1)
    x = torch.randn((1, 8192), generator=gen).to(torch.bfloat16)
    w = (torch.randn((8192, 8192), generator=gen) / 8192**0.5).to(torch.bfloat16)
    for _ in range(3):
        reference_path.gemv_fallback(torch, x, w)
    calls, t0 = 0, time.perf_counter()
    while True:
        reference_path.gemv_fallback(torch, x, w)
        calls += 1
        elapsed = time.perf_counter() - t0
        if elapsed >= seconds or calls >= 20000:
            break
    gbs = gemv_bytes(1, 8192, 8192) * calls / elapsed / 1e9
    return {
        "value": round(gbs, 2),
        "unit": "GB/s",
        "cores": cores,
        "kind": "port",
        "sample": f"{calls} calls of oracle.reference_path.gemv_fallback (torch.mm, the reference's "
        f"ops/gemv/reference.py:12-15) on x[1,8192] @ W[8192,8192]^T bf16, {elapsed:.1f} s, {cores} threads",
        "cpu": _cpu_model(),
    }


def _cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args) -> int:
    """--impl reference: the reference's CPU implementation on the host cores (rank 0 only).

    The reference's path for config 2 is ``torch.mm(x, W.T)`` on host tensors
    (ops/gemv/reference.py:12-15, via oracle/reference_path.py) -- one call covers the whole
    8192 x 8192 weight, whatever N.  The timed region spans about ``--cpu-seconds`` (the
    window of the repo arm's ``cpu_baseline``): ``--steps`` steps of an equal number of
    calls each, the count calibrated from the warm-up calls, so the denominator of the
    driver's ratio is a stable sample rather than a few milliseconds.
    """

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    import torch

    from oracle import reference_path

    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    gen = torch.Generator().manual_seed(1)
    x = torch.randn((1, 8192), generator=gen).to(torch.bfloat16)
    w = (torch.randn((8192, 8192), generator=gen) / 8192**0.5).to(torch.bfloat16)
    warm = max(args.warmup, 3)
    t0 = time.perf_counter()
    for _ in range(warm):
        reference_path.gemv_fallback(torch, x, w)
    per_call = (time.perf_counter() - t0) / warm
    steps = max(1, args.steps)
    calls_per_step = max(1, int(round(args.cpu_seconds / steps / max(per_call, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(steps):
        for _ in range(calls_per_step):
            reference_path.gemv_fallback(torch, x, w)
    elapsed = time.perf_counter() - t0
    calls = steps * calls_per_step
    value = gemv_bytes(1, 8192, 8192) * calls / elapsed / 1e9
    sample = (f"{steps} steps x {calls_per_step} calls of torch.mm(x, W.T) on x[1,8192] @ W[8192,8192]^T bf16 "
              f"(ops/gemv/reference.py:12-15 via oracle/reference_path.py), {elapsed:.1f} s, {cores} threads")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": args.gpus if args.gpus else world,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": round(elapsed / calls * 1e3, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": DATA,
        "config": headline_config(max(1, args.gpus)),
        "cpu_baseline": {"value": round(value, 2), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": sample, "cpu": _cpu_model()},
        "e2e": {"value": round(value, 2), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


PROFILE_CASES = {
    # name: (kind, m, n, k, dtype, distribution)
    "gemv_decode": ("gemv", 1, 8192, 8192, "bf16", "normal/8192"),
    "gemv_decode_m16": ("gemv", 16, 8192, 8192, "bf16", "normal/8192"),
    "gemv_ffn_down_m4": ("gemv", 4, 4096, 14336, "fp16", "normal/14336"),
    "gemm_1024": ("gemm", 1024, 1024, 1024, "bf16", "uniform"),
    "gemm_ffn_up": ("gemm", 4096, 14336, 4096, "fp16", "normal64"),
    "gemm_8192": ("gemm", 8192, 8192, 8192, "bf16", "uniform16"),
    "swiglu_prefill": ("silu_mul", 1024, 11008, 0, "bf16", "normal"),
    "add_rms_norm_prefill": ("add_rms_norm", 2048, 4096, 0, "bf16", "normal"),
    "ffn_swiglu": ("gemm_swiglu", 4096, 14336, 4096, "fp16", "normal64"),
    "paged_b16_c2048": ("paged", 16, 2048, 0, "bf16", "normal"),
    "paged_b16_c2048_cuda_cores": ("paged", 16, 2048, 1, "bf16", "normal"),  # k: kernel choice
    "rms_norm_backward_prefill": ("rms_norm_backward", 2048, 4096, 0, "bf16", "normal"),
    "sdpa_b4_s4096": ("sdpa", 4, 4096, 128, "bf16", "normal"),  # GQA 32 x 8, causal
}


def run_profile(args) -> int:
    """A few launches of one kernel and nothing else of ours: the workload ncu captures."""

    import torch

    from radeon_kernels import _native

    kind, m, n, k, dtype, dist_name = PROFILE_CASES[args.profile]
    ext = _native.extension()
    torch.cuda.set_device(0)
    if kind == "gemv":
        w = seeded((n, k), 1, dist_name, dtype)
        x = seeded((m, k), 2, "normal", dtype)
        out = torch.empty(m, n, dtype=x.dtype, device="cuda")
        launch = lambda: ext.gemv_out(x, w, out, 0)  # noqa: E731
    elif kind == "silu_mul":  # m = tokens, n = hidden
        gate = seeded((m, n), 1, dist_name, dtype)
        up = seeded((m, n), 2, dist_name, dtype)
        launch = lambda: ext.silu_mul(gate, up)  # noqa: E731
    elif kind == "paged":  # m = batch, n = context; GQA 32 x 8, head_dim 128, block 16; k = path
        _native.library().rk_paged_attention_set_path(k)
        maxb = -(-n // 16)
        q = seeded((m, 32, 128), 1, dist_name, dtype)
        kc = seeded((m * maxb, 16, 8, 128), 2, dist_name, dtype)
        vc = seeded((m * maxb, 16, 8, 128), 3, dist_name, dtype)
        tables = torch.arange(m * maxb, device="cuda", dtype=torch.int32).view(m, maxb)
        lens = torch.full((m,), n, dtype=torch.int32, device="cuda")
        launch = lambda: ext.paged_attention_decode(q, kc, vc, tables, lens, 128 ** -0.5)  # noqa: E731
    elif kind == "gemm_swiglu":  # b is [K, 2N]
        a = seeded((m, k), 1, dist_name, dtype)
        b = seeded((k, 2 * n), 2, dist_name, dtype)
        launch = lambda: ext.gemm_swiglu(a, b, 0)  # noqa: E731
    elif kind == "rms_norm_backward":  # with the weight gradient
        dy = seeded((m, n), 1, dist_name, dtype)
        x = seeded((m, n), 2, dist_name, dtype)
        w = seeded((n,), 3, dist_name, dtype)
        launch = lambda: ext.rms_norm_backward(dy, x, w, 1e-6, True)  # noqa: E731
    elif kind == "sdpa":  # m = batch, n = sequence, k = head_dim; 32 query heads over 8 KV heads
        q = seeded((m, 32, n, k), 1, dist_name, dtype)
        kk = seeded((m, 8, n, k), 2, dist_name, dtype)
        v = seeded((m, 8, n, k), 3, dist_name, dtype)
        launch = lambda: ext.sdpa(q, kk, v, True, k ** -0.5)  # noqa: E731
    elif kind == "add_rms_norm":
        x = seeded((m, n), 1, dist_name, dtype)
        r = seeded((m, n), 2, dist_name, dtype)
        w = seeded((n,), 3, dist_name, dtype)
        launch = lambda: ext.add_rms_norm(x, r, w, 1e-6)  # noqa: E731
    else:
        a = seeded((m, k), 1, dist_name, dtype)
        b = seeded((k, n), 2, dist_name, dtype)
        out = torch.empty(m, n, dtype=a.dtype, device="cuda")
        launch = lambda: ext.gemm_out(a, b, out, 0)  # noqa: E731
    for _ in range(args.steps):
        launch()
    torch.cuda.synchronize()
    print(json.dumps({"profile": args.profile, "launches": args.steps, "status": int(ext.device_status())}))
    return 0


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description="B200 GEMM/GEMV hot-path benchmark")
    parser.add_argument("--profile", choices=sorted(PROFILE_CASES), default=None,
                        help="run --steps launches of one kernel only (the case ncu captures)")
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=4000)
    parser.add_argument("--warmup", type=int, default=20)
    parser.add_argument("--e2e-steps", type=int, default=2000)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--cpu-seconds", type=float, default=10.0)
    parser.add_argument("--quick", action="store_true", help="skip the optional 8192^3 suite entry")
    parser.add_argument("--no-suite", action="store_true")
    parser.add_argument("--suite-filter", default=None, help="regex: run only the suite entries it matches")
    args = parser.parse_args(argv)

    if args.impl == "reference":
        return run_reference(args)
    if args.profile:
        return run_profile(args)

    import torch

    from radeon_kernels import _native

    dist = Dist(args.gpus)
    dist.init()
    torch.cuda.set_device(dist.local_rank)
    ext = _native.extension()
    peaks, peak_kind = load_peaks()

    launches_before = _native.library().rk_launch_count()
    with ClockSampler(dist.local_rank) as clocks:
        head = headline(args, dist, ext, peaks, peak_kind)
        end_to_end = e2e(args, dist)
        extra = {} if args.no_suite else suite(args, dist, ext, peaks)
    traffic_key = "gemv_decode_bf16_m1_n8192_k8192" if dist.world == 1 else f"gemv_allgather_bf16_m1_n8192_k8192_w{dist.world}"
    head["roofline"]["traffic"] = load_traffic().get(traffic_key)  # bytes per launch (ncu)
    cpu = cpu_baseline(args.cpu_seconds) if dist.rank == 0 and dist.world == 1 else None
    dist.close()
    if dist.rank != 0:
        return 0
    config = headline_config(dist.world)
    config["launch"] = head.pop("launch")
    line = {
        "metric": METRIC,
        "value": round(head["value"], 1),
        "unit": "GB/s",
        "n_gpus": dist.world,
        "steps": head["steps"],
        "warmup": args.warmup,
        "ms_per_step": round(head["ms_per_step"], 6),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": DATA,
        "config": config,
        "roofline": head["roofline"],
        "e2e": end_to_end,
        "gpu_launches": head["steps"],
        "gpu_launches_note": "per rank: one rk_gemv (N = 1) or rk_gemv_allgather (N > 1) launch per timed step",
        "clocks": clocks.summary(),
        "cpu_baseline": cpu,
        "suite": extra,
        "library_launches_host_counted": int(_native.library().rk_launch_count() - launches_before),
    }
    for key in ("compute_only", "exchange_us_per_step", "weight_sets_per_rank"):
        if key in head:
            line[key] = head[key]
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
