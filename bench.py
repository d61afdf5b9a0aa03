"""Benchmark of the B200 decode-sampling step (BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (one rank per GPU)

Headline workload: 1024 independent rows per GPU of
V=49152 fp32 logits ~N(0,2^2) with Zipf(1.1) histories of 4096 int32 ids; the full
sampling chain (repetition penalty, temperature 1.5, top-k 50, top-p 0.9, softmax,
draw from a per-row uniform) in one fused launch per step.  Rows are sharded
across ranks with no collective in the step ("weak" scaling: 1024 rows per GPU).
Two input sets alternate between steps (2 x 218 MB > the 126 MB L2), so every
step streams its inputs from HBM.

Prints one JSON line (rank 0).  `value` is rows/s over all GPUs with inputs
resident in HBM; `e2e` is the same metric through the C ABI from pinned host
buffers (host->device copies of logits, histories and uniforms and the
device->host read of the tokens inside the timed region); `roofline` relates the
kernel's algorithmic bytes to the measured HBM copy bandwidth; `cpu_baseline`
times the reference's own chain in torch (oracle/torch_chain.py) on this host's
cores on a bounded sample, beside the C restatement (oracle/).
`extras` holds the latency configs (1, 2, 3) and the loop guard (config 5).

--impl reference times only the reference's chain in torch on this host's cores,
on the same 1024-row workload and metric (rank 0; other ranks exit).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

V = 49152
ROWS = 1024
HIST = 4096
METRIC = "sampled rows/s at V=49152 (HBM GB/s vs peak); us per 2-beam decode step"
WORKLOAD = "cfg4: 1024 rows/GPU x V=49152 fp32 N(0,2^2), Zipf(1.1) histories of 4096 int32 ids, T=1.5 top_k=50 top_p=0.9"

# ------------------------------------------------------------------ workloads


def history_with_repeats(rng, n, vocab, repeat_frac=0.3):
    """n ids: (1 - repeat_frac) uniform in [0, vocab), the rest copies of earlier ids."""
    ids = rng.integers(0, vocab, n)
    rep = rng.random(n) < repeat_frac
    rep[0] = False
    src = (rng.random(n) * np.arange(n)).astype(np.int64)
    for j in np.nonzero(rep)[0]:
        ids[j] = ids[src[j]]
    return ids.astype(np.int32)


def zipf_ids(rng, shape, vocab, a=1.1):
    """Zipf(a) ids over [0, vocab): numpy zipf resampled until <= vocab, id = x - 1."""
    x = rng.zipf(a, size=shape)
    bad = x > vocab
    while bad.any():
        x[bad] = rng.zipf(a, size=int(bad.sum()))
        bad = x > vocab
    return (x - 1).astype(np.int32)


def to_bf16_values(x):
    """Round float32 values to bfloat16 (nearest even), returned as float32."""
    b = x.astype(np.float32).view(np.uint32)
    b = ((b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return b.view(np.float32)


def cfg1(seed=0, vocab=V):
    """Config 1: B=1, 2*N(0,1) logits, 20 ids boosted +8, 1024-id history (30 % repeats)."""
    rng = np.random.default_rng(seed)
    x = (2.0 * rng.standard_normal((1, vocab))).astype(np.float32)
    x[0, rng.choice(vocab, 20, replace=False)] += 8.0
    hist = history_with_repeats(rng, 1024, vocab)[None]
    u = rng.random(1).astype(np.float32)
    return dict(logits=x, history=hist, uniforms=u, temperature=1.5, top_p=0.9, keep=1)


def cfg2(seed=1, vocab=V, beams=2, hist_len=2048):
    """Config 2: 2 beams, N(0,2^2) logits, 2048-id histories, running scores U(-200,-10)."""
    rng = np.random.default_rng(seed)
    x = (2.0 * rng.standard_normal((beams, vocab))).astype(np.float32)
    hist = rng.integers(0, vocab, (beams, hist_len)).astype(np.int32)
    running = rng.uniform(-200, -10, beams).astype(np.float32)
    u = rng.random(2 * beams).astype(np.float32)
    return dict(logits=x, history=hist, running=running, uniforms=u, temperature=1.5, top_p=0.9)


def cfg3(seed=2, vocab=V, beams=8, hist_len=8000):
    """Config 3: 8 beams, bf16 N(0,3^2) logits with 1 % of ids +6, 8000-id histories."""
    rng = np.random.default_rng(seed)
    x = (3.0 * rng.standard_normal((beams, vocab))).astype(np.float32)
    x[:, rng.choice(vocab, vocab // 100, replace=False)] += 6.0
    hist = rng.integers(0, vocab, (beams, hist_len)).astype(np.int32)
    running = rng.uniform(-200, -10, beams).astype(np.float32)
    u = rng.random(2 * beams).astype(np.float32)
    return dict(logits=to_bf16_values(x), history=hist, running=running, uniforms=u, temperature=1.5, top_p=0.9)


def cfg4(seed=3, rows=ROWS, vocab=V, hist_len=HIST):
    """Config 4: rows x V N(0,2^2) fp32 logits, Zipf(1.1) histories of 4096 ids."""
    rng = np.random.default_rng(seed)
    x = (2.0 * rng.standard_normal((rows, vocab))).astype(np.float32)
    hist = zipf_ids(rng, (rows, hist_len), vocab)
    u = rng.random(rows).astype(np.float32)
    return dict(logits=x, history=hist, uniforms=u, temperature=1.5, top_p=0.9, keep=1)


def cfg5_tokens(seed=4, rows=256, length=16384, vocab=V, window=64, repeats=3):
    """Config 5: loop-guard histories; rows [0, rows/2) end with one window repeated
    `repeats` times (planted, non-overlapping), the other rows are random."""
    rng = np.random.default_rng(seed)
    t = rng.integers(0, vocab, (rows, length)).astype(np.int32)
    for r in range(rows // 2):
        win = rng.integers(0, vocab, window)
        starts = np.sort(rng.choice((length - window) // window - 1, repeats - 1, replace=False)) * window
        for s in starts:
            t[r, s:s + window] = win
        t[r, length - window:] = win
    return t


def row_bytes(vocab=V, hist=HIST, logit_bytes=4, id_bytes=4):
    """Algorithmic bytes per row of one sampling step: logits + history ids + the
    uniform read; token (8) + kept count (4) + status (4) written."""
    return vocab * logit_bytes + hist * id_bytes + 4 + 8 + 4 + 4


# ------------------------------------------------------------------ helpers


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML every `period` seconds."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, index, period=0.002):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self.period, self._stop, self._thread = period, threading.Event(), None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nvml = None

    def _run(self):
        while not self._stop.is_set():
            self.sample()
            time.sleep(self.period)

    def sample(self):
        if self.nvml is None:
            return
        try:
            self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.h, self.nvml.NVML_CLOCK_SM))
            r = self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            for bit, name in self.REASONS.items():
                if r & bit:
                    self.reasons.add(name)
        except Exception:
            pass

    def __enter__(self):
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._thread.join()
        self.sample()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic():
    """DRAM bytes (read + write) of one stream-kernel launch on this workload, from
    the committed ncu summary (profiles/stream_kernel_cfg4.md), or None."""
    try:
        with open(os.path.join(ROOT, "profiles", "stream_kernel_cfg4.md")) as f:
            for line in f:
                if line.startswith("dram_bytes_per_launch:"):
                    return int(line.split(":")[1])
    except (OSError, ValueError):
        pass
    return None


def cpu_port_rows_per_s(data, seconds=10.0, chunk=64, threads=0):
    """The CPU port of the reference algorithm (oracle/) on all host threads (or
    `threads`), on a bounded sample: chunks of `chunk` rows of the workload until
    `seconds` pass."""
    from oracle import oracle as O
    x, h, u = data["logits"], data["history"], data["uniforms"]
    n = x.shape[0]
    t0 = time.perf_counter()
    rows = 0
    i = 0
    while True:
        s = slice(i, i + chunk)
        O.sample(x[s], u[s], ids=h[s], temperature=1.5, top_p=0.9, cap=0, threads=threads)
        rows += x[s].shape[0]
        i = (i + chunk) % n
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return rows / dt, rows, dt


# ------------------------------------------------------------------ reference arm


def run_reference(args, rank):
    """The reference's own CPU chain (oracle/torch_chain.py: its torch calls, in its
    order, runtime_shared.py:170-202) on this host's cores, over the same 1024-row
    workload per step; rank 0 alone runs and prints."""
    if rank != 0:
        return
    import torch
    from oracle import torch_chain as TC
    data = cfg4()
    threads = os.cpu_count()
    torch.set_num_threads(threads)
    x = torch.from_numpy(data["logits"])
    seen0 = TC.seen_mask(data["history"], V)
    g = torch.Generator().manual_seed(0)

    def step():
        seen = seen0.clone()  # each step starts from the workload's histories
        for r in range(0, ROWS, 64):  # 64 rows per call: the chain's best throughput here
            TC.sample_step(x[r:r + 64], seen[r:r + 64], generator=g)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    value = ROWS * args.steps / dt
    sample = (f"all {ROWS} rows of the workload per step, 64 rows per call: penalty, temperature, top-k, top-p, "
              f"softmax and torch.multinomial in torch on {threads} host threads (runtime_shared.py:170-202)")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args.gpus),
            "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "torch-restatement",
                             "cpu": cpu_model(), "sample": sample},
            "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def workload_config(world):
    """The `config` of both arms' lines."""
    return {"workload": WORKLOAD, "rows_per_gpu": ROWS, "vocab": V, "history_ids": HIST,
            "parallelism": f"row-sharded x{world}, no collective in the step",
            "l2": "two alternating input sets of 218 MB each (> 126 MB L2)"}


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def cpu_baseline(host, seconds):
    """The reference's chain in torch on all host threads and on one, plus the C
    port of the reference algorithm (oracle/), each on a bounded sample."""
    from oracle import torch_chain as TC
    seen = TC.seen_mask(host["history"], V)
    threads = os.cpu_count()
    rps, rows, dt = TC.rows_per_s(host["logits"], seen, seconds=seconds, chunk=64, threads=threads)
    rps1, rows1, dt1 = TC.rows_per_s(host["logits"], seen, seconds=min(seconds, 5.0), chunk=8, threads=1)
    prt, prows, pdt = cpu_port_rows_per_s(host, seconds=min(seconds, 5.0))
    return {"value": rps, "unit": "rows/s", "cores": threads, "kind": "torch-restatement", "cpu": cpu_model(),
            "sample": f"{rows} rows of the workload in {dt:.1f} s, 64 rows per call: the reference's torch chain "
                      f"(runtime_shared.py:170-202, oracle/torch_chain.py)",
            "single_thread": {"value": rps1, "unit": "rows/s", "cores": 1,
                              "sample": f"{rows1} rows in {dt1:.1f} s, 8 rows per call"},
            "c_port": {"value": prt, "unit": "rows/s", "cores": threads, "kind": "port",
                       "sample": f"{prows} rows in {pdt:.1f} s (oracle/ C restatement, OpenMP over rows)"}}


# ------------------------------------------------------------------ our arm


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import __graft_entry__
    sv = __graft_entry__.load_package()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)

    sets = []
    for s in range(2):
        d = cfg4(seed=3 + 1000 * rank + s)
        sets.append(dict(logits=torch.from_numpy(d["logits"]).to(dev), history=torch.from_numpy(d["history"]).to(dev),
                         uniforms=torch.from_numpy(d["uniforms"]).to(dev), host=d))
    outs = [dict(token=torch.empty(ROWS, dtype=torch.int64, device=dev),
                 count=torch.empty(ROWS, dtype=torch.int32, device=dev),
                 status=torch.empty(ROWS, dtype=torch.int32, device=dev)) for _ in range(2)]

    def launch(i):
        d = sets[i & 1]
        sv.sample_step(d["logits"], d["uniforms"], history=d["history"], temperature=1.5, top_p=0.9, top_k=50,
                       keep=1, repetition_penalty=3.1, out=outs[i & 1])

    # The timed steps are one CUDA graph holding the K launches back to back (input
    # sets alternating), as a decode loop runs the step inside its own graph: the
    # device time per step is the kernel plus the launch gap between kernels, not a
    # per-step graph launch or the Python/ctypes call.
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        for i in range(2):
            launch(i)
    stream.wait_stream(side)
    torch.cuda.synchronize()
    timed = torch.cuda.CUDAGraph()
    with torch.cuda.graph(timed):
        for i in range(args.steps):
            launch(i)
    warm = torch.cuda.CUDAGraph()
    with torch.cuda.graph(warm):
        for i in range(max(args.warmup, 3)):
            launch(i)

    def barrier():
        if world > 1:
            dist.barrier()

    warm.replay()
    torch.cuda.synchronize()
    st = outs[0]["status"].max().item()
    if st:
        raise RuntimeError(f"sampling status {st}")
    sampler = ClockSampler(local_rank)
    barrier()
    torch.cuda.synchronize()
    with sampler:
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        timed.replay()
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    total_ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    rows_total = ROWS * world * args.steps
    value = rows_total / (total_ms / 1e3)

    # Roofline of the fused kernel: algorithmic bytes per launch / mean launch time
    # (the timed graph holds only this kernel's launches).
    per_launch = ROWS * row_bytes()
    mean_kern_s = total_ms / args.steps / 1e3
    achieved = per_launch / mean_kern_s / 1e9
    peak, peak_kind = measured_peaks()

    # End to end through the C ABI from pinned host buffers (rank-local).
    host_x = torch.from_numpy(sets[0]["host"]["logits"]).pin_memory()
    host_h = torch.from_numpy(sets[0]["host"]["history"]).pin_memory()
    host_u = torch.from_numpy(sets[0]["host"]["uniforms"]).pin_memory()
    host_tok = torch.empty(ROWS, dtype=torch.int64).pin_memory()
    dx = torch.empty_like(sets[0]["logits"])
    dh = torch.empty_like(sets[0]["history"])
    du = torch.empty_like(sets[0]["uniforms"])
    e2e_steps = max(3, min(args.steps, 20))

    def e2e_step():
        dx.copy_(host_x, non_blocking=True)
        dh.copy_(host_h, non_blocking=True)
        du.copy_(host_u, non_blocking=True)
        o = sv.sample_step(dx, du, history=dh, temperature=1.5, top_p=0.9, out=outs[0])
        host_tok.copy_(o["token"], non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = ROWS * world * e2e_steps / (e2e_ms / 1e3)
    h2d = host_x.numel() * 4 + host_h.numel() * 4 + host_u.numel() * 4
    d2h = ROWS * 8

    extras = latency_extras(sv, dev) if rank == 0 and not args.no_extras else {}
    if rank == 0 and not args.no_extras:
        extras.update(kv_extras(sv, dev))
        extras.update(guard_extras(sv, dev))
        extras.update(advance_extras(sv, dev))
        extras.update(dropin_extras(sv, dev))
    if world > 1 and not args.no_extras:
        extras.update(vocab_sharded_extra(sv, dev, rank, world))  # every rank takes part
        extras.update(vocab_sharded_beam_extra(sv, dev, rank, world))
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(sets[0]["host"], args.cpu_seconds)
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": workload_config(world),
                "timing": "the K timed steps are one CUDA graph of K launches (input sets alternating); "
                          "device time over the graph / K",
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "traffic": profiled_traffic(),
                             "traffic_source": "static, not measured in this run: ncu dram__bytes_read.sum + "
                                               "dram__bytes_write.sum of one launch of this kernel on this workload, "
                                               "read from profiles/stream_kernel_cfg4.md",
                             "peak_source": peak_kind, "algorithmic_bytes_per_launch": per_launch,
                             "mean_launch_us": mean_kern_s * 1e6},
                "cpu_baseline": cpu,
                "e2e": {"value": e2e_value, "unit": "rows/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
                "gpu_launches": args.steps,
                "clocks": sampler.summary(),
                "extras": extras}
        print(json.dumps(line), flush=True)


def graph_time_us(fn, reps=40, per_graph=10):
    """Mean device time of one fn() call, replayed from a CUDA graph that holds
    per_graph calls back to back (after warm-up): a decode loop captures its
    sampling step inside the step's graph, so the host's graph-launch gap is not
    part of the step."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(per_graph):
            fn()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1e3 / (reps * per_graph)


def latency_extras(sv, dev):
    import torch
    out = {}
    d = cfg1()
    x, h, u = (torch.from_numpy(d[k]).to(dev) for k in ("logits", "history", "uniforms"))
    o1 = {}
    sv.sample_step(x, u, history=h, out=o1, dense="probs")
    out["cfg1_us_per_step"] = graph_time_us(lambda: sv.sample_step(x, u, history=h, out=o1, dense="probs"))
    # The same step called eagerly through the Python wrapper and the torch extension:
    # host time per call (submission only) and wall time per call (max of host and GPU).
    import time
    n = 500
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(n):
        sv.sample_step(x, u, history=h, out=o1, dense="probs")
    t1 = time.perf_counter()
    torch.cuda.synchronize()
    t2 = time.perf_counter()
    out["cfg1_eager_host_us_per_call"] = (t1 - t0) / n * 1e6
    out["cfg1_eager_wall_us_per_call"] = (t2 - t0) / n * 1e6
    for name, gen, dt in (("cfg2_beam2_us_per_step", cfg2, torch.float32),
                          ("cfg3_beam8_bf16_us_per_step", cfg3, torch.bfloat16)):
        d = gen()
        x = torch.from_numpy(d["logits"]).to(dev).to(dt)
        h = torch.from_numpy(d["history"]).to(dev)
        rs = torch.from_numpy(d["running"]).to(dev)
        u = torch.from_numpy(d["uniforms"]).to(dev)
        ob = {}
        # The workspace is allocated before capture (the graph then holds no fill).
        ws = sv.beam_workspace(x.shape[0], x.shape[1], dev)
        sv.beam_step(x, rs, u, history=h, out=ob, workspace=ws)
        out[name] = graph_time_us(lambda: sv.beam_step(x, rs, u, history=h, out=ob, workspace=ws))
    # Config 5's sampling rows (256 x V, 16384-token histories as a seen bitmap), on
    # one GPU: the unsharded reference point of the vocab-sharded step.
    xs, us_, bits = cfg5_sample_rows(dev)
    o5 = {}
    sv.sample_step(xs, us_, seen_bits=bits, out=o5)
    out["cfg5_sample_unsharded_us_per_step"] = graph_time_us(lambda: sv.sample_step(xs, us_, seen_bits=bits, out=o5))
    # Config 5's loop guard: warm (the same 16.8 MB each call, L2-resident) and cold
    # (ten copies in turn, 168 MB > the 126 MB L2, so each call reads HBM).
    t = torch.from_numpy(cfg5_tokens()).to(dev)
    lens = torch.full((t.shape[0],), t.shape[1], dtype=torch.int32, device=dev)
    v = torch.empty(t.shape[0], dtype=torch.uint8, device=dev)
    sv.loop_guard(t, lens, out=v)
    out["cfg5_loop_guard_us"] = graph_time_us(lambda: sv.loop_guard(t, lens, out=v))
    out["cfg5_loop_guard_GBps"] = t.numel() * 4 / (out["cfg5_loop_guard_us"] * 1e-6) / 1e9
    copies = [t.clone() for _ in range(10)]
    turn = iter(range(1 << 30))
    out["cfg5_loop_guard_cold_us"] = graph_time_us(lambda: sv.loop_guard(copies[next(turn) % 10], lens, out=v),
                                                   reps=20, per_graph=10)
    out["cfg5_loop_guard_cold_GBps"] = t.numel() * 4 / (out["cfg5_loop_guard_cold_us"] * 1e-6) / 1e9
    del copies
    return out


def kv_extras(sv, dev):
    """The beam KV-cache reorder (runtime_shared.py:388-394) on decoder-sized caches:
    GPTBigCode-1B-like MQA [24 layers, 2 beams, 4096 slots, 128] fp16 with the two
    beams swapped, and StarCoder2-7B-like GQA [32, 8 beams, 4 heads, 2048, 128] bf16
    with every beam taking another's cache.  Moved bytes (read + write of the changed
    rows' keys and values) per second."""
    import torch
    out = {}
    for name, shape, dtype, parents in (
            ("kv_reorder_1b_mqa", (24, 2, 4096, 128), torch.float16, [1, 0]),
            ("kv_reorder_8b_gqa", (32, 8, 4, 2048, 128), torch.bfloat16, [1, 0, 3, 2, 5, 4, 7, 6])):
        keys = torch.randn(shape, device=dev).to(dtype)
        values = torch.randn(shape, device=dev).to(dtype)
        p = torch.tensor(parents, dtype=torch.int64, device=dev)
        length = shape[-2]
        us = graph_time_us(lambda: sv.ops.kv_reorder(keys, values, p, length), reps=10, per_graph=4)
        changed = sum(1 for r, q in enumerate(parents) if q != r)
        moved = 2 * 2 * changed * keys[:, 0].numel() * keys.element_size()
        out[name + "_us"] = us
        out[name + "_GBps"] = moved / (us * 1e-6) / 1e9
        del keys, values
    return out


def guard_extras(sv, dev):
    """One loop-guard check of a single growing sequence at 4096 and 16384 tokens
    (runtime_shared.py:207, every 16 steps): the incremental guard (enter 16 new
    windows, probe the occurrence table) against a full rescan of the row by the
    batched kernel.  Random tokens (no repeat: the probe ends at the first empty
    slot) and a row ending in a loop (the probe verifies three matches)."""
    import torch
    out = {}
    g = np.random.default_rng(11)
    for n in (4096, 16384):
        for kind in ("random", "looping"):
            row = g.integers(0, V, n)
            if kind == "looping":
                row[n - 64 * 3:] = np.tile(row[n - 64:], 3)
            t = torch.from_numpy(row).to(dev)
            table = sv.ops.guard_table(n, dev)
            verdict = torch.zeros(1, dtype=torch.uint8, device=dev)
            sv.ops.loop_guard_incremental(table, t, 0, n - 16, out=verdict)  # the windows already entered
            us = graph_time_us(lambda: sv.ops.loop_guard_incremental(table, t, n - 16, n, out=verdict), reps=20,
                               per_graph=10)
            torch.cuda.synchronize()
            assert bool(verdict.item()) == (kind == "looping")
            out[f"loop_guard_incremental_{n}_{kind}_us"] = us
        lens = torch.full((1,), n, dtype=torch.int32, device=dev)
        v = torch.zeros(1, dtype=torch.uint8, device=dev)
        out[f"loop_guard_rescan_{n}_us"] = graph_time_us(lambda: sv.loop_guard(t[None], lens, out=v), reps=20,
                                                         per_graph=10)
    return out


def advance_extras(sv, dev):
    """The beam loop's per-step decision kernel (sv_beam_advance) at V=49152, step
    1000 of a generation: the decision, the seen-bitmap and history reorder and the
    loop-guard insert, for 2 and 8 beams."""
    import torch
    out = {}
    g = torch.Generator(device=dev).manual_seed(5)
    for beams in (2, 8):
        P, step, words = 2 * beams, 1000, (V + 31) // 32
        o = {"picks": torch.randperm(beams * V, generator=g, device=dev)[:P].contiguous(),
             "scores": -torch.rand(P, generator=g, device=dev) * 50, "n": torch.full((1,), P, dtype=torch.int32,
                                                                                     device=dev),
             "status": torch.zeros(1, dtype=torch.int32, device=dev)}
        stop = torch.tensor([5, 6], dtype=torch.int64, device=dev)
        tails = torch.full((2, beams, 2), -1, dtype=torch.int64, device=dev)
        seen = torch.zeros((2, beams, words), dtype=torch.int32, device=dev)
        hist = torch.zeros((2, beams, 4096), dtype=torch.int32, device=dev)
        whash = torch.zeros((2, beams), dtype=torch.int32, device=dev)
        table = sv.ops.guard_table(beams * 4096, dev)
        run = torch.zeros(beams, device=dev)
        par = torch.zeros(beams, dtype=torch.int64, device=dev)
        tok = torch.zeros(beams, dtype=torch.int64, device=dev)

        def call():
            sv.ops.beam_advance(o, beams=beams, vocab=V, step=step, last=False, stop_ids=stop, eos_id=7,
                                tails_in=tails[0], tails_out=tails[1], running_out=run, parents_out=par,
                                tokens_out=tok, seen_in=seen[0], seen_out=seen[1], hist_in=hist[0],
                                hist_out=hist[1], whash_in=whash[0], whash_out=whash[1], guard_table=table,
                                window=64)
        call()
        out[f"beam_advance_{beams}_us"] = graph_time_us(call, reps=20, per_graph=10)
    return out


class _NoOpDecoding:
    """A scripted decoder for timing the drop-in's loops per token: `step` replays a
    CUDA graph that only stores the fed tokens (the decoder's own work left out) and
    returns fixed N(0, 2^2) logits over V; the beam cache is a GPTBigCode-1B-shaped
    MQA cache [24, beams, capacity, 128] fp16 that the loop reorders on the device
    (sv_kv_reorder) through `reorder_device`.  The three lowest-logit ids serve as
    eos / stop ids, so no generation ends before max_new_tokens."""

    def __init__(self, rows, capacity, dev, vocab=V, seed=7):
        import torch
        g = torch.Generator(device=dev).manual_seed(seed)
        self.logits = torch.randn((rows, vocab), generator=g, device=dev) * 2
        low = torch.argsort(self.logits[0])[:3].tolist()
        self.eos_id, self.stop_ids = low[0], low[1:]
        self.tokens = torch.zeros(rows, dtype=torch.int64, device=dev)
        self.fed = torch.zeros(rows, dtype=torch.int64, device=dev)
        self.keys = torch.zeros((24, rows, capacity, 128), dtype=torch.float16, device=dev) if rows > 1 else None
        self.values = torch.zeros_like(self.keys) if rows > 1 else None
        self.length = 0
        self.graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self.fed.copy_(self.tokens)
        torch.cuda.current_stream().wait_stream(s)
        with torch.cuda.graph(self.graph):
            self.fed.copy_(self.tokens)

    def prefill(self, embeddings, rows, capacity):
        self.length = embeddings.shape[1]
        return self, self.logits

    def step(self, tokens):
        self.tokens.copy_(tokens)
        self.graph.replay()
        self.length += 1
        return self.logits

    def reorder_device(self, parents):
        import __graft_entry__
        __graft_entry__.load_package().kv_reorder(self.keys, self.values, parents, self.length)


def dropin_extras(sv, dev, tokens=512, reps=3):
    """Host-inclusive microseconds per token of the drop-in's `_sample` and
    `_beam_sample` (2 and 8 beams) over the no-op decoder: every kernel launch,
    ctypes call, record read and host replay of a max_new_tokens=512 generation at
    V=49152, wall clock / tokens.  Also the same loops read back every step
    (`_SYNC_EVERY` = 1) to show what the 16-step blocks save, and the cost of the
    decode steps a block issues past an end (0..15, 7.5 on average: each a whole
    loop step plus the decoder's own step)."""
    import importlib
    import time
    import torch
    rs = importlib.import_module(sv.__name__ + ".runtime_shared")
    out = {}
    prefix = torch.zeros((1, 300, 4), device=dev)
    for beams in (1, 2, 8):
        for every in (rs._SYNC_EVERY, 1):
            saved = rs._SYNC_EVERY
            rs._SYNC_EVERY = every
            try:
                times = []
                for r in range(reps + 1):
                    dec = _NoOpDecoding(beams, prefix.shape[1] + tokens, dev)
                    torch.cuda.synchronize()
                    t0 = time.perf_counter()
                    with torch.inference_mode():
                        if beams == 1:
                            gen, reason = rs._sample(dec, prefix, tokens, 1.5, 0.9, dec.stop_ids, dec.eos_id, True,
                                                     lambda step: None)
                        else:
                            gen, reason = rs._beam_sample(dec, prefix, tokens, 1.5, 0.9, beams, dec.stop_ids,
                                                          dec.eos_id, True, lambda step: None)
                    torch.cuda.synchronize()
                    if r:  # the first run warms the caches (pinned buffers, workspaces)
                        times.append((time.perf_counter() - t0) / tokens * 1e6)
                    assert reason == "token_limit" and len(gen) == tokens, (reason, len(gen))
            finally:
                rs._SYNC_EVERY = saved
            name = "dropin_sample" if beams == 1 else f"dropin_beam{beams}"
            out[name + ("_us_per_token" if every > 1 else "_sync_every_step_us_per_token")] = min(times)
    for name in ("dropin_sample", "dropin_beam2", "dropin_beam8"):
        out[name + "_overrun_us_mean"] = 7.5 * out[name + "_us_per_token"]
    out["dropin_config"] = (f"max_new_tokens={tokens}, V={V} fp32, loop guard on, no-op decoder step (CUDA graph), "
                            f"1B-shaped KV cache reordered on the device for beams; wall clock incl. all host work, "
                            f"best of {reps}")
    return out


def _graph_time_ranks(fn, dev, steps):
    """Device time per call of fn (a captured step's replay), max over ranks."""
    import torch
    import torch.distributed as dist
    dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) * 1e3 / steps], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0])


def cfg5_sample_rows(dev, cols=None):
    """Config 5's sampling rows: 256 x V fp32 N(0,2^2) logits (columns `cols` of
    them), uniforms, and the rows' 16384-token histories as a packed seen bitmap
    over the whole vocabulary (the same data on every rank)."""
    import torch
    rows = 256
    g = np.random.default_rng(5)
    x = (2.0 * g.standard_normal((rows, V))).astype(np.float32)
    ids = g.integers(0, V, (rows, 16384))
    u = g.random(rows).astype(np.float32)
    if cols is not None:
        x = np.ascontiguousarray(x[:, cols])
    seen = np.zeros((rows, V), bool)
    seen[np.arange(rows)[:, None], ids] = True
    packed = np.packbits(seen, axis=1, bitorder="little")  # V is a multiple of 32
    bits = torch.from_numpy(np.ascontiguousarray(packed).view(np.int32)).to(dev)
    return torch.from_numpy(x).to(dev), torch.from_numpy(u).to(dev), bits


def vocab_sharded_extra(sv, dev, rank, world, steps=20):
    """Config 5's vocab-sharded sample step: 256 rows, V split across the ranks
    (slice step into the exchange block, one NCCL all-gather, merge on every rank),
    captured as one CUDA graph per rank.  Device time per step, max over ranks."""
    import torch
    import torch.distributed as dist
    cap = 64
    off, w, stride = sv.sharded.slice_bounds(V, rank, world)
    xd, ud, bits = cfg5_sample_rows(dev, slice(off, off + w))
    step = sv.sharded.VocabShardedSampler(xd, ud, offset=off, slice_stride=stride, seen_bits=bits,
                                          capacity=cap).capture()
    try:
        step()
        torch.cuda.synchronize()
        bad = torch.tensor([float(step.out["status"].max().item())], device=dev)
        dist.all_reduce(bad, op=dist.ReduceOp.MAX)
        us = _graph_time_ranks(step, dev, steps)
    finally:
        step.release()
    return {"cfg5_vocab_sharded_us_per_step": us, "cfg5_vocab_sharded_slices": world,
            "cfg5_vocab_sharded_max_status": int(bad.item()), "cfg5_vocab_sharded_graph": True}


def vocab_sharded_beam_extra(sv, dev, rank, world, steps=20):
    """Config 3's beam step with every beam's vocabulary split across the ranks
    (slice statistics, two NCCL all-reduces, slice step, one all-gather, merge),
    captured as one CUDA graph per rank.  Device time per step, max over ranks."""
    import torch
    import torch.distributed as dist
    d = cfg3()
    beams, cap = d["logits"].shape[0], 64
    off, w, stride = sv.sharded.slice_bounds(V, rank, world)
    xd = torch.from_numpy(np.ascontiguousarray(d["logits"][:, off:off + w])).to(dev).to(torch.bfloat16)
    seen = np.zeros((beams, V), bool)
    seen[np.arange(beams)[:, None], d["history"]] = True
    packed = np.packbits(seen, axis=1, bitorder="little")
    bits = torch.from_numpy(np.ascontiguousarray(packed).view(np.int32)).to(dev)
    rs = torch.from_numpy(d["running"]).to(dev)
    ud = torch.from_numpy(d["uniforms"]).to(dev)
    step = sv.sharded.VocabShardedBeamStep(xd, rs, ud, offset=off, vocab=V, slice_stride=stride, seen_bits=bits,
                                           capacity=cap).capture()
    try:
        step()
        torch.cuda.synchronize()
        bad = torch.tensor([float(step.out["status"].max().item())], device=dev)
        dist.all_reduce(bad, op=dist.ReduceOp.MAX)
        us = _graph_time_ranks(step, dev, steps)
    finally:
        step.release()
    return {"cfg3_vocab_sharded_beam_us_per_step": us, "cfg3_vocab_sharded_beam_max_status": int(bad.item()),
            "cfg3_vocab_sharded_beam_graph": True}


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-extras", action="store_true", help="skip the latency configs")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
