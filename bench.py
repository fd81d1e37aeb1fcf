"""KDA core benchmark (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kda|reference]

Workload: chunkwise KDA prefill, B=1, T=4096, H=16,
K=V=128, reference chunk_size 64, fp16 q/k/v, fp32 g/beta, zero S0, fp32
state out.  A step is one ``kda_chunkwise`` call over that batch.  Under
torchrun each rank runs its own batch (weak scaling; the (b, h) recurrences
are independent, so there is no collective on the data path).

Reported, all on the device with CUDA events on the launching stream:

* ``value``     prefill tokens/s of the whole job (sum over ranks; time is the
                max over ranks); 4 rotating input sets (> 3x L2), no flush;
* ``roofline``  the chunkwise kernel against measured HBM bandwidth (the
                workload is HBM-bound: ~116 FLOP/B < ~255 FLOP/B ridge);
* ``e2e``       the same metric through the public API from pinned host
                buffers: H2D of q/k/v/g/beta and D2H of o and S inside the
                timed region, the copies of consecutive steps overlapped with
                compute on three streams (``serial``: all in order on one);
* ``decode``    BASELINE configs[2]: B=64 recurrent single-token steps on
                fp32 [64,16,128,128] states, captured in a CUDA graph (four
                steps on four distinct states: working set 4x L2) and
                replayed, against HBM bandwidth;
* ``mla_decode`` the MLA layer's static-buffer decode step of BASELINE
                configs[4] (B=4, buffer 8192 + 256 latents), CUDA graph,
                against HBM bandwidth (the rest of configs[4], the model
                around it, cannot run on the GPU box: the reference's model code
                does not travel with this repository);
* ``fused_io``  the fused prologue / epilogue kernels of a KDA layer at the
                configs[1] shape, against HBM bandwidth;
* ``long_context`` BASELINE configs[3]: B=8, T=32768 bf16 prefill with a
                fp32 S0, (b, h) sharded over the ranks (strong scaling), with
                and without the final gather of o and S to rank 0;
* ``clocks``    nvidia-smi samples taken inside the timed regions;
* ``cpu_baseline`` the CPU oracle (oracle/kda_oracle.py, a numpy port of the
                reference) on a bounded sample, rank 0 at N=1.

``--impl reference`` times that CPU port alone, with all host cores, on the
same workload and metric (the reference is pure PyTorch with no GPU kernels of
its own; rank 0 only under torchrun).
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "KDA prefill & decode tokens/s per GPU (H16,d128); % of TC/HBM roofline"
CFG1 = dict(B=1, T=4096, H=16, K=128, V=128, C=64)
CFG2 = dict(B=64, H=16, K=128, V=128)
FLOP_PER_TOKEN_HEAD = 180224          # 2*[C(3K+2V) + 3KV] at C=64, K=V=128


def _peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def _traffic(kernel, workload):
    """dram read+write bytes per launch from the committed ncu summary, or None."""
    path = os.path.join(REPO, "profiles", "ncu_traffic.txt")
    try:
        for line in open(path):
            parts = line.split()
            if len(parts) >= 3 and parts[0] == kernel and parts[1] == workload:
                return float(parts[2])
    except OSError:
        pass
    return None


# --------------------------------------------------------------------------- #
# clocks sampled during the timed region
# --------------------------------------------------------------------------- #
class ClockSampler:
    """``nvidia-smi -lms`` in the background for the whole GPU part of the run.

    Samples are kept with their host arrival time; :meth:`mark` brackets each
    timed region and :meth:`summary` reports only samples inside one.  The
    sampler waits for nvidia-smi's first line before returning from
    ``__enter__`` so the short timed regions are covered from their start.
    """

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_MS = 20

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.rows = []
        self.windows = []
        self._t0 = None

    def _reader(self):
        for line in self.proc.stdout:
            self.rows.append((time.perf_counter(), line))

    def __enter__(self):
        import threading
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", str(self.PERIOD_MS)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        threading.Thread(target=self._reader, daemon=True).start()
        t_end = time.perf_counter() + 10.0
        while not self.rows and time.perf_counter() < t_end and self.proc.poll() is None:
            time.sleep(0.01)
        return self

    def start(self):
        self._t0 = time.perf_counter()

    def stop(self):
        if self._t0 is not None:
            # a sample reports the period that ends at its arrival
            self.windows.append((self._t0, time.perf_counter() + self.PERIOD_MS * 1e-3))
            self._t0 = None

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()

    def summary(self):
        rows = []
        for t, line in self.rows:
            if any(a <= t <= b for a, b in self.windows):
                r = [c.strip() for c in line.split(",")]
                if len(r) >= 9:
                    rows.append(r)
        if not rows:
            return None
        num = lambda x: x.replace(".", "", 1).isdigit()  # noqa: E731
        sm = [float(r[1]) for r in rows if num(r[1])]
        mx = [float(r[2]) for r in rows if num(r[2])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


# --------------------------------------------------------------------------- #
# CPU port (oracle) timing -- used by the cpu_baseline leg and --impl reference
# --------------------------------------------------------------------------- #
def _oracle_worker(args):
    """One head of the config-1 workload on one core (spawned process)."""
    T, K, V, C, seed, head = args
    import numpy as np
    from oracle import kda_oracle as O
    rng = np.random.default_rng(seed * 1000 + head)

    def unit(shape):
        x = rng.standard_normal(shape).astype(np.float32)
        return x / np.sqrt((x * x).sum(-1, keepdims=True))
    # fp16-valued q/k/v carried in fp32: the port then runs the reference's
    # fp32-transient arithmetic (kda.py:116), 13x faster in numpy than
    # emulating fp16 transients and 2x faster than the reference's own torch
    # fp16 run on the same CPU -- a conservative (fast) baseline
    q = unit((1, T, 1, K)).astype(np.float16).astype(np.float32)
    k = unit((1, T, 1, K)).astype(np.float16).astype(np.float32)
    v = rng.standard_normal((1, T, 1, V)).astype(np.float16).astype(np.float32)
    a_log = np.log(rng.uniform(1, 16, (1, K))).astype(np.float32)
    x = rng.standard_normal((1, T, 1, K)).astype(np.float32)
    dt = rng.uniform(1e-3, 0.1, (1, K)).astype(np.float32)
    dt_bias = np.log(np.expm1(dt))
    g = (-np.exp(a_log) * np.logaddexp(0, x + dt_bias)).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((1, T, 1))))).astype(np.float32)
    t0 = time.perf_counter()
    O.kda_chunkwise(q, k, v, g, beta, chunk_size=C, state_dtype="f32")
    return time.perf_counter() - t0


def cpu_port_throughput(t_sample, heads, steps=1, warmup=0):
    """Config-1-equivalent tokens/s of the numpy port on ``heads`` host cores.

    A step runs ``heads`` independent heads of length ``t_sample`` in a spawn
    pool (one head per process); a config-1 token is 16 heads, so a step
    covers ``t_sample * heads / 16`` tokens.
    """
    import multiprocessing as mp
    env_keys = ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")
    old = {k: os.environ.get(k) for k in env_keys}
    for k in env_keys:
        os.environ[k] = "1"
    try:
        ctx = mp.get_context("spawn")
        with ctx.Pool(heads) as pool:
            times = []
            for s in range(warmup + steps):
                job = [(t_sample, CFG1["K"], CFG1["V"], CFG1["C"], s, h) for h in range(heads)]
                per_head = pool.map(_oracle_worker, job)
                if s >= warmup:
                    times.append(max(per_head))
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    wall = sum(times) / len(times)
    tokens = t_sample * heads / CFG1["H"]
    return tokens / wall, wall


def cpu_decode_throughput(steps=16):
    """configs[2] on the host: ``oracle.kda_recurrent`` single-token steps on
    the full fp32 state [64, 16, 128, 128] (numpy, one process), ``steps`` of
    them timed and the per-step time extrapolated to the 1024-step workload.
    Returns (tokens/s, s per step)."""
    import numpy as np
    from oracle import kda_oracle as O
    rng = np.random.default_rng(2)
    B, H, K, V = CFG2["B"], CFG2["H"], CFG2["K"], CFG2["V"]
    S = (rng.standard_normal((B, H, K, V)) * 0.02).astype(np.float32)

    def unit(shape):
        x = rng.standard_normal(shape).astype(np.float32)
        return (x / np.sqrt((x * x).sum(-1, keepdims=True))).astype(np.float16)
    toks = []
    for _ in range(steps):
        a_log = np.log(rng.uniform(1, 16, (H, K))).astype(np.float32)
        dt = np.log(np.expm1(rng.uniform(1e-3, 0.1, (H, K)))).astype(np.float32)
        g = (-np.exp(a_log) * np.logaddexp(0, rng.standard_normal((B, 1, H, K)) + dt))
        toks.append((unit((B, 1, H, K)), unit((B, 1, H, K)),
                     rng.standard_normal((B, 1, H, V)).astype(np.float16), g.astype(np.float32),
                     (1 / (1 + np.exp(-rng.standard_normal((B, 1, H))))).astype(np.float32)))
    t0 = time.perf_counter()
    for q, k, v, g, beta in toks:
        _, S = O.kda_recurrent(q, k, v, g, beta, state=S, state_dtype="f32")
    per = (time.perf_counter() - t0) / steps
    return B / per, per


def cpu_long_context_throughput(t_sample, heads):
    """configs[3] on the host: ``oracle.kda_chunkwise`` on bf16-valued fp32
    inputs (the fp32-transient arithmetic the reference intends for bf16,
    ``kda.py:116``), S0 ~ N(0, 0.02), ``heads`` independent heads of
    ``t_sample`` tokens in a spawn pool (one head per process).  A configs[3]
    token is 16 heads, so the sample is ``t_sample * heads / 16`` tokens.
    Returns (tokens/s, wall s)."""
    import numpy as np
    import torch
    from oracle import kda_oracle as O
    from oracle import pool as OP
    kb = importlib.import_module("-kimi-linear-_b200")
    x = kb.synth.make_inputs(1, t_sample, heads, 128, 128, dtype=torch.bfloat16, seed=5,
                             s0_std=0.02)
    f = lambda t: t.float().numpy()  # noqa: E731
    t0 = time.perf_counter()
    OP.chunkwise_by_head(f(x["q"]), f(x["k"]), f(x["v"]), x["g"].numpy(), x["beta"].numpy(),
                         initial_state=x["S0"].numpy(), chunk_size=64, state_dtype="f32",
                         v_dtype="bf16", procs=heads)
    wall = time.perf_counter() - t0
    del O, np
    return t_sample * heads / 16 / wall, wall


# --------------------------------------------------------------------------- #
# GPU legs
# --------------------------------------------------------------------------- #
def _events_time(torch, fn, steps, warmup, clk=None, dist=None):
    """Mean device ms of ``fn`` over ``steps`` runs (CUDA events on the
    current stream), bracketed by synchronize + barrier on both sides.
    Callers make sure the inputs of consecutive runs are not L2-resident
    (rotating input sets or inputs larger than L2)."""
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
        torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    if clk is not None:
        clk.start()
    for i in range(steps):
        starts[i].record()
        fn(i)
        ends[i].record()
    torch.cuda.synchronize()
    if clk is not None:
        clk.stop()
    if dist is not None:
        dist.barrier()
    return sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / steps


PREFILL_SETS = 4   # rotating input sets: 4 x 100 MB of inputs, plus outputs, > 3x L2


def _graph_time(torch, dev, fn, n, steps, warmup, clk=None):
    """Mean device ms per call of ``fn(0) .. fn(n-1)`` captured in one CUDA
    graph (after a warm-up on a side stream, as the decode legs do) and
    replayed; events bracket every replay."""
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for i in range(n):
            fn(i)
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(n):
            fn(i)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    reps = max(1, steps // n)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    if clk is not None:
        clk.start()
    for i in range(reps):
        starts[i].record()
        graph.replay()
        ends[i].record()
    torch.cuda.synchronize()
    if clk is not None:
        clk.stop()
    del graph
    return sum(a.elapsed_time(b) for a, b in zip(starts, ends)) / (reps * n)


def _e2e_pipelined(torch, run, host, outs_h, steps, warmup, clk=None, dist=None, slots=2):
    """End-to-end steps with the PCIe copies of consecutive steps overlapped:
    the H2D of step i + 1 (copy stream, into one of ``slots`` device input
    sets) runs while step i computes (current stream) and step i - 1's
    results are read back (D2H stream).  Every step's inputs and results cross
    PCIe inside the timed region, which runs from an event before the first
    H2D to an event after the last read-back.  Returns mean ms per step."""
    comp = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    bufs = [{n: torch.empty_like(t, device=comp.device) for n, t in host.items()}
            for _ in range(slots)]
    free = [None] * slots              # compute of the slot's previous step done

    def one(i):
        k = i % slots
        with torch.cuda.stream(up):
            if free[k] is not None:
                up.wait_event(free[k])
            for n, t in host.items():
                bufs[k][n].copy_(t, non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(up)
        comp.wait_event(ready)
        outs = run(bufs[k])
        done = torch.cuda.Event()
        done.record(comp)
        free[k] = done
        with torch.cuda.stream(down):
            down.wait_event(done)
            for dst, src in zip(outs_h, outs):
                dst.copy_(src, non_blocking=True)
                src.record_stream(down)

    for i in range(warmup):
        one(i)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
        torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if clk is not None:
        clk.start()
    start.record(comp)
    up.wait_event(start)
    for i in range(steps):
        one(i)
    comp.wait_stream(down)
    end.record(comp)
    torch.cuda.synchronize()
    if clk is not None:
        clk.stop()
    if dist is not None:
        dist.barrier()
    return start.elapsed_time(end) / steps


def bench_prefill(torch, kb, dev, steps, warmup, dist, world, clk):
    """Config 1.  Step i runs on input set i % PREFILL_SETS, so its inputs come
    from HBM and the previous steps' outputs and workspace are written back
    while it runs (the steady state of consecutive layers); no L2 flush."""
    sets = [kb.synth.make_config(1, seed=s, device=dev) for s in range(PREFILL_SETS)]
    f32 = torch.float32

    def step(i):
        x = sets[i % PREFILL_SETS]
        return kb.kda_chunkwise(x["q"], x["k"], x["v"], x["g"], x["beta"],
                                chunk_size=CFG1["C"], state_dtype=f32)

    ms_step = _events_time(torch, step, steps, warmup, clk, dist)
    total = torch.tensor([ms_step], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(total, op=dist.ReduceOp.MAX)
    ms_step = total.item()

    # end to end through the public API from pinned host memory
    x0 = sets[0]
    host = {n: x0[n].cpu().pin_memory() for n in ("q", "k", "v", "g", "beta")}
    o_h = torch.empty((CFG1["B"], CFG1["T"], CFG1["H"], CFG1["V"]), dtype=x0["v"].dtype).pin_memory()
    S_h = torch.empty((CFG1["B"], CFG1["H"], CFG1["K"], CFG1["V"]), dtype=f32).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = o_h.numel() * o_h.element_size() + S_h.numel() * S_h.element_size()

    def e2e_step(i):
        d = {n: t.to(dev, non_blocking=True) for n, t in host.items()}
        o, S = kb.kda_chunkwise(d["q"], d["k"], d["v"], d["g"], d["beta"],
                                chunk_size=CFG1["C"], state_dtype=f32)
        o_h.copy_(o, non_blocking=True)
        S_h.copy_(S, non_blocking=True)

    e2e_steps = max(5, steps // 10)
    serial_ms = _events_time(torch, e2e_step, e2e_steps, 3, clk, dist)

    def run(d):
        return kb.kda_chunkwise(d["q"], d["k"], d["v"], d["g"], d["beta"],
                                chunk_size=CFG1["C"], state_dtype=f32)

    # three runs of e2e_steps, the median reported: a PCIe or host hiccup on a
    # shared machine can slow one run by an order of magnitude
    runs = [_e2e_pipelined(torch, run, host, (o_h, S_h), e2e_steps, 3, clk, dist)
            for _ in range(3)]
    e2e_t = torch.tensor([sorted(runs)[1], serial_ms] + runs, dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    path = kb.chunkwise_path(x0["q"], x0["k"], x0["v"], x0["g"], x0["beta"],
                             chunk_size=CFG1["C"], state_dtype=f32)
    del sets
    return ms_step, tuple(e2e_t.tolist()), h2d, d2h, path


def bench_decode(torch, kb, dev, steps, warmup, clk):
    """Config 2: single-token recurrent steps on fp32 [64,16,128,128] states,
    captured in a CUDA graph the way ``GraphedDecoder`` captures its step
    (``graph_decode.py:269-289``: warm-up on a side stream, then
    ``torch.cuda.graph``).  The graph holds NBUF steps on NBUF distinct states
    (inputs 4 x 64 MiB + outputs 4 x 64 MiB = 512 MiB, four times L2), so every
    step reads its state from HBM and the previous steps' outputs are written
    back while it runs -- the steady state of a decoder walking its layers,
    with no L2 flush inside the timing.  Returns ms per step."""
    NBUF = 4
    B, H, K, V = CFG2["B"], CFG2["H"], CFG2["K"], CFG2["V"]
    x = kb.synth.make_inputs(B, 1, H, K, V, dtype=torch.float16, seed=2, s0_std=0.02,
                             device=dev)
    args = [x[n] for n in ("q", "k", "v", "g", "beta")]
    states = [x["S0"].clone() for _ in range(NBUF)]

    def steps_all():
        return [kb.kda_recurrent(*args, state=st, state_dtype=torch.float32) for st in states]

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(3):
            steps_all()
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = steps_all()
    o_e, S_e = kb.kda_recurrent(*args, state=states[0], state_dtype=torch.float32)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(outs[0][0], o_e) and torch.equal(outs[0][1], S_e), \
        "graph replay differs from eager"
    reps = max(1, steps // NBUF)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    clk.start()
    for i in range(reps):
        starts[i].record()
        graph.replay()
        ends[i].record()
    torch.cuda.synchronize()
    clk.stop()
    ms = sum(a.elapsed_time(b) for a, b in zip(starts, ends)) / (reps * NBUF)
    del graph
    return ms, reps * NBUF


# MLA layer of configs[4] (1.5B hybrid, kimi_linear_1p5b_dense.json full_attn):
# prefill B=4 x T=8192, then decode into a buffer of 8192 + 256 latents
CFG4_MLA = dict(B=4, L=8192 + 256, H=16, KVL=512, DN=128, DV=128, prompt=8192)


def bench_mla_decode(torch, kb, dev, steps, warmup, clk):
    """configs[4]'s MLA decode step (static latent buffer, what GraphedDecoder
    runs per MLA layer): the core of ``MLA._decode_step_static`` through
    ``mla.mla_decode_core``, captured in a CUDA graph of NBUF steps on NBUF
    distinct buffers (4 x 34.6 MB > L2), replayed.  The buffers start with the
    8192-token prompt; every replay advances each buffer's pos by one.
    Returns (ms per step, steps timed, algorithmic bytes per step)."""
    NBUF = 4
    c = CFG4_MLA
    B, L, H, KVL, DN, DV, P = c["B"], c["L"], c["H"], c["KVL"], c["DN"], c["DV"], c["prompt"]
    reps = max(1, min(steps // NBUF, (L - P) // NBUF - warmup - 2))
    g = torch.Generator(device=dev).manual_seed(11)
    f16 = dict(device=dev, dtype=torch.float16)
    w = torch.randn(H * (DN + DV), KVL, generator=g, device=dev).mul_(KVL ** -0.5).half()
    q = torch.randn(B, 1, H, DN, generator=g, device=dev).mul_(0.5).half()
    ck = torch.randn(B, 1, KVL, generator=g, device=dev).half()
    bufs, poss = [], []
    for _ in range(NBUF):
        b = torch.zeros(B, L, KVL, **f16)
        b[:, :P].copy_(torch.randn(B, P, KVL, generator=g, device=dev))
        bufs.append(b)
        poss.append(torch.tensor([P], dtype=torch.int64, device=dev))
    scale = DN ** -0.5

    def steps_all():
        return [kb.mla.mla_decode_core(q, ck, bufs[i], poss[i], w, H, DN, DV, scale)
                for i in range(NBUF)]

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        steps_all()
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        steps_all()
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    pos_mid = int(poss[0].item())
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    clk.start()
    for i in range(reps):
        starts[i].record()
        graph.replay()
        ends[i].record()
    torch.cuda.synchronize()
    clk.stop()
    ms = sum(a.elapsed_time(b) for a, b in zip(starts, ends)) / (reps * NBUF)
    del graph
    # bytes a step must move: the valid latent rows, kv_b_proj.weight, q, c_kv, out
    valid = pos_mid + reps // 2 + 1
    nbytes = B * valid * KVL * 2 + H * (DN + DV) * KVL * 2 + B * H * (DN + DV) * 2 + B * KVL * 2
    return ms, reps * NBUF, nbytes


def bench_fused_io(torch, kb, dev, steps, warmup, clk):
    """The fused prologue (short conv + SiLU + L2 norm of q/k, gates, beta)
    and epilogue (head RMSNorm x weight x sigmoid gate) of one KDA layer at the
    configs[1] shape (B=1, T=4096, H=16, K=V=128, fp16, conv size 4 with bias),
    through ``kda_prologue`` / ``kda_epilogue``.  Four rotating input sets
    (256 MB and 128 MB, both > L2), one call on each captured in a CUDA graph
    and replayed (a call's host work is longer than its kernel, so eager
    timing would measure the host).  Returns (prologue ms, epilogue ms,
    prologue bytes, epilogue bytes): algorithmic bytes = one read of every
    input and one write of every output."""
    B, T, H, K = 1, CFG1["T"], CFG1["H"], CFG1["K"]
    D, cs = H * K, 4
    g = torch.Generator(device=dev).manual_seed(5)
    f16 = torch.float16

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g, device=dev) * scale).to(f16)

    pro = [dict(q=rnd(B, T, D), k=rnd(B, T, D), v=rnd(B, T, D), gk=rnd(B, T, D),
                beta=rnd(B, T, H)) for _ in range(4)]
    # conv weights as the module path passes them: its fp32 copies, cast once
    # per parameter version (fused.projections), so no cast runs per call
    ws = [(torch.randn(D, 1, cs, generator=g, device=dev) * 0.4).to(f16).float()
          for _ in range(3)]
    bs = [(torch.randn(D, generator=g, device=dev) * 0.1).to(f16).float() for _ in range(3)]
    A_log = torch.log(torch.rand(H, K, generator=g, device=dev) * 15 + 1)
    dt_bias = torch.log(torch.expm1(torch.rand(H, K, generator=g, device=dev) * 0.099 + 1e-3))

    def prologue(i):
        x = pro[i % 4]
        return kb.kda_prologue(x["q"], x["k"], x["v"], x["gk"], x["beta"], ws, bs, A_log,
                               dt_bias, H, K, K, 1e-6)

    pro_ms = _graph_time(torch, dev, prologue, 4, steps, warmup, clk)
    del pro
    epi = [dict(o=rnd(B, T, H, K), og=rnd(B, T, D)) for _ in range(4)]
    w = torch.rand(H, K, generator=g, device=dev) + 0.5

    def epilogue(i):
        x = epi[i % 4]
        return kb.kda_epilogue(x["o"], x["og"], w, 1e-6)

    epi_ms = _graph_time(torch, dev, epilogue, 4, steps, warmup, clk)
    del epi
    n = B * T * D
    pro_bytes = 4 * n * 2 + B * T * H * 2 + 3 * n * 2 + n * 4 + B * T * H * 4
    epi_bytes = 3 * n * 2
    return pro_ms, epi_ms, pro_bytes, epi_bytes


def bench_long_context(torch, kb, dev, steps, warmup, dist, world, rank, clk):
    """Config 3: B=8, T=32768, H=16 bf16 prefill with a fp32 S0, (b, h)
    sharded over the ranks (strong scaling), then o and S gathered to rank 0.

    Every rank draws the same full inputs from one seed on its own GPU and
    keeps its slice (input generation is outside the timed region).  Timed on
    the device: the kernel alone (max over ranks), and kernel + gather."""
    c = kb.synth.CONFIGS[3]
    B, T, H, K, V = c["B"], c["T"], c["H"], c["K"], c["V"]
    shard = kb.sharding.plan(B, H, world, rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3)
    # generate per batch row to bound the fp32 transients, keep the local slice
    parts = {n: [] for n in ("q", "k", "v", "g", "beta", "S0")}
    for b in range(B):
        xb = kb.synth.make_inputs(1, T, H, K, V, dtype=c["dtype"], s0_std=c["s0_std"],
                                  device=dev, generator=gen)
        for n in parts:
            parts[n].append(xb[n])
        del xb
    full = {n: torch.cat(v) for n, v in parts.items()}
    del parts
    loc = {n: kb.sharding.take(full[n], shard, "state" if n == "S0" else "seq").contiguous()
           for n in full}
    del full
    torch.cuda.empty_cache()

    def step(i=0):
        return kb.kda_chunkwise(loc["q"], loc["k"], loc["v"], loc["g"], loc["beta"],
                                initial_state=loc["S0"], chunk_size=c["C"],
                                state_dtype=torch.float32)

    # inputs of 5.4 GB (one GPU) or 5.4/N GB per rank: far larger than L2
    ms = _events_time(torch, step, steps, warmup, clk, dist)
    ms_t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = ms_t.item()

    # four time segments per rank: segment i's outputs travel to rank 0 while
    # segment i + 1 computes (all peers' transfers in flight at once)
    segs = 4 if world > 1 else 1

    def step_gather(i):
        kb.sharding.run_shard(loc["q"], loc["k"], loc["v"], loc["g"], loc["beta"], loc["S0"],
                              shard=shard, full_bth=(B, T, H), chunk_size=c["C"],
                              state_dtype=torch.float32, gather_to=0, segments=segs)

    g_steps = max(2, steps // 2)
    ms_g = _events_time(torch, step_gather, g_steps, 1, clk, dist)
    ms_g_t = torch.tensor([ms_g], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(ms_g_t, op=dist.ReduceOp.MAX)
    tokens = B * T
    th = tokens * H
    byts = th * (3 * K * 2 + K * 4 + 4 + V * 2) + 2 * B * H * K * V * 4
    return {"workload": "kda_chunkwise prefill, BASELINE configs[3], (b,h) sharded, "
                        "o and S gathered to rank 0",
            "B": B, "T": T, "H": H, "K": K, "V": V, "dtype": "bf16", "s0": "N(0,0.02) fp32",
            "scaling": "strong", "shard": f"{shard.dim} x{shard.size} per rank",
            "value": tokens / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms,
            "with_gather": {"value": tokens / (ms_g_t.item() * 1e-3), "unit": "tokens/s",
                            "ms_per_step": ms_g_t.item(), "time_segments": segs,
                            "gather": "o and S to rank 0, point-to-point over NCCL, every "
                                      "peer's transfers in flight at once, overlapping "
                                      "the next time segment's compute"},
            "roofline": {"bound": "hbm", "achieved": byts / world / (ms * 1e-3) / 1e9,
                         "unit": "GB/s", "algorithmic_bytes": byts}}


def bench_backward(torch, kb, dev, steps, warmup, clk):
    """configs[1] backward: the gradients of one ``kda_chunkwise`` call (B=1,
    T=4096, H=16, fp16 q/k/v, fp32 state) for random output and final-state
    gradients, through ``ops.kda_backward`` (the chunkwise backward: per-chunk
    prep, the two state chains in one launch, the per-chunk gradients).  Two
    rotating input sets.
    Returns (ms per call, algorithmic bytes: every input read once and every
    gradient written once)."""
    B, T, H, K, V = CFG1["B"], CFG1["T"], CFG1["H"], CFG1["K"], CFG1["V"]
    gen = torch.Generator(device=dev).manual_seed(9)
    sets = []
    for s_ in range(2):
        x = kb.synth.make_config(1, seed=20 + s_, device=dev)
        x["do"] = torch.randn(B, T, H, V, generator=gen, device=dev).half()
        x["dS"] = torch.randn(B, H, K, V, generator=gen, device=dev) * 0.01
        sets.append(x)

    def step(i):
        x = sets[i % 2]
        return kb.ops.kda_backward(x["q"], x["k"], x["v"], x["g"], x["beta"], None, x["do"],
                                   x["dS"])

    ms = _events_time(torch, step, steps, warmup, clk)
    th = B * T * H
    nbytes = th * (3 * K * 2 + K * 4 + 4 + V * 2) + B * H * K * V * 4 \
        + th * (2 * K * 2 + V * 2 + K * 4 + 4)
    return ms, nbytes


def bench_cfg4_decode_layers(torch, kb, dev, steps, warmup, clk):
    """The attention side of one configs[4] decode step at its layer shapes
    (B=4, hidden 2048, 16 KDA heads x 128, conv 4, fp16): one KDA layer's core
    work per token -- fused prologue (conv step from the cache, SiLU, L2 norm,
    gates), the recurrent state update on the fp32 [4, 16, 128, 128] state
    (in place, as GraphedDecoder keeps it) and the fused epilogue -- captured
    in a CUDA graph on NBUF layer states and replayed.  The projections, FFN
    and MLA/KDA output projections (cuBLAS GEMMs of the model) are not part of
    it.  Returns ms per KDA layer per decode step."""
    B, H, K, cs = 4, 16, 128, 4
    D = H * K
    NBUF = 8
    g = torch.Generator(device=dev).manual_seed(13)
    f16 = torch.float16

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g, device=dev) * scale).to(f16)
    layers = []
    for _ in range(NBUF):
        layers.append(dict(
            x=[rnd(B, 1, D) for _ in range(4)], beta=rnd(B, 1, H), og=rnd(B, 1, D),
            hist={n: rnd(B, cs - 1, D) for n in "qkv"},
            w=[(torch.randn(D, 1, cs, generator=g, device=dev) * 0.4).to(f16).float()
               for _ in range(3)],
            b=[(torch.randn(D, generator=g, device=dev) * 0.1).to(f16).float() for _ in range(3)],
            A_log=torch.log(torch.rand(H, K, generator=g, device=dev) * 15 + 1),
            dt=torch.log(torch.expm1(torch.rand(H, K, generator=g, device=dev) * 0.099 + 1e-3)),
            S=torch.randn(B, H, K, K, generator=g, device=dev) * 0.02,
            nw=torch.rand(H, K, generator=g, device=dev) + 0.5))

    def layer(i):
        L = layers[i % NBUF]
        q, k, v, gg, beta, _ = kb.kda_prologue(*L["x"], L["beta"], L["w"], L["b"], L["A_log"],
                                                L["dt"], H, K, K, 1e-6, conv_cache=L["hist"])
        o, _ = kb.kda_recurrent(q, k, v, gg, beta, state=L["S"], state_dtype=torch.float32,
                                inplace=True)
        return kb.kda_epilogue(o, L["og"], L["nw"], 1e-6)

    return _graph_time(torch, dev, layer, NBUF, steps, warmup, clk)


def profile_case(which, reps=3):
    """Three calls of one workload on cuda:0 (the target of the ncu captures
    summarised under profiles/): ``prefill`` = configs[1], ``decode`` = one
    configs[2] step, ``mla`` = one configs[4] MLA decode step (8192-token
    prompt in the static buffer), ``io`` = the fused prologue then the fused
    epilogue at the configs[1] shape (the inputs of ``bench_fused_io``),
    ``bwd`` = the configs[1] backward of ``bench_backward``."""
    import torch
    kb = importlib.import_module("-kimi-linear-_b200")
    kb.load_library()
    dev = torch.device("cuda", 0)
    if which == "prefill":
        x = kb.synth.make_config(1, seed=0, device=dev)
        for _ in range(reps):
            kb.kda_chunkwise(x["q"], x["k"], x["v"], x["g"], x["beta"], chunk_size=CFG1["C"],
                             state_dtype=torch.float32)
    elif which == "bwd":
        B, T, H, K, V = CFG1["B"], CFG1["T"], CFG1["H"], CFG1["K"], CFG1["V"]
        gen = torch.Generator(device=dev).manual_seed(9)
        x = kb.synth.make_config(1, seed=20, device=dev)
        do = torch.randn(B, T, H, V, generator=gen, device=dev).half()
        dS = torch.randn(B, H, K, V, generator=gen, device=dev) * 0.01
        for _ in range(reps):
            kb.ops.kda_backward(x["q"], x["k"], x["v"], x["g"], x["beta"], None, do, dS)
    elif which == "io":
        B, T, H, K = 1, CFG1["T"], CFG1["H"], CFG1["K"]
        D = H * K
        g = torch.Generator(device=dev).manual_seed(5)
        x = {n: torch.randn(B, T, D, generator=g, device=dev).half() for n in ("q", "k", "v", "gk")}
        bl = torch.randn(B, T, H, generator=g, device=dev).half()
        ws = [(torch.randn(D, 1, 4, generator=g, device=dev) * 0.4).half().float()
              for _ in range(3)]
        bs = [(torch.randn(D, generator=g, device=dev) * 0.1).half().float() for _ in range(3)]
        A_log = torch.log(torch.rand(H, K, generator=g, device=dev) * 15 + 1)
        dt_bias = torch.log(torch.expm1(torch.rand(H, K, generator=g, device=dev) * 0.099 + 1e-3))
        for _ in range(reps):
            kb.kda_prologue(x["q"], x["k"], x["v"], x["gk"], bl, ws, bs, A_log, dt_bias, H, K, K,
                            1e-6)
        o = torch.randn(B, T, H, K, generator=g, device=dev).half()
        w = torch.rand(H, K, generator=g, device=dev) + 0.5
        for _ in range(reps):
            kb.kda_epilogue(o, x["q"], w, 1e-6)
    elif which == "mla":
        c = CFG4_MLA
        B, L, H, KVL, DN, DV = c["B"], c["L"], c["H"], c["KVL"], c["DN"], c["DV"]
        g = torch.Generator(device=dev).manual_seed(11)
        w = torch.randn(H * (DN + DV), KVL, generator=g, device=dev).mul_(KVL ** -0.5).half()
        q = torch.randn(B, 1, H, DN, generator=g, device=dev).mul_(0.5).half()
        ck = torch.randn(B, 1, KVL, generator=g, device=dev).half()
        buf = torch.zeros(B, L, KVL, device=dev, dtype=torch.float16)
        buf[:, :c["prompt"]].copy_(torch.randn(B, c["prompt"], KVL, generator=g, device=dev))
        pos = torch.tensor([c["prompt"]], dtype=torch.int64, device=dev)
        for _ in range(reps):
            kb.mla.mla_decode_core(q, ck, buf, pos, w, H, DN, DV, DN ** -0.5)
    else:
        y = kb.synth.make_inputs(CFG2["B"], 1, CFG2["H"], CFG2["K"], CFG2["V"],
                                 dtype=torch.float16, seed=2, s0_std=0.02, device=dev)
        for _ in range(reps):
            kb.kda_recurrent(y["q"], y["k"], y["v"], y["g"], y["beta"], state=y["S0"],
                             state_dtype=torch.float32)
    torch.cuda.synchronize()
    print(f"case {which}: {reps} calls done", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("kda", "reference"), default="kda")
    ap.add_argument("--decode-steps", type=int, default=1024)
    ap.add_argument("--long-steps", type=int, default=4,
                    help="timed steps of the configs[3] leg (0 skips it)")
    ap.add_argument("--mla-steps", type=int, default=128,
                    help="timed steps of the configs[4] MLA decode leg")
    ap.add_argument("--io-steps", type=int, default=50,
                    help="timed calls of the fused prologue / epilogue leg (0 skips it)")
    ap.add_argument("--bwd-steps", type=int, default=6,
                    help="timed calls of the configs[1] backward leg (0 skips it)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--case", choices=("prefill", "decode", "mla", "io", "bwd"),
                    help="profiling target: run the workload three times, print nothing timed")
    a = ap.parse_args()
    if a.case:
        return profile_case(a.case)
    if a.warmup < 3:
        a.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if a.impl == "reference":
        if rank != 0:
            return
        heads = max(1, min(os.cpu_count() or 1, 16))
        t_sample = CFG1["T"]        # the same sample as the cpu_baseline leg of the kda arm
        val, wall = cpu_port_throughput(t_sample, heads, steps=a.steps, warmup=a.warmup)
        line = {
            "metric": METRIC, "value": val, "unit": "tokens/s", "n_gpus": a.gpus,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": wall * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16", "data": "synthetic", "impl": "reference",
            "config": {"workload": "kda_chunkwise prefill, BASELINE configs[1]", **CFG1,
                       "sample": f"{heads} of 16 heads x {t_sample} tokens per step"},
            "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": heads, "kind": "port",
                             "sample": f"{heads} heads x {t_sample} tokens of configs[1] per "
                                       f"step, numpy port of kda.py:58-185, fp32 transients "
                                       f"on fp16-valued inputs"},
            "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return

    import torch
    kb = importlib.import_module("-kimi-linear-_b200")
    kb.load_library()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as td
        td.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                              device_id=dev)
        dist = td

    with ClockSampler(dev.index) as clk:
        ms_step, e2e_ms, h2d, d2h, path = bench_prefill(
            torch, kb, dev, a.steps, a.warmup, dist, world, clk)
        dec_ms, dec_steps = bench_decode(torch, kb, dev, a.decode_steps, a.warmup, clk)
        dec_t = torch.tensor([dec_ms], dtype=torch.float64, device=dev)
        if dist is not None:
            dist.all_reduce(dec_t, op=dist.ReduceOp.MAX)
        dec_ms = dec_t.item()
        mla_ms, mla_steps, mla_bytes = bench_mla_decode(torch, kb, dev, a.mla_steps, a.warmup,
                                                        clk)
        io_ms = bench_fused_io(torch, kb, dev, a.io_steps, a.warmup, clk) \
            if a.io_steps > 0 else None
        bwd = bench_backward(torch, kb, dev, a.bwd_steps, 2, clk) if a.bwd_steps > 0 else None
        cfg4_layer_ms = bench_cfg4_decode_layers(torch, kb, dev, max(64, a.mla_steps), a.warmup,
                                                 clk)
        long_ctx = None
        if a.long_steps > 0:
            long_ctx = bench_long_context(torch, kb, dev, a.long_steps, 3, dist, world,
                                          rank, clk)
    clocks = clk.summary()
    # kernels per prefill call: prep + state pass on the tensor-core path (the
    # ready-flag reset before them is a memset node, not a kernel)
    launches_per_call = 2 if path == "tcgen05" else 1

    hbm, tc, peak_kind = _peaks()
    tokens = CFG1["B"] * CFG1["T"]
    th = tokens * CFG1["H"]
    pre_bytes = th * (2 * CFG1["K"] * 2 + CFG1["V"] * 2 + CFG1["K"] * 4 + 4 + CFG1["V"] * 2) \
        + CFG1["B"] * CFG1["H"] * CFG1["K"] * CFG1["V"] * 4
    pre_flop = th * FLOP_PER_TOKEN_HEAD
    dec_bytes = CFG2["B"] * CFG2["H"] * (2 * CFG2["K"] * CFG2["V"] * 4
                                         + 2 * CFG2["K"] * 2 + CFG2["V"] * 2 + CFG2["K"] * 4
                                         + 4 + CFG2["V"] * 2)

    cpu = cpu_dec = cpu_long = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        heads = max(1, min(os.cpu_count() or 1, 16))
        t_sample = CFG1["T"]
        val, wall = cpu_port_throughput(t_sample, heads, steps=2, warmup=1)
        cpu = {"value": val, "unit": "tokens/s", "cores": heads, "kind": "port",
               "sample": f"{heads} heads x {t_sample} tokens of configs[1] "
                         f"({wall:.2f} s per step), numpy port of kda.py:58-185, fp32 "
                         f"transients on fp16-valued inputs"}
        dval, dper = cpu_decode_throughput()
        cpu_dec = {"value": dval, "unit": "tokens/s", "cores": 1, "kind": "port",
                   "sample": f"16 single-token steps of configs[2] on the full fp32 state "
                             f"[64,16,128,128] ({dper * 1e3:.1f} ms per step), numpy port of "
                             f"kda.py:188-219, extrapolated to the 1024-step workload"}
        lt = 8192
        lval, lwall = cpu_long_context_throughput(lt, heads)
        cpu_long = {"value": lval, "unit": "tokens/s", "cores": heads, "kind": "port",
                    "sample": f"{heads} heads x {lt} tokens of configs[3] ({lwall:.2f} s), "
                              f"numpy port of kda.py:58-185 on bf16-valued fp32 inputs "
                              f"with S0 ~ N(0, 0.02)"}

    if rank == 0:
        ach = pre_bytes / (ms_step * 1e-3) / 1e9
        line = {
            "metric": METRIC,
            "value": world * tokens / (ms_step * 1e-3),
            "unit": "tokens/s",
            "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "kda_chunkwise prefill, BASELINE configs[1] per GPU",
                       **CFG1, "state": "fp32", "parallelism": f"dp{world} over (b,h)",
                       "kernel": path,
                       "l2": "inputs larger than L2: 4 rotating input sets (400 MB) "
                             "plus per-call outputs and workspace; no flush"},
            "roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s",
                         "frac": ach / hbm, "peak_kind": peak_kind,
                         "traffic": _traffic("kda_chunkwise", "cfg1"),
                         "algorithmic_bytes": pre_bytes,
                         "tensor_frac": pre_flop / (ms_step * 1e-3) / (tc * 1e12)},
            "e2e": {"value": world * tokens / (e2e_ms[0] * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms[0],
                    "pipeline": "kda_chunkwise on pinned-host inputs: H2D of step i+1, "
                                "compute of step i and D2H of step i-1 on three streams, "
                                "2 device input slots; timed from before the first H2D "
                                "to after the last D2H; median of three runs",
                    "runs_ms_per_step": list(e2e_ms[2:5]),
                    "serial": {"value": world * tokens / (e2e_ms[1] * 1e-3),
                               "ms_per_step": e2e_ms[1],
                               "timing": "H2D, compute, D2H in order on one stream"}},
            "decode": {"workload": "kda_recurrent single-token step, BASELINE configs[2]",
                       "value": world * CFG2["B"] / (dec_ms * 1e-3), "unit": "tokens/s",
                       "ms_per_step": dec_ms, "steps": dec_steps,
                       "timing": "CUDA graph of 4 single-token steps on 4 distinct "
                                 "64 MiB states (512 MiB working set, 4x L2; no flush), "
                                 "replayed; device time per step",
                       "roofline": {"bound": "hbm", "achieved": dec_bytes / (dec_ms * 1e-3) / 1e9,
                                    "peak": hbm, "unit": "GB/s",
                                    "frac": dec_bytes / (dec_ms * 1e-3) / 1e9 / hbm,
                                    "traffic": None,
                                    "traffic_note": "a single-launch ncu capture leaves the "
                                                    "state write in L2 and under-counts the "
                                                    "steady state; not reported",
                                    "algorithmic_bytes": dec_bytes},
                       "cpu_baseline": cpu_dec},
            "mla_decode": {"workload": "MLA static-buffer decode step of configs[4] "
                                       "(B=4, 16 heads, kv_lora_rank 512, head dims 128, "
                                       "buffer 8192 + 256 latents, fp16)",
                           "value": world * CFG4_MLA["B"] / (mla_ms * 1e-3), "unit": "tokens/s",
                           "ms_per_step": mla_ms, "steps": mla_steps,
                           "timing": "CUDA graph of 4 steps on 4 distinct 34.6 MB buffers, "
                                     "replayed; device time per step",
                           "roofline": {"bound": "hbm",
                                        "achieved": mla_bytes / (mla_ms * 1e-3) / 1e9,
                                        "peak": hbm, "unit": "GB/s",
                                        "frac": mla_bytes / (mla_ms * 1e-3) / 1e9 / hbm,
                                        "algorithmic_bytes": mla_bytes}},
            "fused_io": None if io_ms is None else {
                "workload": "fused KDA prologue (conv 4 + SiLU + q/k L2 norm + gates + beta) "
                            "and epilogue (head RMSNorm x weight x sigmoid gate) at the "
                            "configs[1] shape, fp16, 4 rotating input sets (> L2), "
                            "CUDA graph of one call per set, replayed",
                **{name: {"value": CFG1["T"] / (ms * 1e-3), "unit": "tokens/s",
                          "ms_per_call": ms,
                          "roofline": {"bound": "hbm",
                                       "achieved": nb / (ms * 1e-3) / 1e9,
                                       "peak": hbm, "unit": "GB/s",
                                       "frac": nb / (ms * 1e-3) / 1e9 / hbm,
                                       "algorithmic_bytes": nb}}
                   for name, ms, nb in (("prologue", io_ms[0], io_ms[2]),
                                        ("epilogue", io_ms[1], io_ms[3]))}},
            "long_context": None if long_ctx is None else {**long_ctx,
                                                           "cpu_baseline": cpu_long},
            "backward": None if bwd is None else {
                "workload": "gradients of one kda_chunkwise call at configs[1] (B=1, T=4096, "
                            "H=16, fp16, fp32 state) for random do and dS, ops.kda_backward "
                            "(chunkwise: per-chunk prep, forward and reverse state chains, "
                            "per-chunk gradients; fp32 data, 3xTF32 mma.sync GEMMs)",
                "value": tokens / (bwd[0] * 1e-3), "unit": "tokens/s",
                "ms_per_call": bwd[0],
                "roofline": {"bound": "hbm", "achieved": bwd[1] / (bwd[0] * 1e-3) / 1e9,
                             "peak": hbm, "unit": "GB/s",
                             "frac": bwd[1] / (bwd[0] * 1e-3) / 1e9 / hbm,
                             "algorithmic_bytes": bwd[1],
                             "note": "compute-bound (fp32 GEMMs as 3xTF32 mma.sync, one "
                                     "exponential per pair and channel); the HBM fraction is "
                                     "for reference"}},
            "configs4_decode": {
                "workload": "configs[4] decode step, attention side at its layer shapes "
                            "(B=4, fp16): 18 KDA layers x (fused prologue + recurrent "
                            "state update in place + fused epilogue) and 6 MLA static-buffer "
                            "steps; the model's projection / FFN GEMMs are not included (the "
                            "reference model code does not travel with this repository)",
                "kda_layer_ms": cfg4_layer_ms, "mla_step_ms": mla_ms,
                "attention_ms_per_decode_step": 18 * cfg4_layer_ms + 6 * mla_ms,
                "kda_share": 18 * cfg4_layer_ms / (18 * cfg4_layer_ms + 6 * mla_ms)},
            "gpu_launches": a.steps * launches_per_call,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
