#!/usr/bin/env python
"""Benchmark of the block-diffusion select step: logit rows/sec at V = 8194.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 1|2|3|4|5]

One *step* is one select step (m8than/yapd ``server/engine.py:533-622``) over one
GPU's batch.  The default is configuration 3, the metric's 1/2/4/8-GPU
workload: 256 requests per GPU x 2 CFG rows x 32 positions x V = 8194 bf16
logits with per-request parameters (T in [0.5, 1.2], top-k in {0, 50, 200,
1000}, top-p in [0.8, 1], repetition penalty in [1, 1.5] over histories of
0-2048 tokens), Philox Gumbel noise.  Configuration 1 is 64 requests with
uniform parameters (T 0.8, top-p 0.95, min-p 0.05, penalty 1.2), configuration
2 is configuration 3 with fp32 logits.

The batch runs as the engine runs it, continuous batching through the
engine's own buffers: each request's tokens live in a token buffer, every step
samples the masked positions of the requests that are denoising, unmasks,
writes the block back and moves the requests that were committing to their
next block (the library does all of it in its two kernels).  The requests start
staggered (configurations 2 and 3: U{1..32} masked positions and a random step
counter each), so the batch stays ragged.  A logit row is counted when the step
must read it (masked position of a non-commit request), the metric of the
reference's tick; the line also carries the dense figure (every position
sampled, as the reference's tick reads all of them).

Configuration 4 puts the speech LM head in front of the step: each step first
multiplies the hidden states (512 requests x 2 x 32 rows of 1024, bf16) by the
head weight (8194 x 1024) with cuBLAS into a bf16 logits buffer (the unfused
form, ``server/engine.py:517-520``), then runs the select step on it.

Configuration 5 ("turbo") times the Turbo engine's autoregressive sampler
(``server/engine_ar.py:220-243``) through ``sample_rows``: 256 active rows x
V = 6563 fp32 logits, the engine defaults T 0.8, top-k 1000, top-p 0.95,
repetition penalty 1.2 (``server/engine_ar.py:140-146``); one step = one call.

Under ``torchrun`` each rank runs its own request shard (weak scaling, no
per-step collective); ranks gather their committed tokens with one NCCL
all-gather after timing.  Device time is the max over ranks.

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from yapd_b200 import select as S  # noqa: E402
from yapd_b200 import workloads as WL  # noqa: E402

METRIC = "logit rows/sec at V=8194"
LAUNCHES_PER_STEP = 2  # sample_kernel + unmask_kernel per select step
N_BUFFERS = 5  # rotating logits buffers, total well above the 126 MB L2


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8000)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, default=3, choices=[1, 2, 3, 4, 5])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=16)
    ap.add_argument("--requests", type=int, default=None,
                    help="requests per GPU instead of the configuration's (small cases for profiling)")
    ap.add_argument("--unfused", action="store_true",
                    help="configuration 4: time the cuBLAS head GEMM + select step as the main line")
    return ap.parse_args()


# ----------------------------------------------------------------------- dist

def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


_STDOUT_FD = None


def quiet_stdout():
    """Under torchrun, whatever libraries write to the process's stdout (NCCL's
    version banner) goes to stderr, so that stdout carries only the JSON line."""
    global _STDOUT_FD
    if _STDOUT_FD is None:
        sys.stdout.flush()
        _STDOUT_FD = os.dup(1)
        os.dup2(2, 1)


def emit(line: dict):
    """Print the bench's JSON line on the real stdout."""
    sys.stdout.flush()
    if _STDOUT_FD is not None:
        os.write(_STDOUT_FD, (json.dumps(line) + "\n").encode())
    else:
        print(json.dumps(line), flush=True)


def dist_init(ws, local):
    if ws > 1:
        import torch.distributed as dist
        quiet_stdout()
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        return dist
    torch.cuda.set_device(local)
    return None


# --------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], [], set()
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "samples": len(sm), "reasons": sorted(reasons)}


# ------------------------------------------------------------------ workload

def config_name(cfg: int) -> str:
    return {1: "config1", 2: "config2", 3: "config3", 4: "config4", 5: "turbo"}[cfg]


N_HIDDEN = 3  # rotating hidden-state buffers of config 4 (3 x 64 MB > L2)


def cfg4_chain(inp):
    """Configuration 4's sampling chain, the fused variant's epilogue (BASELINE:
    PMI / CFG / penalty / sample / unmask): temperature, repetition penalty and
    Gumbel-max, no top-k / top-p / min-p.  Every leg of configuration 4 (fused,
    unfused, CPU) samples with it."""
    inp.top_k = torch.zeros(inp.B, dtype=torch.int32)
    inp.top_p = torch.ones(inp.B)
    inp.min_p = torch.zeros(inp.B)
    return inp
LOGIT_PAD = 8200  # config 4 logits row length: V = 8194 rounded up to 8 (16 bytes)


def make_inputs(cfg: int, rank: int, device, requests=None):
    """The per-GPU shard: config defaults, Philox noise (production mode).

    Configuration 4 returns one logits buffer and a ``gemm`` dict holding the
    device operands of the head GEMM that fills it every step."""
    if cfg == 4:
        inp = cfg4_chain(WL.make_config(4, seed=100 + rank, B=requests, explicit_noise=False, lmhead_logits=False))
        g = torch.Generator(device=device).manual_seed(7 + 131 * rank)
        hid = [inp.meta["hidden"].to(device)]
        for _ in range(N_HIDDEN - 1):
            hid.append(torch.randn(hid[0].shape, generator=g, device=device).to(torch.bfloat16))
        # the head weight padded to LOGIT_PAD rows: the GEMM writes 16-byte
        # aligned logits rows (cuBLAS takes its fast path; the select step
        # reads the first V columns of each row through its row stride)
        w = inp.meta["weight"].to(device)
        wp = torch.zeros(LOGIT_PAD, w.shape[1], dtype=w.dtype, device=device)
        wp[: w.shape[0]] = w
        out = torch.empty(hid[0].shape[0], LOGIT_PAD, dtype=torch.bfloat16, device=device)
        gemm = {"hidden": hid, "weight": wp, "weight_v": w, "out": out}
        logits = out.view(inp.logits.shape[0], inp.logits.shape[1], LOGIT_PAD)[:, :, : inp.V]
        return inp, [logits], gemm
    inp = WL.make_config(cfg, seed=100 + rank, B=requests, explicit_noise=False,
                         masked="ragged" if cfg in (2, 3) else "all")
    g = torch.Generator(device=device).manual_seed(7 + 131 * rank)
    bufs = [inp.logits.to(device)]
    for _ in range(N_BUFFERS - 1):
        x = torch.randn(inp.logits.shape, generator=g, device=device) * 2.0
        idx = torch.randint(0, inp.V, (*inp.logits.shape[:2], 3), generator=g, device=device)
        x.scatter_add_(2, idx, torch.full(idx.shape, 8.0, device=device))
        bufs.append(x.to(inp.logits.dtype))
    return inp, bufs, None


class Runner:
    """Continuous batching through the engine buffers, as FlashEngine runs it
    (``server/engine.py:491-622``): each request's tokens live in ``xt_full``;
    a step gathers every request's current block in the kernels, samples its
    masked positions (non-commit requests), unmasks, writes the block back and
    moves the requests that were committing to their next, fully masked block.
    The requests start staggered (configurations 2 and 3: U{1..32} masked
    positions and a random step counter each), so the batch stays ragged.
    ``G`` graphs (Philox offsets 0..G-1, rotating logits buffers) are replayed
    in turn; a device counter accumulates the sampled positions."""

    G = 8

    def __init__(self, inp, bufs, device, total_steps: int, gemm=None, fused: bool = False):
        self.inp, self.bufs, self.dev, self.gemm, self.fused = inp, bufs, device, gemm, fused
        B, L = inp.B, inp.L
        # enough blocks that no request reaches the end of its buffer: a block
        # takes at most K denoising ticks and one commit tick
        n_blocks = total_steps // (inp.num_steps + 1) + 4
        self.n_blocks = n_blocks
        xt_full = torch.full((B, n_blocks * L), inp.mask_id, dtype=torch.int64)
        xt_full[:, :L] = inp.xt
        self.state0 = dict(xt_full=xt_full, k=inp.k_step.clone(), c=inp.is_commit.clone())
        self.xt_full = xt_full.to(device)
        self.k = inp.k_step.to(device).clone()
        self.c = inp.is_commit.to(device).clone()
        self.blk = torch.zeros(B, dtype=torch.int64, device=device)
        self.cache = torch.zeros(B, dtype=torch.int64, device=device)
        self.nsp = torch.full((B,), n_blocks * L, dtype=torch.int64, device=device)
        self.flags = torch.zeros(B, 6, dtype=torch.int64, device=device)
        self.count = torch.zeros(1, dtype=torch.int64, device=device)
        self.eng = S.EngineBuffers(xt_full=self.xt_full, blk_start=self.blk, cache_len=self.cache,
                                   n_speech=self.nsp, flags=self.flags, blk_limit=(n_blocks - 1) * L,
                                   cache_limit=n_blocks * L)
        o = S.SelectOutputs.empty(B, L, device)
        self.out = S.SelectOutputs(xt=o.xt, sampled=o.sampled, pmi=o.pmi, n_unmask=o.n_unmask,
                                   n_mask_after=o.n_mask_after, hit_eos=o.hit_eos, k_step=self.k,
                                   is_commit=self.c)
        # min-p off for every request (configurations 2 and 3): the scalar tells
        # the library so, and the select step runs its grouped kernel alone
        min_p = 0.0 if float(inp.min_p.max()) <= 0.0 else inp.min_p.to(device)
        bf = inp.logits.dtype == torch.bfloat16
        self.kernel = "wsample_kernel" if bf and not isinstance(min_p, float) else "sample_kernel"
        if fused:
            self.kernel = "lm_select_kernel"
        self.kw = dict(cfg_scale=inp.cfg_scale, mask_id=inp.mask_id, stop_id=inp.stop_id,
                       temperature=inp.temperature.to(device), top_k=inp.top_k.to(device),
                       top_p=inp.top_p.to(device), min_p=min_p,
                       rep_penalty=inp.rep_penalty.to(device),
                       history=inp.history_bitmap().to(device), pmi_lambda=inp.pmi_lambda,
                       pos_noise=True, use_quantile=True)
        self.lp = inp.log_prior.to(device)
        self.sched = inp.sched_t.to(device)
        self.q = inp.q_t.to(device)
        self.L = L
        self.ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(self.G)]
        self.gev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                    for _ in range(self.G)] if gemm and not fused else None
        for a, b in self.ev + (self.gev or []):  # torch creates the CUDA events lazily
            a.record()
            b.record()
        torch.cuda.synchronize()
        self.graphs, self.pgraphs = [], []
        self.dense_graph = None

    def restore(self):
        """Back to the starting state (the same steps then replay identically)."""
        self.xt_full.copy_(self.state0["xt_full"])
        self.k.copy_(self.state0["k"])
        self.c.copy_(self.state0["c"])
        self.blk.zero_()
        self.cache.zero_()

    def step(self, k: int, prof: bool = True, dense: bool = False, logits=None, hidden=None):
        """Step k of the cycle; `logits` (already on the device) replaces the
        step's own logits buffer (and, in configuration 4, its head GEMM);
        fused: `hidden` replaces the step's hidden-state buffer."""
        if self.fused:
            h = self.gemm["hidden"][k % len(self.gemm["hidden"])] if hidden is None else hidden
            B, L = self.inp.B, self.L
            kw = {k_: v for k_, v in self.kw.items() if k_ not in ("top_k", "top_p", "min_p")}
            S.lmhead_select_step(h.view(B, 2, L, -1), self.gemm["weight_v"], None, self.k, self.c, self.lp,
                                 self.sched, self.q, seed=1234, offset=k, out=self.out, dense=dense,
                                 prof_events=self.ev[k] if prof else None, engine=self.eng, L=L,
                                 positions_sampled=self.count, **kw)
            return
        if self.gemm and logits is None:
            if prof:
                record_event(self.gev[k][0])
            self.head_gemm(self.gemm["hidden"][k % len(self.gemm["hidden"])])
            if prof:
                record_event(self.gev[k][1])
        S.select_step(self.bufs[k % len(self.bufs)] if logits is None else logits, None, self.k, self.c,
                      self.lp, self.sched, self.q, seed=1234, offset=k, out=self.out, dense=dense,
                      prof_events=self.ev[k] if prof else None, engine=self.eng, L=self.L,
                      positions_sampled=self.count, **self.kw)

    def head_gemm(self, hidden):
        """logits = hidden @ weight.T (cuBLAS bf16, fp32 accumulation) into the
        padded buffer; returns the (B*2, L, V) logits view."""
        torch.mm(hidden, self.gemm["weight"].t(), out=self.gemm["out"])
        return self.bufs[0]

    def capture(self):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for k in range(self.G):
                self.step(k)
            self.step(0, prof=False, dense=True)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        # timed graphs carry no profiling events (an event between kernels adds
        # to the step); a second set records the sample kernel's duration for
        # the roofline; one dense step (every position sampled)
        for k in range(self.G):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.step(k, prof=False)
            self.graphs.append(g)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.step(k)
            self.pgraphs.append(g)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step(0, prof=False, dense=True)
        self.dense_graph = g
        torch.cuda.synchronize()
        self.restore()
        torch.cuda.synchronize()


def record_event(ev):
    """Record a timing event on the current stream; inside a graph capture as
    an event-record node (a plain record there only orders the capture)."""
    from cuda.bindings import runtime as rt
    st = torch.cuda.current_stream()
    err, cap = rt.cudaStreamIsCapturing(rt.cudaStream_t(st.cuda_stream))
    if int(err) != 0:
        raise RuntimeError(f"cudaStreamIsCapturing failed: {err}")
    if cap == rt.cudaStreamCaptureStatus.cudaStreamCaptureStatusActive:
        err, = rt.cudaEventRecordWithFlags(rt.cudaEvent_t(ev.cuda_event), rt.cudaStream_t(st.cuda_stream),
                                           rt.cudaEventRecordExternal)
        if int(err) != 0:
            raise RuntimeError(f"cudaEventRecordWithFlags failed: {err}")
    else:
        ev.record(st)


def event_ms(e0, e1) -> float:
    """Elapsed time between two events recorded by the library (inside a graph,
    so torch's own bookkeeping does not know them)."""
    from cuda.bindings import runtime as rt
    err, ms = rt.cudaEventElapsedTime(rt.cudaEvent_t(e0.cuda_event), rt.cudaEvent_t(e1.cuda_event))
    if int(err) != 0:
        raise RuntimeError(f"cudaEventElapsedTime failed: {err}")
    return float(ms)


def algorithmic_bytes(inp, positions: int) -> int:
    return WL.algorithmic_bytes(inp, 2 * positions, positions, explicit_noise=False)


def roofline_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def tensor_peak():
    """Dense bf16 TFLOP/s: the measured burst figure (a kernel timed alone)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"]), "measured (burst)"
    except Exception:
        return 1590.0, "fallback"


def timed_steps(R, warmup: int, steps: int, dist):
    """Replay `warmup` then `steps` graphs of R's cycle; (device ms of the
    timed steps, positions they sampled) on this rank."""
    for i in range(warmup):
        R.graphs[i % R.G].replay()
    c0 = count_now(R)
    if dist:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        R.graphs[(warmup + i) % R.G].replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1), count_now(R) - c0


def committed_traffic(cfg: int):
    """DRAM bytes per sample-kernel launch from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d.get(config_name(cfg))
    except Exception:
        return None


# ------------------------------------------------------------ CPU baselines

def cpu_head(inp):
    """Configuration 4: the head GEMM on the host cores, as the reference's
    speech head runs before its select step."""
    if inp.meta.get("config") == 4:
        inp.logits = WL.lmhead_logits_of(inp.meta["hidden"], inp.meta["weight"]).view(inp.logits.shape)


def host_cpu() -> dict:
    """The host CPU: model name, physical cores and logical CPUs."""
    model, phys = None, set()
    try:
        cur = {}
        for line in open("/proc/cpuinfo"):
            if ":" not in line:
                if cur:
                    phys.add((cur.get("physical id", "0"), cur.get("core id", cur.get("processor"))))
                cur = {}
                continue
            k, v = [x.strip() for x in line.split(":", 1)]
            cur[k] = v
            if k == "model name" and model is None:
                model = v
        if cur:
            phys.add((cur.get("physical id", "0"), cur.get("core id", cur.get("processor"))))
    except OSError:
        pass
    return {"cpu_model": model, "physical_cores": len(phys) or None, "logical_cpus": os.cpu_count()}


def cpu_threads() -> int:
    """Threads for the CPU arms: one per physical core."""
    n = host_cpu()["physical_cores"] or os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


def cpu_sample(cfg: int, seconds: float, B_s: int = 2):
    """The CPU oracle (the reference algorithm, torch CPU, all host cores) on a
    bounded sample of the same workload: B_s requests, all positions masked."""
    from oracle import select_oracle as O
    cpu_threads()
    inp = WL.make_config(cfg, seed=999, B=B_s, explicit_noise=False)
    if cfg == 4:
        cfg4_chain(inp)
    rows = 2 * inp.B * inp.L
    O.select_step(inp, noise="philox", seed=1, offset=0)
    n, t0 = 0, time.perf_counter()
    while True:
        cpu_head(inp)
        O.select_step(inp, noise="philox", seed=1, offset=n)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return {"value": rows * n / el, "unit": "rows/s", "cores": torch.get_num_threads(),
            "kind": "port", **host_cpu(), "sample": f"{config_name(cfg)} shape with B={B_s} requests, all "
            f"{inp.L} positions masked, {n} steps in {el:.1f} s (torch CPU oracle"
            f"{', after the head GEMM' if cfg == 4 else ''})"}, el / n, rows


# ----------------------------------------------------------------- main arms

def run_reference(args, ws, rank):
    if ws > 1 and rank != 0:
        return
    if args.config == 5:
        return run_reference_turbo(args)
    B_s = 4
    from oracle import select_oracle as O
    cpu_threads()
    inp = WL.make_config(args.config, seed=999, B=B_s, explicit_noise=False)
    if args.config == 4:
        cfg4_chain(inp)
    rows = 2 * inp.B * inp.L
    for i in range(args.warmup):
        cpu_head(inp)
        O.select_step(inp, noise="philox", seed=1, offset=i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        cpu_head(inp)
        O.select_step(inp, noise="philox", seed=1, offset=i)
    el = time.perf_counter() - t0
    v = rows * args.steps / el
    cb = {"value": v, "unit": "rows/s", "cores": torch.get_num_threads(), "kind": "port", **host_cpu(),
          "sample": f"{config_name(args.config)} shape with B={B_s} requests per step, all positions "
                    f"masked (torch CPU oracle of server/engine.py:533-612"
                    f"{', after the head GEMM' if args.config == 4 else ''})"}
    line = {"metric": METRIC, "value": v, "unit": "rows/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": f"{config_name(args.config)} (CPU sample, B={B_s})",
                       "parallelism": "host cores"},
            "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


def count_now(R) -> int:
    torch.cuda.synchronize()
    return int(R.count.item())


def run_ours(args, ws, rank, local):
    dist = dist_init(ws, local)
    dev = torch.device("cuda", local)
    cfg = args.config
    inp, bufs, gemm = make_inputs(cfg, rank, dev, args.requests)
    total = args.warmup + args.steps + Runner.G + args.e2e_steps + 8
    fused = cfg == 4 and not args.unfused
    R = Runner(inp, bufs, dev, total, gemm, fused=fused)
    R.capture()
    G = R.G
    # warm-up (the state evolves: the timed steps see a running batch)
    for i in range(args.warmup):
        R.graphs[i % G].replay()
    c0 = count_now(R)
    if dist:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0.record()
    for i in range(args.steps):
        R.graphs[(args.warmup + i) % G].replay()
    e1.record()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    ck = clocks.stop()
    my_pos = count_now(R) - c0
    # sample-kernel time: one cycle of the profiling graphs, continuing the
    # same running batch after the timed region
    c1 = count_now(R)
    for k in range(G):
        R.pgraphs[(args.warmup + args.steps + k) % G].replay()
    prof_pos = count_now(R) - c1
    order = [(args.warmup + args.steps + k) % G for k in range(G)]
    kern_ms = sum(event_ms(*R.ev[k]) for k in order)
    gemm_ms = [event_ms(*R.gev[k]) for k in order] if R.gev else None
    byt = sum(algorithmic_bytes(inp, 0) for _ in range(G)) + (algorithmic_bytes(inp, prof_pos) -
                                                               algorithmic_bytes(inp, 0))
    achieved = byt / (kern_ms * 1e-3) / 1e9
    # the dense figure: every position of every request sampled (the
    # reference's tick reads all L positions, server/engine.py:533-550)
    nd = max(4, min(32, args.steps // 4))
    cd = count_now(R)
    d0 = torch.cuda.Event(enable_timing=True)
    d1 = torch.cuda.Event(enable_timing=True)
    d0.record()
    for _ in range(nd):
        R.dense_graph.replay()
    d1.record()
    dense_pos = count_now(R) - cd
    dense_ms = d0.elapsed_time(d1)
    if dist:
        t = torch.tensor([ms, float(my_pos), dense_ms, float(dense_pos)], device=dev, dtype=torch.float64)
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm_ = t.clone()
        dist.all_reduce(sm_, op=dist.ReduceOp.SUM)
        ms_max, pos_all = float(mx[0]), float(sm_[1])
        dense_ms_max, dense_pos_all = float(mx[2]), float(sm_[3])
        # final gather of the committed block tokens (the only collective)
        from yapd_b200.shard import gather_committed
        gather_committed(R.out.xt, R.out.xt.shape[0] * ws, dist)
        torch.cuda.synchronize()
    else:
        ms_max, pos_all, dense_ms_max, dense_pos_all = ms, float(my_pos), dense_ms, float(dense_pos)
    rows_all = 2.0 * pos_all
    value = rows_all / (ms_max * 1e-3)

    # ---- configuration 4: the unfused comparison (cuBLAS head GEMM, then
    # the select step) over the same running batch ----
    unf = None
    if fused:
        R2 = Runner(inp, bufs, dev, total, gemm, fused=False)
        R2.capture()
        u_ms, u_pos = timed_steps(R2, args.warmup, args.steps, dist)
        if dist:
            t = torch.tensor([u_ms, float(u_pos)], device=dev, dtype=torch.float64)
            mx = t.clone()
            dist.all_reduce(mx, op=dist.ReduceOp.MAX)
            sm_ = t.clone()
            dist.all_reduce(sm_, op=dist.ReduceOp.SUM)
            u_ms, u_pos = float(mx[0]), float(sm_[1])
        unf = {"value": 2.0 * u_pos / (u_ms * 1e-3), "unit": "rows/s", "ms_per_step": u_ms / args.steps,
               "what": "cuBLAS bf16 head GEMM into 16-byte-aligned bf16 logits rows, then yapd_select_step "
                       "(same inputs, parameters and noise)"}
        del R2
        R.restore()

    # ---- end to end through the public API with host buffers ----
    e2e = run_e2e(R, inp, dev, args.e2e_steps)
    if dist:
        t = torch.tensor([e2e["ms"], float(e2e["rows"])], device=dev, dtype=torch.float64)
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm_ = t.clone()
        dist.all_reduce(sm_, op=dist.ReduceOp.SUM)
        e2e_ms, e2e_rows = float(mx[0]), float(sm_[1])
    else:
        e2e_ms, e2e_rows = e2e["ms"], e2e["rows"]

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu, _, _ = cpu_sample(cfg, args.cpu_seconds)

    if rank == 0:
        peak, peak_kind = roofline_peak()
        traffic = committed_traffic(cfg)
        line = {
            "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16" if inp.logits.dtype == torch.bfloat16 else "f32",
            "data": "synthetic",
            "config": {
                "workload": f"{config_name(cfg)}: {inp.B} requests x 2 CFG rows x {inp.L} positions x "
                            f"V={inp.V} per GPU, continuous batching through the engine buffers "
                            f"({inp.num_steps}-step blocks, requests staggered"
                            f"{': U{1..32} masked and a random step counter at start' if cfg in (2, 3) else ''}), "
                            f"rows of masked positions of non-commit requests",
                "global_batch": inp.B * ws, "seq_len": inp.L, "parallelism": f"request-sharded x{ws}",
                "l2": f"{N_BUFFERS} rotating logits buffers ({N_BUFFERS * inp.logits.numel() * inp.logits.element_size() / 1e6:.0f} MB) > L2",
                "noise": "in-kernel Philox4x32-10 Gumbel",
                "rows_per_step_mean": rows_all / args.steps / ws,
                "dense": {"value": 2.0 * dense_pos_all / (dense_ms_max * 1e-3), "unit": "rows/s",
                          "ms_per_step": dense_ms_max / nd,
                          "note": "every position of every request sampled (the reference's tick)"},
            },
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                         "traffic_source": "profiles/traffic.json (ncu dram__bytes per launch, committed)",
                         "kernel": R.kernel,
                         "kernel_ms_per_launch": kern_ms / G, "bytes_per_launch": byt / G},
            "e2e": {"value": e2e_rows / (e2e_ms * 1e-3), "unit": "rows/s",
                    "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"]},
            "gpu_launches": LAUNCHES_PER_STEP * args.steps,
            "clocks": ck,
            "cpu_baseline": cpu,
        }
        if fused:
            h = gemm["hidden"][0]
            flop = 2.0 * h.shape[0] * h.shape[1] * inp.V  # useful flops: every row, V columns
            kl = kern_ms / G
            tp, tp_kind = tensor_peak()
            ach = flop / (kl * 1e-3) / 1e12
            line["roofline"] = {"bound": "tensor", "achieved": ach, "peak": tp, "unit": "TFLOP/s",
                                "frac": ach / tp, "traffic": committed_traffic(cfg), "peak_kind": tp_kind,
                                "traffic_source": "profiles/traffic.json (ncu dram__bytes per launch, committed)",
                                "kernel": R.kernel, "kernel_ms_per_launch": kl, "flop_per_launch": flop}
            line["config"].update({
                "workload": f"config4 (fused): tcgen05 bf16 head GEMM [{h.shape[0]} x {h.shape[1]}] x "
                            f"[{inp.V} x {h.shape[1]}]^T with the select epilogue on the accumulators "
                            f"(no logits in HBM), then the resolve and state-update kernels; {inp.B} requests "
                            f"x 2 CFG rows x {inp.L} positions, continuous batching; temperature, repetition "
                            f"penalty and Gumbel-max",
                "l2": f"{N_HIDDEN} rotating hidden-state buffers ({N_HIDDEN * h.numel() * 2 / 1e6:.0f} MB) > L2",
                "unfused": unf})
            line["gpu_launches"] = 3 * args.steps
        elif gemm:
            h = gemm["hidden"][0]
            flop = 2.0 * h.shape[0] * h.shape[1] * inp.V  # useful flops (V columns)
            gm = sum(gemm_ms) / G
            line["config"].update({
                "workload": f"config4 (unfused): cuBLAS bf16 head GEMM [{h.shape[0]} x {h.shape[1]}] x "
                            f"[{inp.V} x {h.shape[1]}]^T (weight zero-padded to {LOGIT_PAD} rows) -> "
                            f"bf16 logits rows of stride {LOGIT_PAD}, then the select step; "
                            f"{inp.B} requests x 2 CFG rows x {inp.L} positions, continuous batching",
                "gemm_ms_per_step": gm, "gemm_tflops": flop / (gm * 1e-3) / 1e12,
                "l2": f"{N_HIDDEN} rotating hidden-state buffers ({N_HIDDEN * h.numel() * 2 / 1e6:.0f} MB) "
                      f"and a {inp.logits.numel() * 2 / 1e6:.0f} MB logits buffer > L2"})
            line["gpu_launches"] = (LAUNCHES_PER_STEP + 1) * args.steps
        emit(line)
    if dist:
        del R
        dist.destroy_process_group()


def run_e2e(R, inp, dev, steps):
    """Same metric through select_step with host buffers: every step copies its
    logits (configuration 4: its hidden states) from pinned host memory to the
    device, runs the step on the engine's device-resident state, and reads back
    the flags and the block tokens, the engine tick's one device-to-host sync
    (server/engine.py:635-636)."""
    if R.gemm:
        pin = [h.cpu().pin_memory() for h in R.gemm["hidden"][:2]]
        dhid = torch.empty_like(R.gemm["hidden"][0])
    else:
        pin = [b.cpu().pin_memory() for b in R.bufs[:2]]
    dlog = None if R.gemm else torch.empty(R.bufs[0].shape, dtype=R.bufs[0].dtype, device=dev)
    of = torch.empty(R.flags.shape, dtype=torch.int64).pin_memory()
    ox = torch.empty(R.out.xt.shape, dtype=torch.int64).pin_memory()

    def tick(i):
        if R.fused:
            dhid.copy_(pin[i % 2], non_blocking=True)
            R.step(i % R.G, prof=False, hidden=dhid)
            of.copy_(R.flags, non_blocking=True)
            ox.copy_(R.out.xt, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            return
        if R.gemm:
            dhid.copy_(pin[i % 2], non_blocking=True)
            logits = R.head_gemm(dhid)
        else:
            dlog.copy_(pin[i % 2], non_blocking=True)
            logits = dlog
        R.step(i % R.G, prof=False, logits=logits)
        of.copy_(R.flags, non_blocking=True)
        ox.copy_(R.out.xt, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for i in range(2):
        tick(i)
    c0 = count_now(R)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        tick(i)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    rows = 2 * (count_now(R) - c0)
    h2d = pin[0].numel() * pin[0].element_size()
    d2h = of.numel() * 8 + ox.numel() * 8
    return {"ms": ms, "rows": rows, "h2d": h2d, "d2h": d2h}


TURBO_ROWS, TURBO_V, TURBO_BUFS = 256, 6563, 24  # 24 x 6.7 MB of logits > L2
TURBO_METRIC = "logit rows/sec at V=6563 (Turbo sampler)"


def turbo_inputs(seed: int, R: int = TURBO_ROWS):
    """Turbo rows: logits ~ N(0, 2) with three tokens per row +8 (as the
    block configurations), a 2% bool history, the engine's default parameters."""
    g = torch.Generator().manual_seed(seed)
    logits = WL.make_logits(g, R, 1, TURBO_V).view(R, TURBO_V)
    seen = torch.rand(R, TURBO_V, generator=g) < 0.02
    prm = dict(temperature=torch.full((R,), 0.8), top_k=torch.full((R,), 1000, dtype=torch.int32),
               top_p=torch.full((R,), 0.95), min_p=torch.zeros(R), rep_penalty=torch.full((R,), 1.2))
    return logits, seen, prm


def turbo_oracle_step(logits, seen, prm, i: int):
    """One Turbo step on the host (the oracle's chain of server/engine_ar.py:220-243)."""
    from oracle import select_oracle as O
    R = logits.shape[0]
    G = O.gumbel_from_uniform(torch.rand(R, TURBO_V, generator=torch.Generator().manual_seed(i)))
    return O.sample_tokens(logits, prm["temperature"], prm["top_k"], prm["top_p"], prm["min_p"],
                           prm["rep_penalty"], seen, G, zero_temp="unscaled")


def run_turbo(args, ws, rank, local):
    """Configuration 5 on each rank (weak scaling): sample_rows over the
    engine's active rows, one call (one kernel launch) per step."""
    dist = dist_init(ws, local)
    dev = torch.device("cuda", local)
    logits, seen, prm = turbo_inputs(100 + rank)
    gd = torch.Generator(device=dev).manual_seed(7 + rank)
    bufs = [logits.to(dev)] + [torch.randn(logits.shape, generator=gd, device=dev) * 2.0
                               for _ in range(TURBO_BUFS - 1)]
    kw = {k: v.to(dev) for k, v in prm.items()}
    seen_d = seen.to(dev)
    out = torch.empty(TURBO_ROWS, dtype=torch.int32, device=dev)

    def call(i, x):
        S.sample_rows(x, seen=seen_d, seed=1234, offset=i, out=out, zero_temp_greedy=False, **kw)

    for i in range(3):
        call(i, bufs[i])
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        call(0, bufs[0])
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(TURBO_BUFS):
            call(i, bufs[i])
    reps = max(1, args.steps // TURBO_BUFS)
    steps = reps * TURBO_BUFS
    for _ in range(max(1, -(-args.warmup // TURBO_BUFS))):
        g.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    ck = clocks.stop()
    # kernel time per launch: events around single calls (one launch each)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(TURBO_BUFS)]
    for i in range(TURBO_BUFS):
        ev[i][0].record()
        call(i, bufs[i])
        ev[i][1].record()
    torch.cuda.synchronize()
    kern_ms = sum(a.elapsed_time(b) for a, b in ev) / TURBO_BUFS
    if dist:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
    rows_all = float(TURBO_ROWS * steps * ws)
    value = rows_all / (ms * 1e-3)
    # end to end: logits from pinned host memory, sampled ids back, every step
    pin = [b.cpu().pin_memory() for b in bufs[:2]]
    dl = torch.empty_like(bufs[0])
    ho = torch.empty(TURBO_ROWS, dtype=torch.int32).pin_memory()
    n_e2e = max(2, args.e2e_steps)

    def tick(i):
        dl.copy_(pin[i % 2], non_blocking=True)
        call(i, dl)
        ho.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for i in range(2):
        tick(i)
    e0.record()
    for i in range(n_e2e):
        tick(i)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t[0])
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = turbo_cpu(args.cpu_seconds)
    if rank == 0:
        peak, peak_kind = roofline_peak()
        # logits in, sampled ids out (the bool history is read per candidate only)
        byt = TURBO_ROWS * TURBO_V * 4 + TURBO_ROWS * 4
        ach = byt / (kern_ms * 1e-3) / 1e9
        line = {
            "metric": TURBO_METRIC, "value": value, "unit": "rows/s",
            "n_gpus": ws, "steps": steps, "warmup": args.warmup, "ms_per_step": ms / steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": f"turbo: sample_rows over {TURBO_ROWS} rows x V={TURBO_V} fp32, T 0.8, "
                                   f"top-k 1000, top-p 0.95, rep 1.2 (server/engine_ar.py:220-243)",
                       "global_batch": TURBO_ROWS * ws, "parallelism": f"request-sharded x{ws}",
                       "l2": f"{TURBO_BUFS} rotating logits buffers "
                             f"({TURBO_BUFS * bufs[0].numel() * 4 / 1e6:.0f} MB) > L2",
                       "noise": "in-kernel Philox4x32-10 Gumbel"},
            "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s",
                         "frac": ach / peak, "traffic": None, "peak_kind": peak_kind,
                         "kernel": "sample_kernel", "kernel_ms_per_launch": kern_ms,
                         "bytes_per_launch": byt},
            "e2e": {"value": TURBO_ROWS * ws * n_e2e / (e2e_ms * 1e-3), "unit": "rows/s",
                    "h2d_bytes_per_step": bufs[0].numel() * 4, "d2h_bytes_per_step": TURBO_ROWS * 4},
            "gpu_launches": steps, "clocks": ck, "cpu_baseline": cpu,
        }
        emit(line)
    if dist:
        del g
        dist.destroy_process_group()


def turbo_cpu(seconds: float, R: int = 16):
    """The Turbo chain on the host cores (oracle port) on a bounded sample."""
    cpu_threads()
    logits, seen, prm = turbo_inputs(999, R)
    turbo_oracle_step(logits, seen, prm, 0)
    n, t0 = 0, time.perf_counter()
    while True:
        turbo_oracle_step(logits, seen, prm, n)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return {"value": R * n / el, "unit": "rows/s", "cores": torch.get_num_threads(), "kind": "port",
            **host_cpu(), "sample": f"{R} Turbo rows per call, {n} calls in {el:.1f} s (torch CPU oracle of "
                      f"server/engine_ar.py:220-243)"}


def run_reference_turbo(args, R: int = 16):
    """The reference arm of configuration 5: the Turbo chain on the host cores
    (oracle port), R rows per step."""
    cpu_threads()
    logits, seen, prm = turbo_inputs(999, R)
    for i in range(args.warmup):
        turbo_oracle_step(logits, seen, prm, i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        turbo_oracle_step(logits, seen, prm, i)
    el = time.perf_counter() - t0
    v = R * args.steps / el
    cb = {"value": v, "unit": "rows/s", "cores": torch.get_num_threads(), "kind": "port", **host_cpu(),
          "sample": f"{R} Turbo rows per step (torch CPU oracle of server/engine_ar.py:220-243)"}
    print(json.dumps({"metric": TURBO_METRIC, "value": v, "unit": "rows/s",
                      "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
                      "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
                      "config": {"workload": f"turbo (CPU sample, {R} rows)", "parallelism": "host cores"},
                      "cpu_baseline": cb,
                      "e2e": {"value": v, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
          flush=True)


def main():
    args = parse()
    ws, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, ws, rank)
        return
    if args.config == 5:
        run_turbo(args, ws, rank, local)
        return
    run_ours(args, ws, rank, local)


if __name__ == "__main__":
    main()
