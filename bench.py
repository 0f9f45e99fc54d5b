"""Benchmark of the memory-layer hot path: fwd+bwd tokens/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 1] [--impl reference]

One step = forward + backward of the memory recurrence over one batch of the
configuration's synthetic inputs (seeded; the distributions of the benchmark
config), through the public API ``atlas_rnn_b200.memory_recurrence``.
Multi-GPU (torchrun, one rank per GPU): batch*head units are independent, so
every rank runs its own full copy of the configuration (weak scaling, no
data-path collective); timing is the max over ranks of CUDA-event time.

``--impl reference`` times the reference algorithm on the host cores instead:
the CPU restatement in oracle/ (materialised [N,T,d,d] einsums and log-depth
scalar scans, autograd backward), on a bounded slice of the same workload,
scaled to the whole workload. Under torchrun only rank 0 runs it.

``--config 3`` times the LMM language model instead (one training step of the
12-layer model of the benchmark config: loss, backward, AdamW; bf16 autocast).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from atlas_rnn_b200.workloads import CONFIGS, make_inputs, shrink  # noqa: E402

METRIC = "memory-layer fwd+bwd tokens/sec"
WITH_BUFFER = False  # pass the (zero) carried omega buffer as the modules do after init_state
UNIT = "tokens/s"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ---------------------------------------------------------------------------
# reference arm / CPU baseline: the oracle port on host cores
# ---------------------------------------------------------------------------
def cpu_sample(w, n_units=1, t_tokens=512, min_seconds=10.0, max_reps=50):
    """Time fwd+bwd of the CPU restatement on a slice; returns (tokens/s scaled
    to the full workload, seconds per rep, reps, sample description)."""
    from oracle import memory_ref
    ws = shrink(w, B=1, H=n_units, T=min(t_tokens, w.T))
    inp = make_inputs(ws, seed=0, device="cpu")
    leaf = {k: (v.float().clone().requires_grad_(True) if v is not None else None) for k, v in inp.items()
            if k not in ("dy", "proj")}
    proj = inp["proj"]
    U = leaf["gate"] if w.gate == "window" else None
    u = leaf["gate"] if w.gate == "token" else None
    times = []
    t_start = time.perf_counter()
    while (time.perf_counter() - t_start < min_seconds and len(times) < max_reps) or len(times) < 1:
        for t in leaf.values():
            if t is not None:
                t.grad = None
        t0 = time.perf_counter()
        y, S_end, Z_end, nb = memory_ref.memory_layer(
            leaf["k"], leaf["q"], leaf["v"], leaf["lr"], leaf["decay"], leaf["beta"], u, leaf["S0"], leaf["S0"],
            leaf["Z0"], leaf["omega_buffer"], window=w.window, U=U, fmap_mode=w.fmap_mode,
            fmap_degree=w.fmap_degree, proj=proj)
        y.backward(inp["dy"].float())
        times.append(time.perf_counter() - t0)
    per = statistics.median(times)
    # linear in units and tokens (the log-depth scan does O(T) work)
    full_time = per * (w.N / ws.N) * (w.T / ws.T)
    tok_s = w.B * w.T / full_time
    sample = (f"oracle port fwd+bwd (fp32, torch CPU) on {ws.N} unit(s) x {ws.T} tokens of "
              f"{w.name}, median of {len(times)} reps = {per:.3f} s, scaled linearly to "
              f"{w.N} units x {w.T} tokens")
    return tok_s, per, len(times), sample


def reference_cuda_times(steps=5, warmup=2):
    """The reference's own Omega-16 CUDA kernels (built from its sources into oracle/_ref by
    oracle/ref_cuda.py) fwd+bwd on the shapes of its performance test, CUDA-event timed; or
    the reason they cannot run here."""
    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device"}
    from oracle import ref_cuda
    try:
        ext = ref_cuda.load()
    except Exception as ex:
        return {"unavailable": str(ex)}
    dev = torch.device("cuda", torch.cuda.current_device())
    out = {}
    b16 = lambda t: t.to(torch.bfloat16).contiguous()
    for wr in ref_kernel_workloads():
        x = make_inputs(wr, seed=0, device=dev, state_scale=0.1)
        a = [b16(x[n]) for n in ("k", "q", "v")] + [b16(x["S0"])] + \
            [b16(x[n]) for n in ("lr", "decay", "beta", "gate")] + [b16(x["S0"]), b16(x["Z0"]), b16(x["dy"])]
        m = timed_ms(lambda: ref_cuda.forward_backward(ext, *a), steps, warmup, dev,
                     lambda: torch.cuda.synchronize(dev))
        out[f"B{wr.B}_H{wr.H}_T{wr.T}"] = {"ms_per_step": m, "tokens_per_s": wr.B * wr.T / (m / 1000.0)}
        del x, a
    return {"kernels": "reference atlas_omega.cu forward_exact_kernel + backward_exact_kernel (sm_100a build)",
            "times": out}


def run_reference(args, w):
    """The reference arm: the reference's algorithm (restated in oracle/, the reference being a
    Python package that cannot travel) fwd+bwd on the host cores, rank 0 only. Each step is
    ``REF_REPS`` repetitions of a bounded slice (1 unit x 512 tokens); ms_per_step is that
    measured slice time, and value scales the slice's rate to the whole workload (the work is
    linear in units and tokens), with the factor stated. At N = 1 the line also carries the
    reference's own CUDA kernels timed on the shapes of its performance test."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    REF_REPS = 5
    for _ in range(args.warmup):
        cpu_sample(w, min_seconds=0.0, max_reps=1)
    pers, sample = [], ""
    for _ in range(args.steps):
        _, per, _, sample = cpu_sample(w, min_seconds=0.0, max_reps=REF_REPS)
        pers.append(per)
    per = statistics.median(pers)
    n_units, t_tok = 1, min(512, w.T)
    scale = (w.N / n_units) * (w.T / t_tok)
    value = w.B * w.T / (per * scale)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * per, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(w, ws),
            "slice": {"units": n_units, "tokens": t_tok, "reps_per_step": REF_REPS,
                      "ms_per_rep_median": 1000.0 * per, "scale_to_workload": scale,
                      "ms_per_workload_step_extrapolated": 1000.0 * per * scale,
                      "note": "ms_per_step is the measured slice; value is its rate scaled to the workload"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if ws == 1 and args.config == 1 and not args.no_extra:
        line["reference_kernel_shapes"] = reference_cuda_times()
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clock/throttle samples (every 50 ms, rank 0, all GPUs of the job).

    Sampling starts on entry and waits for the first row, so that the timed region
    that follows is covered; summary() keeps the rows stamped inside
    [mark_start(), mark_end()] (the nearest row when the region is shorter than
    one period).
    """
    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_ids, rank: int):
        self.ids = gpu_ids
        self.rank = rank
        self.proc = None
        import tempfile
        fd, self.path = tempfile.mkstemp(prefix="atlas_bench_clocks_", suffix=".csv")
        os.close(fd)
        self.t0 = self.t1 = None

    def _rows(self):
        import datetime
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 10 and parts[2].replace(".", "").isdigit():
                try:
                    ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                except ValueError:
                    continue
                rows.append((ts, parts[1:]))
        return rows

    def __enter__(self):
        if self.rank != 0:
            return self
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", ",".join(self.ids), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
            deadline = time.time() + 10.0
            while time.time() < deadline and not self._rows():
                time.sleep(0.02)
        except Exception:
            self.proc = None
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()
        if self.proc is not None:  # one more period so the region's last samples land
            time.sleep(0.12)

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        try:
            return self._summary()
        finally:
            try:
                os.unlink(self.path)
            except OSError:
                pass

    def _summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        allrows = self._rows()
        if not allrows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        t0 = self.t0 if self.t0 is not None else allrows[0][0]
        t1 = self.t1 if self.t1 is not None else allrows[-1][0]
        rows = [r for ts, r in allrows if t0 <= ts <= t1]
        if not rows:  # region shorter than one period: the sample nearest to its middle, per GPU
            mid = 0.5 * (t0 + t1)
            best = {}
            for ts, r in allrows:
                if r[0] not in best or abs(ts - mid) < abs(best[r[0]][0] - mid):
                    best[r[0]] = (ts, r)
            rows = [r for _, r in best.values()]
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows)}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def step_api(inp, w, leaves_from, backward=True):
    """One fwd+bwd (or forward only) through the public API. Returns y."""
    from atlas_rnn_b200 import memory_recurrence
    L = leaves_from
    y, S_end, Z_end, nb = memory_recurrence(
        L["k"], L["q"], L["v"], L["lr"], L["decay"], L["beta"], L["gate"], S_ref=inp["S0"], S0=inp["S0"],
        Z0=inp["Z0"], omega_buffer=inp["omega_buffer"] if WITH_BUFFER else None, window=w.window,
        gate_mode="window" if w.gate == "window" else "token", fmap_mode=w.fmap_mode, fmap_degree=w.fmap_degree,
        proj=inp["proj"])
    if backward:
        torch.autograd.backward([y], [L["dy"]])
    return y


def step_seqpar(inp, w, leaves_from, backward=True):
    """One fwd+bwd (or forward only) of this rank's token slice, sequence-parallel over all ranks."""
    from atlas_rnn_b200.parallel import seq_parallel_memory
    L = leaves_from
    y, S_end, Z_end = seq_parallel_memory(L["k"], L["q"], L["v"], L["lr"], L["decay"], L["beta"], S_ref=inp["S0"],
                                          S0=inp["S0"], Z0=inp["Z0"])
    if backward:
        torch.autograd.backward([y], [L["dy"]])
    return y


def traffic_from_profiles(kernel: str, workload: str):
    """Per-launch DRAM bytes recorded from an ncu capture in profiles/ (or None)."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_{workload}.md")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None

# shapes of the reference's own performance test (tests/test_atlas_performance.py:97-204):
# head 64, window 16, bf16, per-token omega gate, momentum -- the only shape its CUDA kernels run
REF_KERNEL_SHAPES = ((8, 14, 512), (4, 14, 16384))


def ref_kernel_workloads():
    return [shrink(CONFIGS[5], B=b, H=h, T=t) for b, h, t in REF_KERNEL_SHAPES]


def timed_ms(fn, steps, warmup, dev, sync):
    """CUDA-event time per call of fn() on the current stream, after warmup calls;
    sync() brackets the region (barrier + synchronize)."""
    for _ in range(warmup):
        fn()
    sync()
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        fn()
    e1.record(st)
    sync()
    return e0.elapsed_time(e1) / steps


def measure_extra(args, ws, rank, dev, sync, max_over_ranks):
    """Numbers added to the default line: the long-context configuration (sequence-parallel
    over the ranks at N > 1) fwd+bwd and forward only, and, at N = 1, this package on the
    shapes of the reference's own CUDA-kernel performance test."""
    out = {}
    w2 = CONFIGS[2]
    w = shard_workload(w2, ws)
    inp = make_inputs(w, seed=100 + rank, device=dev)
    step = step_seqpar if ws > 1 else step_api
    names = ("k", "q", "v", "lr", "decay", "beta", "gate")

    def leaves():
        d = {n: (inp[n].detach().requires_grad_(True) if inp[n] is not None else None) for n in names}
        d["dy"] = inp["dy"]
        return d

    steps = max(3, min(args.steps, 10))
    ms = max_over_ranks(timed_ms(lambda: step(inp, w, leaves()), steps, 3, dev, sync))
    with torch.no_grad():
        fms = max_over_ranks(timed_ms(lambda: step(inp, w, leaves(), backward=False), steps, 3, dev, sync))
    out["long_context"] = {"config": config_dict(w2, ws), "scaling": "strong", "steps": steps,
                           "ms_per_step": ms, "value": w2.B * w2.T / (ms / 1000.0), "unit": UNIT,
                           "forward_only": {"ms_per_step": fms, "value": w2.B * w2.T / (fms / 1000.0)}}
    del inp
    if ws == 1:
        rk = {}
        for wr in ref_kernel_workloads():
            x = make_inputs(wr, seed=0, device=dev, state_scale=0.1)

            def lv():
                d = {n: (x[n].detach().requires_grad_(True) if x[n] is not None else None) for n in names}
                d["dy"] = x["dy"]
                return d
            m = timed_ms(lambda: step_api(x, wr, lv()), 10, 3, dev, sync)
            rk[f"B{wr.B}_H{wr.H}_T{wr.T}"] = {"ms_per_step": m, "tokens_per_s": wr.B * wr.T / (m / 1000.0)}
        out["reference_kernel_shapes"] = {
            "what": "this package fwd+bwd (bf16, head 64, window 16, token gate, momentum) on the shapes of the "
                    "reference's CUDA-kernel performance test; the reference arm times its kernels on the same",
            "ours": rk}
    return out


def run_ours(args, w):
    import torch.distributed as dist
    from atlas_rnn_b200 import _lib
    from atlas_rnn_b200.roofline import kernel_bytes, kernel_flops, step_bytes_per_token, step_flops_per_token

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev)
    _lib.lib()
    # long-context configs with window 1 run sequence-parallel across the ranks (the ranks
    # share one sequence); the others are sharded by batch*head units (each rank runs
    # B/N of the batch). Both are strong scaling: the whole job is the configuration.
    seqpar = ws > 1 and w.window == 1 and w.gate == "none"
    w_full = w
    w = shard_workload(w, ws)
    step = step_seqpar if seqpar else step_api
    inp = make_inputs(w, seed=rank, device=dev)
    names = ("k", "q", "v", "lr", "decay", "beta", "gate")

    def leaves():
        d = {n: (inp[n].detach().requires_grad_(True) if inp[n] is not None else None) for n in names}
        d["dy"] = inp["dy"]
        return d

    def barrier():
        if ws > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    def max_over_ranks(x):
        if ws == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    # ---- device-resident timing (value) with per-kernel event timing
    for _ in range(args.warmup):
        step(inp, w, leaves())
    barrier()
    st = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    props = torch.cuda.get_device_properties(dev)
    my_id = ("GPU-" + str(props.uuid)) if getattr(props, "uuid", None) is not None else str(local)
    ids = [my_id]
    if ws > 1:
        gathered = [None] * ws
        dist.all_gather_object(gathered, my_id)
        ids = gathered
    # timed region: no per-kernel events inside (they would serialise consecutive kernels)
    launches0 = _lib.launch_count()
    with ClockSampler(ids, rank) as clk:
        barrier()
        clk.mark_start()
        ev0.record(st)
        h0 = time.perf_counter()
        for _ in range(args.steps):
            step(inp, w, leaves())
        host_ms = (time.perf_counter() - h0) * 1000.0 / args.steps  # enqueue time per step
        ev1.record(st)
        barrier()
        clk.mark_end()
    ms = ev0.elapsed_time(ev1)
    launches = _lib.launch_count() - launches0
    # per-kernel CUDA-event times from a separate profiled pass
    prof_steps = min(args.steps, 20)
    _lib.profile_enable(True)
    for _ in range(prof_steps):
        step(inp, w, leaves())
    torch.cuda.synchronize(dev)
    kern = _lib.profile_read()
    _lib.profile_enable(False)
    ms = max_over_ranks(ms)
    ms_step = ms / args.steps
    tokens_step = w.B * w.T  # this rank's tokens per step
    value = ws * tokens_step * args.steps / (ms / 1000.0)

    # ---- e2e through the public API with pinned host buffers
    host = {n: inp[n].cpu().pin_memory() for n in names + ("dy",) if inp[n] is not None}
    y_host = torch.empty((w.N, w.T, w.d_v), dtype=w.dtype).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = y_host.numel() * y_host.element_size()

    # pipelined as a deployment runs it: step i + 1's inputs copy in on a copy stream while step i
    # computes (two device buffers), and y goes back on a third stream; every step's copies are
    # inside the timed region
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    dbuf = [{n: torch.empty_like(host[n], device=dev) for n in host} for _ in range(2)]
    yh = [y_host, torch.empty_like(y_host).pin_memory()]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]
    ev_y = [torch.cuda.Event() for _ in range(2)]
    for e in ev_used:
        e.record(st)

    def issue_copy(i):
        j = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_used[j])  # the compute that read this buffer two steps ago is done
            for n in host:
                dbuf[j][n].copy_(host[n], non_blocking=True)
            ev_in[j].record(s_in)

    def e2e_run(n_steps):
        issue_copy(0)
        for i in range(n_steps):
            j = i % 2
            st.wait_event(ev_in[j])
            if i + 1 < n_steps:
                issue_copy(i + 1)
            d = {n: (dbuf[j][n].detach().requires_grad_(n in names) if n in host else None)
                 for n in names + ("dy",)}
            y = step(inp, w, d)
            ev_used[j].record(st)
            ev_y[j].record(st)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_y[j])
                yh[j].copy_(y.detach(), non_blocking=True)
                y.record_stream(s_out)
        st.wait_stream(s_out)

    e2e_run(max(2, args.warmup // 2))
    barrier()
    ev0.record(st)
    s_in.wait_event(ev0)  # the first copy is inside the timed region
    e2e_run(args.steps)
    ev1.record(st)
    barrier()
    e2e_ms = max_over_ranks(ev0.elapsed_time(ev1))
    e2e_value = ws * tokens_step * args.steps / (e2e_ms / 1000.0)

    # ---- forward only, inputs resident (timed separately, as the long-context config asks)
    with torch.no_grad():
        for _ in range(args.warmup):
            step(inp, w, leaves(), backward=False)
        barrier()
        ev0.record(st)
        for _ in range(args.steps):
            step(inp, w, leaves(), backward=False)
        ev1.record(st)
        barrier()
    fwd_ms = max_over_ranks(ev0.elapsed_time(ev1))
    fwd_value = ws * tokens_step * args.steps / (fwd_ms / 1000.0)

    # ---- roofline of the dominant kernel
    top = max(kern.items(), key=lambda kv: kv[1][0])
    top_name, (top_ms, top_n) = top[0], top[1]
    peaks = {}
    ppath = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(ppath):
        peaks = json.load(open(ppath))
    peak_tf = peaks.get("bf16_tflops", 1590.0)
    peak_bw = peaks.get("hbm_gbs", 6650.0)
    chunk = int(kernel_cfg_chunk(w))
    avg_ms = top_ms / max(top_n, 1)
    src = "MEASURED_PEAKS.json" if peaks else "fallback"
    Ff, Fb = step_flops_per_token(w)
    Bf, Bb = step_bytes_per_token(w)
    tok_heads = w.N * w.T
    # Algorithmic work per the benchmark's per-token-head counting (roofline.py): a kernel of
    # the backward pass is credited with the whole backward's bytes and flops, a forward
    # kernel with the forward's -- an upper bound on what that one kernel has to move. The
    # stand-alone feature-map kernels are credited with their own GEMM (x and phi rows).
    is_bwd = top_name.startswith("k_bwd") or top_name == "k_fmap_bwd_tc"
    if top_name in ("k_fmap_fwd_tc", "k_fmap_bwd_tc"):
        alg_flops = kernel_flops(top_name, w, chunk)
        alg_bytes = 2.0 * w.N * w.T * (w.d_k + w.d_phi)
        basis = "the feature-map GEMM of one of k / q: [x; vec(x x^T)] Proj over every token"
    else:
        alg_flops = (Fb if is_bwd else Ff) * tok_heads
        alg_bytes = (Bb if is_bwd else Bf) * tok_heads
        basis = ("the whole " + ("backward" if is_bwd else "forward") + " pass's algorithmic bytes / flops "
                 "(per token-head counting of the benchmark config) over this one kernel's launch time")
    t_hbm = alg_bytes / (peak_bw * 1e9)
    t_tc = alg_flops / (peak_tf * 1e12)
    tflops = alg_flops / (avg_ms / 1000.0) / 1e12
    gbs = alg_bytes / (avg_ms / 1000.0) / 1e9
    traffic = traffic_from_profiles(top_name, w.name)
    try:
        dec_bytes = kernel_bytes(top_name, w, chunk)
    except KeyError:
        dec_bytes = None
    if t_hbm >= t_tc:
        roofline = {"kernel": top_name, "bound": "hbm", "achieved": gbs, "peak": peak_bw, "unit": "GB/s",
                    "frac": gbs / peak_bw, "peak_source": f"{src} hbm_gbs (burst copy)", "traffic": traffic,
                    "algorithmic_bytes_per_launch": alg_bytes, "tensor_tflops": tflops,
                    "tensor_frac": tflops / peak_tf}
    else:
        roofline = {"kernel": top_name, "bound": "tensor", "achieved": tflops, "peak": peak_tf, "unit": "TFLOP/s",
                    "frac": tflops / peak_tf, "peak_source": f"{src} bf16_tflops (burst)", "traffic": traffic,
                    "algorithmic_bytes_per_launch": alg_bytes, "hbm_gbs": gbs}
    roofline.update({"basis": basis, "launch_ms": avg_ms, "algorithmic_flops_per_launch": alg_flops,
                     "kernel_share": top_ms / sum(v[0] for v in kern.values()),
                     "decomposition_bytes_per_launch": dec_bytes,
                     "decomposition_gbs": (dec_bytes / (avg_ms / 1000.0) / 1e9) if dec_bytes else None})
    step_roof_ms = max((Ff + Fb) * tok_heads / (peak_tf * 1e12),
                       (Bf + Bb) * tok_heads / (peaks.get("hbm_gbs", 6650.0) * 1e9)) * 1000.0
    clocks = clk.summary()
    extra = measure_extra(args, ws, rank, dev, barrier, max_over_ranks) if args.config == 1 and not args.no_extra \
        else {}

    if rank == 0:
        cpu = None
        if ws == 1 and not args.no_cpu_baseline:
            v, per, reps, sample = cpu_sample(w, min_seconds=args.cpu_seconds)
            cpu = {"value": v, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port", "sample": sample}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16" if w.dtype == torch.bfloat16 else "f32",
            "data": "synthetic (seeded, benchmark-config distributions)",
            "config": config_dict(w_full, ws),
            "per_rank": {"units": w.N, "tokens": w.T, "batch": w.B},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "forward_only": {"value": fwd_value, "unit": UNIT, "ms_per_step": fwd_ms / args.steps},
            "gpu_launches": launches,
            "host_enqueue_ms_per_step": host_ms,
            "roofline": roofline,
            "step_roofline_ms": step_roof_ms,
            "step_roofline_frac": step_roof_ms / ms_step,
            "kernels_ms_per_step": {k: v[0] / prof_steps for k, v in kern.items() if v[1]},
            "clocks": clocks,
            "cpu_baseline": cpu,
            **extra,
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def shard_workload(w, ws):
    """This rank's part of the configuration at world size ws: a T / ws token slice of
    the long-context (window 1, no gate) configurations, else B / ws of the batch
    (batch*head units are independent; H / ws when B does not divide)."""
    if ws == 1:
        return w
    if w.window == 1 and w.gate == "none":
        assert w.T % ws == 0
        return shrink(w, T=w.T // ws)
    if w.B % ws == 0:
        return shrink(w, B=w.B // ws)
    assert w.H % ws == 0, "batch*head units do not divide over the ranks"
    return shrink(w, H=w.H // ws)


def config_dict(w, ws):
    """The workload description both arms print (same keys and values)."""
    seqpar = w.window == 1 and w.gate == "none"
    tok_heads = w.N * w.T
    return {"workload": w.name, "B": w.B, "H": w.H, "T": w.T, "d_k": w.d_k, "d_phi": w.d_phi, "d_v": w.d_v,
            "window": w.window, "gate": w.gate, "fmap": f"{w.fmap_mode}:{w.fmap_degree}", "momentum": w.momentum,
            "parallelism": ("single GPU" if ws == 1 else
                            f"sequence-parallel x{ws} (T/{ws} per rank, NCCL carry exchange)" if seqpar
                            else f"batch*head sharded x{ws}"),
            "l2": ("inputs exceed L2 (no flush needed)" if tok_heads * (2 * w.d_k + w.d_v) * w.dtype.itemsize > 126e6
                   else "inputs fit L2")}


def kernel_cfg_chunk(w):
    """Tokens per chunk the library picks for this workload (its default rule)."""
    from atlas_rnn_b200.roofline import tc_chunk
    tensor_cores = w.dtype == torch.bfloat16 and w.d_phi == 128 and w.d_v == 128 and w.window <= 16
    if tensor_cores and os.environ.get("ATLAS_MEM_TC", "1") != "0":
        return tc_chunk(w)
    return 32 if w.window - 1 <= 32 else w.window - 1


def run_reference_cuda(args, w):
    """The reference's own Omega-16 CUDA kernels (atlas_pytorch/cuda, built from its sources into
    oracle/_ref by oracle/ref_cuda.py) on the workload they support, fwd+bwd as the reference's
    autograd wrapper runs them; rank 0 only. Also reports how far their y is from ours."""
    ws, rank, local = dist_env()
    if rank != 0:
        return
    if not (w.window == 16 and w.d_k == w.d_phi == w.d_v == 64 and w.gate == "token" and w.fmap_mode == "off"
            and w.dtype == torch.bfloat16 and w.momentum):
        print(json.dumps({"impl": "reference-cuda", "unavailable": "the reference's CUDA kernels run only "
                          "window 16, head 64, bf16, per-token gate, momentum (use --config 5)"}))
        return
    from oracle import ref_cuda
    try:
        ext = ref_cuda.load()
    except Exception as ex:  # not built here
        print(json.dumps({"impl": "reference-cuda", "unavailable": str(ex)}))
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    inp = make_inputs(w, seed=0, device=dev, state_scale=0.1)
    b16 = lambda t: t.to(torch.bfloat16).contiguous()
    args_ref = [b16(inp[n]) for n in ("k", "q", "v")] + [b16(inp["S0"])] + \
        [b16(inp[n]) for n in ("lr", "decay", "beta", "gate")] + [b16(inp["S0"]), b16(inp["Z0"]), b16(inp["dy"])]
    for _ in range(args.warmup):
        ref_cuda.forward_backward(ext, *args_ref)
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        (y_ref, _, _), _ = ref_cuda.forward_backward(ext, *args_ref)
    ev1.record()
    torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1) / args.steps
    from atlas_rnn_b200 import memory_recurrence
    with torch.no_grad():
        y_ours = memory_recurrence(inp["k"], inp["q"], inp["v"], inp["lr"], inp["decay"], inp["beta"], inp["gate"],
                                   S_ref=inp["S0"], S0=inp["S0"], Z0=inp["Z0"], window=16, gate_mode="token")[0]
    diff = ((y_ref.float() - y_ours.float()).norm() / y_ours.float().norm()).item()
    print(json.dumps({"impl": "reference-cuda", "metric": METRIC, "value": w.B * w.T / (ms / 1000.0), "unit": UNIT,
                      "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                      "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
                      "config": {"workload": w.name, "B": w.B, "H": w.H, "T": w.T, "d": 64, "window": 16},
                      "kernels": "reference atlas_omega.cu forward_exact_kernel + backward_exact_kernel (sm_100a)",
                      "y_rel_l2_vs_ours": diff}), flush=True)


LM_C3 = dict(num_tokens=256, dim=768, depth=12, block_type="lmm", heads=12, dim_head=64, ff_mult=4,
             omega_window=8, use_omega_gate=True, use_momentum=True, poly_mode="elementwise", poly_degree=2,
             qkv_conv_kernel=4)
LM_C3_BATCH, LM_C3_SEQ = 16, 8192


def run_lm(args):
    """Config 3: one training step (next-token loss, backward, AdamW) of the 12-layer LMM
    language model (RNNMemoryTransformer, block_type 'lmm'; SwiGLU hidden 2048) on synthetic
    byte tokens under bf16 autocast, random-init weights. N > 1: the global batch is split
    over the ranks (data parallel, gradients all-reduced by DistributedDataParallel)."""
    import torch.distributed as dist
    from atlas_rnn_b200 import RNNMemoryTransformer, _lib

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev)
    B = (args.B or LM_C3_BATCH) // ws
    T = args.T or LM_C3_SEQ
    torch.manual_seed(0)
    model = RNNMemoryTransformer(**LM_C3).to(dev)
    with torch.no_grad():  # N(0, 0.02) weights as the benchmark config states
        for name, p in model.named_parameters():
            if p.dim() > 1:
                p.normal_(0.0, 0.02)
    net = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local]) if ws > 1 else model
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, fused=True)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    tokens = torch.randint(0, 256, (B, T + 1), device=dev, generator=g)
    host_tokens = tokens.cpu().pin_memory()
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()

    def step(tok):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = net(tok, return_loss=True)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()
        return loss

    def barrier():
        if ws > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step(tokens)
    barrier()
    st = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    props = torch.cuda.get_device_properties(dev)
    ids = [("GPU-" + str(props.uuid)) if getattr(props, "uuid", None) is not None else str(local)]
    if ws > 1:
        gathered = [None] * ws
        dist.all_gather_object(gathered, ids[0])
        ids = gathered
    launches0 = _lib.launch_count()
    with ClockSampler(ids, rank) as clk:
        barrier()
        clk.mark_start()
        ev0.record(st)
        for _ in range(args.steps):
            step(tokens)
        ev1.record(st)
        barrier()
        clk.mark_end()
    ms = ev0.elapsed_time(ev1)
    launches = _lib.launch_count() - launches0
    # end to end: tokens from pinned host memory, loss back to the host, every step
    barrier()
    ev0.record(st)
    tok_dev = torch.empty_like(tokens)  # one preallocated device buffer: no allocation inside the region
    for _ in range(args.steps):
        tok_dev.copy_(host_tokens, non_blocking=True)
        loss = step(tok_dev)
        loss_host.copy_(loss.detach().float(), non_blocking=True)
    ev1.record(st)
    barrier()
    e2e_ms = ev0.elapsed_time(ev1)
    if ws > 1:
        t = torch.tensor([ms, e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = t.tolist()
    tok = ws * B * T * args.steps
    if args.torch_profile and rank == 0:  # per-kernel table of one more step (after the timed ones)
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step(tokens)
            torch.cuda.synchronize(dev)
        print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=30, max_name_column_width=70),
              file=sys.stderr, flush=True)
    if rank == 0:
        line = {
            "metric": "LM training tokens/sec", "value": tok / (ms / 1000.0), "unit": UNIT, "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic byte tokens (uniform 0..255), random-init N(0, 0.02) weights",
            "config": {"workload": "lmm_lm_c3", "global_batch": B * ws, "seq_len": T, **LM_C3,
                       "parallelism": f"data-parallel x{ws}", "l2": "activations exceed L2"},
            "e2e": {"value": tok / (e2e_ms / 1000.0), "unit": UNIT,
                    "h2d_bytes_per_step": host_tokens.numel() * host_tokens.element_size(), "d2h_bytes_per_step": 4},
            "gpu_launches": launches, "loss": float(loss_host), "clocks": clk.summary(),
            "peak_mem_gb": torch.cuda.max_memory_allocated(dev) / 1e9,
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", type=int, default=1)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-cuda"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the long-context and reference-kernel-shape numbers of the default line")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--T", type=int, default=None, help="override tokens (for profiling small cases)")
    ap.add_argument("--B", type=int, default=None)
    ap.add_argument("--with-buffer", action="store_true", help="pass the zero omega buffer explicitly")
    ap.add_argument("--torch-profile", action="store_true",
                    help="config 3: print torch.profiler's per-kernel table of one extra step to stderr")
    args = ap.parse_args()
    global WITH_BUFFER
    WITH_BUFFER = args.with_buffer
    if args.config == 3:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference LM runs its memory cells in "
                              "materialised [B,H,T,d,d] torch einsums; config 3 does not fit one GPU that way"}))
            return
        run_lm(args)
        return
    w = CONFIGS[args.config]
    if args.T or args.B:
        w = shrink(w, B=args.B, T=args.T)
    if args.impl == "reference-cuda":
        run_reference_cuda(args, w)
    elif args.impl == "reference":
        run_reference(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()
