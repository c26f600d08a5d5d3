"""Benchmark: encoder-policy forward states/s on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--impl ours|reference]

A step is one policy forward over one batch of B synthetic states (config 2
by default: B=1024 states x N=64 entities x F=32, d=256, 8 heads, FFN 1024,
4 blocks, P=16, bf16 tensor-core path). Under torchrun each rank is one GPU
with its own B states (weak scaling); rank 0 builds the seeded weights and
broadcasts them once over NCCL.

  value  states/s with inputs resident in HBM; per-step CUDA events on the
         launching stream; L2 flushed (256 MiB write) between timed steps;
         whole-job aggregate = world * B * K / max-over-ranks time.
  e2e    the same through the host-buffer API (ow_policy_forward with pinned
         host buffers: H2D of features/counts, D2H of logits/value/actions
         inside every step), wall clock per call, max over ranks.
  roofline  the dominant kernel (largest share of device time, from CUDA
         events the library records around each launch in the timed region).
  cpu_baseline  the CPU oracle (fp32, OpenMP, all host threads) on a bounded
         sample of the same workload, rank 0 at N=1 only.
  weight_broadcast  (N > 1) the library's NCCL broadcast of rank 0's packed
         device weights into every other rank's handle: bytes, device ms, GB/s.
  config5  the same measurement, nested, for config 5 (65,536 states per GPU,
         d=512, 8 blocks): the scale-out workload, so the 1/2/4/8-GPU runs of
         this command trace its scaling and its weight broadcast too.
  true2d  (N = 1) the reference ABI drop-in (True2D self-play forward): device
         and e2e requests/s, the reference's own CUDA build on the same call,
         the MUFU roofline against the measured MUFU rate, the CPU reference.

--impl reference times the reference-side CPU implementation of this path.
The reference repository has no implementation of this network, so that arm
is the repository's CPU port of the spec (oracle, fp32, every host core, the
whole configured batch per step when the run fits its CPU budget).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
PKG = REPO / "orbit-wars-2d-transformer_b200"
for _p in (str(REPO), str(PKG)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "policy-forward states/sec (config {c})"
UNIT = "states/s"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_FLUSH_BYTES = 256 << 20
REFERENCE_RUN_S = 150.0  # CPU time budget of one --impl reference run


def ncu_traffic(config, kernel: str):
    """DRAM bytes per launch of `kernel` from the committed ncu capture of this
    config (profiles/ncu_traffic_c<config>.json, or ncu_traffic_true2d.json for
    config "true2d"), or None."""
    p = REPO / "profiles" / (f"ncu_traffic_c{config}.json" if config != "true2d" else "ncu_traffic_true2d.json")
    if not p.exists():
        return None, None
    d = json.loads(p.read_text())
    k = d.get("kernels", {}).get(kernel)
    return (k["dram_bytes_per_launch"] if k else None), d.get("workload")


def load_peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return dict(PEAKS_FALLBACK), "fallback"


def workload_name(cfg) -> str:
    return (f"{cfg.name}: B={cfg.batch} states x N={cfg.n_entities} entities x F={cfg.features}, d={cfg.d_model}, "
            f"h={cfg.heads}, f={cfg.ffn}, L={cfg.layers}, P={cfg.actions}, counts U[{cfg.count_lo},{cfg.count_hi}]"
            f"{', Gumbel-max actions' if cfg.sample_actions else ''}")


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None
        self.window = None  # (t0, t1) wall-clock bounds of the loaded region

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(1.0)  # let nvidia-smi start sampling before the load begins
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.3)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        if self.path is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        from datetime import datetime
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                clk = float(parts[2])
                smax = float(parts[3])
            except ValueError:
                continue
            if self.window is not None and not (self.window[0] - 0.25 <= ts <= self.window[1] + 0.25):
                continue
            sm.append(clk)
            for n, v in zip(names, parts[6:10]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax, "samples": len(sm),
                "reasons": sorted(reasons)}


def kernel_work(cfg, name: str, m_valid: int, sq_counts: int, batch: int) -> tuple[float, float]:
    """(algorithmic FLOPs, algorithmic HBM bytes) of one launch: every activation
    read and written once, weights counted once (they stay in L2)."""
    d, f, F, P, N, L = cfg.d_model, cfg.ffn, cfg.features, cfg.actions, cfg.n_entities, cfg.layers
    act = 4 if cfg.precision == "f32" else 2          # bf16 activations (f32 on the fp32 path)
    a8 = 1 if cfg.precision == "fp8" else act         # GEMM A operands (e4m3 on the fp8 path)
    ln_out = (act * (L - 1) + 4) / L                  # LN output of the block's last GEMM: f32 after the last layer
    wb = 1 if cfg.precision == "fp8" else act
    xb = 2 if (cfg.precision != "f32" and d == 256) else 4  # the residual stream: bf16 at d = 256, else f32
    M = float(m_valid)
    if name in ("gemm_qkv", "gemm_f32_qkv"):
        return 2.0 * M * 3 * d * d, M * (d * a8 + 3 * d * act) + 3 * d * d * wb
    if name in ("gemm_out_resid_ln", "gemm_f32_out_resid"):
        return 2.0 * M * d * d, M * (d * a8 + 2 * xb * d + d * a8) + d * d * wb
    if name in ("gemm_ffn_up_gelu", "gemm_f32_ffn_up"):
        return 2.0 * M * f * d, M * (d * a8 + f * act) + f * d * wb
    if name in ("gemm_ffn_down_resid_ln", "gemm_f32_ffn_down_resid"):
        return 2.0 * M * d * f, M * (f * a8 + 2 * xb * d + d * ln_out) + d * f * wb
    if name == "ffn_fused":
        return 4.0 * M * d * f, M * (d * a8 + 8 * d + d * ln_out) + 2 * d * f * wb
    if name == "attention":
        return 4.0 * sq_counts * d, M * (3 * d * act + d * act)
    if name == "embed_ln":
        return 2.0 * M * F * d, M * (F * 4 + xb * d + d * a8)
    if name == "heads":
        lb = 4 if cfg.logits_dtype == "f32" else 2
        return 2.0 * M * d * (P + 1), M * (4 * d + 4) + batch * N * (P * lb + 4)
    if name == "layernorm_f32":
        return 0.0, M * d * 8.0
    if name == "quantize_e4m3":
        return 0.0, M * (f + d) / 2 * 3.0
    if name == "scan_counts":
        return 0.0, batch * 8.0
    if name == "state_finalize":
        return 0.0, M * 4.0 + batch * 4.0
    return 0.0, 0.0


def measure_fp8_tflops(dev) -> float | None:
    """Dense e4m3 tensor-core rate of this GPU: torch._scaled_mm (cuBLASLt) on
    8192^3 with bf16 output, best of 10 CUDA-event runs. The fp8 path's roofline
    uses this instead of assuming twice the measured bf16 rate; None when the
    library call is unavailable."""
    import torch
    n = 8192
    try:
        a = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
        b = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn).t()  # column-major B
        one = torch.ones((), device=dev, dtype=torch.float32)
        for _ in range(3):
            torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        best = float("inf")
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1) / 1000.0)
        del a, b
        torch.cuda.empty_cache()
        return 2.0 * n ** 3 / best / 1e12
    except Exception:  # noqa: BLE001 - the fallback is stated in the JSON line
        return None


def gemm_summary(cfg, kernels: dict, m_valid: int, sq_counts: int, batch: int, tc_peak,
                 tc_peak_sustained=None) -> dict | None:
    """The block GEMMs together (QKV, out-projection, FFN up and down): their
    FLOPs over their summed device time, against the measured bf16 peak (burst)
    and, beside it, the measured sustained rate under the power cap (the
    kernels run inside seconds of back-to-back steps)."""
    names = [n for n in kernels if n.startswith("gemm_") or n == "ffn_fused"]
    if not names or not tc_peak:
        return None
    flops = sum(kernel_work(cfg, n, m_valid, sq_counts, batch)[0] * kernels[n]["launches"] for n in names)
    secs = sum(kernels[n]["total_ms"] for n in names) / 1000.0
    t = flops / secs / 1e12
    res = {"kernels": names, "tflops": round(t, 1), "frac_of_peak": round(t / tc_peak, 4),
           "note": "FLOPs 2*M_valid*N*K of the four block GEMMs / their CUDA-event time; per-kernel bounds in kernels"}
    if tc_peak_sustained:
        res["frac_of_sustained_peak"] = round(t / tc_peak_sustained, 4)
    return res


def host_threads() -> int:
    """Every host core this process may run on (torchrun sets OMP_NUM_THREADS=1 for its ranks, so the
    oracle's OpenMP default would be one thread: pass the count explicitly)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline(cfg, weights, feats, counts, target_s: float = 12.0) -> dict:
    """Times the fp32 CPU oracle (OpenMP, all host threads) on a bounded sample of the workload."""
    from oracle import bind
    threads = host_threads()
    n = max(1, min(4, cfg.batch))
    bind.policy_forward(cfg, weights, feats[:n], counts[:n], f64=False, threads=threads)  # warm
    while True:
        t0 = time.perf_counter()
        bind.policy_forward(cfg, weights, feats[:n], counts[:n], f64=False, threads=threads)
        dt = time.perf_counter() - t0
        if dt >= target_s or n >= cfg.batch:
            break
        grow = max(2, int(target_s / max(dt, 1e-3)))
        n = min(cfg.batch, n * grow)
    return {"value": n / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{n} of the {cfg.batch} states of the workload, fp32 CPU oracle (valid rows only), "
                      f"{threads} threads, {dt:.1f} s"}


def run_reference(args, cfg) -> None:
    """The reference-side CPU arm: the fp32 CPU port of the spec on every host core, rank 0 only. Each step
    is the whole configured batch when warm-up + timed steps fit REFERENCE_RUN_S of CPU work (so the arm
    runs the same workload as ours), else a bounded sample of it."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import orbit_wars_b200 as ow
    from oracle import bind
    weights = ow.make_weights(cfg, seed=args.seed)
    feats, counts = ow.make_inputs(cfg, seed=args.seed)
    threads = host_threads()
    n = min(cfg.batch, 16)
    bind.policy_forward(cfg, weights, feats[:n], counts[:n], f64=False, threads=threads)  # warm
    t0 = time.perf_counter()
    bind.policy_forward(cfg, weights, feats[:n], counts[:n], f64=False, threads=threads)
    per_state = (time.perf_counter() - t0) / n
    step_s = REFERENCE_RUN_S / (args.steps + args.warmup)
    n = int(max(1, min(cfg.batch, step_s / max(per_state, 1e-6))))
    for i in range(args.warmup):
        bind.policy_forward(cfg, weights, feats[:n], counts[:n], f64=False, threads=threads)
    times = []
    for i in range(args.steps):
        s = (i * n) % max(1, cfg.batch - n + 1)
        t0 = time.perf_counter()
        bind.policy_forward(cfg, weights, feats[s:s + n], counts[s:s + n], f64=False, threads=threads)
        times.append(time.perf_counter() - t0)
    total = float(np.sum(times))
    value = n * args.steps / total
    sample = (f"{n} states per step (of the {cfg.batch}-state workload), fp32 CPU port of the spec (valid rows "
              f"only), {threads} threads; the reference repository has no implementation of this network")
    line = {
        "impl": "reference", "metric": METRIC.format(c=args.config), "value": value, "unit": UNIT,
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * total / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded SplitMix/Box-Muller features, Xavier-uniform weights)",
        "config": {"workload": workload_name(cfg), "states_per_step": n, "same_config": n == cfg.batch},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


class Ctx:
    """This process's place in the run: rank, device, stream and (N > 1) the library's NCCL communicator."""

    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.comm = None
        self.nccl_log = None
        self.dev = None
        self.stream = None

    def start(self):
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            from datetime import timedelta
            # NCCL's init lines (rank counts of every communicator, torch's and the library's) go to a
            # per-process file and are echoed to stderr at the end: stdout carries one JSON line only
            self.nccl_log = Path(tempfile.gettempdir()) / f"ow_nccl_{os.getpid()}.log"
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
            os.environ["NCCL_DEBUG_FILE"] = str(self.nccl_log)
            dist.init_process_group("nccl", device_id=self.dev, timeout=timedelta(seconds=120))
            # the weight broadcast's communicator: its 128-byte id travels over torch.distributed
            from orbit_wars_b200.policy import Comm
            from orbit_wars_b200.shard import share_comm_id
            uid = share_comm_id(self.rank, Comm.unique_id() if self.rank == 0 else None)
            self.comm = Comm(uid, self.world, self.rank, self.local)
        # one non-default stream carries the library's kernels, torch's copies/flushes and the timing events
        self.stream = torch.cuda.Stream(self.dev)
        torch.cuda.set_stream(self.stream)
        return self

    def barrier(self):
        import torch.distributed as dist
        if self.world > 1:
            dist.barrier()

    def max_over_ranks(self, vals):
        import torch
        import torch.distributed as dist
        t = torch.tensor(vals, dtype=torch.float64, device=self.dev)
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(v) for v in t.tolist()]

    def finish(self):
        import torch.distributed as dist
        if self.world > 1:
            dist.barrier()
            if self.comm is not None:
                self.comm.close()
            dist.destroy_process_group()
            if self.nccl_log is not None and self.nccl_log.exists():
                keep = [ln for ln in self.nccl_log.read_text(errors="replace").splitlines()
                        if "Init COMPLETE" in ln or "nranks" in ln.lower()]
                for ln in keep[:16]:
                    print(ln, file=sys.stderr)
                self.nccl_log.unlink()


def policy_handle(cfg, weights, ctx, io: str, bcast: bool):
    """A handle on this rank's GPU. Rank 0 converts the seeded f32 blob; every other rank starts with no
    weights and receives rank 0's packed device arena over NCCL (the library's ncclBroadcast). Returns the
    handle and, for N > 1 with bcast, the broadcast timing (one warm-up, then three timed broadcasts)."""
    import orbit_wars_b200 as ow
    pol = ow.EncoderPolicy(cfg, weights if ctx.rank == 0 else None, device=ctx.local,
                           stream=ctx.stream.cuda_stream, io=io)
    if ctx.world == 1:
        return pol, None
    pol.broadcast_from(ctx.comm, root=0)
    if not bcast:
        return pol, None
    ms = [pol.broadcast_from(ctx.comm, root=0) for _ in range(3)]
    _, nbytes = pol.device_weights()
    worst = ctx.max_over_ranks([float(np.mean(ms))])[0]
    return pol, {"bytes": int(nbytes), "ms": round(worst, 4), "gbs": round(nbytes / (worst * 1e-3) / 1e9, 1),
                 "nranks": ctx.world, "timing": "device time of one ncclBroadcast of the packed weight arena "
                                                "(ow_policy_broadcast_weights_comm), mean of 3 after a warm-up, "
                                                "max over ranks; in-switch reduction not involved (broadcast)",
                 "what": "rank 0's converted bf16/e4m3 weights + scales + f32 vectors, as the kernels read them"}


def measure_policy(args, cfg, ctx, steps: int, warmup: int, e2e_steps: int, with_cpu: bool,
                   cpu_target_s: float = 12.0) -> dict:
    """One workload: device-resident throughput with per-kernel events, the roofline of the dominant
    kernel, e2e through the host-buffer API, the weight broadcast (N > 1), and the CPU baseline."""
    import torch

    import orbit_wars_b200 as ow
    from orbit_wars_b200.shard import shard_inputs

    dev, stream = ctx.dev, ctx.stream
    weights = ow.make_weights(cfg, seed=args.seed) if ctx.rank == 0 else None
    # this rank's shard of the global batch (world * B states)
    feats, counts = shard_inputs(cfg, args.seed, ctx.rank)
    B = cfg.batch
    m_valid = int(counts.sum())
    sq_counts = int((counts.astype(np.int64) ** 2).sum())

    pol, bcast = policy_handle(cfg, weights, ctx, "device", bcast=True)
    f_d = torch.from_numpy(feats).to(dev)
    c_d = torch.from_numpy(counts).to(dev)
    ldt = torch.bfloat16 if cfg.logits_dtype == "bf16" else torch.float32
    vdt = torch.bfloat16 if cfg.value_dtype == "bf16" else torch.float32
    lg = torch.empty((B, cfg.n_entities, cfg.actions), dtype=ldt, device=dev)
    vv = torch.empty((B,), dtype=vdt, device=dev)
    aa = torch.empty((B, cfg.n_entities), dtype=torch.int32, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def step(i):
        pol.forward_device(f_d.data_ptr(), c_d.data_ptr(), B, lg.data_ptr(), vv.data_ptr(), aa.data_ptr(), seed=i)

    for i in range(warmup):
        flush.zero_()
        step(i)
    pol.synchronize()
    ctx.barrier()
    torch.cuda.synchronize(dev)

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    # per-kernel events on the first timed steps only: an event between two
    # kernels stops the next one from starting early (programmatic dependent
    # launch), so profiled steps run slightly slower than the rest
    prof_steps = min(steps, 20)
    pol.profile_begin(prof_steps)
    with ClockSampler(ctx.local) as clk:
        clk.window = (time.time(), None)
        for i in range(steps):
            flush.zero_()  # L2 flush outside the step's events
            starts[i].record(stream)
            step(warmup + i)
            ends[i].record(stream)
        torch.cuda.synchronize(dev)
        clk.window = (clk.window[0], time.time())
    prof = pol.profile_end()
    pol.synchronize()
    ctx.barrier()
    torch.cuda.synchronize(dev)
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    t_max = ctx.max_over_ranks([float(np.sum(step_ms)) / 1000.0])[0]
    value = ctx.world * B * steps / t_max
    launches = pol.launches_per_forward() * steps
    out_ok = bool(torch.isfinite(lg.float()).all().item() and torch.isfinite(vv.float()).all().item())
    # the device-IO handle's workspace goes before the host-IO handle allocates its own
    # (config 5's activations take about 112 GB per workspace)
    pol.close()
    del f_d, c_d, lg, vv, aa, flush
    torch.cuda.empty_cache()

    # e2e through the host-buffer API (pinned host buffers): the pipelined
    # submit / wait pair, two submissions in flight so one step's upload and
    # download overlap the previous step's forward; every step uploads its
    # features + counts and downloads logits, value and actions
    e2e = None
    if e2e_steps > 0:
        hp, _ = policy_handle(cfg, weights, ctx, "host", bcast=False)
        f_h = torch.from_numpy(feats).pin_memory()
        c_h = torch.from_numpy(counts).pin_memory()
        outs = [(torch.empty((B, cfg.n_entities, cfg.actions), dtype=ldt).pin_memory(),
                 torch.empty((B,), dtype=vdt).pin_memory(),
                 torch.empty((B, cfg.n_entities), dtype=torch.int32).pin_memory()) for _ in range(2)]

        def submit(i):
            lg_h, vv_h, aa_h = outs[i % 2]
            return hp.submit_raw(f_h.data_ptr(), c_h.data_ptr(), B, lg_h.data_ptr(), vv_h.data_ptr(),
                                 aa_h.data_ptr(), seed=i)

        for i in range(warmup):
            hp.wait(submit(i))
        torch.cuda.synchronize(dev)
        ctx.barrier()
        t0 = time.perf_counter()
        prev = None
        for i in range(e2e_steps):
            t = submit(i)
            if prev is not None:
                hp.wait(prev)
            prev = t
        hp.wait(prev)
        t_pipe = time.perf_counter() - t0
        # the same calls one at a time (ow_policy_forward: submit + wait)
        n_sync = min(e2e_steps, 50)
        t0 = time.perf_counter()
        for i in range(n_sync):
            hp.wait(submit(i))
        t_sync = (time.perf_counter() - t0) / n_sync
        t_pipe, t_sync = ctx.max_over_ranks([t_pipe, t_sync])
        lg_h, vv_h, aa_h = outs[0]
        h2d = feats.nbytes + counts.nbytes
        d2h = lg_h.numel() * lg_h.element_size() + vv_h.numel() * vv_h.element_size() + aa_h.numel() * 4
        e2e = {"value": ctx.world * B * e2e_steps / t_pipe, "unit": UNIT, "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h), "steps": e2e_steps,
               "timing": "wall clock over the steps, ow_policy_submit / ow_policy_wait with two submissions in "
                         "flight (pinned host buffers), max over ranks; no L2 flush (each step's working set "
                         "exceeds the 126 MB L2)",
               "synchronous_value": ctx.world * B / t_sync,
               "synchronous_timing": "ow_policy_forward-equivalent submit + wait per step, one at a time"}
        hp.close()
        del f_h, c_h, outs
        torch.cuda.empty_cache()

    # roofline of the dominant kernel: the bound whose roofline time is longer
    # (algorithmic bytes / measured HBM copy rate vs FLOPs / measured bf16 peak)
    peaks, peak_src = load_peaks()
    hbm_peak = float(peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    bf16_peak = float(peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"]))
    tc_peak, fp8_src = bf16_peak, ""
    if cfg.precision == "fp8":
        fp8 = measure_fp8_tflops(ctx.dev)
        if fp8:
            tc_peak, fp8_src = fp8, " (fp8 peak measured here: torch._scaled_mm e4m3 8192^3, best of 10)"
        else:
            tc_peak, fp8_src = 2.0 * bf16_peak, " (fp8 peak = 2x measured bf16: the fp8 GEMM measurement failed)"
    if cfg.precision == "f32":
        tc_peak = None  # the fp32 path runs on CUDA cores
    kernels = {}
    for name, (n_launch, total_ms) in prof.items():  # from the first `prof_steps` timed steps
        flops, nbytes = kernel_work(cfg, name, m_valid, sq_counts, B)
        avg_s = total_ms / 1000.0 / max(n_launch, 1)
        gbs = nbytes / avg_s / 1e9 if avg_s > 0 else 0.0
        tfs = flops / avg_s / 1e12 if avg_s > 0 else 0.0
        t_hbm = nbytes / (hbm_peak * 1e9)
        t_tc = flops / (tc_peak * 1e12) if tc_peak else 0.0
        bound = "tensor" if t_tc > t_hbm else "hbm"
        kernels[name] = {"launches": n_launch, "total_ms": round(total_ms, 4), "avg_us": round(avg_s * 1e6, 2),
                         "bound": bound, "achieved": round(tfs if bound == "tensor" else gbs, 2),
                         "unit": "TFLOP/s" if bound == "tensor" else "GB/s",
                         "tflops": round(tfs, 1), "tensor_frac": round(tfs / tc_peak, 4) if tc_peak else None,
                         "gbs": round(gbs, 1), "hbm_frac": round(gbs / hbm_peak, 4),
                         "roofline_frac": round(max(t_hbm, t_tc) / avg_s, 4) if avg_s > 0 else None}
    total = sum(k["total_ms"] for k in kernels.values()) or 1.0
    for k in kernels.values():
        k["share"] = round(k["total_ms"] / total, 4)
    dom_name = max(kernels, key=lambda k: kernels[k]["total_ms"]) if kernels else None
    roof = None
    if dom_name is not None:
        k = kernels[dom_name]
        peak = tc_peak if k["bound"] == "tensor" else hbm_peak
        traffic, traffic_src = ncu_traffic(int(cfg.name[1]), dom_name)
        roof = {"kernel": dom_name, "bound": k["bound"], "achieved": k["achieved"], "peak": peak, "unit": k["unit"],
                "frac": round(k["achieved"] / peak, 4), "traffic": traffic, "traffic_source": traffic_src,
                "peak_source": peak_src + fp8_src,
                "tensor_frac": k["tensor_frac"], "hbm_frac": k["hbm_frac"],
                "work_per_launch": "algorithmic bytes = every activation read and written once (weights once); "
                                   "FLOPs = 2*M_valid*N*K, M_valid = valid tokens of the batch",
                "timed_steps_profiled": prof_steps}

    cpu = None
    if with_cpu and ctx.rank == 0 and ctx.world == 1:
        cpu = cpu_baseline(cfg, weights, feats, counts, target_s=cpu_target_s)
    tc_sus = (float(peaks.get("bf16_tflops_sustained", PEAKS_FALLBACK["bf16_tflops_sustained"]))
              * tc_peak / bf16_peak) if tc_peak else None
    return {
        "value": value, "ms_per_step": 1000.0 * t_max / steps, "steps": steps, "warmup": warmup,
        "dtype": {"f32": "f32", "bf16": "bf16", "fp8": "e4m3"}[cfg.precision],
        "config": {"workload": workload_name(cfg), "per_gpu_batch": B, "global_batch": B * ctx.world,
                   "valid_tokens_per_gpu": m_valid, "l2": "flushed between timed steps (256 MiB write)",
                   "parallelism": f"dp{ctx.world} (states sharded; weights broadcast over NCCL by the library)",
                   "seed": args.seed},
        "e2e": e2e, "gpu_launches": launches, "roofline": roof, "cpu_baseline": cpu, "clocks": clk.summary(),
        "kernels": kernels, "outputs_finite": out_ok, "weight_broadcast": bcast,
        "gemm": gemm_summary(cfg, kernels, m_valid, sq_counts, B, tc_peak, tc_sus),
    }


def run_ours(args, cfg) -> None:
    import orbit_wars_b200 as ow

    ctx = Ctx().start()
    main = measure_policy(args, cfg, ctx, args.steps, args.warmup, min(args.steps, 200), not args.no_cpu)
    # config 5 (the scale-out workload: 65,536 states per GPU) rides along as a nested object, so the
    # 1/2/4/8-GPU runs of this command also trace config 5's scaling and its weight broadcast
    c5 = None
    if args.config != 5 and not args.no_c5:
        c5 = measure_policy(args, ow.preset(5), ctx, steps=5, warmup=3, e2e_steps=3, with_cpu=not args.no_cpu,
                            cpu_target_s=6.0)
        c5["metric"] = METRIC.format(c=5)
        c5["unit"] = UNIT
    # the True2D drop-in (the reference's own self-play forward, behind its own ABI): one GPU, rank 0
    t2 = None
    if ctx.world == 1 and not args.no_true2d:
        t2 = true2d_measure(args, ctx, steps=50, warmup=5, cpu_target_s=8.0)
    if ctx.rank == 0:
        line = {"metric": METRIC.format(c=args.config), "value": main["value"], "unit": UNIT, "n_gpus": ctx.world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": main["ms_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": main["dtype"],
                "data": "synthetic (seeded SplitMix/Box-Muller features, Xavier-uniform weights)"}
        for k in ("config", "e2e", "gpu_launches", "roofline", "cpu_baseline", "clocks", "kernels", "outputs_finite",
                  "weight_broadcast", "gemm"):
            line[k] = main[k]
        line["config5"] = c5
        line["true2d"] = t2
        print(json.dumps(line), flush=True)
    ctx.finish()


# ---------------------------------------------------------------- True2D drop-in workload
# The reference engine's self-play forward (crates/orbit-wars-core/src/true2d_model.rs:197-283)
# through the reference ABI: a resident population of seeded models
# (True2DTransformer::seeded) and one batch of engine-shaped requests per step,
# forward_many_resident as the engine calls it (cuda_true2d.rs:275-358).
T2_METRIC = "True2D drop-in forward requests/sec (61 layers, 64 rows, 1 head; resident population)"
T2_UNIT = "requests/s"


def true2d_workload(args):
    from orbit_wars_b200 import synth
    from orbit_wars_b200.true2d import True2DShape
    shape = True2DShape()  # config.rs defaults: 61 matrix layers, 64 rows, 1 attention head
    per = shape.parameter_count()
    pop = synth.true2d_population(args.seed, args.models, per)
    x, idx = synth.true2d_requests(args.seed, args.requests, shape.rows, args.models)
    return shape, per, pop, x, idx


def true2d_workload_name(args, shape) -> str:
    return (f"True2D self-play batch: {args.requests} requests x {shape.rows} rows x 7 features, "
            f"population of {args.models} seeded models ({shape.parameter_count():,} f32 weights each, "
            f"{args.models * shape.parameter_count() * 4 / 1e6:.0f} MB resident), "
            f"{shape.layers} matrix layers, {shape.heads} attention head")


def true2d_mufu_per_request(shape, part: str) -> float:
    """MUFU operations per request in a matrix-layer kernel: 5 per cell per layer (one ex2.approx for each
    of the three tanh, their reciprocals on the FMA pipe; ex2.approx and rcp.approx for the gate's sigmoid);
    the post-attention kernel adds the collapse's two exponentials per (row, action, target)."""
    cells = shape.rows * shape.rows
    mid = shape.layers // 2
    if part == "pre":
        return 5.0 * cells * mid
    return 5.0 * cells * (shape.layers - mid) + 2.0 * shape.rows * 12 * shape.rows


def true2d_cpu_reference(args, shape, pop, per, x, target_s: float) -> dict | None:
    """The reference's own CPU forward (native/cuda/orbit_wars_cuda_true2d_smoke.cpp:127-260,
    cpu_reference: 2 requests of one model per call, single-threaded), compiled from the
    reference source into oracle/_ref, run concurrently on every host thread."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle import bind
    if not bind.ref_available():
        return None
    lib = bind.load_ref_cpu()
    games = int(lib.ref_true2d_smoke_games())
    if int(lib.ref_true2d_smoke_weight_count()) != per or shape.heads != 1:
        return None
    threads = host_threads()
    rows_per_call = games * shape.rows * 7
    calls_avail = max(1, x.size // rows_per_call)

    def one(i):
        c = i % calls_avail
        xin = np.ascontiguousarray(x[c * rows_per_call:(c + 1) * rows_per_call])
        w = pop[(i % args.models) * per:(i % args.models + 1) * per]
        out = np.zeros(games * shape.rows * 24, np.float32)
        lib.ref_true2d_cpu_reference(xin.ctypes.data, w.ctypes.data, out.ctypes.data)
        return out

    t0 = time.perf_counter()
    one(0)
    per_call = time.perf_counter() - t0
    # about target_s of wall time when every thread runs calls back to back
    calls = max(threads, min(100000, int(target_s / max(per_call, 1e-6)) * threads))
    with ThreadPoolExecutor(threads) as ex:
        t0 = time.perf_counter()
        list(ex.map(one, range(calls)))
        dt = time.perf_counter() - t0
    return {"value": calls * games / dt, "unit": T2_UNIT, "cores": threads, "kind": "reference",
            "sample": f"{calls * games} requests ({calls} calls of the reference's cpu_reference, {games} requests "
                      f"each, models cycling over the population) on {threads} threads, {dt:.1f} s"}


def run_true2d_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    shape, per, pop, x, idx = true2d_workload(args)
    budget = min(30.0, REFERENCE_RUN_S / (args.steps + args.warmup))
    for _ in range(args.warmup):
        true2d_cpu_reference(args, shape, pop, per, x, target_s=budget)
    vals = []
    for _ in range(args.steps):
        r = true2d_cpu_reference(args, shape, pop, per, x, target_s=budget)
        if r is None:
            print(json.dumps({"impl": "reference", "unavailable":
                              "the reference's cpu_reference was not built from source (make -C oracle ref)"}))
            return
        vals.append(r)
    value = float(np.mean([v["value"] for v in vals]))
    cpu = dict(vals[-1])
    cpu["value"] = value
    line = {
        "impl": "reference", "metric": T2_METRIC, "value": value, "unit": T2_UNIT,
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * args.requests / value, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded True2DTransformer::seeded models)",
        "config": {"workload": true2d_workload_name(args, shape)},
        "cpu_baseline": cpu, "e2e": {"value": value, "unit": T2_UNIT, "h2d_bytes_per_step": 0,
                                     "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def reference_gpu_true2d(args, shape, pop, x, idx, steps: int) -> dict | None:
    """The reference's own CUDA library (native/cuda/orbit_wars_cuda.cu, built from source for
    sm_100a into oracle/_ref) on the same workload and the same ABI call."""
    import ctypes as C
    from orbit_wars_b200 import _lib
    path = REPO / "oracle" / "_ref" / "liborbit_wars_cuda_ref.so"
    if not path.exists():
        return None
    ref = C.CDLL(str(path), mode=2)
    ref.orbit_wars_cuda_true2d_upload_population.restype = _lib.Status
    ref.orbit_wars_cuda_true2d_upload_population.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t,
                                                             _lib.True2DShapeC]
    ref.orbit_wars_cuda_true2d_forward_many_resident.restype = _lib.Status
    ref.orbit_wars_cuda_true2d_forward_many_resident.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                                                 _lib.True2DShapeC]
    _lib.check("reference upload", ref.orbit_wars_cuda_true2d_upload_population(
        pop.ctypes.data, args.models, args.requests, shape.c()))
    out = np.zeros(args.requests * shape.rows * 24, np.float32)

    def call():
        _lib.check("reference forward", ref.orbit_wars_cuda_true2d_forward_many_resident(
            x.ctypes.data, idx.ctypes.data, out.ctypes.data, args.requests, shape.c()))

    for _ in range(3):
        call()
    wall = []
    for _ in range(steps):
        t0 = time.perf_counter()
        call()
        wall.append(time.perf_counter() - t0)
    return {"value": args.requests * steps / float(np.sum(wall)), "unit": T2_UNIT, "steps": steps,
            "timing": "wall clock per synchronous forward_many_resident call (host buffers), same workload",
            "library": "oracle/_ref/liborbit_wars_cuda_ref.so (reference source, nvcc sm_100a)", "output": out}


def true2d_turn(args, lib, shape, steps: int) -> dict:
    """One policy turn on the device through orbit_wars_cuda_true2d_play_many_resident: seeded game states
    (host CSR planets) in, decoded (target row, ship count) pairs out; encoder, forward and decode kernels
    timed by CUDA events. Beside it, the encoder oracle (a C++ restatement of encoder.rs:37-208) on all host
    threads encodes the same batch: the per-turn host work the device encoder removes
    (crates/orbit-wars-trainer/src/main.rs:3599-3667 runs encode_state on 12 threads)."""
    from orbit_wars_b200 import synth
    from oracle import bind
    batch, rg, rp = synth.game_batch(args.seed + 1, max(1, args.requests // 3 + 8), players=4)
    n = min(args.requests, rg.size)
    rg, rp = rg[:n], rp[:n]
    idx = (np.arange(n, dtype=np.uint64) * 2654435761 % args.models).astype(np.uintp)
    for _ in range(3):
        ids, tr, sc = lib.play_population_resident(batch, rg, rp, idx, args.models, shape)
    lib.profile_begin(steps)
    wall = []
    for _ in range(steps):
        t0 = time.perf_counter()
        ids, tr, sc = lib.play_population_resident(batch, rg, rp, idx, args.models, shape)
        wall.append(time.perf_counter() - t0)
    prof = lib.profile_end()
    kern = {k: round(ms * 1000.0 / max(c, 1), 2) for k, (c, ms) in prof.items()}
    threads = host_threads()
    bind.encode_batch(batch, rg, rp, threads=threads)
    t0, reps = time.perf_counter(), 0
    while time.perf_counter() - t0 < 2.0:
        bind.encode_batch(batch, rg, rp, threads=threads)
        reps += 1
    cpu_rate = n * reps / (time.perf_counter() - t0)
    enc_us = kern.get("t2_encode", 0.0)
    h2d = int(batch.planets.nbytes + batch.initial_planets.nbytes + 8 * 3 * (batch.game_count + 1) + 8 * n
              + (0 if batch.comet_planet_ids is None else batch.comet_planet_ids.nbytes) + 8 * n)
    return {"value": n * steps / float(np.sum(wall)), "unit": T2_UNIT, "requests": n, "games": batch.game_count,
            "steps": steps, "timing": "wall clock per synchronous play_many_resident call (host game states in, "
                                      "row ids + target rows + ship counts out)",
            "kernel_avg_us": kern, "encode_requests_per_s_device": round(n / (enc_us * 1e-6), 1) if enc_us else None,
            "encode_requests_per_s_cpu_oracle": round(cpu_rate, 1), "cpu_threads": threads,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": int(n * shape.rows * 4 * (1 + 2 * 12)),
            "commands_per_request": round(float((tr >= 0).sum()) / n, 2)}


def true2d_train(args, lib, shape, samples: int = 64, models: int = 8, steps: int = 3) -> dict:
    """The training step (orbit_wars_cuda_true2d_train_full_attention) on seeded engine-shaped samples: ours
    and, when built, the reference's own CUDA library on the same samples and weights (wall clock per
    synchronous call, host buffers, as the engine calls it), with the agreement of the weight updates."""
    import ctypes as C
    from orbit_wars_b200 import _lib, synth
    rng = np.random.default_rng(args.seed + 7)
    R = shape.rows
    x = rng.uniform(-1.0, 1.0, (samples, R, 7)).astype(np.float32)
    classes = np.array([1.0, 0.75, 0.5, 0.25, 0.0, -1.0], np.float32)
    for i in range(samples):
        act = int(rng.integers(8, R + 1))
        x[i, :act, 0] = rng.choice(classes, act, p=[0.3, 0.15, 0.1, 0.1, 0.25, 0.1])
        x[i, act:, 0] = -0.5
        x[i, act:, 1:] = 0.0
    out = rng.uniform(0.0, 1.0, (samples, R, 24)).astype(np.float32)
    rewards = rng.integers(-2, 3, samples).astype(np.int32)
    tar = (rng.standard_normal((samples, R, 12)) * 0.2).astype(np.float32)
    idx = (np.arange(samples) % models).astype(np.uintp)
    w = synth.true2d_population(args.seed, models, shape.parameter_count())
    kw = dict(batch_sample_count=samples, learning_rate=0.01, reward_normalizer=2.0, send_threshold=0.5)
    ours = lib.train_full_attention(x, out, rewards, tar, idx, w, shape, **kw)
    # timed calls update a working copy in place, as the engine's host buffer is updated (each call takes
    # the same work; the weights move by one SGD step per call)
    wk = np.array(w, dtype=np.float32, copy=True)
    lib.train_full_attention(x, out, rewards, tar, idx, wk, shape, inplace=True, **kw)
    wall = []
    lib.profile_begin(2 * steps)
    for _ in range(steps):
        t0 = time.perf_counter()
        lib.train_full_attention(x, out, rewards, tar, idx, wk, shape, inplace=True, **kw)
        wall.append(time.perf_counter() - t0)
    prof = lib.profile_end()
    res = {"value": samples * steps / float(np.sum(wall)), "unit": "samples/s", "samples": samples, "models": models,
           "steps": steps, "timing": "wall clock per synchronous train_full_attention call (host buffers, updated in place)",
           "phase_ms_per_call": {k: round(ms / max(c, 1), 3) for k, (c, ms) in prof.items()}}
    path = REPO / "oracle" / "_ref" / "liborbit_wars_cuda_ref.so"
    if path.exists():
        ref = C.CDLL(str(path), mode=2)
        fn = ref.orbit_wars_cuda_true2d_train_full_attention
        fn.restype = _lib.Status
        fn.argtypes = [C.c_void_p] * 6 + [C.c_size_t, C.c_size_t, _lib.True2DShapeC, _lib.TrainingConfigC]
        cfg = _lib.TrainingConfigC(samples, 0.01, 2.0, 0.5, 1.0, -0.5, -1.0)
        rwall = []
        for k in range(4):
            wr = np.array(w, dtype=np.float32, copy=True)  # outside the timed region
            t0 = time.perf_counter()
            _lib.check("reference training", fn(x.ctypes.data, out.ctypes.data, rewards.ctypes.data, tar.ctypes.data,
                                                idx.ctypes.data, wr.ctypes.data, samples, models, shape.c(), cfg))
            if k > 0:
                rwall.append(time.perf_counter() - t0)
        d_ref = wr.reshape(models, -1) - w.reshape(models, -1)
        d_ours = ours - w.reshape(models, -1)
        res["reference_value"] = samples * len(rwall) / float(np.sum(rwall))
        res["ours_over_reference"] = round(res["value"] / res["reference_value"], 2)
        res["update_rel_err_vs_reference"] = float(np.abs(d_ours - d_ref).max() / np.abs(d_ref).max())
        res["reference_library"] = "oracle/_ref/liborbit_wars_cuda_ref.so (reference source, nvcc sm_100a)"
    return res


def mufu_peak(sm_mhz: float | None, cells_ex2: float, cells_rcp: float) -> dict | None:
    """The special-function pipe's rate, measured on this GPU (orbit_wars_cuda_mufu_rate: ex2.approx and
    rcp.approx chains, one 1024-thread CTA per SM, clock64 spans), for a kernel that issues ex2 and rcp in
    the ratio cells_ex2 : cells_rcp; at the SM clock sampled during the timed region."""
    import ctypes as C
    from orbit_wars_b200 import _lib
    lib = _lib.load_library()
    res = {}
    for op, name in ((0, "ex2"), (1, "rcp")):
        ops, per_clk, mhz = C.c_double(), C.c_double(), C.c_double()
        st = lib.orbit_wars_cuda_mufu_rate(op, C.byref(ops), C.byref(per_clk), C.byref(mhz))
        if st.code != 0:
            return None
        res[name] = {"ops_per_s": ops.value, "per_clock_per_sm": round(per_clk.value, 3),
                     "probe_sm_mhz": round(mhz.value, 1)}
    import torch
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    mhz = sm_mhz or res["ex2"]["probe_sm_mhz"]
    # time per op mix: cells_ex2 / r_ex2 + cells_rcp / r_rcp  ->  effective ops per clock per SM
    r_e, r_r = res["ex2"]["per_clock_per_sm"], res["rcp"]["per_clock_per_sm"]
    eff = (cells_ex2 + cells_rcp) / (cells_ex2 / r_e + cells_rcp / r_r)
    return {"peak_gops": eff * sms * mhz * 1e6 / 1e9, "per_clock_per_sm": round(eff, 3), "sm_mhz": mhz,
            "probe": res}


def true2d_measure(args, ctx, steps: int, warmup: int, cpu_target_s: float = 12.0) -> dict:
    """The True2D drop-in (reference ABI) on this process's GPU: device kernel phases, e2e through the
    C-ABI call, the reference's own CUDA build on the same call, the reference's CPU forward, the MUFU
    roofline against the measured MUFU rate, a device turn and the training step."""
    import torch

    from orbit_wars_b200 import _lib
    from orbit_wars_b200.true2d import CudaTrue2D

    dev = ctx.dev
    shape, per, pop, x, idx = true2d_workload(args)  # replicas: every rank runs the same workload
    lib = CudaTrue2D()
    lib.upload_population(pop, args.requests, shape)
    out_buf = np.empty(args.requests * shape.rows * 24, np.float32)
    fwd = lib.lib.orbit_wars_cuda_true2d_forward_many_resident
    shape_c = shape.c()

    def step():
        # the engine's call (cuda_true2d.rs:469-487 packs, then forward_many_resident into a host buffer),
        # timed as the reference arm times the reference library: the C-ABI call alone
        _lib.check("cuda_true2d_forward_many_resident",
                   fwd(x.ctypes.data, idx.ctypes.data, out_buf.ctypes.data, args.requests, shape_c))
        return out_buf

    for _ in range(warmup):
        out = step()
    ctx.barrier()
    torch.cuda.synchronize(dev)
    lib.profile_begin(steps)
    wall = []
    with ClockSampler(ctx.local) as clk:
        clk.window = (time.time(), None)
        for _ in range(steps):
            t0 = time.perf_counter()
            out = step()
            wall.append(time.perf_counter() - t0)
        clk.window = (clk.window[0], time.time())
    prof = lib.profile_end()
    ctx.barrier()
    torch.cuda.synchronize(dev)
    dev_s = sum(v[1] for k, v in prof.items() if k.startswith("t2_")) / 1000.0  # kernels only, not the copies
    t_dev, t_wall = ctx.max_over_ranks([dev_s, float(np.sum(wall))])
    value = ctx.world * args.requests * steps / t_dev
    e2e = {"value": ctx.world * args.requests * steps / t_wall, "unit": T2_UNIT,
           "h2d_bytes_per_step": int(x.nbytes + idx.nbytes),
           "d2h_bytes_per_step": int(args.requests * shape.rows * 24 * 4 + 4),
           "timing": "wall clock per synchronous forward_many_resident C-ABI call (host buffers, output buffer reused "
                     "as in the reference arm), max over ranks"}
    kernels, copies = {}, {}
    for name, (n, ms) in prof.items():
        (kernels if name.startswith("t2_") else copies)[name] = {
            "launches": n, "total_ms": round(ms, 4), "avg_us": round(ms * 1000.0 / max(n, 1), 2)}
    total = sum(k["total_ms"] for k in kernels.values()) or 1.0
    for k in kernels.values():
        k["share"] = round(k["total_ms"] / total, 4)
    clocks = clk.summary()
    roof = None
    mufu = {"t2_expand_pre": true2d_mufu_per_request(shape, "pre"),
            "t2_post_collapse": true2d_mufu_per_request(shape, "post")}
    top = max((k for k in mufu if k in kernels), key=lambda k: kernels[k]["total_ms"], default=None)
    if top is not None:
        a = kernels[top]
        ach = mufu[top] * args.requests / (a["avg_us"] * 1e-6) / 1e9
        # per cell and layer 4 ex2 (three tanh, the gate) and 1 rcp (the gate); the collapse adds ex2 only
        cells = shape.rows * shape.rows
        n_layers = shape.layers // 2 if top == "t2_expand_pre" else shape.layers - shape.layers // 2
        ex2 = 4.0 * cells * n_layers + (2.0 * shape.rows * 12 * shape.rows if top == "t2_post_collapse" else 0.0)
        rcp = 1.0 * cells * n_layers
        pk = mufu_peak(clocks.get("sm_mhz"), ex2, rcp)
        traffic, traffic_src = ncu_traffic("true2d", top) if args.requests == 1024 and args.models == 64 else (None, None)
        if pk is not None:
            roof = {"kernel": top, "bound": "mufu", "achieved": round(ach, 1), "peak": round(pk["peak_gops"], 1),
                    "unit": "G MUFU ops/s", "frac": round(ach / pk["peak_gops"], 4), "traffic": traffic,
                    "traffic_unit": "bytes per launch (dram read + write)", "traffic_source": traffic_src,
                    "peak_source": f"measured: ex2/rcp probe {pk['per_clock_per_sm']} ops/clk/SM for this kernel's "
                                   f"ex2:rcp mix x SMs x {pk['sm_mhz']:.0f} MHz (median SM clock sampled during the "
                                   "timed region)", "mufu_probe": pk["probe"],
                    "work_per_launch": f"{mufu[top]:.0f} MUFU ops per request: 5 per cell per matrix layer (ex2 "
                                       "for each of the three tanh, ex2 and rcp for the gate's sigmoid)"
                                       + (" plus two ex2 per (row, action, target) of the collapse" if top ==
                                          "t2_post_collapse" else "")}
    ref_gpu = None
    if ctx.rank == 0 and ctx.world == 1:
        ref_gpu = reference_gpu_true2d(args, shape, pop, x, idx, steps=min(steps, 50))
        if ref_gpu is not None:
            ro = ref_gpu.pop("output")
            ref_gpu["max_abs_diff_vs_ours"] = float(np.abs(ro - out.reshape(-1)).max())
            ref_gpu["ours_e2e_over_reference"] = round(e2e["value"] / ref_gpu["value"], 3)
            ref_gpu["ours_device_over_reference"] = round(value / ref_gpu["value"], 3)
    solo = ctx.rank == 0 and ctx.world == 1
    turn = true2d_turn(args, lib, shape, steps=min(steps, 20)) if solo else None
    train = true2d_train(args, lib, shape) if solo else None
    cpu = true2d_cpu_reference(args, shape, pop, per, x, target_s=cpu_target_s) if solo and not args.no_cpu else None
    return {"metric": T2_METRIC, "value": value, "unit": T2_UNIT, "steps": steps, "warmup": warmup,
            "ms_per_step": 1000.0 * t_dev / steps, "dtype": "f32",
            "data": "synthetic (seeded True2DTransformer::seeded models, N(0,1)/2 request rows)",
            "config": {"workload": true2d_workload_name(args, shape), "requests_per_gpu": args.requests,
                       "models": args.models,
                       "l2": f"population of {args.models * per * 4 / 1e6:.0f} MB > 126 MB L2, read every step",
                       "parallelism": f"replicas x{ctx.world} (the reference ABI is single-device)",
                       "value_timing": "sum of the kernel phases' CUDA events per call (expand and matrix layers, "
                                       "attention, matrix layers and collapse; the row upload excluded; the "
                                       "collapse writes the outputs into mapped host memory as it runs, so its "
                                       "time includes their transfer)"},
            "e2e": e2e, "gpu_launches": 4 * steps, "roofline": roof, "cpu_baseline": cpu,
            "reference_gpu": ref_gpu, "clocks": clocks, "kernels": kernels, "copies": copies, "turn": turn,
            "train": train, "outputs_finite": bool(np.isfinite(out).all())}


def run_true2d(args) -> None:
    ctx = Ctx().start()
    res = true2d_measure(args, ctx, args.steps, args.warmup)
    if ctx.rank == 0:
        line = {"metric": res["metric"], "value": res["value"], "unit": T2_UNIT, "n_gpus": ctx.world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None}
        line.update({k: v for k, v in res.items() if k not in line and k != "metric"})
        print(json.dumps(line), flush=True)
    ctx.finish()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4, 5])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seed", type=int, default=17)
    ap.add_argument("--batch", type=int, default=None, help="override the config's per-GPU batch")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-c5", action="store_true", help="skip the nested config-5 (scale-out) measurement")
    ap.add_argument("--no-true2d", action="store_true", help="skip the nested True2D drop-in measurement")
    ap.add_argument("--workload", default="policy", choices=["policy", "true2d"],
                    help="policy: the encoder-policy forward (default); true2d: the reference ABI drop-in")
    ap.add_argument("--requests", type=int, default=1024, help="true2d: requests per step")
    ap.add_argument("--models", type=int, default=64, help="true2d: resident population size")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.workload == "true2d":
        return run_true2d_reference(args) if args.impl == "reference" else run_true2d(args)
    import orbit_wars_b200 as ow
    cfg = ow.preset(args.config)
    if args.batch:
        cfg = cfg.with_(batch=args.batch)
    if args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
