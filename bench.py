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

--impl reference times the reference-side CPU implementation of this path.
The reference repository has no implementation of this network, so that arm
is the repository's CPU port of the spec (oracle, fp32, all host threads).
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


def ncu_traffic(config: int, kernel: str):
    """DRAM bytes per launch of `kernel` from the committed ncu capture of this
    config (profiles/ncu_traffic_c<config>.json), or None."""
    p = REPO / "profiles" / f"ncu_traffic_c{config}.json"
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


def kernel_work(cfg, name: str, m_valid: int, sq_counts: int, batch: int) -> tuple[str, float]:
    """(bound, algorithmic work per launch): FLOPs for tensor-bound kernels, bytes for HBM-bound ones."""
    d, f, F, P, N = cfg.d_model, cfg.ffn, cfg.features, cfg.actions, cfg.n_entities
    act = 4 if cfg.precision == "f32" else 2
    a8 = 1 if cfg.precision == "fp8" else act
    if name in ("gemm_qkv", "gemm_f32_qkv"):
        return "tensor", 2.0 * m_valid * 3 * d * d
    if name in ("gemm_out_resid_ln", "gemm_f32_out_resid"):
        return "tensor", 2.0 * m_valid * d * d
    if name in ("gemm_ffn_up_gelu", "gemm_f32_ffn_up"):
        return "tensor", 2.0 * m_valid * f * d
    if name in ("gemm_ffn_down_resid_ln", "gemm_f32_ffn_down_resid"):
        return "tensor", 2.0 * m_valid * d * f
    if name == "attention":
        return "tensor", 4.0 * sq_counts * d
    if name == "embed_ln":
        return "hbm", m_valid * (F * 4 + 2 * d * a8)
    if name == "heads":
        lb = 4 if cfg.logits_dtype == "f32" else 2
        return "hbm", m_valid * d * act + batch * N * (P * lb + 4) + batch * 4
    if name == "layernorm_f32":
        return "hbm", m_valid * d * 8.0
    if name == "quantize_e4m3":
        return "hbm", m_valid * (f + d) / 2 * 3.0
    if name == "scan_counts":
        return "hbm", batch * 8.0
    return "hbm", 0.0


def cpu_baseline(cfg, weights, feats, counts, target_s: float = 12.0) -> dict:
    """Times the fp32 CPU oracle (OpenMP, all host threads) on a bounded sample of the workload."""
    from oracle import bind
    threads = bind.max_threads()
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
            "sample": f"{n} of the {cfg.batch} states of the workload, fp32 CPU oracle, {dt:.1f} s"}


def run_reference(args, cfg) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import orbit_wars_b200 as ow
    from oracle import bind
    weights = ow.make_weights(cfg, seed=args.seed)
    feats, counts = ow.make_inputs(cfg, seed=args.seed)
    threads = bind.max_threads()
    # sample size so one step takes ~3 s of CPU work
    n = 4
    t0 = time.perf_counter()
    bind.policy_forward(cfg, weights, feats[:n], counts[:n], f64=False, threads=threads)
    per_state = (time.perf_counter() - t0) / n
    n = int(max(1, min(cfg.batch, 3.0 / max(per_state, 1e-6))))
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
    sample = (f"{n} states per step (of the {cfg.batch}-state workload), fp32 CPU port of the spec, "
              f"{threads} threads; the reference repository has no implementation of this network")
    line = {
        "impl": "reference", "metric": METRIC.format(c=args.config), "value": value, "unit": UNIT,
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * total / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, SPEC.md section 7)",
        "config": {"workload": workload_name(cfg), "sample_states_per_step": n},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, cfg) -> None:
    import torch
    import torch.distributed as dist

    import orbit_wars_b200 as ow

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep NCCL's banner off stdout (one JSON line)
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    from orbit_wars_b200.shard import broadcast_weights, shard_inputs

    # weights: rank 0 builds them, one NCCL broadcast to every rank
    weights = broadcast_weights(cfg, args.seed, rank, device=dev)
    # this rank's shard of the global batch (world * B states)
    feats, counts = shard_inputs(cfg, args.seed, rank)
    B = cfg.batch
    m_valid = int(counts.sum())
    sq_counts = int((counts.astype(np.int64) ** 2).sum())

    # one non-default stream carries the library's kernels, torch's copies/flushes and the timing events
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    pol = ow.EncoderPolicy(cfg, weights, device=local, stream=stream.cuda_stream, io="device")
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

    for i in range(args.warmup):
        flush.zero_()
        step(i)
    pol.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    prof_steps = min(args.steps, 100)
    pol.profile_begin(prof_steps)  # per-kernel events on the first timed steps
    with ClockSampler(local) as clk:
        clk.window = (time.time(), None)
        for i in range(args.steps):
            flush.zero_()  # L2 flush outside the step's events
            starts[i].record(stream)
            step(args.warmup + i)
            ends[i].record(stream)
        torch.cuda.synchronize(dev)
        clk.window = (clk.window[0], time.time())
    prof = pol.profile_end()
    pol.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    t_local = float(np.sum(step_ms)) / 1000.0
    t = torch.tensor([t_local], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    t_max = float(t.item())
    value = world * B * args.steps / t_max
    launches = pol.launches_per_forward() * args.steps
    out_ok = bool(torch.isfinite(lg.float()).all().item() and torch.isfinite(vv.float()).all().item())

    # e2e through the host-buffer API (pinned host buffers)
    e2e = None
    e2e_steps = min(args.steps, 200)
    if not args.no_e2e:
        hp = ow.EncoderPolicy(cfg, weights, device=local, stream=stream.cuda_stream, io="host")
        f_h = torch.from_numpy(feats).pin_memory()
        c_h = torch.from_numpy(counts).pin_memory()
        lg_h = torch.empty((B, cfg.n_entities, cfg.actions), dtype=ldt).pin_memory()
        vv_h = torch.empty((B,), dtype=vdt).pin_memory()
        aa_h = torch.empty((B, cfg.n_entities), dtype=torch.int32).pin_memory()

        def hstep(i):
            hp.forward_raw(f_h.data_ptr(), c_h.data_ptr(), B, lg_h.data_ptr(), vv_h.data_ptr(), aa_h.data_ptr(),
                           seed=i)

        for i in range(args.warmup):
            hstep(i)
        if world > 1:
            dist.barrier()
        wall = []
        for i in range(e2e_steps):
            flush.zero_()
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            hstep(i)
            wall.append(time.perf_counter() - t0)
        te = torch.tensor([float(np.sum(wall))], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        h2d = feats.nbytes + counts.nbytes
        d2h = lg_h.numel() * lg_h.element_size() + vv_h.numel() * vv_h.element_size() + aa_h.numel() * 4
        e2e = {"value": world * B * e2e_steps / float(te.item()), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h), "steps": e2e_steps,
               "timing": "wall clock per synchronous host-buffer call (pinned buffers), max over ranks"}
        hp.close()

    # roofline of the dominant kernel
    peaks, peak_src = load_peaks()
    kernels = {}
    for name, (n_launch, total_ms) in prof.items():  # from the first `prof_steps` timed steps
        bound, work = kernel_work(cfg, name, m_valid, sq_counts, B)
        avg_s = total_ms / 1000.0 / max(n_launch, 1)
        ach = work / avg_s if avg_s > 0 else 0.0
        kernels[name] = {"launches": n_launch, "total_ms": round(total_ms, 4), "avg_us": round(avg_s * 1e6, 2),
                         "bound": bound, "achieved": round(ach / (1e12 if bound == "tensor" else 1e9), 2),
                         "unit": "TFLOP/s" if bound == "tensor" else "GB/s"}
    total = sum(k["total_ms"] for k in kernels.values()) or 1.0
    for k in kernels.values():
        k["share"] = round(k["total_ms"] / total, 4)
    dom_name = max(kernels, key=lambda k: kernels[k]["total_ms"]) if kernels else None
    roof = None
    if dom_name is not None:
        k = kernels[dom_name]
        if k["bound"] == "tensor":
            peak = float(peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"]))
            if cfg.precision == "fp8":
                peak *= 2.0
        else:
            peak = float(peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
        traffic, traffic_src = ncu_traffic(args.config, dom_name)
        roof = {"kernel": dom_name, "bound": k["bound"], "achieved": k["achieved"], "peak": peak, "unit": k["unit"],
                "frac": round(k["achieved"] / peak, 4), "traffic": traffic,
                "traffic_source": traffic_src,
                "peak_source": peak_src + (" (fp8 peak = 2x measured bf16)" if cfg.precision == "fp8" else ""),
                "work_per_launch": "2*M_valid*N*K FLOPs, M_valid = valid tokens of the batch"
                if k["bound"] == "tensor" else "bytes read + written",
                "timed_steps_profiled": prof_steps}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(cfg, weights, feats, counts)

    clocks = clk.summary()
    if rank == 0:
        line = {
            "metric": METRIC.format(c=args.config), "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * t_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": {"f32": "f32", "bf16": "bf16", "fp8": "e4m3"}[cfg.precision],
            "data": "synthetic (seeded SplitMix/Box-Muller, SPEC.md section 7)",
            "config": {"workload": workload_name(cfg), "per_gpu_batch": B, "global_batch": B * world,
                       "valid_tokens_per_gpu": m_valid, "l2": "flushed between timed steps (256 MiB write)",
                       "parallelism": f"dp{world} (states sharded, weights broadcast once over NCCL)",
                       "seed": args.seed},
            "e2e": e2e, "gpu_launches": launches, "roofline": roof, "cpu_baseline": cpu, "clocks": clocks,
            "kernels": kernels, "outputs_finite": out_ok,
            "gemm_tflops_per_gpu": round(cfg.gemm_flops_per_token() * m_valid * args.steps / t_max / 1e12
                                         * (world / world), 2),
        }
        print(json.dumps(line), flush=True)
    pol.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


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
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
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
