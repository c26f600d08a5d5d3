"""CPU checks of bench.py's output contract (no GPU needed).

The reference arm (`--impl reference`) times the fp32 CPU port on the host's
cores, so it runs here: it must print exactly one JSON line with the keys the
driver reads. The roofline's algorithmic work counts are checked against the
GEMM shapes they describe (2 * M * N * K FLOPs per launch).
"""
import json
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def _bench(*args, timeout=300):
    return subprocess.run([sys.executable, str(REPO / "bench.py"), *args], cwd=REPO, capture_output=True,
                          text=True, timeout=timeout)


def test_reference_arm_prints_one_contract_line():
    out = _bench("--impl", "reference", "--config", "1", "--steps", "2", "--warmup", "3")
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert (d["n_gpus"], d["steps"], d["warmup"]) == (1, 2, 3)
    cpu = d["cpu_baseline"]
    assert cpu["value"] == d["value"] and cpu["cores"] >= 1 and cpu["kind"] in ("port", "reference")
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["same_config"] is True


def test_fewer_than_three_warmup_steps_are_refused():
    out = _bench("--impl", "reference", "--config", "1", "--steps", "1", "--warmup", "2", timeout=120)
    assert out.returncode != 0
    assert "--warmup must be >= 3" in out.stderr


def test_gemm_work_is_two_m_n_k():
    sys.path.insert(0, str(REPO))
    import bench
    import orbit_wars_b200 as ow

    cfg = ow.preset(2)
    d, f, m = cfg.d_model, cfg.ffn, 40271
    shapes = {"gemm_qkv": (3 * d, d), "gemm_out_resid_ln": (d, d), "gemm_ffn_up_gelu": (f, d),
              "gemm_ffn_down_resid_ln": (d, f)}
    for name, (n, k) in shapes.items():
        flops, nbytes = bench.kernel_work(cfg, name, m, 0, cfg.batch)
        assert flops == 2.0 * m * n * k, name
        # at least the A operand and the output cross HBM once
        assert nbytes >= m * (k + n) * 1, name
