"""ctypes binding of the CPU oracles (oracle/libow_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, as the checker. The product library never
loads it.

    policy_forward(cfg, weights, features, counts, f64=True)  encoder policy (SPEC.md)
    true2d_forward(...)                                        True2D (true2d_model.rs restatement)
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "libow_oracle.so"
REF_DIR = HERE / "_ref"
_lib = None


class OwoShape(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("n_entities", "features", "d_model", "heads", "ffn", "layers", "actions")]


def build(ref: bool = False) -> None:
    """make -C oracle [ref]: the oracle always; the reference builds only when its source tree exists."""
    target = ["ref"] if ref else []
    subprocess.run(["make", "-s", "-C", str(HERE), *target], check=True)


def load():
    global _lib
    if _lib is not None:
        return _lib
    if not LIB.exists():
        build()
    lib = C.CDLL(str(LIB))
    lib.owo_policy_weight_count.restype = C.c_size_t
    lib.owo_policy_weight_count.argtypes = [C.POINTER(OwoShape)]
    lib.owo_policy_forward.restype = C.c_int
    lib.owo_policy_forward.argtypes = [C.POINTER(OwoShape), C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p,
                                       C.c_int32, C.c_int, C.c_int, C.c_int, C.c_uint64,
                                       C.c_void_p, C.c_void_p, C.c_void_p]
    lib.owo_gumbel.restype = C.c_double
    lib.owo_gumbel.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32]
    lib.owo_philox4x32_10.restype = None
    lib.owo_philox4x32_10.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p]
    lib.owo_max_threads.restype = C.c_int
    lib.owo_true2d_weight_count.restype = C.c_size_t
    lib.owo_true2d_weight_count.argtypes = [C.c_size_t] * 3
    lib.owo_deterministic_weight.restype = C.c_float
    lib.owo_deterministic_weight.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64]
    lib.owo_true2d_seeded.restype = None
    lib.owo_true2d_seeded.argtypes = [C.c_uint64, C.c_void_p, C.c_size_t]
    lib.owo_true2d_forward.restype = C.c_int
    lib.owo_true2d_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t,
                                       C.c_size_t, C.c_size_t, C.c_size_t, C.c_int]
    lib.owo_trainable_forward.restype = C.c_int
    lib.owo_trainable_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p] + [C.c_size_t] * 5
    lib.owo_sinusoid_fill.restype = None
    lib.owo_sinusoid_fill.argtypes = [C.c_void_p, C.c_size_t, C.c_float, C.c_float]
    _lib = lib
    return lib


def shape_of(cfg) -> OwoShape:
    return OwoShape(cfg.n_entities, cfg.features, cfg.d_model, cfg.heads, cfg.ffn, cfg.layers, cfg.actions)


def policy_forward(cfg, weights, features, counts, f64: bool = True, threads: int = 0, sample: bool | None = None,
                   seed: int = 0):
    """Returns (logits f32 [B,N,P], value f32 [B], actions int32 [B,N])."""
    lib = load()
    w = np.ascontiguousarray(weights, dtype=np.float32)
    f = np.ascontiguousarray(features, dtype=np.float32)
    c = np.ascontiguousarray(counts, dtype=np.int32)
    B = c.shape[0]
    logits = np.zeros((B, cfg.n_entities, cfg.actions), dtype=np.float32)
    value = np.zeros((B,), dtype=np.float32)
    actions = np.zeros((B, cfg.n_entities), dtype=np.int32)
    smp = cfg.sample_actions if sample is None else sample
    sh = shape_of(cfg)
    rc = lib.owo_policy_forward(C.byref(sh), w.ctypes.data, w.size, f.ctypes.data, c.ctypes.data, B,
                                1 if f64 else 0, threads, 1 if smp else 0, C.c_uint64(seed),
                                logits.ctypes.data, value.ctypes.data, actions.ctypes.data)
    if rc != 0:
        raise ValueError(f"oracle rejected arguments (rc={rc})")
    return logits, value, actions


def policy_weight_count(cfg) -> int:
    sh = shape_of(cfg)
    return int(load().owo_policy_weight_count(C.byref(sh)))


def gumbel(seed: int, state: int, entity: int, action: int) -> float:
    return float(load().owo_gumbel(seed, state, entity, action))


def philox(counter, k0: int, k1: int) -> list[int]:
    c = np.ascontiguousarray(counter, dtype=np.uint32)
    out = np.zeros(4, dtype=np.uint32)
    load().owo_philox4x32_10(c.ctypes.data, k0, k1, out.ctypes.data)
    return [int(v) for v in out]


def max_threads() -> int:
    return int(load().owo_max_threads())


def true2d_weight_count(layers=61, rows=64, heads=1) -> int:
    return int(load().owo_true2d_weight_count(layers, rows, heads))


def true2d_seeded(seed: int, count: int) -> np.ndarray:
    w = np.zeros(count, dtype=np.float32)
    load().owo_true2d_seeded(seed, w.ctypes.data, count)
    return w


def deterministic_weight(seed: int, row: int, column: int) -> float:
    return float(load().owo_deterministic_weight(seed, row, column))


def sinusoid(n: int, step: float, scale: float = 1.0) -> np.ndarray:
    """v[i] = sinf((float)(i+1) * step) * scale, computed in C like the reference smoke's fixture."""
    out = np.zeros(n, dtype=np.float32)
    load().owo_sinusoid_fill(out.ctypes.data, n, step, scale)
    return out


def true2d_forward(input_rows, all_weights, model_indices=None, layers=61, rows=64, heads=1, threads: int = 0):
    lib = load()
    x = np.ascontiguousarray(input_rows, dtype=np.float32)
    per = true2d_weight_count(layers, rows, heads)
    w = np.ascontiguousarray(all_weights, dtype=np.float32).reshape(-1)
    models = w.size // per
    n = x.size // (rows * 7)
    idx = None if model_indices is None else np.ascontiguousarray(model_indices, dtype=np.uintp)
    out = np.zeros(n * rows * 24, dtype=np.float32)
    rc = lib.owo_true2d_forward(x.ctypes.data, None if idx is None else idx.ctypes.data, w.ctypes.data, models,
                                out.ctypes.data, n, layers, rows, heads, threads)
    if rc != 0:
        raise ValueError(f"oracle rejected arguments (rc={rc})")
    return out


def trainable_forward(input_rows, weights, games, layers, d_model, heads, rows):
    x = np.ascontiguousarray(input_rows, dtype=np.float32)
    w = np.ascontiguousarray(weights, dtype=np.float32)
    out = np.zeros(games * rows * 2, dtype=np.float32)
    rc = load().owo_trainable_forward(x.ctypes.data, w.ctypes.data, out.ctypes.data, games, layers, d_model,
                                      heads, rows)
    if rc != 0:
        raise ValueError(f"oracle rejected arguments (rc={rc})")
    return out


def ref_available() -> bool:
    return (REF_DIR / "libref_true2d_cpu.so").exists()


def load_ref_cpu():
    """The reference smoke's own cpu_reference (built from the reference source into oracle/_ref)."""
    lib = C.CDLL(str(REF_DIR / "libref_true2d_cpu.so"))
    lib.ref_true2d_smoke_weight_count.restype = C.c_size_t
    lib.ref_true2d_smoke_games.restype = C.c_size_t
    lib.ref_true2d_cpu_reference.restype = None
    lib.ref_true2d_cpu_reference.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
    return lib
