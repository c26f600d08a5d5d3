"""ctypes binding of the CPU oracles (oracle/libow_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, as the checker. The product library never
loads it.

    policy_forward(cfg, weights, features, counts, f64=True)  encoder policy (frozen spec)
    true2d_forward(...)                                        True2D (true2d_model.rs restatement)
    encode_batch(batch, request_games, request_players)        state encoder (encoder.rs restatement)
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


class OwoEncoderConfig(C.Structure):
    """The AgentConfig fields the encoder reads (crates/orbit-wars-core/src/config.rs:115-140)."""
    _fields_ = [("max_rows", C.c_size_t), ("initial_planet_slots", C.c_size_t), ("comet_slots", C.c_size_t),
                ("padding_slots", C.c_size_t), ("ship_log_pivot", C.c_float), ("ship_log_cap", C.c_float),
                ("max_players", C.c_size_t), ("owner_class_own", C.c_float), ("owner_class_enemy_1", C.c_float),
                ("owner_class_enemy_2", C.c_float), ("owner_class_enemy_3", C.c_float),
                ("owner_class_neutral", C.c_float), ("owner_class_empty", C.c_float),
                ("owner_class_absent_on_map", C.c_float), ("board_size", C.c_float),
                ("fleet_speed_max", C.c_float)]


def default_encoder_config() -> OwoEncoderConfig:
    """config.rs:1-19 (MAX_ROWS .. FLEET_SPEED_MAX)."""
    return OwoEncoderConfig(64, 40, 20, 4, 1000.0, 100000.0, 4, 1.0, 0.75, 0.5, 0.25, 0.0, -0.5, -1.0, 100.0, 6.0)


# types.rs:6-16
PLANET_DTYPE = np.dtype([("id", "<i4"), ("owner", "<i4"), ("x", "<f4"), ("y", "<f4"), ("radius", "<f4"),
                         ("ships", "<f4"), ("production", "<f4"), ("velocity_x", "<f4"), ("velocity_y", "<f4")])


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
    lib.owo_policy_forward_emulated.restype = C.c_int
    lib.owo_policy_forward_emulated.argtypes = [C.POINTER(OwoShape), C.c_void_p, C.c_size_t, C.c_void_p,
                                                C.c_void_p, C.c_int32, C.c_uint, C.c_int, C.c_void_p, C.c_void_p,
                                                C.c_void_p]
    lib.owo_gumbel_argmax.restype = C.c_int
    lib.owo_gumbel_argmax.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_uint64,
                                      C.c_uint32, C.c_int, C.c_void_p, C.c_void_p]
    lib.owo_round_e4m3.restype = C.c_float
    lib.owo_round_e4m3.argtypes = [C.c_float]
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
    lib.owo_encode_state.restype = C.c_int
    lib.owo_encode_state.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t,
                                     C.c_int32, C.POINTER(OwoEncoderConfig), C.c_void_p, C.c_void_p, C.c_void_p,
                                     C.c_void_p]
    lib.owo_encode_batch.restype = None
    lib.owo_encode_batch.argtypes = [C.c_void_p] * 8 + [C.c_size_t, C.POINTER(OwoEncoderConfig)] + [C.c_void_p] * 5 + [
        C.c_int]
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


# rounding points of owo_policy_forward_emulated (ow_policy_oracle.cpp)
EMU_STORE_BF16, EMU_QUANT_QKV, EMU_QUANT_OUT, EMU_QUANT_UP, EMU_QUANT_DOWN, EMU_VALUE_BF16 = 1, 2, 4, 8, 16, 32
EMU_RESID_BF16 = 64
EMU_QUANT_ALL = EMU_QUANT_QKV | EMU_QUANT_OUT | EMU_QUANT_UP | EMU_QUANT_DOWN


def recipe_mode(cfg) -> int:
    """The full rounding recipe of cfg's precision path (0 for fp32)."""
    if cfg.precision == "f32":
        return 0
    resid = EMU_RESID_BF16 if cfg.d_model == 256 else 0  # the d = 256 tensor-core paths keep x in bf16
    if cfg.precision == "bf16":
        return EMU_STORE_BF16 | resid
    return EMU_STORE_BF16 | EMU_QUANT_ALL | EMU_VALUE_BF16 | resid


def policy_forward_emulated(cfg, weights, features, counts, mode: int | None = None, threads: int = 0):
    """Float64 forward with the precision recipe's rounding points (default: cfg's full recipe).
    Returns (logits f32 [B,N,P], value f32 [B], greedy actions int32 [B,N])."""
    lib = load()
    w = np.ascontiguousarray(weights, dtype=np.float32)
    f = np.ascontiguousarray(features, dtype=np.float32)
    c = np.ascontiguousarray(counts, dtype=np.int32)
    B = c.shape[0]
    logits = np.zeros((B, cfg.n_entities, cfg.actions), dtype=np.float32)
    value = np.zeros((B,), dtype=np.float32)
    actions = np.zeros((B, cfg.n_entities), dtype=np.int32)
    m = recipe_mode(cfg) if mode is None else int(mode)
    sh = shape_of(cfg)
    rc = lib.owo_policy_forward_emulated(C.byref(sh), w.ctypes.data, w.size, f.ctypes.data, c.ctypes.data, B, m,
                                         threads, logits.ctypes.data, value.ctypes.data, actions.ctypes.data)
    if rc != 0:
        raise ValueError(f"oracle rejected arguments (rc={rc})")
    return logits, value, actions


def gumbel_argmax(logits, counts, seed: int, state_base: int = 0, threads: int = 0):
    """Gumbel-max actions of the given logits [B,N,P] under the spec's Philox noise, and the top-two gap
    per entity (inf for padded entities). Returns (actions int32 [B,N], gap f32 [B,N])."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    c = np.ascontiguousarray(counts, dtype=np.int32)
    B, N, P = lg.shape
    actions = np.zeros((B, N), np.int32)
    gap = np.zeros((B, N), np.float32)
    rc = load().owo_gumbel_argmax(lg.ctypes.data, c.ctypes.data, B, N, P, C.c_uint64(seed), state_base, threads,
                                  actions.ctypes.data, gap.ctypes.data)
    if rc != 0:
        raise ValueError(f"oracle rejected arguments (rc={rc})")
    return actions, gap


def round_e4m3(v: float) -> float:
    return float(load().owo_round_e4m3(v))


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


def _planets(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=PLANET_DTYPE)


def encode_state(planets, initial_planets, comet_planet_ids, player: int, cfg: OwoEncoderConfig | None = None):
    """encode_state (encoder.rs:37-125) for one request -> (rows [R, 7] f32, ids [R] int32, flags [R] uint8,
    ships [R] f32, error code); error 0 = encoded, else the EncodeError index + 1 with empty rows."""
    cfg = cfg or default_encoder_config()
    p, i = _planets(planets), _planets(initial_planets)
    cm = np.ascontiguousarray(comet_planet_ids if comet_planet_ids is not None else [], dtype=np.int32)
    R = min(int(cfg.max_rows), 64)
    rows = np.zeros((R, 7), np.float32)
    ids = np.zeros(R, np.int32)
    flags = np.zeros(R, np.uint8)
    ships = np.zeros(R, np.float32)
    e = load().owo_encode_state(p.ctypes.data, p.size, i.ctypes.data, i.size, cm.ctypes.data, cm.size, int(player),
                                C.byref(cfg), rows.ctypes.data, ids.ctypes.data, flags.ctypes.data, ships.ctypes.data)
    return rows, ids, flags, ships, int(e)


def encode_batch(batch, request_games, request_players, cfg: OwoEncoderConfig | None = None, threads: int = 0):
    """A CSR batch (attributes planets, planet_offsets, initial_planets, initial_offsets, comet_planet_ids,
    comet_offsets) -> (rows [n, R, 7], ids [n, R], flags [n, R], ships [n, R], errors [n])."""
    cfg = cfg or default_encoder_config()
    p, i = _planets(batch.planets), _planets(batch.initial_planets)
    po = np.ascontiguousarray(batch.planet_offsets, dtype=np.uint64)
    io = np.ascontiguousarray(batch.initial_offsets, dtype=np.uint64)
    cm = None if batch.comet_planet_ids is None else np.ascontiguousarray(batch.comet_planet_ids, dtype=np.int32)
    co = None if batch.comet_offsets is None else np.ascontiguousarray(batch.comet_offsets, dtype=np.uint64)
    rg = np.ascontiguousarray(request_games, dtype=np.uint32)
    rp = np.ascontiguousarray(request_players, dtype=np.int32)
    n = rg.size
    R = min(int(cfg.max_rows), 64)
    rows = np.zeros((n, R, 7), np.float32)
    ids = np.zeros((n, R), np.int32)
    flags = np.zeros((n, R), np.uint8)
    ships = np.zeros((n, R), np.float32)
    errors = np.zeros(n, np.int32)
    load().owo_encode_batch(p.ctypes.data, po.ctypes.data, i.ctypes.data, io.ctypes.data,
                            None if cm is None else cm.ctypes.data, None if co is None else co.ctypes.data,
                            rg.ctypes.data, rp.ctypes.data, n, C.byref(cfg), rows.ctypes.data, ids.ctypes.data,
                            flags.ctypes.data, ships.ctypes.data, errors.ctypes.data, threads)
    return rows, ids, flags, ships, errors
