"""Host mirror of the engine's binding to the True2D GPU ABI.

Follows crates/orbit-wars-trainer/src/cuda_true2d.rs: the same five symbols
looked up at open (:10-15, :360-451), the same argument checks before each
call (:104-147, :149-173, :175-228, :230-273, :275-358) and the same output
unpacking with a finiteness check (:522-557). Outputs come back as
[requests, rows, 12, 2] arrays of (target_fraction, send_fraction).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from .games import ENCODE_ERRORS, GameBatch, default_config

INPUT_FEATURES = 7        # config.rs TRUE2D_INPUT_FEATURES
TARGETS = 12              # TRUE2D_ACTION_TARGETS_PER_SOURCE
OUTPUT_FEATURES = 24
ENGINE_SYMBOLS = (
    "orbit_wars_cuda_true2d_forward",
    "orbit_wars_cuda_true2d_forward_many",
    "orbit_wars_cuda_true2d_upload_population",
    "orbit_wars_cuda_true2d_forward_many_resident",
    "orbit_wars_cuda_true2d_train_full_attention",
)


@dataclass(frozen=True)
class True2DShape:
    layers: int = 61
    rows: int = 64
    heads: int = 1

    def c(self) -> _lib.True2DShapeC:
        return _lib.True2DShapeC(self.layers, self.rows, self.heads)

    def parameter_count(self) -> int:
        """true2d_model.rs:111-126."""
        cells = self.rows * self.rows
        return (INPUT_FEATURES * 2 + 2 * self.rows + cells + 1 + self.layers * cells * 12
                + self.heads * 7 + 6 + 2 * self.rows * TARGETS + 5 * TARGETS)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def unpack_outputs(out: np.ndarray, requests: int, shape: True2DShape) -> np.ndarray:
    if not np.all(np.isfinite(out)):
        raise _lib.OwError("cuda_true2d_unpack", 2, "cuda_true2d_non_finite_output")
    return out.reshape(requests, shape.rows, TARGETS, 2)


class CudaTrue2D:
    def __init__(self, path=None):
        self.lib = _lib.load_library(path)
        for s in ENGINE_SYMBOLS:  # open() fails when any engine symbol is missing
            getattr(self.lib, s)

    @classmethod
    def open_from_environment(cls) -> "CudaTrue2D":
        return cls()

    def forward_packed(self, input_rows, weights, game_count: int, shape: True2DShape = True2DShape()) -> np.ndarray:
        x, w = _f32(input_rows), _f32(weights)
        if x.size != game_count * shape.rows * INPUT_FEATURES:
            raise ValueError("cuda_true2d_input_count_mismatch")
        if w.size != shape.parameter_count():
            raise ValueError("cuda_true2d_weight_count_mismatch")
        out = np.zeros(game_count * shape.rows * OUTPUT_FEATURES, dtype=np.float32)
        _lib.check("cuda_true2d_forward", self.lib.orbit_wars_cuda_true2d_forward(
            x.ctypes.data, w.ctypes.data, out.ctypes.data, game_count, shape.c()))
        return unpack_outputs(out, game_count, shape)

    def upload_population(self, population: np.ndarray, request_capacity: int,
                          shape: True2DShape = True2DShape()) -> None:
        if request_capacity == 0:
            raise ValueError("cuda_true2d_upload_request_capacity_zero")
        w = _f32(population).reshape(-1, shape.parameter_count())
        _lib.check("cuda_true2d_upload_population", self.lib.orbit_wars_cuda_true2d_upload_population(
            w.ctypes.data, w.shape[0], request_capacity, shape.c()))

    def forward_population_packed(self, input_rows, model_indices, population,
                                  shape: True2DShape = True2DShape()) -> np.ndarray:
        idx = np.ascontiguousarray(model_indices, dtype=np.uintp)
        n = idx.size
        if n == 0:
            return np.zeros((0, shape.rows, TARGETS, 2), dtype=np.float32)
        w = _f32(population).reshape(-1, shape.parameter_count())
        x = _f32(input_rows)
        if x.size != n * shape.rows * INPUT_FEATURES:
            raise ValueError("cuda_true2d_many_input_count_mismatch")
        if np.any(idx >= w.shape[0]):
            raise ValueError("cuda_true2d_many_model_index_out_of_range")
        out = np.zeros(n * shape.rows * OUTPUT_FEATURES, dtype=np.float32)
        _lib.check("cuda_true2d_forward_many", self.lib.orbit_wars_cuda_true2d_forward_many(
            x.ctypes.data, idx.ctypes.data, w.ctypes.data, out.ctypes.data, n, w.shape[0], shape.c()))
        return unpack_outputs(out, n, shape)

    def forward_population_resident_packed(self, input_rows, model_indices, population_size: int,
                                           shape: True2DShape = True2DShape()) -> np.ndarray:
        idx = np.ascontiguousarray(model_indices, dtype=np.uintp)
        n = idx.size
        if n == 0:
            return np.zeros((0, shape.rows, TARGETS, 2), dtype=np.float32)
        x = _f32(input_rows)
        if x.size != n * shape.rows * INPUT_FEATURES:
            raise ValueError("cuda_true2d_resident_input_count_mismatch")
        if np.any(idx >= population_size):
            raise ValueError("cuda_true2d_resident_model_index_out_of_range")
        out = np.zeros(n * shape.rows * OUTPUT_FEATURES, dtype=np.float32)
        _lib.check("cuda_true2d_forward_many_resident", self.lib.orbit_wars_cuda_true2d_forward_many_resident(
            x.ctypes.data, idx.ctypes.data, out.ctypes.data, n, shape.c()))
        return unpack_outputs(out, n, shape)

    def profile_begin(self, max_calls: int) -> None:
        """Arms device timing of each kernel of the next `max_calls` forward calls."""
        _lib.check("cuda_true2d_profile_begin", self.lib.orbit_wars_cuda_true2d_profile_begin(int(max_calls)))

    def profile_end(self) -> dict:
        """{kernel: (launches, total_ms)} over the calls since profile_begin."""
        cap = 16
        arr = (_lib.KernelTimingC * cap)()
        n = C.c_int32(0)
        _lib.check("cuda_true2d_profile_end", self.lib.orbit_wars_cuda_true2d_profile_end(arr, cap, C.byref(n)))
        return {arr[i].name.decode(): (int(arr[i].launches), float(arr[i].total_ms)) for i in range(n.value)}

    def _decode_bufs(self, n: int, rows: int, row_planet_ids, row_flags, source_ships):
        ids = np.ascontiguousarray(row_planet_ids, dtype=np.int32).reshape(n, rows)
        own = np.ascontiguousarray(row_flags, dtype=np.uint8).reshape(n, rows)
        ships = np.ascontiguousarray(source_ships, dtype=np.float32).reshape(n, rows)
        tr = np.empty((n, rows, TARGETS), dtype=np.int32)
        sc = np.empty((n, rows, TARGETS), dtype=np.int32)
        return ids, own, ships, tr, sc

    def decode_population_resident(self, input_rows, model_indices, population_size: int, row_planet_ids,
                                   row_flags, source_ships, shape: True2DShape = True2DShape(),
                                   with_outputs: bool = False):
        """Resident forward + device decode: (target_rows, ship_counts[, outputs]) per (request, row, slot);
        target_rows -1 / ship_counts 0 where the decoder skips (decoder.rs:85-124). row_flags per row:
        ROW_OWNED (the planet belongs to the player) | ROW_ABSENT (the planet is not on the map)."""
        idx = np.ascontiguousarray(model_indices, dtype=np.uintp)
        n = idx.size
        x = _f32(input_rows)
        if x.size != n * shape.rows * INPUT_FEATURES:
            raise ValueError("cuda_true2d_decode_input_count_mismatch")
        if np.any(idx >= population_size):
            raise ValueError("cuda_true2d_decode_model_index_out_of_range")
        ids, own, ships, tr, sc = self._decode_bufs(n, shape.rows, row_planet_ids, row_flags, source_ships)
        out = np.zeros(n * shape.rows * OUTPUT_FEATURES, dtype=np.float32) if with_outputs else None
        _lib.check("cuda_true2d_decode_many_resident", self.lib.orbit_wars_cuda_true2d_decode_many_resident(
            x.ctypes.data, idx.ctypes.data, ids.ctypes.data, own.ctypes.data, ships.ctypes.data, tr.ctypes.data,
            sc.ctypes.data, None if out is None else out.ctypes.data, n, shape.c()))
        return (tr, sc, out.reshape(n, shape.rows, TARGETS, 2)) if with_outputs else (tr, sc)

    def decode_outputs(self, outputs, row_planet_ids, row_flags, source_ships, rows: int = 64):
        """Device decode of given outputs [n, rows, 12, 2] -> (target_rows, ship_counts)."""
        o = _f32(outputs)
        n = o.size // (rows * OUTPUT_FEATURES)
        ids, own, ships, tr, sc = self._decode_bufs(n, rows, row_planet_ids, row_flags, source_ships)
        _lib.check("cuda_true2d_decode_outputs", self.lib.orbit_wars_cuda_true2d_decode_outputs(
            o.ctypes.data, ids.ctypes.data, own.ctypes.data, ships.ctypes.data, tr.ctypes.data, sc.ctypes.data,
            n, rows))
        return tr, sc


    # ---- training step (orbit_wars_cuda.cu:2823-3330) ---------------------------------------------------------
    def train_full_attention(self, input_rows, output_rows, rewards, target_action_rewards, model_indices,
                             all_weights, shape: True2DShape = True2DShape(), batch_sample_count: int = 64,
                             learning_rate: float = 1e-3, reward_normalizer: float = 1.0, send_threshold: float = 0.5,
                             owner_class_own: float = 1.0, owner_class_empty: float = -0.5,
                             owner_class_absent_on_map: float = -1.0, inplace: bool = False) -> np.ndarray:
        """One SGD step; returns the updated weights (models x parameter_count): a new array, or with
        inplace=True the given float32 C-contiguous array itself, updated where it lies (as the engine's
        host buffer is)."""
        x = _f32(input_rows)
        o = _f32(output_rows)
        r = np.ascontiguousarray(rewards, dtype=np.int32)
        tar = _f32(target_action_rewards)
        idx = np.ascontiguousarray(model_indices, dtype=np.uintp)
        if inplace:
            w = all_weights
            if not (isinstance(w, np.ndarray) and w.dtype == np.float32 and w.flags.c_contiguous):
                raise ValueError("inplace training needs a float32 C-contiguous weight array")
        else:
            w = np.array(all_weights, dtype=np.float32, copy=True, order="C")
        n = idx.size
        models = w.size // shape.parameter_count()
        cfg = _lib.TrainingConfigC(batch_sample_count, learning_rate, reward_normalizer, send_threshold,
                                   owner_class_own, owner_class_empty, owner_class_absent_on_map)
        _lib.check("cuda_true2d_train_full_attention", self.lib.orbit_wars_cuda_true2d_train_full_attention(
            x.ctypes.data, o.ctypes.data, r.ctypes.data, tar.ctypes.data, idx.ctypes.data, w.ctypes.data, n, models,
            shape.c(), cfg))
        return w.reshape(models, shape.parameter_count())

    # ---- device encoder (encoder.rs:37-208) ----------------------------------------------------------------
    @staticmethod
    def _requests(request_games, request_players):
        rg = np.ascontiguousarray(request_games, dtype=np.uint32)
        rp = np.ascontiguousarray(request_players, dtype=np.int32)
        if rg.shape != rp.shape or rg.ndim != 1:
            raise ValueError("encode_request_shape_mismatch")
        return rg, rp

    def encode_states(self, batch: GameBatch, request_games, request_players, config=None, strict: bool = True):
        """encode_state for every request on the device -> EncodedRows(rows [n, R, 7], row_planet_ids [n, R],
        row_flags [n, R], row_ships [n, R], errors [n]). strict: raise when a request fails to encode
        (the call's BAD_ARGUMENT); otherwise return its empty rows with its error code."""
        cfg = config if config is not None else default_config()
        rg, rp = self._requests(request_games, request_players)
        n, R = rg.size, int(cfg.max_rows)
        rows = np.empty((n, R, INPUT_FEATURES), np.float32)
        ids = np.empty((n, R), np.int32)
        flags = np.empty((n, R), np.uint8)
        ships = np.empty((n, R), np.float32)
        errors = np.empty(n, np.int32)
        bc = batch.c()
        st = self.lib.orbit_wars_cuda_encode_states(C.byref(bc), rg.ctypes.data, rp.ctypes.data, n, C.byref(cfg),
                                                    rows.ctypes.data, ids.ctypes.data, flags.ctypes.data,
                                                    ships.ctypes.data, errors.ctypes.data)
        if st.code != 0 and (strict or not (st.message or b"").startswith(b"encode failed")):
            _lib.check("cuda_encode_states", st)
        return EncodedRows(rows, ids, flags, ships, errors)

    def play_population_resident(self, batch: GameBatch, request_games, request_players, model_indices,
                                 population_size: int, shape: True2DShape = True2DShape(), config=None,
                                 with_rows: bool = False, with_outputs: bool = False):
        """Encode + resident forward + decode on the device, one call:
        (row_planet_ids [n, R], target_rows [n, R, 12], ship_counts [n, R, 12][, rows][, outputs])."""
        cfg = config if config is not None else default_config()
        rg, rp = self._requests(request_games, request_players)
        idx = np.ascontiguousarray(model_indices, dtype=np.uintp)
        n, R = rg.size, shape.rows
        if idx.size != n:
            raise ValueError("cuda_true2d_play_model_index_count_mismatch")
        if np.any(idx >= population_size):
            raise ValueError("cuda_true2d_play_model_index_out_of_range")
        ids = np.empty((n, R), np.int32)
        tr = np.empty((n, R, TARGETS), np.int32)
        sc = np.empty((n, R, TARGETS), np.int32)
        rows = np.empty((n, R, INPUT_FEATURES), np.float32) if with_rows else None
        out = np.empty((n, R, TARGETS, 2), np.float32) if with_outputs else None
        bc = batch.c()
        _lib.check("cuda_true2d_play_many_resident", self.lib.orbit_wars_cuda_true2d_play_many_resident(
            C.byref(bc), rg.ctypes.data, rp.ctypes.data, idx.ctypes.data, n, C.byref(cfg), ids.ctypes.data,
            tr.ctypes.data, sc.ctypes.data, None, None if rows is None else rows.ctypes.data,
            None if out is None else out.ctypes.data, shape.c()))
        res = (ids, tr, sc)
        if with_rows:
            res += (rows,)
        if with_outputs:
            res += (out,)
        return res


@dataclass
class EncodedRows:
    rows: np.ndarray
    row_planet_ids: np.ndarray
    row_flags: np.ndarray
    row_ships: np.ndarray
    errors: np.ndarray

    def error_names(self) -> list[str]:
        return [ENCODE_ERRORS[int(e)] for e in self.errors]
