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
        cap = 8
        arr = (_lib.KernelTimingC * cap)()
        n = C.c_int32(0)
        _lib.check("cuda_true2d_profile_end", self.lib.orbit_wars_cuda_true2d_profile_end(arr, cap, C.byref(n)))
        return {arr[i].name.decode(): (int(arr[i].launches), float(arr[i].total_ms)) for i in range(n.value)}

    def _decode_bufs(self, n: int, rows: int, row_planet_ids, source_owned, source_ships):
        ids = np.ascontiguousarray(row_planet_ids, dtype=np.int32).reshape(n, rows)
        own = np.ascontiguousarray(source_owned, dtype=np.uint8).reshape(n, rows)
        ships = np.ascontiguousarray(source_ships, dtype=np.float32).reshape(n, rows)
        tr = np.empty((n, rows, TARGETS), dtype=np.int32)
        sc = np.empty((n, rows, TARGETS), dtype=np.int32)
        return ids, own, ships, tr, sc

    def decode_population_resident(self, input_rows, model_indices, population_size: int, row_planet_ids,
                                   source_owned, source_ships, shape: True2DShape = True2DShape(),
                                   with_outputs: bool = False):
        """Resident forward + device decode: (target_rows, ship_counts[, outputs]) per (request, row, slot);
        target_rows -1 / ship_counts 0 where the decoder skips (decoder.rs:85-124)."""
        idx = np.ascontiguousarray(model_indices, dtype=np.uintp)
        n = idx.size
        x = _f32(input_rows)
        if x.size != n * shape.rows * INPUT_FEATURES:
            raise ValueError("cuda_true2d_decode_input_count_mismatch")
        if np.any(idx >= population_size):
            raise ValueError("cuda_true2d_decode_model_index_out_of_range")
        ids, own, ships, tr, sc = self._decode_bufs(n, shape.rows, row_planet_ids, source_owned, source_ships)
        out = np.zeros(n * shape.rows * OUTPUT_FEATURES, dtype=np.float32) if with_outputs else None
        _lib.check("cuda_true2d_decode_many_resident", self.lib.orbit_wars_cuda_true2d_decode_many_resident(
            x.ctypes.data, idx.ctypes.data, ids.ctypes.data, own.ctypes.data, ships.ctypes.data, tr.ctypes.data,
            sc.ctypes.data, None if out is None else out.ctypes.data, n, shape.c()))
        return (tr, sc, out.reshape(n, shape.rows, TARGETS, 2)) if with_outputs else (tr, sc)

    def decode_outputs(self, outputs, row_planet_ids, source_owned, source_ships, rows: int = 64):
        """Device decode of given outputs [n, rows, 12, 2] -> (target_rows, ship_counts)."""
        o = _f32(outputs)
        n = o.size // (rows * OUTPUT_FEATURES)
        ids, own, ships, tr, sc = self._decode_bufs(n, rows, row_planet_ids, source_owned, source_ships)
        _lib.check("cuda_true2d_decode_outputs", self.lib.orbit_wars_cuda_true2d_decode_outputs(
            o.ctypes.data, ids.ctypes.data, own.ctypes.data, ships.ctypes.data, tr.ctypes.data, sc.ctypes.data,
            n, rows))
        return tr, sc

