"""Game states for the device encoder: planets and the CSR batch the C ABI takes.

    batch = GameBatch.from_games([(planets, initial_planets, comet_ids), ...])
    rows = CudaTrue2D().encode_states(batch, request_games, request_players)

A planet is the engine's Planet (crates/orbit-wars-core/src/types.rs:6-16) as a
numpy record of PLANET_DTYPE, 36 bytes, the layout of OrbitWarsPlanet.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib

PLANET_DTYPE = np.dtype([("id", "<i4"), ("owner", "<i4"), ("x", "<f4"), ("y", "<f4"), ("radius", "<f4"),
                         ("ships", "<f4"), ("production", "<f4"), ("velocity_x", "<f4"), ("velocity_y", "<f4")])
assert PLANET_DTYPE.itemsize == 36

NO_PLANET_ID = -1   # types.rs:3
ROW_OWNED = 1       # ORBIT_WARS_ROW_OWNED
ROW_ABSENT = 2      # ORBIT_WARS_ROW_ABSENT
# ORBIT_WARS_ENCODE_*: EncodeError (encoder.rs:29-35) in declaration order after 0 = encoded
ENCODE_ERRORS = ("Ok", "InvalidConfig", "InvalidOwnerClass", "MissingHomePlanet", "RowOverflow")


def planets(rows) -> np.ndarray:
    """[(id, owner, x, y, radius, ships, production, velocity_x, velocity_y), ...] -> PLANET_DTYPE array."""
    if isinstance(rows, np.ndarray) and rows.dtype == PLANET_DTYPE:
        return np.ascontiguousarray(rows)
    return np.array([tuple(r) for r in rows], dtype=PLANET_DTYPE)


def default_config() -> _lib.EncoderConfigC:
    """orbit_wars_encoder_config_default: the defaults of crates/orbit-wars-core/src/config.rs:1-19."""
    cfg = _lib.EncoderConfigC()
    _lib.load_library().orbit_wars_encoder_config_default(C.byref(cfg))
    return cfg


@dataclass
class GameBatch:
    """OrbitWarsGameBatch: game g's planets are planets[planet_offsets[g]:planet_offsets[g + 1]], and so on."""
    planets: np.ndarray
    planet_offsets: np.ndarray
    initial_planets: np.ndarray
    initial_offsets: np.ndarray
    comet_planet_ids: np.ndarray | None = None
    comet_offsets: np.ndarray | None = None

    def __post_init__(self):
        self.planets = np.ascontiguousarray(self.planets, dtype=PLANET_DTYPE)
        self.initial_planets = np.ascontiguousarray(self.initial_planets, dtype=PLANET_DTYPE)
        self.planet_offsets = np.ascontiguousarray(self.planet_offsets, dtype=np.uint64)
        self.initial_offsets = np.ascontiguousarray(self.initial_offsets, dtype=np.uint64)
        if self.comet_planet_ids is not None:
            self.comet_planet_ids = np.ascontiguousarray(self.comet_planet_ids, dtype=np.int32)
            self.comet_offsets = np.ascontiguousarray(self.comet_offsets, dtype=np.uint64)

    @property
    def game_count(self) -> int:
        return self.planet_offsets.size - 1

    @classmethod
    def from_games(cls, games) -> "GameBatch":
        """games: iterable of (planets, initial_planets[, comet_planet_ids])."""
        ps, inits, comets = [], [], []
        any_comets = False
        for g in games:
            ps.append(planets(g[0]) if len(g[0]) else np.zeros(0, PLANET_DTYPE))
            inits.append(planets(g[1]) if len(g[1]) else np.zeros(0, PLANET_DTYPE))
            c = np.asarray(g[2] if len(g) > 2 and g[2] is not None else [], dtype=np.int32)
            any_comets |= c.size > 0
            comets.append(c)

        def csr(parts, dtype):
            off = np.zeros(len(parts) + 1, np.uint64)
            off[1:] = np.cumsum([p.size for p in parts])
            return (np.concatenate(parts) if parts else np.zeros(0, dtype)), off

        p, po = csr(ps, PLANET_DTYPE)
        i, io = csr(inits, PLANET_DTYPE)
        c, co = csr(comets, np.int32) if any_comets else (None, None)
        return cls(p, po, i, io, c, co)

    def c(self) -> _lib.GameBatchC:
        """The ctypes struct; valid while this batch is alive."""
        # zero-length arrays still need a valid pointer; keep the stand-ins alive on self
        self._keep = [np.zeros(1, PLANET_DTYPE), np.zeros(1, PLANET_DTYPE)]
        p = self.planets.ctypes.data if self.planets.size else self._keep[0].ctypes.data
        i = self.initial_planets.ctypes.data if self.initial_planets.size else self._keep[1].ctypes.data
        cm = None
        if self.comet_planet_ids is not None:
            if self.comet_planet_ids.size == 0:
                self._keep.append(np.zeros(1, np.int32))
                cm = self._keep[-1].ctypes.data
            else:
                cm = self.comet_planet_ids.ctypes.data
        return _lib.GameBatchC(p, self.planet_offsets.ctypes.data, i, self.initial_offsets.ctypes.data, cm,
                               None if self.comet_offsets is None else self.comet_offsets.ctypes.data,
                               self.game_count)
