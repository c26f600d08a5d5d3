"""CPU restatement of the engine decoder's geometry-free part (test infrastructure).

crates/orbit-wars-core/src/decoder.rs:85-124 with target_row_from_fraction
(:457-461) and EncodedState::active_row_indices (encoder.rs:14-26): for each
request, active source rows owned by the player and on the map (planet_by_id
finds them, :93-98), each of the 12 target slots: target row from the fraction
over the active rows, skipped when it is the source or its planet is not on
the map (:112-114); send fraction clamped to [0, 1], skipped when <= 0; ship
count floor(ships * send), skipped when < 1. Row flags: 1 = the row's planet
belongs to the player, 2 = the row's planet is not on the map. Used only to
check the device decode.
"""
from __future__ import annotations

import numpy as np

NO_PLANET_ID = -1  # types.rs:3
TARGETS = 12
OWNED, ABSENT = 1, 2


def as_i32(v) -> int:
    """Rust's saturating `f32 as i32` (NaN -> 0)."""
    if np.isnan(v):
        return 0
    return int(min(max(float(v), -2147483648.0), 2147483647.0))


def decode(outputs, row_planet_ids, row_flags, source_ships):
    """outputs [n, rows, 12, 2] f32 -> (target_rows, ship_counts) [n, rows, 12] int32 (-1 / 0 when skipped)."""
    out = np.asarray(outputs, dtype=np.float32)
    n, rows = out.shape[:2]
    ids = np.asarray(row_planet_ids, dtype=np.int32).reshape(n, rows)
    flags = np.asarray(row_flags).astype(np.int64).reshape(n, rows)
    ships = np.asarray(source_ships, dtype=np.float32).reshape(n, rows)
    tr = np.full((n, rows, TARGETS), -1, dtype=np.int32)
    sc = np.zeros((n, rows, TARGETS), dtype=np.int32)
    for r in range(n):
        active = [i for i in range(rows) if ids[r, i] != NO_PLANET_ID]
        if not active:
            continue
        for s in range(rows):
            if ids[r, s] == NO_PLANET_ID or (flags[r, s] & (OWNED | ABSENT)) != OWNED:
                continue
            for a in range(TARGETS):
                tf, sf = out[r, s, a, 0], out[r, s, a, 1]
                if not (np.isfinite(tf) and np.isfinite(sf)):
                    raise ValueError("NonFiniteModelOutput")
                scaled = int(np.floor(np.float32(min(max(tf, np.float32(0)), np.float32(1))) * np.float32(len(active))))
                target = active[min(scaled, len(active) - 1)]
                if target == s or flags[r, target] & ABSENT:
                    continue
                send = np.float32(min(max(sf, np.float32(0)), np.float32(1)))
                if send <= 0:
                    continue
                count = as_i32(np.floor(np.float32(ships[r, s] * send)))
                if count < 1:
                    continue
                tr[r, s, a] = target
                sc[r, s, a] = count
    return tr, sc
