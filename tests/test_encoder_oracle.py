"""The encoder oracle (oracle/encoder_oracle.cpp) pinned to the reference's own
encoder and scaler tests (crates/orbit-wars-core/src/encoder.rs:210-324,
scaler.rs:14-37), cross-checked against a pure-Python restatement of
encode_state on small synthetic games, and the encoder ABI's host-side checks
(no GPU needed)."""
import ctypes as C
import math

import numpy as np
import pytest

import orbit_wars_b200 as ow
from orbit_wars_b200 import games, synth
from oracle import bind

CFG = bind.default_encoder_config()
OWN, E1, E2, E3, NEUTRAL, EMPTY, ABSENT = 1.0, 0.75, 0.5, 0.25, 0.0, -0.5, -1.0


def planet(pid, owner, x, y, ships):
    """encoder.rs:214-226: radius 1, production 1, velocity (3, -1.5)."""
    return (pid, owner, x, y, 1.0, ships, 1.0, 3.0, -1.5)


def test_row_zero_is_home_planet_and_initial_rows_are_distance_sorted():
    initial = [planet(10, 1, 10.0, 10.0, 10.0), planet(20, -1, 20.0, 10.0, 10.0), planet(30, -1, 90.0, 90.0, 10.0)]
    rows, ids, _, _, err = bind.encode_state(initial, initial, [], 1)
    assert err == 0
    assert list(ids[:3]) == [10, 20, 30]
    assert rows[0, 0] == OWN and rows[1, 0] == NEUTRAL
    f32 = np.float32
    assert rows[0, 2] == f32(0.1) and rows[0, 3] == f32(0.1) and rows[0, 4] == f32(0.2)
    assert rows[0, 5] == f32(0.5) and rows[0, 6] == f32(-0.25)
    assert rows[1, 2] == f32(0.2) and rows[1, 3] == f32(0.1) and rows[1, 4] == f32(0.2)
    assert rows[1, 5] == f32(0.5) and rows[1, 6] == f32(-0.25)


def test_owner_class_encodes_three_enemies_neutral_absent_and_empty_rows():
    initial = [planet(10, 0, 10.0, 10.0, 10.0), planet(20, 1, 20.0, 10.0, 10.0), planet(30, 2, 30.0, 10.0, 10.0),
               planet(40, 3, 40.0, 10.0, 10.0), planet(50, -1, 50.0, 10.0, 10.0), planet(60, -1, 60.0, 10.0, 10.0)]
    current = [p for p in initial if p[0] != 60]
    rows, ids, flags, _, err = bind.encode_state(current, initial, [], 0)
    assert err == 0
    assert list(rows[:6, 0]) == [OWN, E1, E2, E3, NEUTRAL, ABSENT]
    assert rows[CFG.initial_planet_slots, 0] == EMPTY
    assert np.all(rows[5, 1:] == 0.0)
    assert flags[5] == games.ROW_ABSENT and flags[0] == games.ROW_OWNED and flags[1] == 0


def test_owner_class_for_player_one_maps_single_lower_id_enemy_to_enemy_one():
    initial = [planet(10, 1, 10.0, 10.0, 10.0), planet(20, 0, 20.0, 10.0, 10.0)]
    rows, _, _, _, err = bind.encode_state(initial, initial, [], 1)
    assert err == 0 and rows[0, 0] == OWN and rows[1, 0] == E1


def test_official_initial_planets_can_have_neutral_home_owner():
    initial = [planet(10, -1, 10.0, 10.0, 10.0), planet(20, -1, 20.0, 10.0, 10.0)]
    current = [planet(10, 0, 10.0, 10.0, 10.0), planet(20, -1, 20.0, 10.0, 10.0)]
    rows, ids, _, _, err = bind.encode_state(current, initial, [], 0)
    assert err == 0 and ids[0] == 10 and rows[0, 0] == OWN


def ship_scaled(ships):
    p = [planet(1, 0, 10.0, 10.0, ships)]
    return bind.encode_state(p, p, [], 0)[0][0, 1]


def test_ship_scaler_known_answers():
    """scaler.rs:19-36: 0 -> 0; pivot -> 0.9 and 2 x cap -> 1 within 1e-6."""
    assert ship_scaled(0.0) == 0.0
    assert abs(ship_scaled(CFG.ship_log_pivot) - 0.9) < 1e-6
    assert abs(ship_scaled(CFG.ship_log_cap * 2.0) - 1.0) < 1e-6
    assert ship_scaled(-5.0) == 0.0 and ship_scaled(float("nan")) == 0.0 and ship_scaled(float("inf")) == 1.0


def test_nan_distances_order_as_on_x86():
    """total_cmp on the reference's x86-64 NaNs: a NaN coordinate propagates its (positive) NaN, sorted after
    every number; inf - inf gives the default NaN 0xFFC00000, sorted before every number."""
    nan, inf = float("nan"), float("inf")
    g = [planet(1, 0, 10.0, 10.0, 1.0), planet(2, -1, nan, 10.0, 1.0), planet(3, -1, 30.0, 10.0, 1.0),
         planet(4, -1, 12.0, 11.0, 1.0)]
    assert list(bind.encode_state(g, g, [], 0)[1][:4]) == [1, 4, 3, 2]
    g = [planet(1, 0, inf, 10.0, 1.0), planet(2, -1, inf, 20.0, 1.0), planet(3, -1, 10.0, 10.0, 1.0),
         planet(4, -1, -inf, 5.0, 1.0)]
    assert list(bind.encode_state(g, g, [], 0)[1][:4]) == [1, 2, 3, 4]


def test_errors():
    p = [planet(1, 0, 10.0, 10.0, 5.0), planet(2, 1, 20.0, 10.0, 5.0)]
    assert bind.encode_state(p, p, [], 3)[4] == 3  # MissingHomePlanet
    assert bind.encode_state([], [], [], 0)[4] == 3
    bad_owner = [planet(1, 0, 10.0, 10.0, 5.0), planet(2, 7, 20.0, 10.0, 5.0)]
    rows, ids, _, _, err = bind.encode_state(bad_owner, bad_owner, [], 0)
    assert err == 2 and np.all(ids == -1) and np.all(rows[:, 0] == EMPTY)  # InvalidOwnerClass, empty rows
    # a player id outside 0..3 owns its home (owner == player), but any other owner is invalid
    big = [planet(1, 9, 10.0, 10.0, 5.0), planet(2, -1, 20.0, 10.0, 5.0)]
    assert bind.encode_state(big, big, [], 9)[4] == 0
    big.append(planet(3, 1, 30.0, 10.0, 5.0))
    assert bind.encode_state(big, big, [], 9)[4] == 2
    cfg = bind.default_encoder_config()
    cfg.padding_slots = 5  # slots no longer sum to max_rows
    assert bind.encode_state(p, p, [], 0, cfg)[4] == 1


# ---- pure-Python restatement of encode_state (encoder.rs:37-208), small cases only ---------------------------
def total_key(v):
    b = int(np.array([v], np.float32).view(np.int32)[0])
    return b ^ ((b >> 31) & 0x7FFFFFFF)


def py_encode(cur, init, comets, player):
    f32 = np.float32
    R = 64
    rows = np.zeros((R, 7), np.float32)
    rows[:, 0] = EMPTY
    ids = np.full(R, -1, np.int32)
    home = next((p for p in cur if p["owner"] == player), None)
    if home is None:
        return rows, ids, 3

    def d2(p):
        dx = f32(p["x"]) - f32(home["x"])
        dy = f32(p["y"]) - f32(home["y"])
        return f32(f32(dx * dx) + f32(dy * dy))

    def owner_class(owner):
        if owner < 0:
            return NEUTRAL
        if owner == player:
            return OWN
        if player < 0 or owner >= 4 or player >= 4:
            return None
        return (E1, E2, E3)[[c for c in range(4) if c != player].index(owner)]

    def ship_log(s):
        s = f32(max(s, f32(0.0))) if not np.isnan(s) else f32(0.0)
        if s <= 1000.0:
            return f32(f32(f32(0.9) * np.log(f32(1.0) + s)) / np.log(f32(1001.0)))
        up = f32(np.log(f32(s / f32(1000.0))) / np.log(f32(100.0)))
        return f32(f32(0.9) + f32(f32(0.1) * min(max(up, f32(0.0)), f32(1.0))))

    order = []
    order.append(home["id"])
    rest = sorted([p for p in init if p["id"] != home["id"]], key=lambda p: total_key(d2(p)))
    order += [p["id"] for p in rest[:39]]
    comet_rows = sorted([p for p in cur if p["id"] in list(comets)],
                        key=lambda p: (list(comets).index(p["id"]), total_key(d2(p))))
    assign = list(enumerate(order)) + [(40 + k, p["id"]) for k, p in enumerate(comet_rows[:20])]
    for row, pid in assign:
        ids[row] = pid
        c = next((p for p in cur if p["id"] == pid), None)
        if c is None:
            rows[row] = (ABSENT, 0, 0, 0, 0, 0, 0)
            continue
        oc = owner_class(int(c["owner"]))
        if oc is None:
            rows[:] = 0
            rows[:, 0] = EMPTY
            ids[:] = -1
            return rows, ids, 2
        rows[row] = (oc, ship_log(f32(c["ships"])), f32(c["x"]) / f32(100.0), f32(c["y"]) / f32(100.0),
                     min(max(f32(c["production"]) / f32(5.0), 0.0), 1.0),
                     min(max(f32(c["velocity_x"]) / f32(6.0), -1.0), 1.0),
                     min(max(f32(c["velocity_y"]) / f32(6.0), -1.0), 1.0))
    return rows, ids, 0


def test_oracle_matches_python_restatement_on_synthetic_games():
    batch, rg, rp = synth.game_batch(7, 24, players=4, max_groups=12)
    rows, ids, flags, ships, errors = bind.encode_batch(batch, rg, rp)
    po, io, co = batch.planet_offsets, batch.initial_offsets, batch.comet_offsets
    for r in range(rg.size):
        g = int(rg[r])
        cur = batch.planets[po[g]:po[g + 1]]
        init = batch.initial_planets[io[g]:io[g + 1]]
        cm = batch.comet_planet_ids[co[g]:co[g + 1]]
        prow, pids, perr = py_encode(cur, init, cm, int(rp[r]))
        assert perr == errors[r]
        assert np.array_equal(pids, ids[r])
        # ship_log_percent: glibc logf vs numpy's float32 log may differ in the last bit
        np.testing.assert_array_equal(np.delete(prow, 1, axis=1), np.delete(rows[r], 1, axis=1))
        np.testing.assert_allclose(prow[:, 1], rows[r][:, 1], rtol=0, atol=2e-7)


def test_oracle_properties_on_synthetic_games():
    batch, rg, rp = synth.game_batch(3, 64, players=2)
    rows, ids, flags, ships, errors = bind.encode_batch(batch, rg, rp)
    assert np.all(errors == 0)
    assert np.all(rows[:, 0, 0] == OWN) and np.all(flags[:, 0] == games.ROW_OWNED)
    # empty rows exactly where there is no id; absent rows exactly where the flag says so
    assert np.array_equal(ids == -1, rows[..., 0] == EMPTY)
    assert np.array_equal(flags == games.ROW_ABSENT, rows[..., 0] == ABSENT)
    assert np.all(ids[:, 60:] == -1)  # padding rows


def test_encoder_config_default_matches_config_rs():
    lib = ow.load_library()
    got = games.default_config()
    want = bind.default_encoder_config()
    for name, _ in bind.OwoEncoderConfig._fields_:
        assert getattr(got, name) == getattr(want, name), name
    assert lib is not None


def test_encode_abi_rejects_bad_arguments_before_the_device():
    """Config and batch checks return BAD_ARGUMENT (1) without touching a device."""
    lib = ow.load_library()
    batch, rg, rp = synth.game_batch(1, 2, players=2)
    n = rg.size
    out = [np.zeros((n, 64, 7), np.float32), np.zeros((n, 64), np.int32), np.zeros((n, 64), np.uint8)]
    cfg = games.default_config()
    cfg.comet_slots = 21
    bc = batch.c()
    st = lib.orbit_wars_cuda_encode_states(C.byref(bc), rg.ctypes.data, rp.ctypes.data, n, C.byref(cfg),
                                           out[0].ctypes.data, out[1].ctypes.data, out[2].ctypes.data, None, None)
    assert st.code == 1 and b"config" in st.message
    cfg = games.default_config()
    bad_rg = rg.copy()
    bad_rg[0] = 99
    st = lib.orbit_wars_cuda_encode_states(C.byref(bc), bad_rg.ctypes.data, rp.ctypes.data, n, C.byref(cfg),
                                           out[0].ctypes.data, out[1].ctypes.data, out[2].ctypes.data, None, None)
    assert st.code == 1 and b"out of range" in st.message
    bad_off = batch.planet_offsets.copy()
    bad_off[1], bad_off[2] = bad_off[2], bad_off[1]
    b2 = ow.GameBatch(batch.planets, bad_off, batch.initial_planets, batch.initial_offsets,
                      batch.comet_planet_ids, batch.comet_offsets)
    bc2 = b2.c()
    st = lib.orbit_wars_cuda_encode_states(C.byref(bc2), rg.ctypes.data, rp.ctypes.data, n, C.byref(cfg),
                                           out[0].ctypes.data, out[1].ctypes.data, out[2].ctypes.data, None, None)
    assert st.code == 1 and b"offsets" in st.message


def test_total_order_key_matches_rust_total_cmp():
    vals = np.array([-np.inf, -1.0, -0.0, 0.0, 1e-45, 1.0, np.inf, np.nan], np.float32)
    keys = [total_key(v) for v in vals]
    assert keys == sorted(keys) and len(set(keys)) == len(keys)
    assert math.isnan(vals[-1])
