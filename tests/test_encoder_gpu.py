"""Device encoder (orbit_wars_cuda_encode_states) and the fused device turn
(orbit_wars_cuda_true2d_play_many_resident) against the encoder oracle
(oracle/encoder_oracle.cpp, a restatement of crates/orbit-wars-core/src/
encoder.rs:37-208) and the reference's own encoder tests.

Tolerance: planet ids, row flags, ships, errors and six of the seven features
are bit-exact; ship_log_percent (feature 1) is within 2e-7 absolute, since the
device's ln (double, rounded to f32) and glibc's logf may differ in the last
bit of a value <= 1."""
import numpy as np
import pytest

import orbit_wars_b200 as ow
from orbit_wars_b200 import games, synth
from oracle import bind
from oracle import decode as dec

pytestmark = pytest.mark.gpu
SHAPE = ow.True2DShape(61, 64, 1)
SHIP_ATOL = 2e-7


def assert_matches_oracle(got: ow.EncodedRows, want):
    rows, ids, flags, ships, errors = want
    assert np.array_equal(got.errors, errors)
    assert np.array_equal(got.row_planet_ids, ids)
    assert np.array_equal(got.row_flags, flags)
    assert np.array_equal(got.row_ships, ships, equal_nan=True)
    np.testing.assert_array_equal(np.delete(got.rows, 1, axis=2), np.delete(rows, 1, axis=2))
    np.testing.assert_allclose(got.rows[..., 1], rows[..., 1], rtol=0, atol=SHIP_ATOL)


def planet(pid, owner, x, y, ships):
    return (pid, owner, x, y, 1.0, ships, 1.0, 3.0, -1.5)


def test_reference_encoder_known_answers_on_device():
    lib = ow.CudaTrue2D()
    initial = [planet(10, 1, 10.0, 10.0, 10.0), planet(20, -1, 20.0, 10.0, 10.0), planet(30, -1, 90.0, 90.0, 10.0)]
    # encoder.rs:228-255 and :257-292 in one batch
    initial2 = [planet(10, 0, 10.0, 10.0, 10.0), planet(20, 1, 20.0, 10.0, 10.0), planet(30, 2, 30.0, 10.0, 10.0),
                planet(40, 3, 40.0, 10.0, 10.0), planet(50, -1, 50.0, 10.0, 10.0), planet(60, -1, 60.0, 10.0, 10.0)]
    current2 = [p for p in initial2 if p[0] != 60]
    batch = ow.GameBatch.from_games([(initial, initial), (current2, initial2)])
    e = lib.encode_states(batch, [0, 1], [1, 0])
    assert list(e.errors) == [0, 0]
    assert list(e.row_planet_ids[0, :3]) == [10, 20, 30]
    f32 = np.float32
    assert e.rows[0, 0, 0] == 1.0 and e.rows[0, 1, 0] == 0.0
    assert tuple(e.rows[0, 0, 2:]) == (f32(0.1), f32(0.1), f32(0.2), f32(0.5), f32(-0.25))
    assert tuple(e.rows[0, 1, 2:]) == (f32(0.2), f32(0.1), f32(0.2), f32(0.5), f32(-0.25))
    assert list(e.rows[1, :6, 0]) == [1.0, 0.75, 0.5, 0.25, 0.0, -1.0]
    assert e.rows[1, 40, 0] == -0.5 and np.all(e.rows[1, 5, 1:] == 0.0)
    # :294-305 and :307-323
    b3 = ow.GameBatch.from_games([
        ([planet(10, 1, 10.0, 10.0, 10.0), planet(20, 0, 20.0, 10.0, 10.0)],) * 2,
        ([planet(10, 0, 10.0, 10.0, 10.0), planet(20, -1, 20.0, 10.0, 10.0)],
         [planet(10, -1, 10.0, 10.0, 10.0), planet(20, -1, 20.0, 10.0, 10.0)])])
    e3 = lib.encode_states(b3, [0, 1], [1, 0])
    assert e3.rows[0, 0, 0] == 1.0 and e3.rows[0, 1, 0] == 0.75
    assert e3.row_planet_ids[1, 0] == 10 and e3.rows[1, 0, 0] == 1.0


@pytest.mark.parametrize("seed,games_n,players,max_groups", [(1, 300, 4, 10), (2, 200, 2, 14), (3, 57, 4, 12)])
def test_encode_matches_oracle_on_synthetic_games(seed, games_n, players, max_groups):
    batch, rg, rp = synth.game_batch(seed, games_n, players=players, max_groups=max_groups)
    got = ow.CudaTrue2D().encode_states(batch, rg, rp)
    assert_matches_oracle(got, bind.encode_batch(batch, rg, rp))
    assert np.mean(got.rows[..., 1] == bind.encode_batch(batch, rg, rp)[0][..., 1]) > 0.99


def test_encode_edge_cases_match_oracle():
    nan, inf = float("nan"), float("inf")
    g = []
    # 0: NaN / inf / negative ships and a NaN coordinate (total_cmp puts NaN distances last)
    g.append(([planet(1, 0, 10.0, 10.0, nan), planet(2, 1, nan, 10.0, inf), planet(3, -1, 30.0, 10.0, -4.0),
               planet(4, 2, 12.0, 11.0, 1e9)],
              [planet(1, 0, 10.0, 10.0, 0.0), planet(2, -1, nan, 10.0, 0.0), planet(3, -1, 30.0, 10.0, 0.0),
               planet(4, -1, 12.0, 11.0, 0.0)]))
    # 1: duplicate ids (the first planet with an id wins the lookup), ties in distance
    g.append(([planet(5, 0, 50.0, 50.0, 3.0), planet(6, 1, 60.0, 50.0, 3.0), planet(6, 2, 40.0, 50.0, 3.0),
               planet(7, -1, 50.0, 60.0, 3.0)],
              [planet(7, -1, 50.0, 60.0, 0.0), planet(6, -1, 60.0, 50.0, 0.0), planet(8, -1, 40.0, 50.0, 0.0),
               planet(5, -1, 50.0, 50.0, 0.0)]))
    # 2: more than 39 initial planets (truncated) and more than 20 comets (truncated), comets listed twice
    cur = [planet(0, 3, 50.0, 50.0, 9.0)] + [planet(100 + k, -1, 50.0 + k * 0.7, 40.0, k) for k in range(30)]
    init = [planet(k, -1, (k * 37) % 100, (k * 53) % 100, 0.0) for k in range(70)]
    comets = [100 + (k * 7) % 30 for k in range(30)] + [100, 101]
    g.append((cur, init, comets))
    # 3: missing home; 4: invalid owner; 5: no initial planets at all
    g.append(([planet(1, 1, 10.0, 10.0, 1.0)], [planet(1, 1, 10.0, 10.0, 1.0)]))
    g.append(([planet(1, 0, 10.0, 10.0, 1.0), planet(2, 5, 20.0, 10.0, 1.0)], [planet(2, -1, 20.0, 10.0, 1.0)]))
    g.append(([planet(1, 2, 10.0, 10.0, 1.0), planet(2, 0, 20.0, 20.0, 1.0)], []))
    # 6: infinite coordinates: inf - inf is x86's default NaN (sign bit set), which total_cmp sorts first
    inf_game = [planet(1, 0, inf, 10.0, 1.0), planet(2, -1, inf, 20.0, 1.0), planet(3, -1, 10.0, 10.0, 1.0),
                planet(4, -1, -inf, 5.0, 1.0)]
    g.append((inf_game, inf_game))
    batch = ow.GameBatch.from_games(g)
    rg = [0, 0, 1, 1, 1, 2, 3, 4, 5, 5, 6]
    rp = [0, 1, 0, 1, 2, 3, 0, 0, 2, 0, 0]
    got = ow.CudaTrue2D().encode_states(batch, rg, rp, strict=False)
    want = bind.encode_batch(batch, rg, rp)
    assert_matches_oracle(got, want)
    assert list(got.errors) == [0, 0, 0, 0, 0, 0, 3, 2, 0, 0, 0]
    assert list(got.row_planet_ids[0, :4]) == [1, 4, 3, 2]  # the NaN distance last
    assert list(got.row_planet_ids[10, :4]) == [1, 2, 3, 4]  # the default NaN first
    with pytest.raises(ow.OwError) as e:
        ow.CudaTrue2D().encode_states(batch, rg, rp)
    assert e.value.code == 1 and "MissingHomePlanet" in str(e.value)


def test_encode_large_game_uses_dynamic_shared_memory():
    rng = np.random.default_rng(9)
    n_p = 3000
    cur = np.zeros(n_p, games.PLANET_DTYPE)
    cur["id"] = rng.permutation(n_p)
    cur["owner"] = rng.integers(-1, 4, n_p)
    cur["x"], cur["y"] = rng.uniform(0, 100, n_p), rng.uniform(0, 100, n_p)
    cur["ships"] = rng.uniform(0, 5000, n_p)
    cur["production"] = rng.integers(1, 6, n_p)
    init = cur.copy()
    init["owner"] = -1
    comets = cur["id"][rng.choice(n_p, 400, replace=False)]
    batch = ow.GameBatch.from_games([(cur, init, comets)] * 3)
    rg, rp = [0, 1, 2, 2], [0, 1, 2, 3]
    got = ow.CudaTrue2D().encode_states(batch, rg, rp)
    assert_matches_oracle(got, bind.encode_batch(batch, rg, rp))


def test_play_matches_encode_forward_decode():
    lib = ow.CudaTrue2D()
    models = 5
    pop = synth.true2d_population(21, models, SHAPE.parameter_count())
    batch, rg, rp = synth.game_batch(4, 40, players=4)
    n = rg.size
    idx = (np.arange(n) * 7 % models).astype(np.uintp)
    lib.upload_population(pop, n, SHAPE)
    ids, tr, sc, rows, out = lib.play_population_resident(batch, rg, rp, idx, models, SHAPE, with_rows=True,
                                                          with_outputs=True)
    e = lib.encode_states(batch, rg, rp)
    assert np.array_equal(rows, e.rows) and np.array_equal(ids, e.row_planet_ids)
    ref_out = lib.forward_population_resident_packed(e.rows, idx, models, SHAPE)
    assert np.array_equal(out, ref_out)
    rtr, rsc = dec.decode(out, e.row_planet_ids, e.row_flags, e.row_ships)
    assert np.array_equal(tr, rtr) and np.array_equal(sc, rsc)
    assert (tr >= 0).sum() > 50
    ids2, tr2, sc2 = lib.play_population_resident(batch, rg, rp, idx, models, SHAPE)
    assert np.array_equal(ids2, ids) and np.array_equal(tr2, tr) and np.array_equal(sc2, sc)


def test_profile_counts_the_encoder():
    lib = ow.CudaTrue2D()
    pop = synth.true2d_population(2, 2, SHAPE.parameter_count())
    batch, rg, rp = synth.game_batch(5, 8, players=2)
    idx = (np.arange(rg.size) % 2).astype(np.uintp)
    lib.upload_population(pop, rg.size, SHAPE)
    lib.profile_begin(4)
    lib.play_population_resident(batch, rg, rp, idx, 2, SHAPE)
    prof = lib.profile_end()
    assert prof["t2_encode"][0] == 1 and prof["t2_attention"][0] == 1
