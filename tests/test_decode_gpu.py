"""Device decode of the True2D outputs (orbit_wars_cuda_true2d_decode_*): the
geometry-free part of crates/orbit-wars-core/src/decoder.rs:85-124, against the
reference's own decoder tests and a CPU restatement (oracle/decode.py); bit-exact."""
import numpy as np
import pytest

import orbit_wars_b200 as ow
from orbit_wars_b200 import synth
from oracle import decode as dec

pytestmark = pytest.mark.gpu
SHAPE = ow.True2DShape(61, 64, 1)


def scenario(ships_src, target_fraction, send_fraction):
    """decoder.rs:505-549: planet 1 (owned, row 0) and planet 2 (not owned, row 1); every output
    (target_fraction, send_fraction) except the source row's slots 1..11, which send nothing."""
    out = np.zeros((1, 64, 12, 2), np.float32)
    out[..., 0] = target_fraction
    out[..., 1] = send_fraction
    out[0, 0, 1:, 1] = 0.0
    ids = np.full((1, 64), -1, np.int32)
    ids[0, :2] = (1, 2)
    owned = np.zeros((1, 64), np.uint8)
    owned[0, 0] = 1
    ships = np.zeros((1, 64), np.float32)
    ships[0, :2] = (ships_src, 5.0)
    return out, ids, owned, ships


def test_reference_decoder_known_answers():
    lib = ow.CudaTrue2D()
    # decoder_sends_owned_source_to_selected_target: 10 ships * 0.5 -> 5 to row 1 (planet 2)
    tr, sc = lib.decode_outputs(*scenario(10.0, 0.75, 0.5))
    assert (tr >= 0).sum() == 1 and tr[0, 0, 0] == 1 and sc[0, 0, 0] == 5
    # ... and with target fraction 0 the target is the source row: no command
    tr, sc = lib.decode_outputs(*scenario(10.0, 0.0, 0.5))
    assert (tr >= 0).sum() == 0 and sc.sum() == 0
    # decoder_ignores_fractional_ship_launches: floor(3 * 0.2) = 0 -> no command
    tr, sc = lib.decode_outputs(*scenario(3.0, 0.75, 0.2))
    assert (tr >= 0).sum() == 0


def random_decode_inputs(rng, n, rows=64):
    """Row flags: 1 = owned by the player, 2 = not on the map (both set is contradictory and never decoded)."""
    ids = np.where(rng.random((n, rows)) < 0.6, rng.integers(0, 50, (n, rows)), -1).astype(np.int32)
    ids[0, :] = -1  # a request with no planet at all
    owned = (rng.random((n, rows)) < 0.5).astype(np.uint8)
    absent = (rng.random((n, rows)) < 0.1).astype(np.uint8)
    ships = (rng.random((n, rows)) * 120.0).astype(np.float32)
    return ids, owned | (absent << 1), ships


def test_decode_outputs_matches_restatement():
    rng = np.random.default_rng(3)
    n = 37
    out = rng.random((n, 64, 12, 2), dtype=np.float32)
    out[..., 0] = out[..., 0] * 1.4 - 0.2  # fractions outside [0, 1] are clamped
    out[..., 1] = out[..., 1] * 1.4 - 0.2
    ids, owned, ships = random_decode_inputs(rng, n)
    tr, sc = ow.CudaTrue2D().decode_outputs(out, ids, owned, ships)
    rtr, rsc = dec.decode(out, ids, owned, ships)
    assert np.array_equal(tr, rtr) and np.array_equal(sc, rsc)
    assert (tr >= 0).sum() > 100


def test_decode_many_resident_matches_forward_and_restatement():
    rng = np.random.default_rng(5)
    lib = ow.CudaTrue2D()
    models, n = 3, 20
    pop = synth.true2d_population(11, models, SHAPE.parameter_count())
    x, idx = synth.true2d_requests(13, n, SHAPE.rows, models)
    lib.upload_population(pop, n, SHAPE)
    ids, owned, ships = random_decode_inputs(rng, n)
    tr, sc, out = lib.decode_population_resident(x, idx, models, ids, owned, ships, SHAPE, with_outputs=True)
    ref_out = lib.forward_population_resident_packed(x, idx, models, SHAPE)
    assert np.array_equal(out, ref_out)
    rtr, rsc = dec.decode(out, ids, owned, ships)
    assert np.array_equal(tr, rtr) and np.array_equal(sc, rsc)
    tr2, sc2 = lib.decode_population_resident(x, idx, models, ids, owned, ships, SHAPE)
    assert np.array_equal(tr2, tr) and np.array_equal(sc2, sc)


def test_absent_target_and_source_are_skipped():
    """decoder.rs:93-95 and :112-114: a source or target whose planet is not on the map gives no command."""
    out, ids, owned, ships = scenario(10.0, 0.75, 0.5)
    flags = owned.copy()
    flags[0, 1] = 2  # the target planet (row 1) left the map
    tr, sc = ow.CudaTrue2D().decode_outputs(out, ids, flags, ships)
    assert (tr >= 0).sum() == 0 and sc.sum() == 0
    rtr, _ = dec.decode(out, ids, flags, ships)
    assert (rtr >= 0).sum() == 0
    flags = owned.copy()
    flags[0, 0] = 3  # owned but absent: no source
    tr, _ = ow.CudaTrue2D().decode_outputs(out, ids, flags, ships)
    assert (tr >= 0).sum() == 0


def test_non_finite_output_is_rejected():
    out, ids, owned, ships = scenario(10.0, 0.75, 0.5)
    out[0, 0, 3, 1] = np.nan  # an owned, active source's slot
    with pytest.raises(ow.OwError) as e:
        ow.CudaTrue2D().decode_outputs(out, ids, owned, ships)
    assert e.value.code == 2
    # a non-finite output of a row the decoder skips is ignored, as in the reference
    out, ids, owned, ships = scenario(10.0, 0.75, 0.5)
    out[0, 5, 3, 1] = np.nan
    tr, _ = ow.CudaTrue2D().decode_outputs(out, ids, owned, ships)
    assert tr[0, 0, 0] == 1
