"""Pins the CPU oracles against known answers and the reference's own code."""
import numpy as np
import pytest

from tests.golden.make_true2d_golden import fixture_inputs

# Random123 known-answer vectors for Philox4x32-10 (Salmon et al., SC'11).
PHILOX_KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


@pytest.mark.parametrize("ctr,key,expect", PHILOX_KAT)
def test_philox_known_answers(oracle, ctr, key, expect):
    assert tuple(oracle.philox(ctr, *key)) == expect


def test_gumbel_uses_spec_counter_layout(oracle):
    # G for (seed, state 3, entity 5, action 6): word 2 of philox((1, 5, 3, 0), seed).
    seed = 0x0123456789ABCDEF
    words = oracle.philox((6 // 4, 5, 3, 0), seed & 0xFFFFFFFF, seed >> 32)
    u = (words[6 % 4] + 0.5) / 2**32
    assert oracle.gumbel(seed, 3, 5, 6) == pytest.approx(-np.log(-np.log(u)), abs=1e-12)


def test_true2d_parameter_count(oracle):
    # true2d_model.rs:669 MULTI_TARGET_HEAD_PARAMETER_COUNT
    assert oracle.true2d_weight_count(61, 64, 1) == 3_004_120


def test_true2d_oracle_matches_reference_cpu_reference_golden(oracle):
    """Golden outputs of the reference smoke's cpu_reference (tests/golden/make_true2d_golden.py)."""
    g = np.load(__import__("pathlib").Path(__file__).parent / "golden" / "true2d_smoke_fixture.npz")
    x, w1, w2 = fixture_inputs()
    assert np.float64(x.astype(np.float64).sum()) == pytest.approx(float(g["input_sum"]), rel=0, abs=1e-9)
    assert np.array_equal(w1[:16], g["w_a_head"]) and np.array_equal(w2[:16], g["w_b_head"])
    for w, key in ((w1, "out_model_a"), (w2, "out_model_b")):
        out = oracle.true2d_forward(x, w)
        assert np.abs(out - g[key]).max() <= 1e-6
    # many-model path: request r uses model_indices[r]
    out = oracle.true2d_forward(x, np.concatenate([w1, w2]), model_indices=[1, 0])
    assert np.abs(out[: 64 * 24] - g["out_model_b"][: 64 * 24]).max() <= 1e-6
    assert np.abs(out[64 * 24:] - g["out_model_a"][64 * 24:]).max() <= 1e-6


def test_true2d_output_invariants_seeded(oracle):
    """true2d_model.rs:672-708: outputs in [0,1], per-row send sum <= 1 + 1e-6 (seeded model 19)."""
    n = oracle.true2d_weight_count()
    w = oracle.true2d_seeded(19, n)
    rng = np.random.default_rng(0)
    x = rng.uniform(-1, 1, size=(2, 64, 7)).astype(np.float32)
    out = oracle.true2d_forward(x, w).reshape(2, 64, 12, 2)
    assert np.all((out >= 0) & (out <= 1))
    assert np.all(out[..., 1].sum(-1) <= 1 + 1e-6)


def test_deterministic_weight_range_and_mix(oracle):
    # deterministic_weight(seed,row,col) = 2*mix/(2^64-1) - 1; matches the package's synth mixer
    import orbit_wars_b200.synth as synth
    for seed, row, col in [(19, 0, 0), (23, 0, 17), (17, 1, 123456)]:
        u = float(synth.u01(seed, row, col))
        assert oracle.deterministic_weight(seed, row, col) == pytest.approx(np.float32(u * 2 - 1), abs=1e-6)


def test_trainable_oracle_shape_and_range(oracle):
    """model.rs:470-497: legacy outputs are sigmoid values in (0, 1)."""
    d, heads, layers, rows = 32, 4, 3, 64
    n = 2 * d + d + layers * d + 2 * d
    w = (np.sin(np.arange(1, n + 1) * 0.3) * 0.25).astype(np.float32)
    x = np.sin(np.arange(1, 2 * rows * 2 + 1) * 0.7).astype(np.float32)
    out = oracle.trainable_forward(x, w, 2, layers, d, heads, rows)
    assert out.shape == (2 * rows * 2,) and np.all((out > 0) & (out < 1))


def test_true2d_seeded_generator_matches_oracle(oracle):
    """The package's numpy True2DTransformer::seeded (bench workload) is bit-exact with the oracle's C one."""
    from orbit_wars_b200 import synth
    for seed in (0, 17, 123456789):
        assert np.array_equal(synth.true2d_seeded(seed, 50_000), oracle.true2d_seeded(seed, 50_000))


def test_e4m3_rounding_matches_torch(oracle):
    """The recipe emulation's e4m3 (RNE, saturating at 448) against torch.float8_e4m3fn."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(0)
    v = np.concatenate([rng.standard_normal(4000) * s for s in (1e-3, 0.05, 1.0, 30.0, 300.0)] +
                       [np.array([0.0, 448.0, 449.0, 464.0, 465.0, 1e4, 2.0**-10, 1.5 * 2.0**-9, 2.5 * 2.0**-9,
                                  -0.5 * 2.0**-9, 0.0625 * 1.0625, 1.0625, 1.1875])]).astype(np.float32)
    expect = torch.from_numpy(np.clip(v, -448, 448)).to(torch.float8_e4m3fn).float().numpy()
    got = np.array([oracle.round_e4m3(float(x)) for x in v], np.float32)
    assert np.array_equal(got, expect)


def _c3_case(batch=24):
    import orbit_wars_b200 as ow
    from tests.util import representable_embedding, representable_weights
    cfg = ow.preset(3).with_(batch=batch)
    w = representable_embedding(cfg, representable_weights(cfg, ow.make_weights(cfg, seed=11, affine_noise=True)))
    feats, counts = ow.make_inputs(cfg, batch=batch, seed=21)
    return cfg, w, feats, counts


def test_emulation_without_rounding_is_the_truth(oracle):
    from tests.util import rel_err, valid_mask
    cfg, w, feats, counts = _c3_case(8)
    truth = oracle.policy_forward(cfg, w, feats, counts, f64=True, sample=False)
    emu = oracle.policy_forward_emulated(cfg, w, feats, counts, mode=0)
    m = valid_mask(counts, cfg.n_entities)
    assert rel_err(emu[0][m], truth[0][m]) <= 1e-6 and rel_err(emu[1], truth[1]) <= 1e-6


def test_fp8_recipe_floor(oracle):
    """The fp8 recipe, computed exactly, loses more than 3e-2 on logits against the float64 truth (so no
    implementation of it meets 3e-2 there); bf16 storage alone stays well inside 1e-2."""
    from tests.util import rel_err, valid_mask
    cfg, w, feats, counts = _c3_case(24)
    truth = oracle.policy_forward(cfg, w, feats, counts, f64=True, sample=False)
    m = valid_mask(counts, cfg.n_entities)
    fp8 = oracle.policy_forward_emulated(cfg, w, feats, counts)
    bf16 = oracle.policy_forward_emulated(cfg, w, feats, counts, mode=oracle.EMU_STORE_BF16)
    assert rel_err(fp8[0][m], truth[0][m]) > 3e-2
    assert rel_err(bf16[0][m], truth[0][m]) < 1e-2 and rel_err(bf16[1], truth[1]) < 1e-2


def test_gumbel_argmax_replays_the_noise(oracle):
    rng = np.random.default_rng(2)
    B, N, P, seed = 3, 5, 16, 0xABCDEF0123
    logits = rng.standard_normal((B, N, P)).astype(np.float32)
    counts = np.array([5, 0, 3], np.int32)
    acts, gap = oracle.gumbel_argmax(logits, counts, seed, state_base=7)
    for b in range(B):
        for j in range(N):
            if j >= counts[b]:
                assert acts[b, j] == -1 and np.isinf(gap[b, j])
                continue
            s = [float(logits[b, j, p]) + oracle.gumbel(seed, 7 + b, j, p) for p in range(P)]
            assert acts[b, j] == int(np.argmax(s))
            top = sorted(s)[-2:]
            assert gap[b, j] == pytest.approx(top[1] - top[0], rel=1e-5, abs=1e-6)
