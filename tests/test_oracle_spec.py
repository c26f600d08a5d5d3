"""Cross-checks the C++ encoder-policy oracle against the numpy restatement."""
import numpy as np
import pytest

import orbit_wars_b200 as ow
from orbit_wars_b200.synth import split_weights
from tests import spec_numpy
from tests.util import rel_err


def small(cfg, **kw):
    return cfg.with_(**kw)


@pytest.mark.parametrize("pid", [1, 2, 4])
def test_oracle_f64_matches_numpy(oracle, pid):
    cfg = ow.preset(pid)
    cfg = small(cfg, layers=1, d_model=128, heads=4, ffn=256) if pid != 1 else cfg
    w = ow.make_weights(cfg, seed=5, affine_noise=True)
    counts = np.array([0, 1, cfg.n_entities, cfg.count_lo, (cfg.count_lo + cfg.count_hi) // 2], dtype=np.int32)
    feats, counts = ow.make_inputs(cfg, batch=counts.size, seed=9, counts=counts)
    lg, v, a = oracle.policy_forward(cfg, w, feats, counts, f64=True, sample=False)
    nlg, nv, na = spec_numpy.forward(cfg, split_weights(cfg, w), feats, counts)
    assert rel_err(lg, nlg) < 1e-6
    assert rel_err(v, nv) < 1e-6
    assert np.array_equal(a, na)


def test_oracle_f32_close_to_f64(oracle):
    cfg = ow.preset(1)
    w = ow.make_weights(cfg, seed=3, affine_noise=True)
    feats, counts = ow.make_inputs(cfg, batch=16, seed=4)
    l64, v64, _ = oracle.policy_forward(cfg, w, feats, counts, f64=True)
    l32, v32, _ = oracle.policy_forward(cfg, w, feats, counts, f64=False)
    assert rel_err(l32, l64) < 1e-5 and rel_err(v32, v64) < 1e-5


def test_oracle_masks(oracle):
    cfg = ow.preset(1)
    w = ow.make_weights(cfg, seed=3)
    feats, counts = ow.make_inputs(cfg, batch=8, seed=4)
    lg, v, a = oracle.policy_forward(cfg, w, feats, counts)
    pad = np.arange(cfg.n_entities)[None, :] >= counts[:, None]
    assert np.all(lg[pad] == 0) and np.all(a[pad] == -1)
    assert np.all((a[~pad] >= 0) & (a[~pad] < cfg.actions))


def test_padding_content_does_not_leak(oracle):
    """Garbage in padded feature slots must not change any output."""
    cfg = ow.preset(1)
    w = ow.make_weights(cfg, seed=3)
    feats, counts = ow.make_inputs(cfg, batch=6, seed=4)
    dirty = feats.copy()
    pad = np.arange(cfg.n_entities)[None, :] >= counts[:, None]
    dirty[pad] = 123.0
    r1 = oracle.policy_forward(cfg, w, feats, counts)
    r2 = oracle.policy_forward(cfg, w, dirty, counts)
    for x, y in zip(r1, r2):
        assert np.array_equal(x, y)


def test_gumbel_sampling_statistics(oracle):
    """With all-zero logits Gumbel-max is uniform over actions."""
    cfg = ow.preset(4).with_(layers=1, d_model=128, heads=4, ffn=256)
    w = ow.make_weights(cfg, seed=1)
    w[:] = 0.0  # every logit 0 -> argmax decided by the noise alone
    feats, counts = ow.make_inputs(cfg, batch=64, seed=2)
    _, _, a = oracle.policy_forward(cfg, w, feats, counts, sample=True, seed=77)
    valid = a[a >= 0]
    hist = np.bincount(valid, minlength=cfg.actions) / valid.size
    assert np.all(np.abs(hist - 1.0 / cfg.actions) < 0.02)


def test_oracle_rejects_bad_counts(oracle):
    cfg = ow.preset(1)
    w = ow.make_weights(cfg)
    feats, counts = ow.make_inputs(cfg, batch=2)
    counts[1] = cfg.n_entities + 1
    with pytest.raises(ValueError):
        oracle.policy_forward(cfg, w, feats, counts)
