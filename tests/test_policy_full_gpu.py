"""Full configured batches against the CPU oracle, with the seeded f32 weights
exactly as the benchmark builds them (no pre-rounding: the GPU quantises its
own weights, so the comparison covers weight storage as well as arithmetic).

  C2  all 1,024 states (seed 17)                    bf16 <= 1e-2 vs the float64 truth
  C3  the first 1,024 of its 4,096 states           fp8  within the recipe's own error vs the truth
  C4  the first 256 of its 8,192 states, Gumbel     bf16 <= 1e-2; actions replayed from the GPU logits
  C5  the first 256 of its 65,536 states per GPU    bf16 <= 1e-2

The first k states of a configured batch are the states a full-batch run sees
first (inputs are keyed by the global state index), so a subset is a slice of
the benchmark's own workload.
"""
import numpy as np
import pytest

import orbit_wars_b200 as ow
from tests.util import (TOL, check_fp8_against_recipe, near_tie_mask, rel_err, representable_embedding,
                        representable_weights, valid_mask)

pytestmark = pytest.mark.gpu

SEED = 17
CASES = [(2, 1024), (3, 1024), (4, 256), (5, 256)]
TIE_MARGIN = {"bf16": 5e-2, "fp8": 1.5e-1}


@pytest.mark.parametrize("pid,batch", CASES)
def test_configured_batch_matches_oracle(oracle, pid, batch):
    cfg = ow.preset(pid).with_(batch=batch)
    w = ow.make_weights(cfg, seed=SEED)
    feats, counts = ow.make_inputs(cfg, batch=batch, seed=SEED)
    with ow.EncoderPolicy(cfg, w) as pol:
        g_lg, g_v, g_a = pol.forward(feats, counts, seed=SEED)
    m = valid_mask(counts, cfg.n_entities)
    # masks and indices bit-exact
    assert np.all(g_lg[~m] == 0.0) and np.all(g_a[~m] == -1)
    assert np.all((g_a[m] >= 0) & (g_a[m] < cfg.actions))
    truth = oracle.policy_forward(cfg, w, feats, counts, f64=True, sample=False)
    if cfg.precision == "fp8":
        # the recipe computed exactly, from the weights as the fp8 model stores them
        recipe = oracle.policy_forward_emulated(cfg, representable_embedding(cfg, representable_weights(cfg, w)),
                                                feats, counts)
        r = check_fp8_against_recipe(g_lg, g_v, truth, recipe, m)
        print(f"{cfg.name} x{batch}: " + "; ".join(f"{k} vs truth {v['vs_truth']:.2e} (recipe {v['recipe']:.2e})"
                                                   for k, v in r.items()))
        return
    e_l, e_v = rel_err(g_lg[m], truth[0][m]), rel_err(g_v, truth[1])
    assert e_l <= TOL[cfg.precision] and e_v <= TOL[cfg.precision], (e_l, e_v)
    if cfg.sample_actions:
        # Gumbel-max over the GPU's own (bf16) logits with the spec's Philox noise
        acts, gap = oracle.gumbel_argmax(g_lg, counts, SEED)
        clear = m & (gap > 1e-4)
        assert np.array_equal(g_a[clear], acts[clear])
        assert clear.sum() >= 0.999 * m.sum()
    else:
        keep = m & ~near_tie_mask(truth[0], counts, cfg.n_entities, TIE_MARGIN[cfg.precision])
        agree = float((g_a[keep] == truth[2][keep]).mean())
        assert agree >= 0.999, agree
    print(f"{cfg.name} x{batch}: logits rel {e_l:.2e} value rel {e_v:.2e}")
