"""Shared comparison helpers for parity tests (tolerances: SPEC.md section 8)."""
from __future__ import annotations

import numpy as np

TOL = {"f32": 1e-4, "bf16": 1e-2, "fp8": 3e-2}


def rel_err(a, b) -> float:
    """max|a-b| / max(max|b|, 1e-6)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    if b.size == 0:
        return 0.0
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-6))


def valid_mask(counts, n_entities):
    return np.arange(n_entities)[None, :] < np.asarray(counts)[:, None]


def argmax_agreement(actions_a, actions_b, counts, n_entities) -> float:
    m = valid_mask(counts, n_entities)
    if m.sum() == 0:
        return 1.0
    return float((np.asarray(actions_a)[m] == np.asarray(actions_b)[m]).mean())


def near_tie_mask(logits, counts, n_entities, margin):
    """Valid entities whose top-2 logits are within `margin` (argmax may legitimately flip)."""
    s = np.sort(np.asarray(logits, dtype=np.float64), axis=-1)
    gap = s[..., -1] - s[..., -2]
    return valid_mask(counts, n_entities) & (gap < margin)
