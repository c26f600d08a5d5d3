"""The Chebyshev-moment attention of t2_attention_moments (csrc/orbit_wars_true2d.cu),
restated in float64 numpy and checked against the direct softmax of the
reference's attention layer (true2d_model.rs:463-544: rank-1 scores
q_i k_j, no scale, no mask).

What is pinned here is the method and its two rules, not the CUDA code (the GPU
tests compare the kernel with the oracle):
  * the series cut P(|b|) = ceil(8.5 sqrt(|b|) + 7) drops at most 1e-16 of
    e^|b| for |b| in [1e-12, 1e3] (tabulated e^-|b| I_k(|b|) from scipy);
  * Miller's backward recurrence from k = P with the sums taken on the way
    down gives E[m] to near double rounding on ordinary and adversarial cell
    values (most cells at one end) for |b| up to the 470 cut-off.
"""
import math

import numpy as np
import pytest

BETA_MAX = 470.0


def order(beta: float) -> int:
    p = int(math.ceil(8.5 * math.sqrt(beta) + 7.0))
    return (p + 3) & ~3


def moments(x: np.ndarray, p: int):
    """mu_k = sum_j T_k(x_j), k = 0 .. p + 1, and nu_k = (mu_{k+1} + mu_{|k-1|}) / 2, k = 0 .. p."""
    mu = np.zeros(p + 2)
    tp, tc = x.copy(), np.ones_like(x)
    for k in range(p + 2):
        mu[k] = tc.sum()
        tp, tc = tc, 2.0 * x * tc - tp
    nu = np.empty(p + 1)
    nu[0] = mu[1]
    nu[1:] = 0.5 * (mu[2:p + 2] + mu[0:p])
    return mu, nu


def moment_mean(m: np.ndarray, a: np.ndarray) -> np.ndarray:
    """E_i[m] = sum_j m_j e^(a_i m_j) / sum_j e^(a_i m_j) by the moment method, in float64."""
    lo, hi = float(m.min()), float(m.max())
    c, h = 0.5 * (lo + hi), 0.5 * (hi - lo)
    if h == 0.0:
        return np.full(a.shape, lo)
    b = a * h
    p = order(float(np.abs(b).max()))
    mu, nu = moments((m - c) / h, p)
    out = np.empty_like(a)
    for i, bi in enumerate(b):
        if abs(bi) < 1e-6:
            ratio = (nu[0] + bi * 0.5 * (mu[0] + mu[2])) / (mu[0] + bi * mu[1])
        else:
            step, z, z1, sf, sp = 2.0 / bi, 1.0, 0.0, 0.0, 0.0
            for k in range(p, 0, -1):
                sf += z * mu[k]
                sp += z * nu[k]
                z, z1 = k * step * z + z1, z
                if abs(z) > 1e180:
                    z, z1, sf, sp = z * 1e-180, z1 * 1e-180, sf * 1e-180, sp * 1e-180
            ratio = (z * nu[0] + 2.0 * sp) / (z * mu[0] + 2.0 * sf)
        out[i] = c + h * ratio
    return out


def direct_mean(m: np.ndarray, a: np.ndarray) -> np.ndarray:
    s = a[:, None] * m[None, :]
    s -= s.max(axis=1, keepdims=True)
    e = np.exp(s)
    return (e * m[None, :]).sum(axis=1) / e.sum(axis=1)


def test_series_cut_rule():
    ive = pytest.importorskip("scipy.special").ive
    for beta in np.logspace(-12, 3, 600):
        p = order(beta)
        tail = 2.0 * ive(np.arange(p + 1, p + 600), beta).sum()
        assert tail <= 1e-16, (beta, p, tail)
    assert order(BETA_MAX) <= 192


@pytest.mark.parametrize("kind", ["tanh", "ends", "two_points", "constant"])
@pytest.mark.parametrize("beta", [1e-9, 1e-3, 0.7, 9.0, 60.0, 300.0, 470.0])
def test_moment_mean_matches_direct_softmax(kind, beta):
    rng = np.random.default_rng(int(beta * 1000) % 9973 + len(kind))
    n = 1024
    if kind == "tanh":
        m = np.tanh(rng.standard_normal(n) * 1.5)
    elif kind == "ends":
        m = np.where(rng.random(n) < 0.995, -0.97, 0.99) + rng.standard_normal(n) * 1e-3
    elif kind == "two_points":
        m = np.where(rng.random(n) < 0.5, -0.4, 0.6)
    else:
        m = np.full(n, 0.25)
    h = 0.5 * (m.max() - m.min())
    # queries spanning [-|b|max, |b|max] with the cut-off query at an end, as q is affine in m
    a = np.linspace(-1.0, 1.0, 257) * (beta / h if h > 0 else beta)
    got = moment_mean(m, a)
    want = direct_mean(m, a)
    assert np.abs(got - want).max() <= 1e-11, (kind, beta, np.abs(got - want).max())
