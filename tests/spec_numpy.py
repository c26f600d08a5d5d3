"""Second, independent float64 restatement of the encoder-policy spec (weight layout,
forward, heads) in numpy, used to cross-check the C++ oracle. Test-only."""
from __future__ import annotations

import math

import numpy as np


def _ln(x, g, b):
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    return (x - mu) / np.sqrt(var + 1e-5) * g + b


def _gelu(x):
    erf = np.vectorize(math.erf)
    return 0.5 * x * (1.0 + erf(x / math.sqrt(2.0)))


def forward(cfg, tensors: dict, features: np.ndarray, counts: np.ndarray):
    """Greedy forward: returns (logits [B,N,P], value [B], actions [B,N])."""
    T = {k: np.asarray(v, dtype=np.float64) for k, v in tensors.items()}
    B, N = counts.shape[0], cfg.n_entities
    d, H = cfg.d_model, cfg.heads
    hd = d // H
    logits = np.zeros((B, N, cfg.actions))
    value = np.zeros(B)
    actions = np.full((B, N), -1, dtype=np.int32)
    for b in range(B):
        c = int(counts[b])
        x = features[b].astype(np.float64) @ T["W_e"].T + T["b_e"]
        for l in range(cfg.layers):
            a = _ln(x, T[f"ln1_g.{l}"], T[f"ln1_b.{l}"])
            qkv = a @ T[f"W_qkv.{l}"].T + T[f"b_qkv.{l}"]
            o = np.zeros((N, d))
            if c > 0:
                for h in range(H):
                    q = qkv[:, h * hd:(h + 1) * hd]
                    k = qkv[:c, d + h * hd:d + (h + 1) * hd]
                    v = qkv[:c, 2 * d + h * hd:2 * d + (h + 1) * hd]
                    s = q @ k.T / math.sqrt(hd)
                    s = np.exp(s - s.max(-1, keepdims=True))
                    o[:, h * hd:(h + 1) * hd] = (s / s.sum(-1, keepdims=True)) @ v
            x = x + o @ T[f"W_o.{l}"].T + T[f"b_o.{l}"]
            a = _ln(x, T[f"ln2_g.{l}"], T[f"ln2_b.{l}"])
            x = x + _gelu(a @ T[f"W_1.{l}"].T + T[f"b_1.{l}"]) @ T[f"W_2.{l}"].T + T[f"b_2.{l}"]
        y = _ln(x, T["lnf_g"], T["lnf_b"])
        lg = y[:c] @ T["W_p"].T + T["b_p"]
        logits[b, :c] = lg
        actions[b, :c] = np.argmax(lg, axis=-1)
        pooled = y[:c].mean(0) if c > 0 else np.zeros(d)
        value[b] = float(pooled @ T["W_v"][0] + T["b_v"][0])
    return logits, value, actions
