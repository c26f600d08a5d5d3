"""Seeded synthetic inputs and weights.

Random source: the reference's SplitMix-style mix
(crates/orbit-wars-core/src/true2d_model.rs:653-663), keyed by
(seed, tensor id, index) and scaled to U[0, 1]; Box-Muller for N(0, 1).
Default seed 17 is the reference's DEFAULT_SEED (crates/orbit-wars-core/src/model.rs:10).
"""
from __future__ import annotations

import numpy as np

from .presets import PolicyConfig

MASK64 = (1 << 64) - 1
ROW_FACTOR = 0x9E3779B97F4A7C15
COL_FACTOR = 0xBF58476D1CE4E5B9
MIX_FACTOR = 0x94D049BB133111EB
TENSOR_FEATURES, TENSOR_COUNTS, TENSOR_ONEHOT, TENSOR_WEIGHTS = 1, 2, 3, 100
TENSOR_TRUE2D_ROWS, TENSOR_TRUE2D_MODELS = 4, 5
DEFAULT_SEED = 17


def mix64(seed: int, tensor: int, idx) -> np.ndarray:
    idx = np.asarray(idx, dtype=np.uint64)
    base = np.uint64((int(seed) ^ ((int(tensor) * ROW_FACTOR) & MASK64)) & MASK64)
    with np.errstate(over="ignore"):
        x = base ^ (idx * np.uint64(COL_FACTOR))
        x ^= x >> np.uint64(30)
        x = x * np.uint64(COL_FACTOR)
        x ^= x >> np.uint64(27)
        x = x * np.uint64(MIX_FACTOR)
        x ^= x >> np.uint64(31)
    return x


def u01(seed: int, tensor: int, idx) -> np.ndarray:
    return mix64(seed, tensor, idx).astype(np.float64) / float(MASK64)


def normal(seed: int, tensor: int, idx) -> np.ndarray:
    idx = np.asarray(idx, dtype=np.uint64)
    u1 = np.maximum(u01(seed, tensor, idx * np.uint64(2)), 1e-300)
    u2 = u01(seed, tensor, idx * np.uint64(2) + np.uint64(1))
    return np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)


def counts_for(cfg: PolicyConfig, batch: int, seed: int = DEFAULT_SEED, state_offset: int = 0) -> np.ndarray:
    u = u01(seed, TENSOR_COUNTS, np.arange(state_offset, state_offset + batch, dtype=np.uint64))
    span = cfg.count_hi - cfg.count_lo + 1
    c = cfg.count_lo + np.floor(u * span).astype(np.int64)
    return np.minimum(c, cfg.count_hi).astype(np.int32)


def make_inputs(cfg: PolicyConfig, batch: int | None = None, seed: int = DEFAULT_SEED,
                counts: np.ndarray | None = None, state_offset: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """features f32 [B, N, F] (padded entities are 0) and counts int32 [B] of
    global states state_offset .. state_offset+B-1 (a rank's shard of a larger batch)."""
    B = cfg.batch if batch is None else int(batch)
    N, F = cfg.n_entities, cfg.features
    cnt = counts_for(cfg, B, seed, state_offset) if counts is None else np.asarray(counts, dtype=np.int32)
    feats = np.zeros((B, N, F), dtype=np.float32)
    valid = np.arange(N)[None, :] < cnt[:, None]          # [B, N]
    b_idx, j_idx = np.nonzero(valid)
    slot = ((b_idx.astype(np.uint64) + np.uint64(state_offset)) * np.uint64(N) + j_idx.astype(np.uint64))
    chunk = 1 << 20
    for s in range(0, slot.size, chunk):
        sl = slot[s:s + chunk]
        idx = sl[:, None] * np.uint64(F) + np.arange(F, dtype=np.uint64)[None, :]
        vals = normal(seed, TENSOR_FEATURES, idx).astype(np.float32)
        if cfg.onehot_features:
            half = F // 2
            vals[:, half:] = 0.0
            blocks = (F - half) // 4
            kidx = sl[:, None] * np.uint64(4) + np.arange(blocks, dtype=np.uint64)[None, :]
            cls = np.minimum(np.floor(4.0 * u01(seed, TENSOR_ONEHOT, kidx)), 3).astype(np.int64)
            rows = np.arange(sl.size)[:, None]
            vals[rows, half + 4 * np.arange(blocks)[None, :] + cls] = 1.0
        feats[b_idx[s:s + chunk], j_idx[s:s + chunk]] = vals
    return feats, cnt


def tensor_list(cfg: PolicyConfig) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, shape, kind) of every tensor of the weight blob, in order.

    kind: 'mat' (Xavier), 'bias', 'ln_g', 'ln_b'.
    """
    d, F, f, P = cfg.d_model, cfg.features, cfg.ffn, cfg.actions
    out = [("W_e", (d, F), "mat"), ("b_e", (d,), "bias")]
    for l in range(cfg.layers):
        out += [
            (f"ln1_g.{l}", (d,), "ln_g"), (f"ln1_b.{l}", (d,), "ln_b"),
            (f"W_qkv.{l}", (3 * d, d), "mat"), (f"b_qkv.{l}", (3 * d,), "bias"),
            (f"W_o.{l}", (d, d), "mat"), (f"b_o.{l}", (d,), "bias"),
            (f"ln2_g.{l}", (d,), "ln_g"), (f"ln2_b.{l}", (d,), "ln_b"),
            (f"W_1.{l}", (f, d), "mat"), (f"b_1.{l}", (f,), "bias"),
            (f"W_2.{l}", (d, f), "mat"), (f"b_2.{l}", (d,), "bias"),
        ]
    out += [("lnf_g", (d,), "ln_g"), ("lnf_b", (d,), "ln_b"),
            ("W_p", (P, d), "mat"), ("b_p", (P,), "bias"), ("W_v", (1, d), "mat"), ("b_v", (1,), "bias")]
    return out


def weight_count(cfg: PolicyConfig) -> int:
    return int(sum(np.prod(s) for _, s, _ in tensor_list(cfg)))


def make_weights(cfg: PolicyConfig, seed: int = DEFAULT_SEED, affine_noise: bool = False) -> np.ndarray:
    """Flat f32 weight blob: Xavier-uniform matrices; biases 0 and LN (1, 0) unless affine_noise."""
    parts = []
    for k, (_, shape, kind) in enumerate(tensor_list(cfg)):
        n = int(np.prod(shape))
        tid = TENSOR_WEIGHTS + k
        if kind == "mat":
            out_f, in_f = shape
            a = np.sqrt(6.0 / (in_f + out_f))
            parts.append(((2.0 * u01(seed, tid, np.arange(n, dtype=np.uint64)) - 1.0) * a).astype(np.float32))
        elif not affine_noise:
            parts.append(np.full(n, 1.0 if kind == "ln_g" else 0.0, dtype=np.float32))
        else:
            r = 0.1 * (2.0 * u01(seed, tid, np.arange(n, dtype=np.uint64)) - 1.0)
            parts.append((r + (1.0 if kind == "ln_g" else 0.0)).astype(np.float32))
    return np.concatenate(parts)


def split_weights(cfg: PolicyConfig, blob: np.ndarray) -> dict[str, np.ndarray]:
    out, at = {}, 0
    for name, shape, _ in tensor_list(cfg):
        n = int(np.prod(shape))
        out[name] = blob[at:at + n].reshape(shape)
        at += n
    return out


# ---------------------------------------------------------------- True2D drop-in workloads

def true2d_seeded(seed: int, count: int) -> np.ndarray:
    """True2DTransformer::seeded (true2d_model.rs:159-169): weight[i] =
    deterministic_weight(seed, 0, i) * 0.02, deterministic_weight(:653-663) =
    mix / u64::MAX * 2 - 1 rounded to f32 as the reference does."""
    x = u01(seed, 0, np.arange(count, dtype=np.uint64)).astype(np.float32)
    return (x * np.float32(2.0) - np.float32(1.0)) * np.float32(0.02)


def true2d_population(seed: int, models: int, count: int) -> np.ndarray:
    """`models` seeded True2D models back to back (model k uses seed + k)."""
    return np.concatenate([true2d_seeded(seed + k, count) for k in range(models)]) if models else \
        np.zeros(0, np.float32)


def true2d_requests(seed: int, requests: int, rows: int, models: int) -> tuple[np.ndarray, np.ndarray]:
    """Engine-shaped request rows (requests x rows x 7, N(0,1)/2) and seeded
    model indices uniform over the population."""
    n = requests * rows * 7
    x = (normal(seed, TENSOR_TRUE2D_ROWS, np.arange(n, dtype=np.uint64)) * 0.5).astype(np.float32)
    idx = (u01(seed, TENSOR_TRUE2D_MODELS, np.arange(requests, dtype=np.uint64)) * models).astype(np.uintp)
    return x, np.minimum(idx, models - 1).astype(np.uintp)



def game_batch(seed: int, games: int, players: int = 4, min_groups: int = 5, max_groups: int = 10,
               comet_prob: float = 0.5, absent_prob: float = 0.02):
    """Seeded Orbit Wars-shaped game states for the device encoder -> (GameBatch, request_games, request_players).

    Per game: 5..10 planet groups (config.rs MAP_MIN/MAX_PLANET_GROUPS), each one planet mirrored into the
    four quadrants of the 100 x 100 board outside the sun (so equal distances, and the encoder's tie order,
    are common); 40% of groups orbit the centre at 0.03 rad per turn (DEFAULT_ANGULAR_VELOCITY) and are
    shown rotated to a random turn with their tangential velocity; owners and log-uniform ships (0 .. 2e5,
    across SHIP_LOG_PIVOT and SHIP_LOG_CAP) are random; player p's home is group 0, quadrant p. With
    probability comet_prob a group of four comets (speed 4, some above fleet_speed_max) is on the map, its
    ids listed in a shuffled comet list that also names a departed comet. absent_prob of the non-home
    initial planets are missing from the current planets (absent_on_map rows). One request per
    (game, player) for every player that owns a planet.
    """
    from .games import GameBatch, PLANET_DTYPE

    rng = np.random.default_rng(seed)
    quadrant = ((1, 1), (-1, 1), (1, -1), (-1, -1))
    cur_parts, init_parts, comet_parts = [], [], []
    req_g, req_p = [], []
    for g in range(games):
        groups = int(rng.integers(min_groups, max_groups + 1))
        step = int(rng.integers(0, 500))
        init, cur = [], []
        for k in range(groups):
            while True:
                dx, dy = rng.uniform(8.0, 45.0, 2)
                if np.hypot(dx, dy) > 17.0:
                    break
            radius = float(rng.uniform(1.0, 3.0))
            prod = float(rng.integers(1, 6))
            ships0 = float(rng.integers(5, 40))
            orbit = k > 0 and rng.random() < 0.4
            for q, (sx, sy) in enumerate(quadrant):
                pid = 4 * k + q
                x0, y0 = 50.0 + sx * dx, 50.0 + sy * dy
                owner0 = q if (k == 0 and q < players and g % 2 == 0) else -1
                init.append((pid, owner0, x0, y0, radius, ships0, prod, 0.0, 0.0))
                x, y, vx, vy = x0, y0, 0.0, 0.0
                if orbit:
                    a = 0.03 * step
                    ca, sa = np.cos(a), np.sin(a)
                    rx, ry = x0 - 50.0, y0 - 50.0
                    x, y = 50.0 + ca * rx - sa * ry, 50.0 + sa * rx + ca * ry
                    vx, vy = -0.03 * (y - 50.0), 0.03 * (x - 50.0)
                if k == 0 and q < players:
                    owner = q
                else:
                    owner = int(rng.choice([-1, -1, -1] + list(range(players))))
                ships = float(np.expm1(rng.uniform(0.0, np.log(2e5)))) if rng.random() > 0.05 else 0.0
                if k > 0 and rng.random() < absent_prob:
                    continue
                cur.append((pid, owner, x, y, radius, ships, prod, vx, vy))
        comets = []
        if rng.random() < comet_prob:
            base = 1000 + 10 * int(rng.integers(0, 50))
            speed = 4.0 if rng.random() < 0.7 else 7.5
            for q, (sx, sy) in enumerate(quadrant):
                cx, cy = rng.uniform(0.0, 100.0, 2)
                ang = rng.uniform(0, 2 * np.pi)
                cur.append((base + q, int(rng.choice([-1, -1] + list(range(players)))), cx, cy, 1.0,
                            float(rng.integers(0, 60)), 1.0, speed * np.cos(ang), speed * np.sin(ang)))
            comets = [base + q for q in range(4)] + [base + 9]
            rng.shuffle(comets)
        cur_parts.append(np.array(cur, dtype=PLANET_DTYPE))
        init_parts.append(np.array(init, dtype=PLANET_DTYPE))
        comet_parts.append(np.array(comets, dtype=np.int32))
        owners = {int(p[1]) for p in cur}
        for p in range(players):
            if p in owners:
                req_g.append(g)
                req_p.append(p)
    batch = GameBatch.from_games(list(zip(cur_parts, init_parts, comet_parts)))
    if batch.comet_planet_ids is None:
        batch.comet_planet_ids = np.zeros(0, np.int32)
        batch.comet_offsets = np.zeros(games + 1, np.uint64)
    return batch, np.array(req_g, np.uint32), np.array(req_p, np.int32)
