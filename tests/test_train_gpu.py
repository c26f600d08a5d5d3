"""True2D training step (orbit_wars_cuda_true2d_train_full_attention) against the
reference's own CUDA build (native/cuda/orbit_wars_cuda.cu:2823-3330, compiled
from its source for sm_100a into oracle/_ref) on the same samples.

Both implementations take one full-batch SGD step per model. They sum the
per-sample gradients in different orders (the reference per weight over
samples and cells, this build through per-model partials), so the weight
updates agree to f32 rounding: the gate is max|dW_ours - dW_ref| <= 2e-3 x
max|dW_ref| over every weight of every model."""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest

import orbit_wars_b200 as ow
from orbit_wars_b200 import _lib, synth

pytestmark = pytest.mark.gpu
REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "liborbit_wars_cuda_ref.so"
OWN, EMPTY, ABSENT = 1.0, -0.5, -1.0
CLASSES = np.array([OWN, 0.75, 0.5, 0.25, 0.0, ABSENT], np.float32)
GATE = 2e-3


def samples(seed, n, shape, models):
    """Engine-shaped training samples: owner classes from the encoder's set (empty padding rows at the end),
    features in [-1, 1], stored outputs in [0, 1], int rewards in [-2, 2] (some 0), target action rewards."""
    rng = np.random.default_rng(seed)
    R = shape.rows
    x = rng.uniform(-1.0, 1.0, (n, R, 7)).astype(np.float32)
    for s in range(n):
        active = int(rng.integers(2, R + 1))
        x[s, :active, 0] = rng.choice(CLASSES, active, p=[0.3, 0.15, 0.1, 0.1, 0.25, 0.1])
        x[s, 0, 0] = OWN
        x[s, active:, 0] = EMPTY
        x[s, active:, 1:] = 0.0
    out = rng.uniform(0.0, 1.0, (n, R, 24)).astype(np.float32)
    rewards = rng.integers(-2, 3, n).astype(np.int32)
    tar = (rng.standard_normal((n, R, 12)) * 0.2).astype(np.float32)
    tar[rng.random((n, R, 12)) < 0.3] = 0.0
    idx = rng.integers(0, models, n).astype(np.uintp)
    return x, out, rewards, tar, idx


def ref_train(x, out, rewards, tar, idx, w, shape, batch, lr, norm, thr):
    ref = C.CDLL(str(REF_LIB), mode=2)
    fn = ref.orbit_wars_cuda_true2d_train_full_attention
    fn.restype = _lib.Status
    fn.argtypes = [C.c_void_p] * 6 + [C.c_size_t, C.c_size_t, _lib.True2DShapeC, _lib.TrainingConfigC]
    wr = np.array(w, dtype=np.float32, copy=True)
    cfg = _lib.TrainingConfigC(batch, lr, norm, thr, OWN, EMPTY, ABSENT)
    _lib.check("reference training", fn(x.ctypes.data, out.ctypes.data, rewards.ctypes.data, tar.ctypes.data,
                                        idx.ctypes.data, wr.ctypes.data, idx.size, wr.size // shape.parameter_count(),
                                        shape.c(), cfg))
    return wr.reshape(-1, shape.parameter_count())


def check(shape, models, n, seed, batch=64, lr=0.05, norm=2.0, thr=0.5, scale=0.3):
    rng = np.random.default_rng(seed + 100)
    if shape == ow.True2DShape():
        w = synth.true2d_population(seed, models, shape.parameter_count())
    else:
        w = (rng.standard_normal(models * shape.parameter_count()) * scale).astype(np.float32)
    x, out, rewards, tar, idx = samples(seed, n, shape, models)
    w0 = w.reshape(models, -1)
    ours = ow.CudaTrue2D().train_full_attention(x, out, rewards, tar, idx, w, shape, batch_sample_count=batch,
                                                learning_rate=lr, reward_normalizer=norm, send_threshold=thr)
    ref = ref_train(x, out, rewards, tar, idx, w, shape, batch, lr, norm, thr)
    d_ours, d_ref = ours - w0, ref - w0
    scale_ref = np.abs(d_ref).max()
    assert scale_ref > 0.0
    err = np.abs(d_ours - d_ref).max() / scale_ref
    assert err <= GATE, f"{shape} models={models} n={n}: update rel err {err:.3e}"
    return ours, err


needs_ref = pytest.mark.skipif(not REF_LIB.exists(), reason="reference CUDA library not built (make -C oracle ref)")


@needs_ref
@pytest.mark.parametrize("layers,rows,heads,models,n", [(5, 8, 2, 3, 10), (4, 16, 1, 2, 7), (3, 2, 3, 1, 4)])
def test_small_shapes_match_reference_build(layers, rows, heads, models, n):
    check(ow.True2DShape(layers, rows, heads), models, n, seed=layers * 10 + rows)


@needs_ref
def test_full_shape_matches_reference_build_with_chunks():
    """61 layers, 64 rows, 1 head; 6 samples over 2 models in chunks of 4."""
    check(ow.True2DShape(), 2, 6, seed=5, batch=4, lr=0.01)


def test_deterministic_and_chunk_invariant():
    shape = ow.True2DShape(5, 8, 2)
    rng = np.random.default_rng(1)
    w = (rng.standard_normal(3 * shape.parameter_count()) * 0.3).astype(np.float32)
    x, out, rewards, tar, idx = samples(9, 12, shape, 3)
    lib = ow.CudaTrue2D()
    a = lib.train_full_attention(x, out, rewards, tar, idx, w, shape, batch_sample_count=64, learning_rate=0.05)
    b = lib.train_full_attention(x, out, rewards, tar, idx, w, shape, batch_sample_count=64, learning_rate=0.05)
    assert np.array_equal(a, b)
    c = lib.train_full_attention(x, out, rewards, tar, idx, w, shape, batch_sample_count=1, learning_rate=0.05)
    d_a, d_c = a - w.reshape(3, -1), c - w.reshape(3, -1)
    assert np.abs(d_a - d_c).max() <= 1e-4 * np.abs(d_a).max()


def test_zero_rewards_leave_weights_unchanged():
    """Reward 0 and target action rewards 0: every loss term is scaled by 0."""
    shape = ow.True2DShape(4, 8, 1)
    rng = np.random.default_rng(2)
    w = (rng.standard_normal(2 * shape.parameter_count()) * 0.3).astype(np.float32)
    x, out, rewards, tar, idx = samples(3, 5, shape, 2)
    rewards[:] = 0
    tar[:] = 0.0
    new = ow.CudaTrue2D().train_full_attention(x, out, rewards, tar, idx, w, shape)
    assert np.array_equal(new, w.reshape(2, -1))


def test_training_rejects_bad_batches():
    shape = ow.True2DShape(4, 8, 1)
    x, out, rewards, tar, idx = samples(3, 2, shape, 1)
    w = np.zeros(shape.parameter_count(), np.float32)
    idx[1] = 4
    with pytest.raises(ow.OwError) as e:
        ow.CudaTrue2D().train_full_attention(x, out, rewards, tar, idx, w, shape)
    assert e.value.code == 1 and "out of range" in str(e.value)
    idx[1] = 0
    with pytest.raises(ow.OwError) as e:
        ow.CudaTrue2D().train_full_attention(x, out, rewards, tar, idx, w, shape, learning_rate=0.0)
    assert e.value.code == 1
