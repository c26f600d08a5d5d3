"""GPU parity of the True2D drop-in (include/orbit_wars_cuda.h) against the
CPU oracle (pinned to the reference's cpu_reference) and, when present, the
reference's own CUDA library built from source into oracle/_ref.

Gate: max abs diff <= 5e-4, the reference's own (config.rs:111,
orbit_wars_cuda_true2d_smoke.cpp:24); outputs in [0, 1]; per-row send sum <= 1 + 1e-6.
"""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest

import orbit_wars_b200 as ow
from orbit_wars_b200 import _lib
from tests.golden.make_true2d_golden import fixture_inputs

pytestmark = pytest.mark.gpu
GATE = 5e-4
SHAPE = ow.True2DShape(61, 64, 1)
REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "liborbit_wars_cuda_ref.so"


def invariants(out):
    out = out.reshape(-1, 64, 12, 2)
    assert np.all(np.isfinite(out))
    assert np.all((out >= 0) & (out <= 1))
    assert np.all(out[..., 1].sum(-1) <= 1 + 1e-6)


def test_single_model_matches_golden():
    g = np.load(Path(__file__).parent / "golden" / "true2d_smoke_fixture.npz")
    x, w1, w2 = fixture_inputs()
    t2 = ow.CudaTrue2D()
    for w, key in ((w1, "out_model_a"), (w2, "out_model_b")):
        out = t2.forward_packed(x, w, 2, SHAPE).reshape(-1)
        invariants(out)
        assert np.abs(out - g[key]).max() <= GATE
        assert np.abs(out - g[key]).max() <= 2e-5  # fp32 single-pass softmax: far inside the gate


def test_many_and_resident_paths(oracle):
    rng = np.random.default_rng(1)
    n_models, n_req = 3, 9
    per = SHAPE.parameter_count()
    pop = np.concatenate([oracle.true2d_seeded(19 + i, per) * (1 + 20 * i) for i in range(n_models)])
    x = rng.uniform(-1, 1, size=(n_req, 64, 7)).astype(np.float32)
    idx = rng.integers(0, n_models, size=n_req).astype(np.uintp)
    ref = oracle.true2d_forward(x, pop, model_indices=idx)
    t2 = ow.CudaTrue2D()
    many = t2.forward_population_packed(x, idx, pop, SHAPE).reshape(-1)
    invariants(many)
    assert np.abs(many - ref).max() <= GATE
    t2.upload_population(pop, request_capacity=16, shape=SHAPE)
    res = t2.forward_population_resident_packed(x, idx, n_models, SHAPE).reshape(-1)
    assert np.abs(res - ref).max() <= GATE
    assert np.array_equal(res, many)


def test_heads_and_rows_variants(oracle):
    rng = np.random.default_rng(2)
    for layers, rows, heads in ((4, 64, 3), (3, 16, 1), (5, 2, 2)):
        shape = ow.True2DShape(layers, rows, heads)
        w = (rng.standard_normal(shape.parameter_count()) * 0.3).astype(np.float32)
        x = rng.uniform(-1, 1, size=(3, rows, 7)).astype(np.float32)
        ref = oracle.true2d_forward(x, w, layers=layers, rows=rows, heads=heads)
        out = ow.CudaTrue2D().forward_packed(x, w, 3, shape).reshape(-1)
        assert np.abs(out - ref).max() <= GATE, (layers, rows, heads)


def attn_offset(layers, rows):
    """Offset of the attention weights in the True2D weight vector (true2d_model.rs:111-126): input_pair[14],
    src_emb[rows], tgt_emb[rows], pair_emb[rows^2], expand_bias[1], matrix[layers x rows^2 x 12]."""
    return 14 + 2 * rows + rows * rows + 1 + layers * rows * rows * 12


def test_attention_paths_match_oracle(oracle):
    """One batch whose requests take the Chebyshev-moment attention (|b|max from about 1e-8 to a few
    hundred) and the direct attention (|b|max beyond 470), against the oracle's direct f32 softmax."""
    layers, rows, heads = 4, 64, 2
    shape = ow.True2DShape(layers, rows, heads)
    per = shape.parameter_count()
    rng = np.random.default_rng(7)
    base = (rng.standard_normal(per) * 0.3).astype(np.float32)
    a0 = attn_offset(layers, rows)
    scales = (1e-4, 0.3, 2.0, 6.0, 14.0, 60.0)  # wq, bq, wk of each head: |b|max ~ 2 scale^2 h
    pop = []
    for sc in scales:
        w = base.copy()
        for h in range(heads):
            w[a0 + 7 * h:a0 + 7 * h + 3] = sc * rng.uniform(0.5, 1.0, 3) * rng.choice([-1.0, 1.0], 3)
        pop.append(w)
    pop = np.concatenate(pop)
    n = 2 * len(scales)
    x = rng.uniform(-1, 1, (n, rows, 7)).astype(np.float32)
    idx = (np.arange(n) % len(scales)).astype(np.uintp)
    ref = oracle.true2d_forward(x, pop, model_indices=idx, layers=layers, rows=rows, heads=heads)
    out = ow.CudaTrue2D().forward_population_packed(x, idx, pop, shape).reshape(-1)
    err = np.abs(out - ref).reshape(n, -1).max(axis=1)
    assert np.all(np.isfinite(out))
    assert err.max() <= GATE, err


def test_rows_beyond_one_query_chunk(oracle):
    """More cells than one CTA's 4,096 queries (80 and 128 rows): the direct attention runs several query
    chunks, all over keys staged before any chunk writes its outputs."""
    rng = np.random.default_rng(11)
    for layers, rows, heads in ((3, 80, 1), (2, 128, 2)):
        shape = ow.True2DShape(layers, rows, heads)
        w = (rng.standard_normal(shape.parameter_count()) * 0.3).astype(np.float32)
        x = rng.uniform(-1, 1, size=(2, rows, 7)).astype(np.float32)
        ref = oracle.true2d_forward(x, w, layers=layers, rows=rows, heads=heads)
        out = ow.CudaTrue2D().forward_packed(x, w, 2, shape).reshape(-1)
        assert np.abs(out - ref).max() <= GATE, (layers, rows, heads)


def test_constant_mid_state(oracle):
    """Zero expand and matrix weights leave every cell at 0: one cell value, so every softmax weight is equal."""
    shape = ow.True2DShape(3, 16, 2)
    rng = np.random.default_rng(3)
    w = np.zeros(shape.parameter_count(), np.float32)
    a0 = attn_offset(3, 16)
    w[a0:] = rng.standard_normal(w.size - a0).astype(np.float32) * 0.5
    x = rng.uniform(-1, 1, size=(2, 16, 7)).astype(np.float32)
    ref = oracle.true2d_forward(x, w, layers=3, rows=16, heads=2)
    out = ow.CudaTrue2D().forward_packed(x, w, 2, shape).reshape(-1)
    assert np.abs(out - ref).max() <= 1e-6


def test_resident_errors():
    lib = _lib.load_library()
    x = np.zeros(64 * 7, np.float32)
    out = np.zeros(64 * 24, np.float32)
    idx = np.zeros(1, np.uintp)
    t2 = ow.CudaTrue2D()
    per = SHAPE.parameter_count()
    t2.upload_population(np.zeros(per, np.float32), request_capacity=1, shape=SHAPE)
    idx2 = np.zeros(2, np.uintp)
    x2 = np.zeros(2 * 64 * 7, np.float32)
    out2 = np.zeros(2 * 64 * 24, np.float32)
    st = lib.orbit_wars_cuda_true2d_forward_many_resident(x2.ctypes.data, idx2.ctypes.data, out2.ctypes.data, 2,
                                                          SHAPE.c())
    assert st.code == 2 and b"capacity" in st.message
    idx[0] = 5
    st = lib.orbit_wars_cuda_true2d_forward_many_resident(x.ctypes.data, idx.ctypes.data, out.ctypes.data, 1,
                                                          SHAPE.c())
    assert st.code == 1
    st = lib.orbit_wars_cuda_true2d_train_full_attention(x.ctypes.data, out.ctypes.data, x.ctypes.data, x.ctypes.data,
                                                         idx.ctypes.data, x.ctypes.data, 1, 1, SHAPE.c(),
                                                         _lib.TrainingConfigC())
    assert st.code == 1  # a zero training config is an invalid batch, as in the reference


def test_trainable_legacy_matches_oracle(oracle):
    lib = _lib.load_library()
    d, heads, layers, rows, games = 32, 4, 3, 64, 3
    n = 2 * d + d + layers * d + 2 * d
    w = (np.sin(np.arange(1, n + 1) * 0.3) * 0.25).astype(np.float32)
    x = np.sin(np.arange(1, games * rows * 2 + 1) * 0.7).astype(np.float32)
    out = np.zeros(games * rows * 2, np.float32)
    _lib.check("trainable", lib.orbit_wars_cuda_trainable_forward(
        x.ctypes.data, w.ctypes.data, out.ctypes.data, games, _lib.TransformerShapeC(layers, d, heads, rows)))
    ref = oracle.trainable_forward(x, w, games, layers, d, heads, rows)
    assert np.abs(out - ref).max() <= 1e-5


@pytest.mark.skipif(not REF_LIB.exists(), reason="reference CUDA library not built (make -C oracle ref)")
@pytest.mark.parametrize("d,heads,layers,games", [(32, 4, 3, 3), (64, 8, 2, 5), (16, 1, 1, 1)])
def test_trainable_legacy_matches_reference_gpu_build(d, heads, layers, games):
    """The legacy TrainableTransformer forward against the reference's own kernels
    (native/cuda/orbit_wars_cuda.cu:2468-2582, built from source for sm_100a).

    The reference writes 2 floats per row packed at the front of its output but copies back
    rows x 24 floats (.cu:2481, :2570), so its host buffer gets 24 floats per row and only
    the first games x rows x 2 are compared."""
    ref = C.CDLL(str(REF_LIB), mode=2)
    ref.orbit_wars_cuda_trainable_forward.restype = _lib.Status
    ref.orbit_wars_cuda_trainable_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                                      _lib.TransformerShapeC]
    lib = _lib.load_library()
    rows = 64
    n = 2 * d + d + layers * d + 2 * d
    w = (np.sin(np.arange(1, n + 1) * 0.37) * 0.3).astype(np.float32)
    x = np.cos(np.arange(1, games * rows * 2 + 1) * 0.61).astype(np.float32)
    shape = _lib.TransformerShapeC(layers, d, heads, rows)
    out_ref = np.zeros(games * rows * 24, np.float32)
    _lib.check("reference trainable", ref.orbit_wars_cuda_trainable_forward(x.ctypes.data, w.ctypes.data,
                                                                            out_ref.ctypes.data, games, shape))
    out = np.zeros(games * rows * 2, np.float32)
    _lib.check("trainable", lib.orbit_wars_cuda_trainable_forward(x.ctypes.data, w.ctypes.data, out.ctypes.data,
                                                                  games, shape))
    assert np.abs(out - out_ref[:games * rows * 2]).max() <= 1e-5


def test_identity_copy():
    torch = pytest.importorskip("torch")
    lib = _lib.load_library()
    a = torch.randn(3, 64, 7, device="cuda")
    b = torch.zeros_like(a)
    _lib.check("identity", lib.orbit_wars_cuda_encode_identity_batch(a.data_ptr(), b.data_ptr(), 3, 64, 7))
    assert torch.equal(a, b)


@pytest.mark.skipif(not REF_LIB.exists(), reason="reference CUDA library not built (make -C oracle ref)")
def test_matches_reference_gpu_build():
    """Same inputs through the reference's own kernels (built from its source for sm_100a)."""
    ref = C.CDLL(str(REF_LIB), mode=2)
    ref.orbit_wars_cuda_true2d_forward.restype = _lib.Status
    ref.orbit_wars_cuda_true2d_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, _lib.True2DShapeC]
    x, w1, _ = fixture_inputs()
    out_ref = np.zeros(2 * 64 * 24, np.float32)
    _lib.check("reference true2d", ref.orbit_wars_cuda_true2d_forward(x.ctypes.data, w1.ctypes.data,
                                                                      out_ref.ctypes.data, 2, SHAPE.c()))
    ours = ow.CudaTrue2D().forward_packed(x, w1, 2, SHAPE).reshape(-1)
    assert np.abs(ours - out_ref).max() <= GATE


def test_profile_counts_each_kernel():
    """Device timing hooks: the row upload and three kernel phases per call, every call counted (the outputs
    of a synchronous host-buffer call leave inside the collapse kernel, written to mapped host memory)."""
    lib = ow.CudaTrue2D()
    x = (np.sin(np.arange(3 * 64 * 7) * 0.3) * 0.5).astype(np.float32)
    from orbit_wars_b200 import synth
    w = synth.true2d_population(5, 2, SHAPE.parameter_count())
    lib.upload_population(w, 3, SHAPE)
    lib.profile_begin(4)
    for _ in range(4):
        lib.forward_population_resident_packed(x, np.array([0, 1, 1], np.uintp), 2, SHAPE)
    prof = lib.profile_end()
    assert set(prof) == {"copy_rows_h2d", "t2_expand_pre", "t2_attention", "t2_post_collapse"}
    assert all(n == 4 and ms > 0 for n, ms in prof.values())
    assert lib.profile_end() == {}
