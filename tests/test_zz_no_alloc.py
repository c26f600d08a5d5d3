"""The allocation-free True2D forward (orbit_wars_cuda_true2d_forward_noalloc).

Some callers of the drop-in cannot allocate device memory: an engine whose
device memory is all reserved by its own pool, or a self-play loop that must
not pay cudaMalloc/cudaFree's implicit device-wide synchronisation between
turns. This entry point takes device buffers and keeps its scratch in a fixed
1 MiB array inside the library. It must produce what the allocating entry
point produces (and what the CPU oracle computes), call after call (the shared
array keeps the previous call's contents), up to the documented maximum, take
no device memory while it runs, and refuse work that does not fit.

The file sorts last so a stop-at-first-failure run has run every other test
before it; it also passes alone in a fresh process.
"""
import numpy as np
import pytest

import orbit_wars_b200 as ow
from orbit_wars_b200 import _lib

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
SHAPE = ow.True2DShape(61, 64, 1)
TOL = 5e-4  # the True2D parity gate used by the other True2D tests
MAX_GAMES_64 = 63  # 63 x (64^2 + 1) = 258,111 <= 262,080 floats of scratch


def _allocating_forward(lib, x, w, games, shape=SHAPE):
    out = np.zeros(games * shape.rows * 24, np.float32)
    _lib.check("orbit_wars_cuda_true2d_forward", lib.orbit_wars_cuda_true2d_forward(
        x.ctypes.data, w.ctypes.data, out.ctypes.data, games, shape.c()))
    return out


def _noalloc_forward(lib, x_dev, w_dev, out_dev, games, shape=SHAPE):
    st = lib.orbit_wars_cuda_true2d_forward_noalloc(x_dev.data_ptr(), w_dev.data_ptr(), out_dev.data_ptr(),
                                                    games, shape.c(), torch.cuda.current_stream().cuda_stream)
    _lib.check("orbit_wars_cuda_true2d_forward_noalloc", st)


def _weights(rng, shape):
    return (rng.standard_normal(shape.parameter_count()) * 0.05).astype(np.float32)


def test_noalloc_matches_allocating_entry_point_two_calls(oracle):
    lib = _lib.load_library()
    rng = np.random.default_rng(7)
    w = _weights(rng, SHAPE)
    w_dev = torch.from_numpy(w).cuda()
    for games in (5, 3):  # two calls in a row on the shared scratch
        x = rng.uniform(-1, 1, size=(games, 64, 7)).astype(np.float32)
        ref = _allocating_forward(lib, x, w, games)
        x_dev = torch.from_numpy(x).cuda()
        out_dev = torch.full((games * 64 * 24,), float("nan"), device="cuda")
        _noalloc_forward(lib, x_dev, w_dev, out_dev, games)
        torch.cuda.synchronize()
        out = out_dev.cpu().numpy()
        assert np.all(np.isfinite(out))
        assert np.abs(out - ref).max() <= TOL
        # and against the CPU oracle (the restatement pinned to the reference's cpu_reference)
        assert np.abs(out - oracle.true2d_forward(x, w)).max() <= TOL


def test_noalloc_takes_no_device_memory():
    """After one warm-up call (which loads the device code), further calls leave the device's free
    memory unchanged: nothing is allocated per call."""
    lib = _lib.load_library()
    rng = np.random.default_rng(3)
    games = 4
    w_dev = torch.from_numpy(_weights(rng, SHAPE)).cuda()
    x_dev = torch.from_numpy(rng.uniform(-1, 1, size=(games, 64, 7)).astype(np.float32)).cuda()
    out_dev = torch.zeros(games * 64 * 24, device="cuda")
    _noalloc_forward(lib, x_dev, w_dev, out_dev, games)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(5):
        _noalloc_forward(lib, x_dev, w_dev, out_dev, games)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before


def test_noalloc_at_the_documented_maximum():
    lib = _lib.load_library()
    rng = np.random.default_rng(11)
    w = _weights(rng, SHAPE)
    x = rng.uniform(-1, 1, size=(MAX_GAMES_64, 64, 7)).astype(np.float32)
    ref = _allocating_forward(lib, x, w, MAX_GAMES_64)
    out_dev = torch.full((MAX_GAMES_64 * 64 * 24,), float("nan"), device="cuda")
    _noalloc_forward(lib, torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), out_dev, MAX_GAMES_64)
    torch.cuda.synchronize()
    assert np.abs(out_dev.cpu().numpy() - ref).max() <= TOL


def test_noalloc_more_than_64_rows():
    """96 rows = 9,216 cells per request: the attention takes the direct kernel for every request and
    reads the per-request path flags kept in the shared array."""
    lib = _lib.load_library()
    shape = ow.True2DShape(61, 96, 1)
    rng = np.random.default_rng(5)
    w = _weights(rng, shape)
    w_dev = torch.from_numpy(w).cuda()
    for games in (2, 1):
        x = rng.uniform(-1, 1, size=(games, 96, 7)).astype(np.float32)
        ref = _allocating_forward(lib, x, w, games, shape)
        out_dev = torch.full((games * 96 * 24,), float("nan"), device="cuda")
        _noalloc_forward(lib, torch.from_numpy(x).cuda(), w_dev, out_dev, games, shape)
        torch.cuda.synchronize()
        assert np.abs(out_dev.cpu().numpy() - ref).max() <= TOL


def test_noalloc_rejects_work_beyond_the_scratch():
    lib = _lib.load_library()
    games = MAX_GAMES_64 + 1  # 64 x (64^2 + 1) = 262,208 floats > 262,080
    x = torch.zeros(games * 64 * 7, device="cuda")
    w = torch.zeros(SHAPE.parameter_count(), device="cuda")
    out = torch.zeros(games * 64 * 24, device="cuda")
    st = lib.orbit_wars_cuda_true2d_forward_noalloc(x.data_ptr(), w.data_ptr(), out.data_ptr(), games, SHAPE.c(),
                                                    torch.cuda.current_stream().cuda_stream)
    assert st.code == 1 and b"scratch" in st.message
