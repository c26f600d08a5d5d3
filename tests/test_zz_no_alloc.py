"""The allocation-free True2D forward (orbit_wars_cuda_true2d_forward_noalloc).

Some callers of the drop-in cannot allocate device memory: an engine whose
device memory is all reserved by its own pool, or a self-play loop that must
not pay cudaMalloc/cudaFree's implicit device-wide synchronisation between
turns. This entry point takes device buffers and keeps its scratch in a fixed
1 MiB array inside the library. It must produce what the allocating entry
point produces, call after call (the shared array keeps the previous call's
contents), and refuse work that does not fit.

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


def _allocating_forward(lib, x, w, games):
    out = np.zeros(games * 64 * 24, np.float32)
    _lib.check("orbit_wars_cuda_true2d_forward", lib.orbit_wars_cuda_true2d_forward(
        x.ctypes.data, w.ctypes.data, out.ctypes.data, games, SHAPE.c()))
    return out


def test_noalloc_matches_allocating_entry_point_two_calls():
    lib = _lib.load_library()
    rng = np.random.default_rng(7)
    w = (rng.standard_normal(SHAPE.parameter_count()) * 0.05).astype(np.float32)
    w_dev = torch.from_numpy(w).cuda()
    stream = torch.cuda.current_stream()
    for games in (5, 3):  # two calls in a row on the shared scratch
        x = rng.uniform(-1, 1, size=(games, 64, 7)).astype(np.float32)
        ref = _allocating_forward(lib, x, w, games)
        x_dev = torch.from_numpy(x).cuda()
        out_dev = torch.full((games * 64 * 24,), float("nan"), device="cuda")
        st = lib.orbit_wars_cuda_true2d_forward_noalloc(x_dev.data_ptr(), w_dev.data_ptr(), out_dev.data_ptr(),
                                                        games, SHAPE.c(), stream.cuda_stream)
        _lib.check("orbit_wars_cuda_true2d_forward_noalloc", st)
        torch.cuda.synchronize()
        out = out_dev.cpu().numpy()
        assert np.all(np.isfinite(out))
        assert np.abs(out - ref).max() <= TOL


def test_noalloc_rejects_work_beyond_the_scratch():
    lib = _lib.load_library()
    games = 64  # 64 x (64^2 + 1) = 262,208 floats > 262,080
    x = torch.zeros(games * 64 * 7, device="cuda")
    w = torch.zeros(SHAPE.parameter_count(), device="cuda")
    out = torch.zeros(games * 64 * 24, device="cuda")
    st = lib.orbit_wars_cuda_true2d_forward_noalloc(x.data_ptr(), w.data_ptr(), out.data_ptr(), games, SHAPE.c(),
                                                    torch.cuda.current_stream().cuda_stream)
    assert st.code == 1 and b"scratch" in st.message
