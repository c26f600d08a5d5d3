"""CPU-side checks of the C ABI library: it loads, exports every declared
symbol, validates arguments before touching a device, and fails loudly (no
CPU fallback) when no GPU is present."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

import orbit_wars_b200 as ow
from orbit_wars_b200 import _lib
from orbit_wars_b200.policy import to_config_c

REPO = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for h in (REPO / "include").glob("*.h"):
        txt = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b((?:ow_policy|ow_selftest|ow_comm|ow_nccl|orbit_wars)_\w+)\s*\(", txt))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    return _lib.load_library()


def test_every_declared_symbol_is_exported(lib):
    syms = declared_symbols()
    assert len(syms) >= 17
    for s in syms:
        assert hasattr(lib, s), s
        assert s in _lib.SIGNATURES, f"{s} missing from the ctypes signature table"


def test_engine_symbols_resolve_with_rtld_now():
    lib = C.CDLL(str(_lib.library_path()), mode=2)  # RTLD_NOW like cuda_true2d.rs:360
    for s in ow.true2d.ENGINE_SYMBOLS:
        getattr(lib, s)


@pytest.mark.parametrize("pid", [1, 2, 3, 4, 5])
def test_presets_match_host_configs(lib, pid):
    c = _lib.PolicyConfigC()
    _lib.check("preset", lib.ow_policy_preset(pid, C.byref(c)))
    want = to_config_c(ow.preset(pid))
    for name, _ in _lib.PolicyConfigC._fields_:
        assert getattr(c, name) == getattr(want, name), name
    n = C.c_size_t()
    _lib.check("weight_count", lib.ow_policy_weight_count(C.byref(c), C.byref(n)))
    assert n.value == ow.weight_count(ow.preset(pid))


def test_bad_configs_are_bad_arguments(lib):
    base = to_config_c(ow.preset(2))
    for field, val in [("heads", 7), ("n_entities", 200), ("d_model", 100), ("actions", 40), ("precision", 9),
                       ("batch_capacity", 0), ("layers", 0), ("io", 5)]:
        c = _lib.PolicyConfigC.from_buffer_copy(base)
        setattr(c, field, val)
        n = C.c_size_t()
        st = lib.ow_policy_weight_count(C.byref(c), C.byref(n))
        assert st.code == 1, field


def test_create_validates_before_device(lib):
    cfg = ow.preset(1)
    c = to_config_c(cfg)
    w = np.zeros(ow.weight_count(cfg) - 1, dtype=np.float32)
    h = C.c_void_p()
    st = lib.ow_policy_create(C.byref(c), w.ctypes.data_as(_lib.FP), w.size, 0, None, C.byref(h))
    assert st.code == 1 and b"weight_count" in st.message
    w = np.zeros(ow.weight_count(cfg), dtype=np.float32)
    w[5] = np.nan
    st = lib.ow_policy_create(C.byref(c), w.ctypes.data_as(_lib.FP), w.size, 0, None, C.byref(h))
    assert st.code == 1 and b"non-finite" in st.message
    st = lib.ow_policy_forward(None, None, None, 1, None, None, None, 0)
    assert st.code == 1


def test_no_gpu_means_runtime_error_not_fallback(lib):
    pytest.importorskip("torch")
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    cfg = ow.preset(1)
    with pytest.raises(ow.OwError) as e:
        ow.EncoderPolicy(cfg, ow.make_weights(cfg))
    assert e.value.code == 2
    st = lib.orbit_wars_cuda_status()
    assert st.code == 2


def test_true2d_abi_validates_arguments(lib):
    shape = _lib.True2DShapeC(61, 64, 1)
    st = lib.orbit_wars_cuda_true2d_forward(None, None, None, 1, shape)
    assert st.code == 1
    bad = _lib.True2DShapeC(0, 64, 1)
    x = np.zeros(64 * 7, np.float32)
    st = lib.orbit_wars_cuda_true2d_forward(x.ctypes.data, x.ctypes.data, x.ctypes.data, 1, bad)
    assert st.code == 1
    st = lib.orbit_wars_cuda_true2d_forward_many_resident(x.ctypes.data, x.ctypes.data, x.ctypes.data, 0, shape)
    assert st.code == 1
    st = lib.orbit_wars_cuda_encode_identity_batch(None, None, 1, 1, 1)
    assert st.code == 1


def test_nccl_resolves_at_run_time(lib):
    """The weight broadcast's NCCL is found without linking it (no GPU needed to load it)."""
    import ctypes as C
    v = C.c_int()
    st = lib.ow_nccl_version(C.byref(v))
    assert st.code == 0, st.message
    assert v.value >= 21800


def test_broadcast_validates_arguments(lib):
    import ctypes as C
    assert lib.ow_policy_broadcast_weights(None, 2).code == 1
    assert lib.ow_policy_broadcast_weights_comm(None, None, 0, None).code == 1
    h = C.c_void_p()
    assert lib.ow_comm_init_rank(None, 128, 2, 0, 0, C.byref(h)).code == 1
    uid = C.create_string_buffer(128)
    assert lib.ow_comm_init_rank(uid, 128, 2, 2, 0, C.byref(h)).code == 1  # rank outside [0, nranks)
    assert lib.ow_comm_unique_id(uid, 16).code == 1  # id buffer too short
