"""ctypes binding of liborbit_wars_cuda.so (both C ABIs).

The library is built in-tree by orbit-wars-2d-transformer_b200/build.py.
$ORBIT_WARS_CUDA_LIB_PATH overrides the path, as in the reference engine's
loader (crates/orbit-wars-trainer/src/cuda_true2d.rs:8-9, :98-102).
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_ENV = "ORBIT_WARS_CUDA_LIB_PATH"
_DEFAULT = Path(__file__).resolve().parent / "lib" / "liborbit_wars_cuda.so"
_lib = None


class OwError(RuntimeError):
    """A non-zero status {code, message} from the library (1 BAD_ARGUMENT, 2 RUNTIME_ERROR)."""

    def __init__(self, op: str, code: int, message: str):
        super().__init__(f"{op}: code={code} message={message}")
        self.op, self.code, self.message = op, code, message


class Status(C.Structure):
    _fields_ = [("code", C.c_int), ("message", C.c_char_p)]


class PolicyConfigC(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "batch_capacity", "n_entities", "features", "d_model", "heads", "ffn", "layers", "actions",
        "precision", "sample_actions", "logits_dtype", "value_dtype", "io")]


class True2DShapeC(C.Structure):
    _fields_ = [("layer_count", C.c_size_t), ("row_count", C.c_size_t), ("head_count", C.c_size_t)]


class TransformerShapeC(C.Structure):
    _fields_ = [("layer_count", C.c_size_t), ("d_model", C.c_size_t), ("head_count", C.c_size_t),
                ("row_count", C.c_size_t)]


class TrainingConfigC(C.Structure):
    _fields_ = [("batch_sample_count", C.c_size_t), ("learning_rate", C.c_float),
                ("reward_normalizer", C.c_float), ("send_threshold", C.c_float),
                ("owner_class_own", C.c_float), ("owner_class_empty", C.c_float),
                ("owner_class_absent_on_map", C.c_float)]


class EncoderConfigC(C.Structure):
    """OrbitWarsEncoderConfig (include/orbit_wars_cuda.h)."""
    _fields_ = [("max_rows", C.c_size_t), ("initial_planet_slots", C.c_size_t), ("comet_slots", C.c_size_t),
                ("padding_slots", C.c_size_t), ("ship_log_pivot", C.c_float), ("ship_log_cap", C.c_float),
                ("max_players", C.c_size_t), ("owner_class_own", C.c_float), ("owner_class_enemy_1", C.c_float),
                ("owner_class_enemy_2", C.c_float), ("owner_class_enemy_3", C.c_float),
                ("owner_class_neutral", C.c_float), ("owner_class_empty", C.c_float),
                ("owner_class_absent_on_map", C.c_float), ("board_size", C.c_float),
                ("fleet_speed_max", C.c_float)]


class GameBatchC(C.Structure):
    """OrbitWarsGameBatch (include/orbit_wars_cuda.h): CSR game states."""
    _fields_ = [("planets", C.c_void_p), ("planet_offsets", C.c_void_p), ("initial_planets", C.c_void_p),
                ("initial_offsets", C.c_void_p), ("comet_planet_ids", C.c_void_p), ("comet_offsets", C.c_void_p),
                ("game_count", C.c_size_t)]


class KernelTimingC(C.Structure):
    _fields_ = [("name", C.c_char_p), ("launches", C.c_int32), ("total_ms", C.c_float)]


P = C.c_void_p
FP = C.POINTER(C.c_float)
SZ = C.c_size_t

SIGNATURES = {
    # include/ow_policy.h
    "ow_policy_preset": (Status, [C.c_int, C.POINTER(PolicyConfigC)]),
    "ow_policy_weight_count": (Status, [C.POINTER(PolicyConfigC), C.POINTER(SZ)]),
    "ow_policy_create": (Status, [C.POINTER(PolicyConfigC), FP, SZ, C.c_int, P, C.POINTER(P)]),
    "ow_policy_set_weights": (Status, [P, FP, SZ]),
    "ow_policy_forward": (Status, [P, P, P, C.c_int32, P, P, P, C.c_uint64]),
    "ow_policy_submit": (Status, [P, P, P, C.c_int32, P, P, P, C.c_uint64, C.POINTER(C.c_int64)]),
    "ow_policy_wait": (Status, [P, C.c_int64]),
    "ow_policy_synchronize": (Status, [P]),
    "ow_policy_device_weights": (Status, [P, C.POINTER(P), C.POINTER(SZ)]),
    "ow_policy_launches_per_forward": (Status, [P, C.POINTER(C.c_int32)]),
    "ow_policy_profile_begin": (Status, [P, C.c_int32]),
    "ow_policy_profile_end": (Status, [P, C.POINTER(KernelTimingC), C.c_int32, C.POINTER(C.c_int32)]),
    "ow_policy_destroy": (None, [P]),
    "ow_comm_unique_id": (Status, [P, SZ]),
    "ow_comm_init_rank": (Status, [P, SZ, C.c_int, C.c_int, C.c_int, C.POINTER(P)]),
    "ow_comm_init_all": (Status, [P, C.c_int, P]),
    "ow_comm_info": (Status, [P, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "ow_comm_destroy": (None, [P]),
    "ow_policy_broadcast_weights_comm": (Status, [P, P, C.c_int, FP]),
    "ow_policy_broadcast_weights": (Status, [P, C.c_int]),
    "ow_nccl_version": (Status, [C.POINTER(C.c_int)]),
    "ow_selftest_gemm": (Status, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P, P, P, P, P, P, P, P, C.c_int, P, P,
                                  P, P]),
    "ow_selftest_ffn": (Status, [C.c_int, C.c_int, C.c_int, P, P, P, P, P, P, P, P, P, C.c_int, P]),
    "ow_selftest_attention": (Status, [C.c_int, C.c_int, C.c_int, C.c_int, P, P, P, P]),
    # include/orbit_wars_cuda.h
    "orbit_wars_cuda_status": (Status, []),
    "orbit_wars_cuda_encode_identity_batch": (Status, [P, P, SZ, SZ, SZ]),
    "orbit_wars_cuda_trainable_forward": (Status, [P, P, P, SZ, TransformerShapeC]),
    "orbit_wars_cuda_true2d_forward": (Status, [P, P, P, SZ, True2DShapeC]),
    "orbit_wars_cuda_true2d_forward_many": (Status, [P, P, P, P, SZ, SZ, True2DShapeC]),
    "orbit_wars_cuda_true2d_upload_population": (Status, [P, SZ, SZ, True2DShapeC]),
    "orbit_wars_cuda_true2d_forward_many_resident": (Status, [P, P, P, SZ, True2DShapeC]),
    "orbit_wars_cuda_true2d_forward_noalloc": (Status, [P, P, P, SZ, True2DShapeC, P]),
    "orbit_wars_cuda_true2d_decode_many_resident": (Status, [P, P, P, P, P, P, P, P, SZ, True2DShapeC]),
    "orbit_wars_cuda_true2d_decode_outputs": (Status, [P, P, P, P, P, P, SZ, SZ]),
    "orbit_wars_encoder_config_default": (None, [C.POINTER(EncoderConfigC)]),
    "orbit_wars_cuda_encode_states": (Status, [C.POINTER(GameBatchC), P, P, SZ, C.POINTER(EncoderConfigC), P, P, P, P,
                                               P]),
    "orbit_wars_cuda_true2d_play_many_resident": (
        Status, [C.POINTER(GameBatchC), P, P, P, SZ, C.POINTER(EncoderConfigC), P, P, P, P, P, P, True2DShapeC]),
    "orbit_wars_cuda_true2d_profile_begin": (Status, [C.c_int32]),
    "orbit_wars_cuda_mufu_rate": (Status, [C.c_int32, C.POINTER(C.c_double), C.POINTER(C.c_double),
                                           C.POINTER(C.c_double)]),
    "orbit_wars_cuda_true2d_profile_end": (Status, [C.POINTER(KernelTimingC), C.c_int32, C.POINTER(C.c_int32)]),
    "orbit_wars_cuda_true2d_train_full_attention": (
        Status, [P, P, P, P, P, P, SZ, SZ, True2DShapeC, TrainingConfigC]),
}


def library_path() -> Path:
    env = os.environ.get(LIB_ENV)
    return Path(env) if env else _DEFAULT


def load_library(path: str | os.PathLike | None = None):
    """Loads the library (RTLD_NOW, like the engine) and binds every declared symbol.

    Raises OwError if the library is missing: there is no fallback path.
    """
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else library_path()
    if not p.exists():
        raise OwError("load_library", 2, f"library not built: {p} (run orbit-wars-2d-transformer_b200/build.py)")
    lib = C.CDLL(str(p), mode=os.RTLD_NOW | os.RTLD_LOCAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def check(op: str, st: Status) -> None:
    if st.code != 0:
        raise OwError(op, st.code, (st.message or b"").decode(errors="replace"))


def ptr(a) -> int | None:
    """Raw address of a numpy array or torch tensor (None passes NULL)."""
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data
