"""orbit_wars_b200: host side of the B200 policy-forward library.

The compute lives in lib/liborbit_wars_cuda.so (hand-written sm_100a CUDA
behind a C ABI, include/ow_policy.h and include/orbit_wars_cuda.h); this
package loads it with ctypes and mirrors the engine-facing interfaces:

  EncoderPolicy       entity-encoder policy forward (ow_policy_*)
  CudaTrue2D          mirror of the engine's Rust binding to the True2D ABI
                      (crates/orbit-wars-trainer/src/cuda_true2d.rs), plus the
                      device encoder / decode around it
  GameBatch           game states for the device encoder (games.py)
  presets / synth     the five documented workloads and their seeded inputs

There is no CPU fallback: if the library or a GPU is missing, calls raise.
"""
from .presets import PolicyConfig, preset, PRESETS
from .synth import make_inputs, make_weights, weight_count
from ._lib import OwError, load_library, library_path
from .policy import EncoderPolicy
from .true2d import CudaTrue2D, EncodedRows, True2DShape
from .games import GameBatch, PLANET_DTYPE

__all__ = [
    "PolicyConfig", "preset", "PRESETS", "make_inputs", "make_weights", "weight_count",
    "OwError", "load_library", "library_path", "EncoderPolicy", "CudaTrue2D", "True2DShape",
    "EncodedRows", "GameBatch", "PLANET_DTYPE",
]
