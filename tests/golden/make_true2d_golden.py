"""Generates tests/golden/true2d_smoke_fixture.npz from the REFERENCE's own code.

Runs cpu_reference() of the reference smoke
(native/cuda/orbit_wars_cuda_true2d_smoke.cpp:127-260), compiled from the
reference source into oracle/_ref by `make -C oracle ref`, on that smoke's own
fixture: 2 games x 64 rows x 7 features with input[i] = sin((i+1)*0.11) and
two models with weights[i] = 0.02*sin((i+1)*0.17) and 0.02*sin((i+1)*0.23)
(orbit_wars_cuda_true2d_smoke.cpp:279-291). The inputs are regenerated in C by
the oracle's owo_sinusoid_fill so the fixture stores only outputs plus
checksums of the inputs.

    make -C oracle ref && python tests/golden/make_true2d_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))
from oracle import bind  # noqa: E402


def fixture_inputs():
    n_w = bind.true2d_weight_count(61, 64, 1)
    x = bind.sinusoid(2 * 64 * 7, 0.11)
    w1 = bind.sinusoid(n_w, 0.17, 0.02)
    w2 = bind.sinusoid(n_w, 0.23, 0.02)
    return x, w1, w2


def main() -> None:
    if not bind.ref_available():
        raise SystemExit("oracle/_ref/libref_true2d_cpu.so missing: run `make -C oracle ref` with the reference tree")
    ref = bind.load_ref_cpu()
    x, w1, w2 = fixture_inputs()
    assert ref.ref_true2d_smoke_weight_count() == w1.size
    outs = []
    for w in (w1, w2):
        o = np.zeros(2 * 64 * 24, dtype=np.float32)
        ref.ref_true2d_cpu_reference(x.ctypes.data, w.ctypes.data, o.ctypes.data)
        outs.append(o)
    np.savez_compressed(
        Path(__file__).with_name("true2d_smoke_fixture.npz"),
        out_model_a=outs[0], out_model_b=outs[1],
        input_sum=np.float64(x.astype(np.float64).sum()), w_a_sum=np.float64(w1.astype(np.float64).sum()),
        w_b_sum=np.float64(w2.astype(np.float64).sum()), input_head=x[:16], w_a_head=w1[:16], w_b_head=w2[:16],
    )
    print("wrote true2d_smoke_fixture.npz", outs[0][:6], outs[1][:6])


if __name__ == "__main__":
    main()
