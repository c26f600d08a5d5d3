"""Runs N device-IO forwards of a preset with nothing else on the stream, for
profilers (one forward = the launch sequence of ow_policy_forward).

    python -m orbit_wars_b200.profile_forward --config 2 --forwards 4 [--batch B]
    python -m orbit_wars_b200.profile_forward --workload true2d --forwards 4 [--requests R --models M]

The True2D workload is the drop-in's forward_many_resident on seeded models
(61 layers, 64 rows, 1 head): R requests over a resident population of M.

ncu's --launch-skip/--launch-count then select whole forwards: the launches
per forward are printed at the end.
"""
from __future__ import annotations

import argparse

import torch

from . import preset, make_inputs, make_weights
from .policy import EncoderPolicy


def true2d(a) -> None:
    import numpy as np

    from . import synth
    from .true2d import CudaTrue2D, True2DShape
    shape = True2DShape()
    lib = CudaTrue2D()
    pop = synth.true2d_population(17, a.models, shape.parameter_count())
    x, idx = synth.true2d_requests(17, a.requests, shape.rows, a.models)
    lib.upload_population(pop, a.requests, shape)
    for _ in range(a.forwards):
        out = lib.forward_population_resident_packed(x, idx, a.models, shape)
    print(f"true2d: {a.forwards} forwards of {a.requests} requests, finite={bool(np.isfinite(out).all())}")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="policy", choices=["policy", "true2d"])
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--forwards", type=int, default=4)
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--requests", type=int, default=1024)
    ap.add_argument("--models", type=int, default=64)
    a = ap.parse_args()
    if a.workload == "true2d":
        return true2d(a)
    cfg = preset(a.config)
    if a.batch:
        cfg = cfg.with_(batch=a.batch)
    w = make_weights(cfg, seed=17)
    feats, counts = make_inputs(cfg, seed=17)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    pol = EncoderPolicy(cfg, w, stream=stream.cuda_stream, io="device")
    f = torch.from_numpy(feats).cuda()
    c = torch.from_numpy(counts).cuda()
    ldt = torch.bfloat16 if cfg.logits_dtype == "bf16" else torch.float32
    vdt = torch.bfloat16 if cfg.value_dtype == "bf16" else torch.float32
    lg = torch.empty((cfg.batch, cfg.n_entities, cfg.actions), dtype=ldt, device="cuda")
    v = torch.empty((cfg.batch,), dtype=vdt, device="cuda")
    act = torch.empty((cfg.batch, cfg.n_entities), dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    for i in range(a.forwards):
        pol.forward_device(f.data_ptr(), c.data_ptr(), cfg.batch, lg.data_ptr(), v.data_ptr(), act.data_ptr(), seed=i)
    pol.synchronize()
    print(f"{cfg.name}: {a.forwards} forwards, {pol.launches_per_forward()} launches per forward")
    pol.close()


if __name__ == "__main__":
    main()
