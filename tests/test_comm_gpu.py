"""The library's weight broadcast (include/ow_policy.h, "Weight broadcast over NCCL").

A receiver created without weights must, after the broadcast, compute exactly
what the root computes. The multi-GPU cases need two devices and skip on one;
the one-rank communicator runs everywhere (the broadcast is then a copy onto
itself and must change nothing).
"""
import numpy as np
import pytest

import orbit_wars_b200 as ow
from orbit_wars_b200.policy import Comm, broadcast_weights_all

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _case(batch=32):
    cfg = ow.preset(2).with_(batch=batch)
    w = ow.make_weights(cfg, seed=23)
    feats, counts = ow.make_inputs(cfg, batch=batch, seed=29)
    return cfg, w, feats, counts


def test_one_rank_communicator_keeps_the_weights():
    cfg, w, feats, counts = _case()
    with ow.EncoderPolicy(cfg, w, device=0) as pol:
        before = pol.forward(feats, counts)
        comm = Comm(Comm.unique_id(), 1, 0, 0)
        ms = pol.broadcast_from(comm, root=0)
        after = pol.forward(feats, counts)
        comm.close()
    assert ms >= 0.0
    for a, b in zip(before, after):
        assert np.array_equal(a, b)


def test_weightless_handle_is_zero_until_filled():
    cfg, w, feats, counts = _case(8)
    with ow.EncoderPolicy(cfg, None, device=0) as pol:
        lg, v, a = pol.forward(feats, counts)
    m = np.arange(cfg.n_entities)[None, :] < counts[:, None]
    assert np.all(lg == 0.0) and np.all(v == 0.0)
    assert np.all(a[m] == 0) and np.all(a[~m] == -1)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_broadcast_fills_a_receiver_on_another_gpu():
    cfg, w, feats, counts = _case()
    root = ow.EncoderPolicy(cfg, w, device=0)
    recv = ow.EncoderPolicy(cfg, None, device=1)
    broadcast_weights_all([root, recv])
    want = root.forward(feats, counts)
    got = recv.forward(feats, counts)
    for a, b in zip(want, got):
        assert np.array_equal(a, b)
    root.close()
    recv.close()
