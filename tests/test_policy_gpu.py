"""GPU parity of the encoder-policy forward against the CPU oracle.

Tolerances: fp32 rel <= 1e-4 and bf16 <= 1e-2 against the float64 truth, on
logits and value. fp8: the recipe itself loses about 4.7e-2 against the truth,
so the fp8 path is held to the recipe's own error on the same inputs (the
oracle's exact emulation of the recipe; tests/util.py gives the gate). Greedy argmax agreement >= 99.9% (ties within the precision's noise
excluded); masks bit-exact.
"""
import numpy as np
import pytest

import orbit_wars_b200 as ow
from tests.util import (TOL, check_fp8_against_recipe, argmax_agreement, near_tie_mask, rel_err, representable_embedding,
                        representable_weights, valid_mask)

pytestmark = pytest.mark.gpu

# (preset, states compared) -- sizes the float64 oracle finishes in seconds
CASES = [(1, 64), (2, 48), (3, 48), (4, 12), (5, 4)]
TIE_MARGIN = {"f32": 1e-5, "bf16": 5e-2, "fp8": 1.5e-1}


def edge_counts(cfg, batch, seed):
    _, counts = ow.make_inputs(cfg, batch=batch, seed=seed)
    counts[0] = 0
    counts[1] = 1
    counts[2] = cfg.n_entities
    if batch > 3:
        counts[3] = 15 if cfg.n_entities > 16 else cfg.n_entities  # ragged vs the 16-row attention blocks
    return counts


def check_parity(cfg, gpu, ref, counts):
    g_lg, g_v, g_a = gpu
    r_lg, r_v, r_a = ref
    m = valid_mask(counts, cfg.n_entities)
    # masks and indices bit-exact
    assert np.all(g_lg[~m] == 0.0)
    assert np.all(g_a[~m] == -1)
    assert np.all((g_a[m] >= 0) & (g_a[m] < cfg.actions))
    tol = TOL[cfg.precision]
    e_l = rel_err(g_lg[m], r_lg[m])
    e_v = rel_err(g_v, r_v)
    assert e_l <= tol and e_v <= tol, f"logits rel err {e_l:.3e}, value rel err {e_v:.3e} (tol {tol})"
    return e_l, e_v


def check_fp8_parity(cfg, gpu, truth, recipe, counts):
    """fp8: masks as everywhere; values against the truth within the recipe's own error (tests/util.py)."""
    m = valid_mask(counts, cfg.n_entities)
    assert np.all(gpu[0][~m] == 0.0) and np.all(gpu[2][~m] == -1)
    assert np.all((gpu[2][m] >= 0) & (gpu[2][m] < cfg.actions))
    r = check_fp8_against_recipe(gpu[0], gpu[1], truth, recipe, m)
    print(f"{cfg.name}: " + "; ".join(f"{k} vs truth {v['vs_truth']:.2e} (recipe alone {v['recipe']:.2e}, "
                                       f"rms {v['vs_truth_rms']:.2e} / {v['recipe_rms']:.2e}), "
                                       f"vs recipe {v['vs_recipe']:.2e}" for k, v in r.items()))
    return r["logits"]["vs_truth"], r["value"]["vs_truth"]


def model_weights(cfg, seed, affine_noise=True):
    """Seeded weights as the path's model holds them (bf16 / per-channel e4m3
    matrices, bf16 embedding): GPU and oracle get the identical blob."""
    w = ow.make_weights(cfg, seed=seed, affine_noise=affine_noise)
    return representable_embedding(cfg, representable_weights(cfg, w))


@pytest.mark.parametrize("pid,batch", CASES)
def test_policy_matches_oracle(oracle, pid, batch):
    cfg = ow.preset(pid).with_(batch=batch)
    w = model_weights(cfg, seed=11)
    counts = edge_counts(cfg, batch, seed=21)
    feats, counts = ow.make_inputs(cfg, batch=batch, seed=21, counts=counts)
    with ow.EncoderPolicy(cfg, w) as pol:
        gpu = pol.forward(feats, counts, seed=5)
    ref = oracle.policy_forward(cfg, w, feats, counts, f64=True, sample=False)
    if cfg.precision == "fp8":
        e_l, e_v = check_fp8_parity(cfg, gpu, ref, oracle.policy_forward_emulated(cfg, w, feats, counts), counts)
    else:
        e_l, e_v = check_parity(cfg, gpu, ref, counts)
    if not cfg.sample_actions and cfg.precision != "fp8":
        m = valid_mask(counts, cfg.n_entities) & ~near_tie_mask(ref[0], counts, cfg.n_entities,
                                                                 TIE_MARGIN[cfg.precision])
        agree = float((gpu[2][m] == ref[2][m]).mean()) if m.any() else 1.0
        assert agree >= 0.999, f"argmax agreement {agree:.4f}"
        assert argmax_agreement(gpu[2], ref[2], counts, cfg.n_entities) >= 0.99
    print(f"{cfg.name}: logits rel {e_l:.2e} value rel {e_v:.2e}")


def test_gumbel_actions_replicate_spec(oracle):
    """C4 sampling: actions == argmax(gpu logits + G) with G from the spec's Philox stream."""
    cfg = ow.preset(4).with_(batch=8)
    w = ow.make_weights(cfg, seed=2)
    feats, counts = ow.make_inputs(cfg, batch=8, seed=3)
    seed = 0xABCDEF0123
    with ow.EncoderPolicy(cfg, w) as pol:
        lg, _, a = pol.forward(feats, counts, seed=seed)
    m = valid_mask(counts, cfg.n_entities)
    agree = total = 0
    for b in range(cfg.batch):
        for j in range(int(counts[b])):
            g = np.array([oracle.gumbel(seed, b, j, p) for p in range(cfg.actions)])
            s = lg[b, j].astype(np.float64) + g
            top2 = np.sort(s)[-2:]
            if top2[1] - top2[0] < 1e-4:
                continue
            total += 1
            agree += int(np.argmax(s) == a[b, j])
    assert total > 0 and agree == total
    assert np.all(a[~m] == -1)


def test_device_io_matches_host_io():
    torch = pytest.importorskip("torch")
    cfg = ow.preset(2).with_(batch=64)
    w = ow.make_weights(cfg, seed=4)
    feats, counts = ow.make_inputs(cfg, batch=64, seed=6)
    with ow.EncoderPolicy(cfg, w) as pol:
        h_lg, h_v, h_a = pol.forward(feats, counts)
    stream = torch.cuda.current_stream()
    with ow.EncoderPolicy(cfg, w, io="device", stream=stream.cuda_stream) as pol:
        f = torch.from_numpy(feats).cuda()
        c = torch.from_numpy(counts).cuda()
        lg = torch.empty((64, cfg.n_entities, cfg.actions), dtype=torch.bfloat16, device="cuda")
        v = torch.empty((64,), dtype=torch.float32, device="cuda")
        a = torch.empty((64, cfg.n_entities), dtype=torch.int32, device="cuda")
        pol.forward_device(f.data_ptr(), c.data_ptr(), 64, lg.data_ptr(), v.data_ptr(), a.data_ptr())
        pol.synchronize()
        assert np.array_equal(lg.float().cpu().numpy(), h_lg)
        assert np.array_equal(v.cpu().numpy(), h_v)
        assert np.array_equal(a.cpu().numpy(), h_a)


def test_full_batch_properties():
    """Config-2 full batch: deterministic, permutation-equivariant, padding-invariant (bit-exact)."""
    cfg = ow.preset(2)
    w = ow.make_weights(cfg, seed=17)
    feats, counts = ow.make_inputs(cfg, seed=17)
    names = ("logits", "value", "actions")

    def same(x, y, what):
        for n, a, b in zip(names, x, y):
            if not np.array_equal(a, b):
                diff = np.argwhere(a != b)
                raise AssertionError(f"{what}: {n} differs at {len(diff)} places, first {diff[:3].tolist()}")

    with ow.EncoderPolicy(cfg, w) as pol:
        r1 = pol.forward(feats, counts)
        r2 = pol.forward(feats, counts)
        same(r1, r2, "repeat")
        perm = np.random.default_rng(0).permutation(cfg.batch)
        r3 = pol.forward(feats[perm], counts[perm])
        same(tuple(x[perm] for x in r1), r3, "permutation")
        dirty = feats.copy()
        dirty[~valid_mask(counts, cfg.n_entities)] = 77.0
        r4 = pol.forward(dirty, counts)
        same(r1, r4, "padding")
        assert np.all(np.isfinite(r1[0])) and np.all(np.isfinite(r1[1]))


def test_bad_count_is_rejected():
    cfg = ow.preset(1)
    w = ow.make_weights(cfg)
    feats, counts = ow.make_inputs(cfg, batch=4)
    counts[2] = cfg.n_entities + 3
    with ow.EncoderPolicy(cfg, w) as pol:
        with pytest.raises(ow.OwError) as e:
            pol.forward(feats, counts)
        assert e.value.code == 1
        # the handle stays usable after a rejected call
        counts[2] = 1
        pol.forward(feats, counts)


def test_device_side_bad_count_reports_runtime_error():
    torch = pytest.importorskip("torch")
    cfg = ow.preset(2).with_(batch=8)
    w = ow.make_weights(cfg)
    feats, counts = ow.make_inputs(cfg, batch=8)
    counts[3] = -4
    stream = torch.cuda.current_stream()
    with ow.EncoderPolicy(cfg, w, io="device", stream=stream.cuda_stream) as pol:
        f = torch.from_numpy(feats).cuda()
        c = torch.from_numpy(counts).cuda()
        lg = torch.empty((8, cfg.n_entities, cfg.actions), dtype=torch.bfloat16, device="cuda")
        v = torch.empty((8,), dtype=torch.float32, device="cuda")
        a = torch.empty((8, cfg.n_entities), dtype=torch.int32, device="cuda")
        pol.forward_device(f.data_ptr(), c.data_ptr(), 8, lg.data_ptr(), v.data_ptr(), a.data_ptr())
        with pytest.raises(ow.OwError) as e:
            pol.synchronize()
        assert e.value.code == 2
        pol.synchronize()  # error word cleared; handle usable


def test_fused_ffn_matches_two_kernel_path(monkeypatch):
    """Config-2 full batch (315 row tiles, several per CTA), f32 residual stream
    (ORBIT_WARS_X_F32=1): the fused FFN kernel (ORBIT_WARS_FFN_FUSED=1) against the
    up-projection + down-projection kernels. Each CTA starts the hidden-chunk walk at its own chunk, so the
    down-projection sums the same terms in another order: outputs agree to f32
    rounding, far inside the bf16 tolerance, and each path repeats bit for bit."""
    cfg = ow.preset(2)
    w = ow.make_weights(cfg, seed=17)
    feats, counts = ow.make_inputs(cfg, seed=17)
    monkeypatch.setenv("ORBIT_WARS_X_F32", "1")  # the fused FFN kernel keeps the residual stream in f32
    with ow.EncoderPolicy(cfg, w) as pol:
        two = pol.forward(feats, counts)
        assert pol.launches_per_forward() == 3 + 5 * cfg.layers + 1
    monkeypatch.setenv("ORBIT_WARS_FFN_FUSED", "1")
    with ow.EncoderPolicy(cfg, w) as pol:
        fused = pol.forward(feats, counts)
        again = pol.forward(feats, counts)
        assert pol.launches_per_forward() == 3 + 4 * cfg.layers + 1
    for a, b in zip(fused, again):
        assert np.array_equal(a, b)
    m = valid_mask(counts, cfg.n_entities)
    assert rel_err(fused[0][m], two[0][m]) <= 1e-2 and rel_err(fused[1], two[1]) <= 1e-2
    assert float((fused[2][m] == two[2][m]).mean()) >= 0.99


def test_bf16_and_f32_residual_streams_agree(monkeypatch):
    """Config 2: the default bf16 residual stream (16-warp LayerNorm epilogue) and the f32 one
    (ORBIT_WARS_X_F32=1) agree within the bf16 tolerance, and both repeat bit for bit."""
    cfg = ow.preset(2).with_(batch=256)
    w = ow.make_weights(cfg, seed=19)
    feats, counts = ow.make_inputs(cfg, batch=256, seed=19)
    outs = {}
    for mode in ("0", "1"):
        monkeypatch.setenv("ORBIT_WARS_X_F32", mode)
        with ow.EncoderPolicy(cfg, w) as pol:
            a = pol.forward(feats, counts)
            b = pol.forward(feats, counts)
        for u, v in zip(a, b):
            assert np.array_equal(u, v)
        outs[mode] = a
    m = valid_mask(counts, cfg.n_entities)
    assert rel_err(outs["0"][0][m], outs["1"][0][m]) <= 1e-2
    assert rel_err(outs["0"][1], outs["1"][1]) <= 1e-2


def test_submit_wait_pipeline():
    """Pipelined host IO: two submissions in flight give the synchronous forward's
    outputs bit for bit; a third submit before a wait and unknown tickets are rejected."""
    cfg = ow.preset(2).with_(batch=96)
    w = ow.make_weights(cfg, seed=3)
    fa, ca = ow.make_inputs(cfg, seed=4)
    fb, cb = ow.make_inputs(cfg, seed=5)
    with ow.EncoderPolicy(cfg, w) as pol:
        ref_a = pol.forward(fa, ca, seed=1)
        ref_b = pol.forward(fb, cb, seed=2)
        bufs = []
        for f, c in ((fa, ca), (fb, cb)):
            lg = np.empty((cfg.batch, cfg.n_entities, cfg.actions), np.uint16)
            v = np.empty((cfg.batch,), np.float32)
            a = np.empty((cfg.batch, cfg.n_entities), np.int32)
            bufs.append((np.ascontiguousarray(f), np.ascontiguousarray(c, dtype=np.int32), lg, v, a))
        tickets = [pol.submit_raw(f.ctypes.data, c.ctypes.data, cfg.batch, lg.ctypes.data, v.ctypes.data,
                                  a.ctypes.data, seed=s) for (f, c, lg, v, a), s in zip(bufs, (1, 2))]
        f, c, lg, v, a = bufs[0]
        with pytest.raises(ow.OwError) as e:
            pol.submit_raw(f.ctypes.data, c.ctypes.data, cfg.batch, lg.ctypes.data, v.ctypes.data, a.ctypes.data)
        assert e.value.code == 1
        with pytest.raises(ow.OwError):
            pol.wait(tickets[1] + 5)
        for t in tickets:
            pol.wait(t)
        with pytest.raises(ow.OwError):
            pol.wait(tickets[0])  # already waited for
        for (f, c, lg, v, a), ref in zip(bufs, (ref_a, ref_b)):
            assert np.array_equal((lg.astype(np.uint32) << 16).view(np.float32), ref[0])
            assert np.array_equal(v, ref[1]) and np.array_equal(a, ref[2])
        # the handle keeps working synchronously afterwards
        again = pol.forward(fa, ca, seed=1)
        assert np.array_equal(again[0], ref_a[0])


@pytest.mark.parametrize("pid,batch", [(4, 256), (2, 1024)])
def test_split_device_forward_matches_host(pid, batch):
    """A device-IO forward of 64+ states runs as two halves on two streams; its
    outputs equal the unsplit host-IO forward bit for bit, Gumbel-sampled actions
    included (keys use the global state index)."""
    torch = pytest.importorskip("torch")
    cfg = ow.preset(pid).with_(batch=batch)
    w = ow.make_weights(cfg, seed=8)
    feats, counts = ow.make_inputs(cfg, batch=batch, seed=9)
    seed = 0x1234567
    with ow.EncoderPolicy(cfg, w) as pol:
        h_lg, h_v, h_a = pol.forward(feats, counts, seed=seed)
    stream = torch.cuda.Stream()
    with ow.EncoderPolicy(cfg, w, io="device", stream=stream.cuda_stream) as pol:
        f = torch.from_numpy(feats).cuda()
        c = torch.from_numpy(counts).cuda()
        ldt = torch.bfloat16 if cfg.logits_dtype == "bf16" else torch.float32
        vdt = torch.bfloat16 if cfg.value_dtype == "bf16" else torch.float32
        lg = torch.empty((batch, cfg.n_entities, cfg.actions), dtype=ldt, device="cuda")
        v = torch.empty((batch,), dtype=vdt, device="cuda")
        a = torch.empty((batch, cfg.n_entities), dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        pol.forward_device(f.data_ptr(), c.data_ptr(), batch, lg.data_ptr(), v.data_ptr(), a.data_ptr(), seed=seed)
        pol.synchronize()
        assert np.array_equal(lg.float().cpu().numpy(), h_lg)
        assert np.array_equal(v.float().cpu().numpy(), h_v)
        assert np.array_equal(a.cpu().numpy(), h_a)
