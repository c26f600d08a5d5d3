"""Masked attention launches (ow_selftest_attention) against a plain PyTorch
fp32 reference: per state and head, softmax(Q K^T / sqrt(32)) V over the
state's own rows, on the packed token layout. Both device kernels are run: the
tcgen05 kernel (S and P in tensor memory, the forward's default) and the
mma.sync kernel it replaced."""
import numpy as np
import pytest

from orbit_wars_b200 import _lib

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TC, MMA = 0, 1


def run(kernel, counts, n_entities, heads, qkv):
    lib = _lib.load_library()
    batch = len(counts)
    d = 32 * heads
    cnt = torch.tensor(counts, dtype=torch.int32, device="cuda")
    out = torch.full((batch * n_entities, d), float("nan"), device="cuda", dtype=torch.bfloat16)
    st = lib.ow_selftest_attention(kernel, batch, n_entities, heads, _lib.ptr(cnt), _lib.ptr(qkv), _lib.ptr(out),
                                   torch.cuda.current_stream().cuda_stream)
    _lib.check("ow_selftest_attention", st)
    return out[: int(sum(counts))]


def reference(counts, heads, qkv):
    d = 32 * heads
    rows = int(sum(counts))
    q = qkv[:rows, :d].float()
    k = qkv[:rows, d:2 * d].float()
    v = qkv[:rows, 2 * d:].float()
    out = torch.zeros(rows, d, device="cuda")
    r0 = 0
    for c in counts:
        if c:
            for h in range(heads):
                cs = slice(32 * h, 32 * h + 32)
                s = q[r0:r0 + c, cs] @ k[r0:r0 + c, cs].T / 32 ** 0.5
                out[r0:r0 + c, cs] = torch.softmax(s, dim=1) @ v[r0:r0 + c, cs]
        r0 += c
    return out


def make_qkv(counts, n_entities, heads, scale, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    d = 32 * heads
    qkv = (torch.randn(len(counts) * n_entities, 3 * d, device="cuda", generator=g) * scale).bfloat16()
    qkv[int(sum(counts)):] = 0  # rows past the batch: zero, as a fresh forward workspace holds
    return qkv


def check(counts, n_entities, heads, scale=1.0, seed=0, tol=1.2e-2):
    qkv = make_qkv(counts, n_entities, heads, scale, seed)
    ref = reference(counts, heads, qkv)
    den = max(ref.abs().max().item(), 1e-6)
    outs = {}
    for kernel in (TC, MMA):
        out = run(kernel, counts, n_entities, heads, qkv).float()
        assert torch.isfinite(out).all(), f"kernel {kernel}: non-finite output"
        err = (out - ref).abs().max().item() / den
        assert err <= tol, f"kernel {kernel}: rel err {err:.3e} > {tol}"
        outs[kernel] = out
    diff = (outs[TC] - outs[MMA]).abs().max().item() / den
    assert diff <= tol, f"tcgen05 vs mma.sync: {diff:.3e}"


def rng_counts(batch, lo, hi, seed):
    return np.random.default_rng(seed).integers(lo, hi + 1, size=batch).tolist()


@pytest.mark.parametrize("batch,n,heads,lo", [(1024, 64, 8, 16), (96, 32, 4, 8), (150, 96, 12, 24),
                                              (120, 128, 16, 32)])
def test_config_shapes(batch, n, heads, lo):
    check(rng_counts(batch, lo, n, batch + n), n, heads, seed=batch)


@pytest.mark.parametrize("n,heads", [(64, 8), (128, 16)])
def test_ragged_counts_with_empty_and_full_states(n, heads):
    rng = np.random.default_rng(n)
    counts = rng.integers(0, n + 1, size=400)
    counts[rng.random(400) < 0.2] = 0
    counts[rng.random(400) < 0.1] = 1
    counts[rng.random(400) < 0.1] = n
    check(counts.tolist(), n, heads, seed=n + 1)


@pytest.mark.parametrize("c", [1, 2, 3])
def test_many_states_per_tile(c):
    # 128 / c states share a 128-row query tile (state indices up to 127 in the mask)
    check([c] * 700, 64, 8, seed=c)


def test_tiny_batches():
    check([1], 64, 8)
    check([0, 5, 0], 64, 8)
    check([64], 64, 8)
    # a batch without valid rows launches and returns cleanly for both kernels
    qkv = make_qkv([0, 0], 64, 8, 1.0, 0)
    for kernel in (TC, MMA):
        assert run(kernel, [0, 0], 64, 8, qkv).shape[0] == 0


def test_large_scores():
    # scores of several tens: the mask's -2^20 offset must still dominate
    check(rng_counts(300, 16, 64, 5), 64, 8, scale=2.5, seed=5, tol=2e-2)


def test_all_full_states():
    check([128] * 64, 128, 16, seed=9)
    check([64] * 256, 64, 8, seed=10)


@pytest.mark.parametrize("n,heads", [(64, 8), (128, 16)])
def test_state_results_independent_of_position(n, heads):
    # each state sits at its own block of a tile and its keys are summed in blocks
    # aligned to its first row, so moving it in the batch changes no output bit
    counts = rng_counts(200, n // 4, n, n)
    qkv = make_qkv(counts, n, heads, 1.0, 21)
    for lead in ([7], [n, 3], [1, 1, 1]):
        counts2 = lead + counts
        qkv2 = make_qkv(counts2, n, heads, 1.0, 22)
        skip = sum(lead)
        qkv2[skip:skip + sum(counts)] = qkv[:sum(counts)]
        a = run(TC, counts, n, heads, qkv)
        b = run(TC, counts2, n, heads, qkv2)[skip:]
        assert torch.equal(a, b), f"lead {lead}: {(a != b).sum().item()} values differ"


def test_repeatable():
    counts = rng_counts(512, 16, 64, 3)
    qkv = make_qkv(counts, 64, 8, 1.0, 3)
    a = run(TC, counts, 64, 8, qkv)
    b = run(TC, counts, 64, 8, qkv)
    assert torch.equal(a, b)
