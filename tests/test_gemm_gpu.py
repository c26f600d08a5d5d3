"""Single tcgen05 GEMM launches (ow_selftest_gemm) against a plain PyTorch fp32
reference of the same op, for every epilogue the forward uses."""
import numpy as np
import pytest

from orbit_wars_b200 import _lib

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

BF16, FP8 = 1, 2
EPI_BIAS, EPI_GELU, EPI_LN, EPI_LN16 = 0, 1, 2, 3
PAIR = 16  # epilogue flag: the CTA-pair (cta_group::2) kernel
LN_BF16, LN_E4M3, LN_F32 = 0, 1, 2


def call(precision, epi, m, n, k, a, w, bias, out=None, resid=None, g=None, b=None, ln_out=None, ln_mode=0,
         ln_scale=None, a_scale=None, b_scale=None):
    lib = _lib.load_library()
    p = _lib.ptr
    st = lib.ow_selftest_gemm(precision, epi, m, n, k, p(a), p(w), p(bias), p(out), p(resid), p(g), p(b), p(ln_out),
                              ln_mode, p(ln_scale), p(a_scale), p(b_scale), torch.cuda.current_stream().cuda_stream)
    _lib.check("ow_selftest_gemm", st)


def close(x, ref, rel, what=""):
    diff = (x.float() - ref).abs()
    err = diff.max().item() / max(ref.abs().max().item(), 1e-6)
    if not err <= rel:
        bad = torch.nonzero(~(diff <= rel * max(ref.abs().max().item(), 1e-6)))
        rows = torch.unique(bad[:, 0]).tolist() if bad.ndim == 2 else []
        cols = torch.unique(bad[:, 1]).tolist() if bad.ndim == 2 else []
        raise AssertionError(f"{what}: rel err {err:.3e} > {rel}; {bad.shape[0]} bad, rows {rows[:8]}.. ({len(rows)}), "
                             f"cols {cols[:8]}.. ({len(cols)})")
    return err


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (300, 768, 256), (1000, 384, 256), (77, 256, 1024)])
def test_bf16_bias(m, n, k):
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).bfloat16()
    bias = torch.randn(n, device="cuda", generator=g)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    call(BF16, EPI_BIAS, m, n, k, a, w, bias, out=out)
    ref = a.float() @ w.float().T + bias
    close(out, ref, 8e-3)


@pytest.mark.parametrize("epi,n,m", [(EPI_BIAS, 768, 5000), (EPI_GELU, 1024, 4111), (EPI_BIAS, 256, 129)])
def test_weight_stationary_matches_streaming(monkeypatch, epi, n, m):
    """K = 256 bias / GELU GEMMs keep each CTA's slice of W in shared memory;
    the same MMAs in the same order as the streaming kernel, so the same bits."""
    k = 256
    g = torch.Generator(device="cuda").manual_seed(n + m)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) / 16).bfloat16()
    bias = torch.randn(n, device="cuda", generator=g)
    outs = []
    for ws in ("1", "0"):
        monkeypatch.setenv("ORBIT_WARS_GEMM_WS", ws)
        out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        call(BF16, epi, m, n, k, a, w, bias, out=out)
        outs.append(out)
    assert torch.equal(outs[0], outs[1])
    ref = a.float() @ w.float().T + bias
    if epi == EPI_GELU:
        ref = torch.nn.functional.gelu(ref)
    close(outs[0], ref, 8e-3)


def test_bf16_gelu():
    m, n, k = 513, 1024, 256
    a = torch.randn(m, k, device="cuda").bfloat16()
    w = (torch.randn(n, k, device="cuda") / 16).bfloat16()
    bias = torch.randn(n, device="cuda")
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    call(BF16, EPI_GELU, m, n, k, a, w, bias, out=out)
    ref = torch.nn.functional.gelu(a.float() @ w.float().T + bias)
    close(out, ref, 8e-3)


@pytest.mark.parametrize("n", [128, 256, 384, 512])
@pytest.mark.parametrize("ln_mode", [LN_BF16, LN_F32])
def test_bf16_resid_ln(n, ln_mode):
    m, k = 333, 1024 if n != 384 else 256
    a = torch.randn(m, k, device="cuda").bfloat16()
    w = (torch.randn(n, k, device="cuda") / k ** 0.5).bfloat16()
    bias = torch.randn(n, device="cuda") * 0.1
    resid = torch.randn(m, n, device="cuda")
    resid0 = resid.clone()
    gam = 1 + 0.1 * torch.randn(n, device="cuda")
    bet = 0.1 * torch.randn(n, device="cuda")
    ln_out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16 if ln_mode == LN_BF16 else torch.float32)
    call(BF16, EPI_LN, m, n, k, a, w, bias, resid=resid, g=gam, b=bet, ln_out=ln_out, ln_mode=ln_mode)
    x_ref = resid0 + a.float() @ w.float().T + bias
    close(resid, x_ref, 1e-4, "x")
    y_ref = torch.nn.functional.layer_norm(x_ref, (n,), gam, bet, eps=1e-5)
    close(ln_out, y_ref, 8e-3 if ln_mode == LN_BF16 else 1e-4, "ln")


def quant_rows(x):
    s = (x.abs().amax(dim=1).clamp_min(1e-30) / 448.0)
    q = (x / s[:, None]).to(torch.float8_e4m3fn)
    return q, s


@pytest.mark.parametrize("epi,n", [(EPI_BIAS, 768), (EPI_GELU, 1024)])
def test_fp8_bias_gelu(epi, n):
    m, k = 260, 256
    a, sa = quant_rows(torch.randn(m, k, device="cuda"))
    w, sw = quant_rows(torch.randn(n, k, device="cuda") / 16)
    bias = torch.randn(n, device="cuda")
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    call(FP8, epi, m, n, k, a, w, bias, out=out, a_scale=sa, b_scale=sw)
    ref = (a.float() * sa[:, None]) @ (w.float() * sw[:, None]).T + bias
    if epi == EPI_GELU:
        ref = torch.nn.functional.gelu(ref)
    close(out, ref, 8e-3)


def test_fp8_resid_ln():
    m, n, k = 200, 256, 1024
    a, sa = quant_rows(torch.randn(m, k, device="cuda"))
    w, sw = quant_rows(torch.randn(n, k, device="cuda") / 32)
    bias = torch.randn(n, device="cuda") * 0.1
    resid = torch.randn(m, n, device="cuda")
    resid0 = resid.clone()
    gam = torch.ones(n, device="cuda")
    bet = torch.zeros(n, device="cuda")
    ln_out = torch.empty(m, n, device="cuda", dtype=torch.uint8)
    ln_scale = torch.empty(m, device="cuda")
    call(FP8, EPI_LN, m, n, k, a, w, bias, resid=resid, g=gam, b=bet, ln_out=ln_out, ln_mode=LN_E4M3,
         ln_scale=ln_scale, a_scale=sa, b_scale=sw)
    x_ref = resid0 + (a.float() * sa[:, None]) @ (w.float() * sw[:, None]).T + bias
    close(resid, x_ref, 1e-4)
    y_ref = torch.nn.functional.layer_norm(x_ref, (n,), gam, bet, eps=1e-5)
    y = ln_out.view(torch.float8_e4m3fn).float() * ln_scale[:, None]
    close(y, y_ref, 7e-2)
    # the quantisation point itself follows the recipe: scale absmax/448 per row, and e4m3 codes that equal
    # RNE(y / scale) except where y sits within f32 rounding of a rounding boundary (then one step away)
    close(ln_scale, y_ref.abs().amax(dim=1) / 448.0, 1e-5, "scale")
    q = ln_out.view(torch.float8_e4m3fn).float()
    q_ref = (y_ref / ln_scale[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn).float()
    off = q != q_ref
    assert off.float().mean().item() <= 1e-2
    step = torch.clamp(q_ref.abs(), min=2.0 ** -6) * 2.0 ** -3
    assert torch.all((q - q_ref).abs()[off] <= step[off] * 1.0001)


@pytest.mark.parametrize("epi,n", [(EPI_BIAS, 768), (EPI_GELU, 1024)])
def test_bf16_repeatable(epi, n):
    """Two launches on the same inputs give bit-identical outputs."""
    m, k = 40000, 256
    a = torch.randn(m, k, device="cuda").bfloat16()
    w = (torch.randn(n, k, device="cuda") / 16).bfloat16()
    bias = torch.randn(n, device="cuda")
    o1 = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    o2 = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    call(BF16, epi, m, n, k, a, w, bias, out=o1)
    call(BF16, epi, m, n, k, a, w, bias, out=o2)
    bad = torch.nonzero(o1.view(torch.int16) != o2.view(torch.int16))
    assert bad.shape[0] == 0, f"{bad.shape[0]} differing elements, first {bad[:4].tolist()}"


def test_bf16_resid_ln_repeatable_many_tiles():
    """The LayerNorm epilogue at 315 row tiles (several per CTA) repeats bit for bit:
    its staging tiles are refilled only after every value read from them is consumed."""
    m, n, k = 40271, 256, 1024
    a = torch.randn(m, k, device="cuda").bfloat16()
    w = (torch.randn(n, k, device="cuda") / 32).bfloat16()
    bias = torch.randn(n, device="cuda") * 0.1
    resid0 = torch.randn(m, n, device="cuda")
    gam = 1 + 0.1 * torch.randn(n, device="cuda")
    bet = 0.1 * torch.randn(n, device="cuda")
    outs = []
    for _ in range(2):
        resid = resid0.clone()
        ln_out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        call(BF16, EPI_LN, m, n, k, a, w, bias, resid=resid, g=gam, b=bet, ln_out=ln_out, ln_mode=LN_BF16)
        outs.append((resid, ln_out))
    x_ref = resid0 + a.float() @ w.float().T + bias
    close(outs[0][0], x_ref, 1e-4, "x")
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


@pytest.mark.parametrize("m,k", [(333, 1024), (1000, 256), (40271, 1024)])
@pytest.mark.parametrize("ln_mode", [LN_BF16, LN_F32])
def test_bf16_resid16_ln(m, k, ln_mode):
    """bf16 residual stream, 16-warp LayerNorm epilogue (d = 256): x += a.w^T + bias in place (bf16), the
    LayerNorm of the f32 sum -> ln_out; repeated launches are bit-identical."""
    n = 256
    g = torch.Generator(device="cuda").manual_seed(m + k + ln_mode)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).bfloat16()
    bias = torch.randn(n, device="cuda", generator=g) * 0.1
    resid0 = torch.randn(m, n, device="cuda", generator=g).bfloat16()
    gam = 1 + 0.1 * torch.randn(n, device="cuda", generator=g)
    bet = 0.1 * torch.randn(n, device="cuda", generator=g)
    outs = []
    for _ in range(2):
        resid = resid0.clone()
        ln_out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16 if ln_mode == LN_BF16 else torch.float32)
        call(BF16, EPI_LN16, m, n, k, a, w, bias, resid=resid, g=gam, b=bet, ln_out=ln_out, ln_mode=ln_mode)
        outs.append((resid, ln_out))
    x_ref = resid0.float() + a.float() @ w.float().T + bias
    close(outs[0][0], x_ref, 8e-3, "x")
    y_ref = torch.nn.functional.layer_norm(x_ref, (n,), gam, bet, eps=1e-5)
    close(outs[0][1], y_ref, 8e-3 if ln_mode == LN_BF16 else 1e-4, "ln")
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


def test_fp8_resid16_ln():
    m, n, k = 700, 256, 1024
    a, sa = quant_rows(torch.randn(m, k, device="cuda"))
    w, sw = quant_rows(torch.randn(n, k, device="cuda") / 32)
    bias = torch.randn(n, device="cuda") * 0.1
    resid0 = torch.randn(m, n, device="cuda").bfloat16()
    resid = resid0.clone()
    gam = torch.ones(n, device="cuda")
    bet = torch.zeros(n, device="cuda")
    ln_out = torch.empty(m, n, device="cuda", dtype=torch.uint8)
    ln_scale = torch.empty(m, device="cuda")
    call(FP8, EPI_LN16, m, n, k, a, w, bias, resid=resid, g=gam, b=bet, ln_out=ln_out, ln_mode=LN_E4M3,
         ln_scale=ln_scale, a_scale=sa, b_scale=sw)
    x_ref = resid0.float() + (a.float() * sa[:, None]) @ (w.float() * sw[:, None]).T + bias
    close(resid, x_ref, 8e-3, "x")
    y_ref = torch.nn.functional.layer_norm(x_ref, (n,), gam, bet, eps=1e-5)
    close(ln_scale, y_ref.abs().amax(dim=1) / 448.0, 1e-5, "scale")
    q = ln_out.view(torch.float8_e4m3fn).float()
    q_ref = (y_ref / ln_scale[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn).float()
    off = q != q_ref
    assert off.float().mean().item() <= 1e-2
    step = torch.clamp(q_ref.abs(), min=2.0 ** -6) * 2.0 ** -3
    assert torch.all((q - q_ref).abs()[off] <= step[off] * 1.0001)


@pytest.mark.parametrize("m", [77, 333, 40271])
@pytest.mark.parametrize("epi,n,k", [(EPI_BIAS, 768, 256), (EPI_GELU, 1024, 256), (EPI_BIAS, 256, 1024)])
def test_pair_bias_gelu(m, epi, n, k):
    """CTA-pair kernel (256-row tiles over two SMs) against torch fp32 and the single-CTA kernel."""
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n + k)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).bfloat16()
    bias = torch.randn(n, device="cuda", generator=g)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    one = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    call(BF16, epi | PAIR, m, n, k, a, w, bias, out=out)
    call(BF16, epi, m, n, k, a, w, bias, out=one)
    ref = a.float() @ w.float().T + bias
    if epi == EPI_GELU:
        ref = torch.nn.functional.gelu(ref)
    close(out, ref, 8e-3)
    close(out, one.float(), 8e-3, "vs single-CTA")


@pytest.mark.parametrize("m,k", [(200, 256), (40271, 1024)])
@pytest.mark.parametrize("ln_mode", [LN_BF16, LN_F32])
def test_pair_resid16_ln(m, k, ln_mode):
    n = 256
    g = torch.Generator(device="cuda").manual_seed(m + k + 11 * ln_mode)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).bfloat16()
    bias = torch.randn(n, device="cuda", generator=g) * 0.1
    resid0 = torch.randn(m, n, device="cuda", generator=g).bfloat16()
    gam = 1 + 0.1 * torch.randn(n, device="cuda", generator=g)
    bet = 0.1 * torch.randn(n, device="cuda", generator=g)
    outs = []
    for _ in range(2):
        resid = resid0.clone()
        ln_out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16 if ln_mode == LN_BF16 else torch.float32)
        call(BF16, EPI_LN16 | PAIR, m, n, k, a, w, bias, resid=resid, g=gam, b=bet, ln_out=ln_out, ln_mode=ln_mode)
        outs.append((resid, ln_out))
    x_ref = resid0.float() + a.float() @ w.float().T + bias
    close(outs[0][0], x_ref, 8e-3, "x")
    y_ref = torch.nn.functional.layer_norm(x_ref, (n,), gam, bet, eps=1e-5)
    close(outs[0][1], y_ref, 8e-3 if ln_mode == LN_BF16 else 1e-4, "ln")
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


def test_pair_fp8():
    m, n, k = 700, 256, 1024
    a, sa = quant_rows(torch.randn(m, k, device="cuda"))
    w, sw = quant_rows(torch.randn(n, k, device="cuda") / 32)
    bias = torch.randn(n, device="cuda") * 0.1
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    call(FP8, EPI_BIAS | PAIR, m, n, k, a, w, bias, out=out, a_scale=sa, b_scale=sw)
    ref = (a.float() * sa[:, None]) @ (w.float() * sw[:, None]).T + bias
    close(out, ref, 8e-3)
    resid0 = torch.randn(m, n, device="cuda").bfloat16()
    resid = resid0.clone()
    ln_out = torch.empty(m, n, device="cuda", dtype=torch.uint8)
    ln_scale = torch.empty(m, device="cuda")
    call(FP8, EPI_LN16 | PAIR, m, n, k, a, w, bias, resid=resid, g=torch.ones(n, device="cuda"),
         b=torch.zeros(n, device="cuda"), ln_out=ln_out, ln_mode=LN_E4M3, ln_scale=ln_scale, a_scale=sa, b_scale=sw)
    x_ref = resid0.float() + ref
    close(resid, x_ref, 8e-3, "x")
    y_ref = torch.nn.functional.layer_norm(x_ref, (n,), eps=1e-5)
    close(ln_scale, y_ref.abs().amax(dim=1) / 448.0, 1e-5, "scale")


def ffn_call(m, f, ln, w1, b1, w2, b2, x, g, b, ln_out, ln_mode):
    lib = _lib.load_library()
    p = _lib.ptr
    st = lib.ow_selftest_ffn(m, 256, f, p(ln), p(w1), p(b1), p(w2), p(b2), p(x), p(g), p(b), p(ln_out), ln_mode,
                             torch.cuda.current_stream().cuda_stream)
    _lib.check("ow_selftest_ffn", st)


@pytest.mark.parametrize("m,f,ln_mode", [(77, 1024, LN_BF16), (5000, 512, LN_F32), (40271, 1024, LN_BF16)])
def test_fused_ffn(m, f, ln_mode):
    """Fused up-projection + GELU + down-projection + residual + LayerNorm (d = 256)
    against the same op in PyTorch fp32 with the hidden layer rounded to bf16 as
    the kernel keeps it; 40,271 rows = 315 tiles, several per CTA; repeats bit for bit."""
    d = 256
    g = torch.Generator(device="cuda").manual_seed(m + f)
    ln = torch.randn(m, d, device="cuda", generator=g).bfloat16()
    w1 = (torch.randn(f, d, device="cuda", generator=g) * 0.06).bfloat16()
    w2 = (torch.randn(d, f, device="cuda", generator=g) * 0.03).bfloat16()
    b1 = torch.randn(f, device="cuda", generator=g) * 0.1
    b2 = torch.randn(d, device="cuda", generator=g) * 0.1
    x0 = torch.randn(m, d, device="cuda", generator=g)
    gam = 1 + 0.1 * torch.randn(d, device="cuda", generator=g)
    bet = 0.1 * torch.randn(d, device="cuda", generator=g)
    outs = []
    for _ in range(2):
        x = x0.clone()
        lo = torch.empty(m, d, device="cuda", dtype=torch.bfloat16 if ln_mode == LN_BF16 else torch.float32)
        ffn_call(m, f, ln, w1, b1, w2, b2, x, gam, bet, lo, ln_mode)
        outs.append((x, lo))
    h = torch.nn.functional.gelu(ln.float() @ w1.float().T + b1).bfloat16().float()
    x_ref = x0 + h @ w2.float().T + b2
    close(outs[0][0], x_ref, 2e-3, "x")
    y_ref = torch.nn.functional.layer_norm(x_ref, (d,), gam, bet, eps=1e-5)
    close(outs[0][1], y_ref, 8e-3 if ln_mode == LN_BF16 else 2e-3, "ln")
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
