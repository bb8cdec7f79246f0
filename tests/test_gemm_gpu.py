"""The tcgen05 GEMM (every epilogue, bf16 and e4m3 operands) against a plain PyTorch fp32
reference of the same op, at the encoder's shapes (`nano` 192/576/768, `small`
512/1536/2048) with ragged row counts (B·65 rows is never a multiple of the 128-row tile)."""

import ctypes

import pytest

torch = pytest.importorskip("torch")

from marina_b200 import _lib

pytestmark = pytest.mark.gpu

EPI_BIAS, EPI_GELU_BF16, EPI_GELU_E4M3, EPI_RESIDUAL = 0, 1, 2, 3
EPI_GELU_TANH_BF16, EPI_GELU_TANH_E4M3 = 5, 6
EPI_GELU_E4M3X2, EPI_GELU_TANH_E4M3X2 = 7, 8

# (M, N, K): QKV, out-proj, FFN1, FFN2 of both nets; M = positions x 65. Shapes with N % 256 == 0
# run on single CTAs and on CTA pairs (`pair` 0 and 1), whatever the planning rule would pick.
SHAPES = [
    (65 * 3, 576, 192), (65 * 3, 192, 192), (65 * 3, 768, 192), (65 * 3, 192, 768),
    (65 * 7, 1536, 512), (65 * 7, 512, 512), (65 * 7, 2048, 512), (65 * 7, 512, 2048),
    (1, 256, 64), (128, 128, 128), (65 * 64, 1536, 512),
    # CTA-pair tiles (N % 256 == 0, K >= 1024): one, two and ragged 256-row blocks
    (65 * 3, 512, 1024), (130, 256, 1024), (65 * 9, 512, 2048), (1, 256, 1024),
]


def _run(fp8, epi, a, b, bias, out, ldo, m, n, k, scale=1.0, inv_q=1.0, pair=-1):
    """One GEMM through the test library; `pair` -1 the planning rule, 0 single CTAs, 1 CTA pairs."""
    lib = _lib.load_test()
    status = torch.zeros(1, dtype=torch.int32, device=a.device)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.mrn_test_gemm(int(fp8), epi, pair, a.data_ptr(), b.data_ptr(), bias.data_ptr(), out.data_ptr(), ldo, m,
                           n, k, scale, inv_q, ctypes.c_void_p(status.data_ptr()), ctypes.c_void_p(stream))
    assert rc == 0, lib.mrn_test_last_error().decode()
    torch.cuda.synchronize()
    assert int(status.item()) == 0, f"device status {int(status.item())}"


def _pairs(shapes):
    """(m, n, k, pair) for each shape: single CTAs, and CTA pairs where N % 256 == 0."""
    return [(m, n, k, p) for m, n, k in shapes for p in ((0, 1) if n % 256 == 0 else (0,))]


def _within(got, ref, tol, what=""):
    """Elementwise |got - ref| <= tol; on failure report the worst elements."""
    err = (got - ref).abs()
    bad = err > tol
    if bool(bad.any()):
        idx = bad.nonzero()[:8].tolist()
        worst = int((err - tol).argmax())
        r, c = divmod(worst, got.shape[1])
        raise AssertionError(f"{what}: {int(bad.sum())} elements out of tolerance; worst at ({r}, {c}): got "
                             f"{float(got[r, c])}, ref {float(ref[r, c])}, tol {float(tol[r, c])}; first {idx}")


def _operands(m, n, k, fp8, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(m, k, device="cuda", generator=g)
    b = torch.randn(n, k, device="cuda", generator=g) * 0.05
    bias = torch.randn(n, device="cuda", generator=g) * 0.1
    if fp8:
        a8 = a.to(torch.float8_e4m3fn)
        b8 = (b * 8).to(torch.float8_e4m3fn)
        return a8.view(torch.uint8), b8.view(torch.uint8), a8.float(), b8.float(), bias
    ab, bb = a.to(torch.bfloat16), b.to(torch.bfloat16)
    return ab, bb, ab.float(), bb.float(), bias


def _x2_split(v):
    """Two-term e4m3 of `v` (already in code units): hi = e4m3(v), lo = e4m3(v - hi)."""
    hi = v.clamp(-448, 448).to(torch.float8_e4m3fn)
    lo = (v - hi.float()).to(torch.float8_e4m3fn)
    return hi, lo


def _x2_operands(m, n, k, seed):
    """A as two-term e4m3 [m, 2k] (each row's hi codes, then its lo codes), B as e4m3; the float
    values are hi + lo and the B codes."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(m, k, device="cuda", generator=g) * (448.0 / 6.0)
    b = torch.randn(n, k, device="cuda", generator=g) * 0.05
    bias = torch.randn(n, device="cuda", generator=g) * 0.1
    hi, lo = _x2_split(a)
    a2 = torch.cat([hi.view(torch.uint8), lo.view(torch.uint8)], 1).contiguous()
    b8 = (b * 8).to(torch.float8_e4m3fn)
    return a2, b8.view(torch.uint8), hi.float() + lo.float(), b8.float(), hi.float(), bias


@pytest.mark.parametrize("m,n,k,pair", _pairs(SHAPES))
def test_two_term_operands(cuda, m, n, k, pair):
    """Two-term e4m3 A: the product is (hi + lo) . b, held to the bf16 output's rounding, which is
    far below what dropping the lo term would cost (about 2^-5 of each product)."""
    a2, b, af, bf, hif, bias = _x2_operands(m, n, k, seed=m + 2 * n + k)
    scale = 2.0 ** -12
    out = torch.full((m, n), float("nan"), device=cuda, dtype=torch.bfloat16)
    _run(2, EPI_BIAS, a2, b, bias, out, n, m, n, k, scale=scale, pair=pair)
    ref = (af @ bf.T) * scale + bias
    tol = ref.abs() * 2 ** -8 + 1e-4 * float(ref.abs().max())
    _within(out.float(), ref, tol, "two-term bias")
    # the tolerance has the power to see a dropped lo term
    hi_only = (hif @ bf.T) * scale + bias
    assert not bool(((hi_only - ref).abs() <= tol).all())
    x0 = torch.randn(m, n, device=cuda).half()
    x = x0.clone()
    _run(2, EPI_RESIDUAL, a2, b, bias, x, n, m, n, k, scale=scale, pair=pair)
    delta = (af @ bf.T) * scale + bias
    ref = x0.float() + delta
    _within(x.float(), ref, (ref.abs() + delta.abs()) * 2 ** -10 + 2 ** -14, "two-term residual")


@pytest.mark.parametrize("m,n,k,pair", _pairs([s for s in SHAPES if s[1] in (768, 2048, 256)]))
@pytest.mark.parametrize("epi", [EPI_GELU_E4M3X2, EPI_GELU_TANH_E4M3X2], ids=["erf", "tanh"])
def test_gelu_two_term_epilogue(cuda, m, n, k, pair, epi):
    """GELU into two-term e4m3 [m, 2n] (hi codes in columns [0, n), lo codes in [n, 2n)), from
    two-term operands, as FFN1 of the fp8x2 precision writes FFN2's input."""
    a2, b, af, bf, _, bias = _x2_operands(m, n, k, seed=19 + epi)
    scale, q = 2.0 ** -12, 0.01  # output value = (hi + lo) * q
    out = torch.full((m, 2 * n + 32), 0x55, device=cuda, dtype=torch.uint8)
    _run(2, epi, a2, b, bias, out, 2 * n + 32, m, n, k, scale=scale, inv_q=1.0 / q, pair=pair)
    approx = "tanh" if epi == EPI_GELU_TANH_E4M3X2 else "none"
    ref = torch.nn.functional.gelu((af @ bf.T) * scale + bias, approximate=approx)
    assert float(ref.abs().max()) < 448 * q
    codes = out[:, :2 * n].view(torch.float8_e4m3fn).float()
    got = (codes[:, :n] + codes[:, n:]) * q
    # the residual after one e4m3 step rounded to e4m3 (or to the subnormal step 2^-9)
    _within(got, ref, ref.abs() * 2 ** -8 + q * 2 ** -10 + 1e-5, "two-term GELU")
    assert bool((out[:, 2 * n:] == 0x55).all())


@pytest.mark.parametrize("fp8", [False, True], ids=["bf16", "e4m3"])
@pytest.mark.parametrize("m,n,k,pair", _pairs(SHAPES))
def test_bias_epilogue(cuda, fp8, m, n, k, pair):
    a, b, af, bf, bias = _operands(m, n, k, fp8, seed=m + n + k)
    scale = 0.125 if fp8 else 1.0
    out = torch.full((m, n), float("nan"), device=cuda, dtype=torch.bfloat16)
    _run(fp8, EPI_BIAS, a, b, bias, out, n, m, n, k, scale=scale, pair=pair)
    ref = (af @ bf.T) * scale + bias
    err = (out.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item() + 1e-3, err


@pytest.mark.parametrize("m,n,k,pair", _pairs([s for s in SHAPES if s[1] in (768, 2048, 256)]))
def test_gelu_bf16_epilogue(cuda, m, n, k, pair):
    a, b, af, bf, bias = _operands(m, n, k, False, seed=7)
    out = torch.zeros((m, n), device=cuda, dtype=torch.bfloat16)
    _run(False, EPI_GELU_BF16, a, b, bias, out, n, m, n, k, pair=pair)
    ref = torch.nn.functional.gelu(af @ bf.T + bias)
    err = (out.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item() + 1e-3, err


@pytest.mark.parametrize("m,n,k,pair", _pairs([s for s in SHAPES if s[1] in (768, 2048, 256)]))
def test_gelu_e4m3_epilogue(cuda, m, n, k, pair):
    a, b, af, bf, bias = _operands(m, n, k, True, seed=11)
    scale, q = 0.125, 0.05  # output value = code * q
    out = torch.zeros((m, n), device=cuda, dtype=torch.uint8)
    _run(True, EPI_GELU_E4M3, a, b, bias, out, n, m, n, k, scale=scale, inv_q=1.0 / q, pair=pair)
    ref = torch.nn.functional.gelu((af @ bf.T) * scale + bias)
    got = out.view(torch.float8_e4m3fn).float() * q
    # one e4m3 rounding step (3 mantissa bits) plus saturation at 448 * q
    tol = ref.abs() * 0.0625 + q * 2 ** -6
    ref_sat = ref.clamp(-448 * q, 448 * q)
    assert bool(((got - ref_sat).abs() <= tol + 1e-6).all())


@pytest.mark.parametrize("m,n,k", [s for s in SHAPES if s[1] in (768, 2048, 256)])
def test_gelu_tanh_epilogues(cuda, m, n, k):
    """The tanh-form GELU (cards trained with it) against torch's approximate="tanh" GELU."""
    a, b, af, bf, bias = _operands(m, n, k, False, seed=13)
    out = torch.zeros((m, n), device=cuda, dtype=torch.bfloat16)
    _run(False, EPI_GELU_TANH_BF16, a, b, bias, out, n, m, n, k)
    ref = torch.nn.functional.gelu(af @ bf.T + bias, approximate="tanh")
    assert bool(((out.float() - ref).abs() <= ref.abs() * 2 ** -8 + 1e-5).all())
    a, b, af, bf, bias = _operands(m, n, k, True, seed=17)
    scale, q = 0.125, 0.05
    out8 = torch.zeros((m, n), device=cuda, dtype=torch.uint8)
    _run(True, EPI_GELU_TANH_E4M3, a, b, bias, out8, n, m, n, k, scale=scale, inv_q=1.0 / q)
    ref = torch.nn.functional.gelu((af @ bf.T) * scale + bias, approximate="tanh")
    got = out8.view(torch.float8_e4m3fn).float() * q
    ref_sat = ref.clamp(-448 * q, 448 * q)
    assert bool(((got - ref_sat).abs() <= ref.abs() * 0.0625 + q * 2 ** -6 + 1e-6).all())


@pytest.mark.parametrize("fp8", [False, True], ids=["bf16", "e4m3"])
@pytest.mark.parametrize("m,n,k,pair", _pairs([s for s in SHAPES if s[1] in (192, 512, 128)]))
def test_residual_epilogue(cuda, fp8, m, n, k, pair):
    a, b, af, bf, bias = _operands(m, n, k, fp8, seed=3)
    scale = 0.125 if fp8 else 1.0
    x0 = torch.randn(m, n, device=cuda).half()  # the residual stream is f16
    x = x0.clone()
    _run(fp8, EPI_RESIDUAL, a, b, bias, x, n, m, n, k, scale=scale, pair=pair)
    delta = (af @ bf.T) * scale + bias
    ref = x0.float() + delta
    # the f16 sum of x and the f16-rounded update: at most an f16 half-ulp of each, plus the
    # GEMM's own accumulation order where x and the update cancel; a sum below f16's smallest
    # normal (2^-14) may come back flushed to zero from the L2's f16 reduce-add
    _within(x.float(), ref, (ref.abs() + delta.abs()) * 2 ** -10 + 2 ** -14, "residual")


def test_rows_beyond_m_untouched(cuda):
    m, n, k = 65 * 3, 576, 192
    a, b, af, bf, bias = _operands(m, n, k, False, seed=5)
    out = torch.full((m + 128, n), 7.0, device=cuda, dtype=torch.bfloat16)
    _run(False, EPI_BIAS, a, b, bias, out, n, m, n, k)
    assert bool((out[m:] == 7.0).all())


def _layernorm(x, gamma, beta, eps, e4m3, inv_q, out):
    lib = _lib.load_test()
    rows, d = x.shape
    rc = lib.mrn_test_layernorm(x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), eps, int(e4m3), inv_q,
                                out.data_ptr(), rows, d, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.mrn_test_last_error().decode()
    torch.cuda.synchronize()


def _norm_inputs(m, d, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (torch.randn(m, d, device="cuda", generator=g) * 2.0 + 0.3).half()  # the f16 residual stream
    gamma = 1.0 + 0.2 * torch.randn(d, device="cuda", generator=g)
    beta = 0.1 * torch.randn(d, device="cuda", generator=g)
    return x, gamma, beta


@pytest.mark.parametrize("e4m3", [0, 1, 2], ids=["bf16", "e4m3", "e4m3x2"])
@pytest.mark.parametrize("m,d", [(65 * 7, 512), (65 * 3, 192), (1, 512), (65 * 64, 512), (130, 1024)])
def test_layernorm_kernel(cuda, e4m3, m, d):
    """The LayerNorm kernel against torch fp32 LayerNorm of the same f16 rows."""
    x, gamma, beta = _norm_inputs(m, d, seed=m + d)
    q, eps = 0.02, 1e-5
    out = torch.zeros((m, 2 * d if e4m3 == 2 else d), device=cuda, dtype=torch.uint8 if e4m3 else torch.bfloat16)
    _layernorm(x, gamma, beta, eps, e4m3, 1.0 / q, out)
    ref = torch.nn.functional.layer_norm(x.float(), (d,), gamma, beta, eps)
    if e4m3 == 2:
        codes = out.view(torch.float8_e4m3fn).float()
        got = (codes[:, :d] + codes[:, d:]) * q
        _within(got, ref, ref.abs() * 2 ** -8 + q * 2 ** -10 + 1e-5, "layernorm two-term e4m3")
    elif e4m3:
        got = out.view(torch.float8_e4m3fn).float() * q
        _within(got, ref, ref.abs() * 0.0625 + q * 2 ** -6 + 1e-5, "layernorm e4m3")
    else:
        _within(out.float(), ref, ref.abs() * 2 ** -8 + 1e-4, "layernorm bf16")
