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

# (M, N, K): QKV, out-proj, FFN1, FFN2 of both nets; M = positions x 65.
SHAPES = [
    (65 * 3, 576, 192), (65 * 3, 192, 192), (65 * 3, 768, 192), (65 * 3, 192, 768),
    (65 * 7, 1536, 512), (65 * 7, 512, 512), (65 * 7, 2048, 512), (65 * 7, 512, 2048),
    (1, 256, 64), (128, 128, 128), (65 * 64, 1536, 512),
    # CTA-pair tiles (N % 256 == 0, K >= 1024): one, two and ragged 256-row blocks
    (65 * 3, 512, 1024), (130, 256, 1024), (65 * 9, 512, 2048), (1, 256, 1024),
]


def _run(fp8, epi, a, b, bias, out, ldo, m, n, k, scale=1.0, inv_q=1.0):
    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device=a.device)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.mrn_test_gemm(int(fp8), epi, a.data_ptr(), b.data_ptr(), bias.data_ptr(), out.data_ptr(), ldo, m, n, k,
                           scale, inv_q, ctypes.c_void_p(status.data_ptr()), ctypes.c_void_p(stream))
    assert rc == 0, lib.mrn_test_last_error().decode()
    torch.cuda.synchronize()
    assert int(status.item()) == 0, f"device status {int(status.item())}"


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


@pytest.mark.parametrize("fp8", [False, True], ids=["bf16", "e4m3"])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_bias_epilogue(cuda, fp8, m, n, k):
    a, b, af, bf, bias = _operands(m, n, k, fp8, seed=m + n + k)
    scale = 0.125 if fp8 else 1.0
    out = torch.full((m, n), float("nan"), device=cuda, dtype=torch.bfloat16)
    _run(fp8, EPI_BIAS, a, b, bias, out, n, m, n, k, scale=scale)
    ref = (af @ bf.T) * scale + bias
    err = (out.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item() + 1e-3, err


@pytest.mark.parametrize("m,n,k", [s for s in SHAPES if s[1] in (768, 2048, 256)])
def test_gelu_bf16_epilogue(cuda, m, n, k):
    a, b, af, bf, bias = _operands(m, n, k, False, seed=7)
    out = torch.zeros((m, n), device=cuda, dtype=torch.bfloat16)
    _run(False, EPI_GELU_BF16, a, b, bias, out, n, m, n, k)
    ref = torch.nn.functional.gelu(af @ bf.T + bias)
    err = (out.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item() + 1e-3, err


@pytest.mark.parametrize("m,n,k", [s for s in SHAPES if s[1] in (768, 2048, 256)])
def test_gelu_e4m3_epilogue(cuda, m, n, k):
    a, b, af, bf, bias = _operands(m, n, k, True, seed=11)
    scale, q = 0.125, 0.05  # output value = code * q
    out = torch.zeros((m, n), device=cuda, dtype=torch.uint8)
    _run(True, EPI_GELU_E4M3, a, b, bias, out, n, m, n, k, scale=scale, inv_q=1.0 / q)
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
@pytest.mark.parametrize("m,n,k", [s for s in SHAPES if s[1] in (192, 512, 128)])
def test_residual_epilogue(cuda, fp8, m, n, k):
    a, b, af, bf, bias = _operands(m, n, k, fp8, seed=3)
    scale = 0.125 if fp8 else 1.0
    x0 = torch.randn(m, n, device=cuda).half()  # the residual stream is f16
    x = x0.clone()
    _run(fp8, EPI_RESIDUAL, a, b, bias, x, n, m, n, k, scale=scale)
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


def _run_ln(fp8, a, b, bias, gamma, beta, x, h, m, d, k, scale, eps, inv_q):
    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device=a.device)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.mrn_test_gemm_ln(int(fp8), a.data_ptr(), b.data_ptr(), bias.data_ptr(), gamma.data_ptr(),
                              beta.data_ptr(), x.data_ptr(), h.data_ptr(), m, d, k, scale, eps, inv_q,
                              ctypes.c_void_p(status.data_ptr()), ctypes.c_void_p(stream))
    assert rc == 0, lib.mrn_test_last_error().decode()
    torch.cuda.synchronize()
    assert int(status.item()) == 0, f"device status {int(status.item())}"


# (M, d, K): out-proj and FFN2 of both nets (clusters of 4 x 128 and 2 x 96 columns), ragged and
# single-row blocks, several row blocks per cluster, and the other CTA slicings (d = 64, 256,
# 384, 1024: clusters of 1, 2, 3, 8).
LN_SHAPES = [
    (65 * 7, 512, 512), (65 * 7, 512, 2048), (65 * 3, 192, 192), (65 * 3, 192, 768),
    (1, 512, 512), (128, 512, 512), (65 * 64, 512, 2048), (65 * 256, 192, 768),
    (65 * 5, 64, 128), (65 * 5, 256, 512), (65 * 5, 384, 384), (65 * 2, 1024, 1024),
]


@pytest.mark.parametrize("fp8", [False, True], ids=["bf16", "e4m3"])
@pytest.mark.parametrize("m,d,k", LN_SHAPES)
def test_residual_layernorm_epilogue(cuda, fp8, m, d, k):
    """x (f16) += a.b^T*scale + bias, h = LN(x)*gamma + beta, against torch fp32 of the same op."""
    a, b, af, bf, bias = _operands(m, d, k, fp8, seed=m + 3 * d + k)
    g = torch.Generator(device="cuda").manual_seed(d + k)
    gamma = 1.0 + 0.2 * torch.randn(d, device=cuda, generator=g)
    beta = 0.1 * torch.randn(d, device=cuda, generator=g)
    scale, eps = (0.125 if fp8 else 1.0), 1e-5
    x0 = (torch.randn(m, d, device=cuda, generator=g) + 0.5).half()  # f16 stream, mean away from zero
    x = torch.cat([x0, torch.full((64, d), 3.0, device=cuda, dtype=torch.float16)])  # rows past m stay
    h = torch.full((m + 64, d), 0x55 if fp8 else 7.0, device=cuda, dtype=torch.uint8 if fp8 else torch.bfloat16)
    q = 0.02
    _run_ln(fp8, a, b, bias, gamma, beta, x, h, m, d, k, scale, eps, 1.0 / q)
    delta = (af @ bf.T) * scale + bias
    ref_x = x0.float() + delta
    # one rounding of the f32 sum to f16, plus the accumulation-order difference of the GEMM
    # itself (which dominates where x_old and the update cancel): the plain residual test's bound
    _within(x[:m].float(), ref_x, (ref_x.abs() + delta.abs()) * 2 ** -10 + 1e-6, "residual stream")
    assert bool((x[m:] == 3.0).all())
    # h is the LayerNorm of the rows as stored in the f16 stream (checked just above)
    ref_h = torch.nn.functional.layer_norm(x[:m].float(), (d,), gamma, beta, eps)
    if fp8:
        got = h[:m].view(torch.float8_e4m3fn).float() * q
        ref_sat = ref_h.clamp(-448 * q, 448 * q)
        assert bool(((got - ref_sat).abs() <= ref_h.abs() * 0.0625 + q * 2 ** -6 + 1e-5).all())
        assert bool((h[m:] == 0x55).all())
    else:
        got = h[:m].float()
        assert bool(((got - ref_h).abs() <= ref_h.abs() * 2 ** -8 + 1e-3).all())
        assert bool((h[m:] == 7.0).all())


def test_residual_layernorm_rejects_unsplittable_width(cuda):
    """d = 160 has no 64/96/128-column CTA slice; the plan is refused, nothing is launched."""
    m, d, k = 65, 160, 64
    a, b, _, _, bias = _operands(m, d, k, False, seed=1)
    ones = torch.ones(d, device=cuda)
    x = torch.zeros(m, d, device=cuda, dtype=torch.float16)
    h = torch.zeros(m, d, device=cuda, dtype=torch.bfloat16)
    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    rc = lib.mrn_test_gemm_ln(0, a.data_ptr(), b.data_ptr(), bias.data_ptr(), ones.data_ptr(), ones.data_ptr(),
                              x.data_ptr(), h.data_ptr(), m, d, k, 1.0, 1e-5, 1.0, ctypes.c_void_p(status.data_ptr()),
                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc != 0 and "slice" in lib.mrn_test_last_error().decode()


def _layernorm(x, gamma, beta, eps, e4m3, inv_q, out):
    lib = _lib.load()
    rows, d = x.shape
    rc = lib.mrn_test_layernorm(x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), eps, int(e4m3), inv_q,
                                out.data_ptr(), rows, d, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.mrn_test_last_error().decode()
    torch.cuda.synchronize()


def _run_norm(epi, x, gamma, beta, eps, a_inv_q, b, bias, out, ldo, m, n, k, scale, inv_q):
    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device=x.device)
    rc = lib.mrn_test_gemm_norm(epi, x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), eps, a_inv_q, b.data_ptr(),
                                bias.data_ptr(), out.data_ptr(), ldo, m, n, k, scale, inv_q,
                                ctypes.c_void_p(status.data_ptr()),
                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    if rc != 0:
        return lib.mrn_test_last_error().decode()
    torch.cuda.synchronize()
    assert int(status.item()) == 0, f"device status {int(status.item())}"
    return None


def _norm_inputs(m, d, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (torch.randn(m, d, device="cuda", generator=g) * 2.0 + 0.3).half()  # the f16 residual stream
    gamma = 1.0 + 0.2 * torch.randn(d, device="cuda", generator=g)
    beta = 0.1 * torch.randn(d, device="cuda", generator=g)
    return x, gamma, beta


@pytest.mark.parametrize("e4m3", [False, True], ids=["bf16", "e4m3"])
@pytest.mark.parametrize("m,d", [(65 * 7, 512), (65 * 3, 192), (1, 512), (65 * 64, 512), (130, 1024)])
def test_layernorm_kernel(cuda, e4m3, m, d):
    """The LayerNorm kernel against torch fp32 LayerNorm of the same f16 rows."""
    x, gamma, beta = _norm_inputs(m, d, seed=m + d)
    q, eps = 0.02, 1e-5
    out = torch.zeros((m, d), device=cuda, dtype=torch.uint8 if e4m3 else torch.bfloat16)
    _layernorm(x, gamma, beta, eps, e4m3, 1.0 / q, out)
    ref = torch.nn.functional.layer_norm(x.float(), (d,), gamma, beta, eps)
    if e4m3:
        got = out.view(torch.float8_e4m3fn).float() * q
        _within(got, ref, ref.abs() * 0.0625 + q * 2 ** -6 + 1e-5, "layernorm e4m3")
    else:
        _within(out.float(), ref, ref.abs() * 2 ** -8 + 1e-4, "layernorm bf16")


# (M, N): QKV and FFN1 of `small` (K = d = 512) with one, two and ragged 256-row blocks, fewer
# (block, tile) units than CTA pairs, and many blocks per pair (both A buffers reused).
NORM_SHAPES = [
    (65 * 7, 1536), (65 * 7, 2048), (1, 256), (256, 256), (257, 512), (65 * 64, 1536), (65 * 131, 2048),
    (65 * 1024, 1536), (65 * 1024, 2048),
]


@pytest.mark.parametrize("epi", [EPI_BIAS, EPI_GELU_E4M3, EPI_GELU_TANH_E4M3], ids=["bias", "gelu", "gelu_tanh"])
@pytest.mark.parametrize("m,n", NORM_SHAPES)
def test_norm_gemm_matches_layernorm_then_gemm(cuda, epi, m, n):
    """A normalised inside the GEMM: the same e4m3 A as the LayerNorm kernel writes, so the output
    equals LayerNorm kernel -> GEMM; that A agrees with torch's LayerNorm, and the output with torch
    fp32 of the GEMM on it."""
    k, eps, qa = 512, 1e-5, 0.02
    x, gamma, beta = _norm_inputs(m, k, seed=m + n)
    g = torch.Generator(device="cuda").manual_seed(n)
    b8 = (torch.randn(n, k, device=cuda, generator=g) * 0.4).to(torch.float8_e4m3fn)
    bias = torch.randn(n, device=cuda, generator=g) * 0.1
    scale, q = qa * 0.05, 0.05
    e4m3_out = epi != EPI_BIAS
    odt = torch.uint8 if e4m3_out else torch.bfloat16
    h = torch.zeros((m, k), device=cuda, dtype=torch.uint8)
    _layernorm(x, gamma, beta, eps, True, 1.0 / qa, h)
    want = torch.zeros((m, n), device=cuda, dtype=odt)
    _run(True, epi, h, b8.view(torch.uint8), bias, want, n, m, n, k, scale=scale, inv_q=1.0 / q)
    sentinel = 0x55 if e4m3_out else 7.0
    got = torch.full((m + 64, n), sentinel, device=cuda, dtype=odt)
    err = _run_norm(epi, x, gamma, beta, eps, 1.0 / qa, b8.view(torch.uint8), bias, got, n, m, n, k, scale, 1.0 / q)
    assert err is None, err
    assert bool((got[m:] == sentinel).all()), "rows past M were written"
    got = got[:m]
    if e4m3_out:
        g32, w32 = got.view(torch.float8_e4m3fn).float(), want.view(torch.float8_e4m3fn).float()
    else:
        g32, w32 = got.float(), want.float()
    # Same A, same accumulation per output element: identical up to the MMA's internal order on
    # the 256-row (CTA pair) against the 128-row tile, at most one output rounding step apart.
    same = (g32 == w32).float().mean().item()
    assert same >= 0.999, f"only {same:.4%} of outputs identical to LayerNorm -> GEMM"
    _within(g32, w32, w32.abs() * (0.0625 if e4m3_out else 2 ** -7) + 1e-6, "norm gemm vs layernorm -> gemm")
    # A itself: the LayerNorm kernel's e4m3 rows, within one e4m3 step of torch's LayerNorm (a
    # value on a rounding boundary may round either way, and one flipped code of a large A value
    # moves a whole output row by a step times |b|, so the GEMM is checked from this A).
    a_ref = h.view(torch.float8_e4m3fn).float()
    ln = torch.nn.functional.layer_norm(x.float(), (k,), gamma, beta, eps)
    _within(a_ref * qa, ln, ln.abs() * 0.0625 + qa * 2 ** -6 + 1e-5, "normalised A vs torch")
    acc = (a_ref @ b8.float().T) * scale + bias
    if epi == EPI_BIAS:
        _within(g32, acc, acc.abs() * 2 ** -7 + 1e-3, "norm gemm vs torch")
    else:
        ref = torch.nn.functional.gelu(acc, approximate="tanh" if epi == EPI_GELU_TANH_E4M3 else "none")
        _within(g32 * q, ref, ref.abs() * 0.0625 + q * 2 ** -6 + 2e-3, "norm gemm vs torch")


def test_norm_gemm_rejects_unsupported_shape(cuda):
    """K = 192 (nano) has no normalised-A instantiation: the plan is refused, nothing is launched."""
    m, n, k = 65, 576, 192
    x, gamma, beta = _norm_inputs(m, k, seed=2)
    b = torch.zeros((n, k), device=cuda, dtype=torch.uint8)
    bias = torch.zeros(n, device=cuda)
    out = torch.zeros((m, n), device=cuda, dtype=torch.bfloat16)
    err = _run_norm(EPI_BIAS, x, gamma, beta, 1e-5, 1.0, b, bias, out, n, m, n, k, 1.0, 1.0)
    assert err is not None and "gemm+norm" in err


def _run_mlp(tanh, h, w1, b1, w2, b2, x, m, d, ff, s1, inv_q, s2):
    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device=h.device)
    rc = lib.mrn_test_mlp(int(tanh), h.data_ptr(), w1.data_ptr(), b1.data_ptr(), w2.data_ptr(), b2.data_ptr(),
                          x.data_ptr(), m, d, ff, s1, inv_q, s2, ctypes.c_void_p(status.data_ptr()),
                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    if rc != 0:
        return lib.mrn_test_last_error().decode()
    torch.cuda.synchronize()
    assert int(status.item()) == 0, f"device status {int(status.item())}"
    return None


# (M, ff) with d = 512: one row, ragged and exact 128-row tiles, fewer tiles than CTA pairs, many
# tiles per pair (all hidden-chunk slots reused), and the smallest and a middle ff.
MLP_SHAPES = [(1, 2048), (65 * 3, 2048), (128, 2048), (129, 512), (65 * 64, 2048), (65 * 1024, 2048),
              (65 * 37, 1024), (65 * 512, 512)]


@pytest.mark.parametrize("tanh", [False, True], ids=["erf", "tanh"])
@pytest.mark.parametrize("m,ff", MLP_SHAPES)
def test_fused_mlp_matches_two_gemms(cuda, tanh, m, ff):
    """FFN1 -> GELU -> FFN2 -> residual in one kernel against the two GEMM launches it replaces
    (the same e4m3 hidden values and the same accumulation order, so the same x), and against
    torch fp32 of the same op on the hidden tensor the first GEMM writes."""
    d = 512
    g = torch.Generator(device="cuda").manual_seed(m + ff + int(tanh))
    h = (torch.randn(m, d, device=cuda, generator=g) * 2.0).to(torch.float8_e4m3fn)
    w1 = (torch.randn(ff, d, device=cuda, generator=g) * 0.5).to(torch.float8_e4m3fn)
    w2 = (torch.randn(d, ff, device=cuda, generator=g) * 0.5).to(torch.float8_e4m3fn)
    b1 = torch.randn(ff, device=cuda, generator=g) * 0.1
    b2 = torch.randn(d, device=cuda, generator=g) * 0.1
    s1, q, s2 = 0.01, 0.02, 0.0005
    x0 = torch.randn(m, d, device=cuda, generator=g).half()
    # the two launches it replaces
    f = torch.zeros((m, ff), device=cuda, dtype=torch.uint8)
    _run(True, EPI_GELU_TANH_E4M3 if tanh else EPI_GELU_E4M3, h.view(torch.uint8), w1.view(torch.uint8), b1, f, ff,
         m, ff, d, scale=s1, inv_q=1.0 / q)
    want = x0.clone()
    _run(True, EPI_RESIDUAL, f, w2.view(torch.uint8), b2, want, d, m, d, ff, scale=s2)
    # the fused kernel; rows past m stay
    x = torch.cat([x0, torch.full((64, d), 3.0, device=cuda, dtype=torch.float16)])
    err = _run_mlp(tanh, h.view(torch.uint8), w1.view(torch.uint8), b1, w2.view(torch.uint8), b2, x, m, d, ff, s1,
                   1.0 / q, s2)
    assert err is None, err
    assert bool((x[m:] == 3.0).all()), "rows past M were written"
    got, ref = x[:m].float(), want.float()
    same = (got == ref).float().mean().item()
    assert same >= 0.999, f"only {same:.4%} of x identical to the two-launch path"
    delta = ref - x0.float()
    _within(got, ref, (ref.abs() + delta.abs()) * 2 ** -10 + 2 ** -14, "fused mlp vs two launches")
    # torch fp32 from the hidden tensor the first launch wrote
    ref32 = x0.float() + (f.view(torch.float8_e4m3fn).float() @ w2.float().T) * s2 + b2
    d32 = ref32 - x0.float()
    _within(got, ref32, (ref32.abs() + d32.abs()) * 2 ** -10 + 2 ** -14, "fused mlp vs torch")


def test_fused_mlp_rejects_unsupported_shape(cuda):
    """d = 192 (nano) has no fused instantiation: the plan is refused, nothing is launched."""
    m, d, ff = 65, 192, 768
    z8 = torch.zeros((ff, d), device=cuda, dtype=torch.uint8)
    b = torch.zeros(ff, device=cuda)
    x = torch.zeros((m, d), device=cuda, dtype=torch.float16)
    err = _run_mlp(False, z8, z8, b, z8, b, x, m, d, ff, 1.0, 1.0, 1.0)
    assert err is not None and "mlp" in err
