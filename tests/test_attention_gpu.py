"""The attention kernel against a plain PyTorch fp32 softmax attention on the same bf16 Q, K, V
(per position and head, 65 tokens; head_dim 64 and 32), through the test library."""

import ctypes

import pytest

torch = pytest.importorskip("torch")

from marina_b200 import _lib

pytestmark = pytest.mark.gpu

T = 65


def _attention(qkv, positions, d, heads, e4m3, inv_q):
    """`e4m3`: 0 bf16 output, 1 e4m3 codes, 2 two-term e4m3 codes (rows of 2d bytes)."""
    lib = _lib.load_test()
    out = torch.full((positions * T + 16, 2 * d if e4m3 == 2 else d), 0x55 if e4m3 else 7.0, device=qkv.device,
                     dtype=torch.uint8 if e4m3 else torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=qkv.device)
    rc = lib.mrn_test_attention(qkv.data_ptr(), out.data_ptr(), positions, d, heads, int(e4m3), inv_q,
                                ctypes.c_void_p(status.data_ptr()),
                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.mrn_test_last_error().decode()
    torch.cuda.synchronize()
    assert int(status.item()) == 0, f"device status {int(status.item())}"
    return out


def _reference(qkv, positions, d, heads):
    """fp32 softmax attention, and the P-weighted mean of |V| that bounds what rounding the
    probabilities to bf16 (the kernel's tensor-core path, relative error <= 2^-9 each) can move
    an output by."""
    hd = d // heads
    x = qkv.float().view(positions, T, 3, heads, hd)
    q, k, v = x[:, :, 0].transpose(1, 2), x[:, :, 1].transpose(1, 2), x[:, :, 2].transpose(1, 2)
    p = torch.softmax(q @ k.transpose(-1, -2) / hd ** 0.5, dim=-1)
    out = (p @ v).transpose(1, 2).reshape(positions * T, d)
    w = (p @ v.abs()).transpose(1, 2).reshape(positions * T, d)
    return out, w


# small (8 x 64) and nano (6 x 32) heads; one position, a few, and more items than CTAs
@pytest.mark.parametrize("d,heads", [(512, 8), (192, 6)])
@pytest.mark.parametrize("positions", [1, 3, 37, 300])
@pytest.mark.parametrize("e4m3", [0, 1, 2], ids=["bf16", "e4m3", "e4m3x2"])
def test_attention_matches_torch(cuda, d, heads, positions, e4m3):
    g = torch.Generator(device="cuda").manual_seed(positions * 7 + d)
    # scores of a few units, so the softmax is far from uniform
    qkv = (torch.randn(positions * T, 3 * d, device=cuda, generator=g) * 1.5).to(torch.bfloat16)
    ref, w = _reference(qkv, positions, d, heads)
    q = 0.02  # e4m3 codes up to 448 q: every output in range
    out = _attention(qkv, positions, d, heads, e4m3, 1.0 / q)
    rows = positions * T
    if e4m3 == 2:
        # hi + lo: the residual after one e4m3 step, itself rounded to e4m3 (or to the subnormal
        # step 2^-9), plus the bf16 rounding of P
        codes = out[:rows].view(torch.float8_e4m3fn).float()
        got = (codes[:, :d] + codes[:, d:]) * q
        assert float(ref.abs().max()) < 448 * q
        tol = ref.abs() * 2 ** -8 + q * 2 ** -10 + w * 2 ** -8 + 1e-4
        assert bool((out[rows:] == 0x55).all())
    elif e4m3:
        got = out[:rows].view(torch.float8_e4m3fn).float() * q
        assert float(ref.abs().max()) < 448 * q
        # one e4m3 step of the output, plus the bf16 rounding of P
        tol = ref.abs() * 0.0625 + q * 2 ** -6 + w * 2 ** -8 + 1e-4
        assert bool((out[rows:] == 0x55).all())
    else:
        got = out[:rows].float()
        # one bf16 rounding of the output, plus the bf16 rounding of P
        tol = ref.abs() * 2 ** -8 + w * 2 ** -8 + 1e-4
        assert bool((out[rows:] == 7.0).all())
    err = (got - ref).abs()
    bad = err > tol
    if bool(bad.any()):
        idx = bad.nonzero()[:6].tolist()
        where = [(r % T, c // (d // heads), c % (d // heads), float(got[r, c]), float(ref[r, c])) for r, c in idx]
        raise AssertionError(f"{int(bad.sum())} out of tolerance, max err {float(err.max())}; "
                             f"(token, head, col, got, ref): {where}")
