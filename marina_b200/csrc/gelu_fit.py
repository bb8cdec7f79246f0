"""Coefficients of the GELU epilogues in gemm.cuh (run: python marina_b200/csrc/gelu_fit.py).

The epilogues evaluate the exact GELU of `torch.nn.GELU()` (src/net/cuda/kernels.cu:62-65 in the
reference, `0.5 x (1 + erf(x / sqrt 2))`) in the form

    GELU(x) = x Phi(x) = relu(x) - |x| Phi(-|x|),    Phi(-a) = 2^(-g(a)),   g(a) = -log2 Phi(-a),

so each element costs one hardware base-2 exponential and a polynomial for g. g is smooth and
convex on a >= 0 (g(0) = 1, g(a) ~ a^2 / (2 ln 2) for large a); it is fitted here by least
squares on Chebyshev nodes of [0, A] and the argument is clamped at A, past which Phi(-a) is
below 3.4e-6 (A = 4.5) / 1.9e-8 (A = 5.5) and the term it feeds is under half an output ulp.

Two fits: degree 7 on [0, 5.5] for the f32 epilogue (bf16 outputs; |GELU error| <= 4.4e-6
relative with f32 arithmetic), and degree 4 on [0, 4.5] for the packed-f16 epilogue whose
outputs are rounded to e4m3 (relative error <= 1.0e-2 in f16 arithmetic, dominated by the f16
rounding of x itself, so a higher degree buys nothing there; one e4m3 step is 12.5%; past the
bound Phi(-a) < 3.4e-6). The printed constants are the negated
coefficients, so the Horner chain yields -g(a) and feeds the exponential directly.
"""

import numpy as np
from scipy.special import log_ndtr, ndtr


def g(a):
    return -log_ndtr(-a) / np.log(2.0)


def fit(degree, bound, nodes=4000):
    t = np.cos(np.pi * (np.arange(nodes) + 0.5) / nodes)
    a = (t + 1.0) * bound / 2.0
    coef, *_ = np.linalg.lstsq(np.vander(a, degree + 1, increasing=True), g(a), rcond=None)
    return coef


def horner(coef, a, dtype):
    a = a.astype(dtype)
    p = dtype(coef[-1])
    for c in coef[-2::-1]:
        p = (p * a + dtype(c)).astype(dtype)
    return p


def gelu_error(coef, bound, dtype):
    """Max |error| relative to |GELU(x)| (for |GELU(x)| > 1e-3) over x in [-9, 9]."""
    x = np.linspace(-9.0, 9.0, 400001)
    exact = x * ndtr(x)
    xd = x.astype(dtype)
    a = np.minimum(np.abs(xd), dtype(bound))
    q = np.exp2(-horner(coef, a, dtype).astype(np.float32)).astype(dtype)
    y = (np.maximum(xd, dtype(0)) - (np.abs(xd) * q).astype(dtype)).astype(dtype).astype(np.float64)
    big = np.abs(exact) > 1e-3
    return float((np.abs(y - exact)[big] / np.abs(exact[big])).max())


def main():
    for name, degree, bound, dtype in (("kGeluF32", 7, 5.5, np.float32), ("kGeluF16", 4, 4.5, np.float16)):
        coef = fit(degree, bound)
        print(f"// {name}: degree {degree} on [0, {bound}], max relative GELU error "
              f"{gelu_error(coef, bound, dtype):.2e} in {np.dtype(dtype).name}")
        print(f"constexpr float {name}Bound = {bound}f;")
        for k, c in enumerate(coef):
            print(f"constexpr float {name}_{k} = {-c:.9e}f;")


if __name__ == "__main__":
    main()
