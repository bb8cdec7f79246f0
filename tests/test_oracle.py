"""Pin the CPU oracle (the C restatement of src/net/cpu.rs) before it is trusted:
the reference's own known-answer tests for the primitives (src/net/cpu.rs:377-420,
src/net/gemm.rs:132-159), an independent float64 PyTorch implementation of the whole
forward pass, and the committed golden output of the `nano` configuration."""

import math
from pathlib import Path

import numpy as np
import pytest

import oracle
from marina_b200 import chess, model, weights
from tests.torch_reference import forward64, priors_from_logits, softmax

GOLDEN = Path(__file__).parent / "golden"


@pytest.fixture(scope="module")
def lib():
    return oracle.load()


def test_primitives_match_definitions(lib):
    """src/net/cpu.rs:377-420."""
    assert abs(lib.oracle_gelu(0.0)) < 1e-7
    assert abs(lib.oracle_gelu(1.0) - 0.841345) < 1e-5
    assert abs(lib.oracle_gelu(-1.0) + 0.158655) < 1e-5
    assert abs(lib.oracle_gelu(3.0) - 2.99595) < 1e-5
    assert abs(lib.oracle_gelu_tanh(0.0)) < 1e-7
    assert abs(lib.oracle_gelu_tanh(1.0) - 0.841192) < 1e-5
    assert abs(lib.oracle_gelu_tanh(-1.0) + 0.158808) < 1e-5
    assert abs(lib.oracle_gelu_tanh(3.0) - 2.99636) < 1e-5

    row = np.array([1, 2, 3, 4], np.float32)
    out = np.zeros(4, np.float32)
    g, b = np.ones(4, np.float32), np.zeros(4, np.float32)
    lib.oracle_layer_norm(oracle.fp(row), oracle.fp(out), oracle.fp(g), oracle.fp(b), 1, 4, 1e-5)
    assert abs(out.sum()) < 1e-5 and abs(out[3] - 1.34164) < 1e-4

    w = np.array([1, 2, 3, 4, 5, 6], np.float32)
    bias = np.array([0.5, -0.5], np.float32)
    x = np.array([1, 1, 1, 0, 1, 0], np.float32)
    y = np.zeros(4, np.float32)
    lib.oracle_linear(oracle.fp(x), oracle.fp(y), oracle.fp(w), oracle.fp(bias), 2, 3, 2, 1)
    assert y.tolist() == [6.5, 14.5, 2.5, 4.5]

    for v in [-80.0, -10.0, -1.0, -0.1, 0.0, 0.1, 1.0, 5.0, 20.0, 80.0]:
        rel = abs(lib.oracle_exp_fast(v) - math.exp(v)) / math.exp(v)
        assert rel < 3e-7, (v, rel)

    s = np.array([1, 2, 3], np.float32)
    lib.oracle_softmax(oracle.fp(s), 3)
    assert abs(s.sum() - 1) < 1e-6 and abs(s[2] - 0.66524) < 1e-4


def test_erf_within_abramowitz_stegun_bound(lib):
    for v in np.linspace(-4, 4, 81):
        assert abs(lib.oracle_erf(float(v)) - math.erf(v)) < 3e-7


def test_sgemm_matches_a_hand_computation(lib):
    """src/net/gemm.rs:145-153: c starts at 0.5."""
    a = np.array([1, 1, 1, 0, 1, 0], np.float32)
    w = np.array([1, 2, 3, 4, 5, 6], np.float32)
    c = np.full(4, 0.5, np.float32)
    lib.oracle_sgemm_nt(2, 3, 2, oracle.fp(a), oracle.fp(w), oracle.fp(c))
    assert c.tolist() == [6.5, 15.5, 2.5, 5.5]


@pytest.mark.parametrize("m,k,n", [(37, 53, 29), (130, 64, 96), (5, 512, 73)])
def test_sgemm_agrees_with_naive(lib, m, k, n):
    """src/net/gemm.rs:155-159, plus shapes that exercise the 4x32 blocking and its tails."""
    a = (((np.arange(m * k) * 7) % 11) / 11.0 - 0.5).astype(np.float32)
    w = (((np.arange(n * k) * 5) % 13) / 13.0 - 0.5).astype(np.float32)
    c = np.zeros(m * n, np.float32)
    lib.oracle_sgemm_nt(m, k, n, oracle.fp(a), oracle.fp(w), oracle.fp(c))
    expect = a.reshape(m, k).astype(np.float64) @ w.reshape(n, k).astype(np.float64).T
    assert np.abs(c.reshape(m, n) - expect).max() < 1e-4


def _tiny_arch():
    return model.Architecture(64, 2, 2, 128)


def _tiny_tanh_arch():
    return model.Architecture(64, 2, 2, 128, gelu=model.GELU_TANH)


@pytest.mark.parametrize("arch_fn,n,threads", [(_tiny_arch, 9, 1), (_tiny_tanh_arch, 7, 2), (model.nano, 5, 3)])
def test_forward_matches_float64_reference(arch_fn, n, threads):
    arch = arch_fn()
    w = weights.random_init(arch, seed=3, std=0.05, bias_std=0.05, norm_std=0.1)
    boards, legal, counts, _ = chess.random_positions(11, n)
    net = oracle.OracleNetwork(arch, w, threads=threads)
    policy, value = net.logits(boards)
    ref_p, ref_v = forward64(arch, w, boards)
    assert np.abs(policy - ref_p).max() < 2e-4
    assert np.abs(value - ref_v).max() < 2e-4
    priors, wdl = net.evaluate(boards, legal)
    assert np.abs(priors - priors_from_logits(ref_p, legal)).max() < 2e-5
    assert np.abs(wdl - softmax(ref_v)).max() < 2e-5
    for p in range(n):
        assert abs(priors[p].sum() - 1) < 1e-5 and (priors[p, counts[p]:] == 0).all()


def test_thread_count_does_not_change_results():
    arch = model.nano()
    w = weights.random_init(arch, seed=0)
    boards, legal, _, _ = chess.random_positions(1, 600)
    a = oracle.OracleNetwork(arch, w, threads=1).evaluate(boards, legal)
    b = oracle.OracleNetwork(arch, w, threads=4).evaluate(boards, legal)
    assert (a[0] == b[0]).all() and (a[1] == b[1]).all()


def test_golden_nano_config():
    """Config 0: nano net, N(0, 0.02) weights (seed 0), 64 random-playout positions (seed 1):
    the oracle reproduces the committed golden WDL and legal-move policy."""
    g = np.load(GOLDEN / "nano_b64.npz")
    arch = model.nano()
    w = weights.random_init(arch, seed=0)
    boards, legal, counts, _ = chess.random_positions(1, 64, 0, 80)
    assert (boards == g["boards"]).all() and (legal == g["legal"]).all()
    priors, wdl = oracle.OracleNetwork(arch, w, threads=2).evaluate(boards, legal)
    assert np.abs(priors - g["priors"]).max() < 1e-6
    assert np.abs(wdl - g["wdl"]).max() < 1e-6
    ref_p, ref_v = forward64(arch, w, boards)
    assert np.abs(g["priors"] - priors_from_logits(ref_p, legal)).max() < 1e-5
    assert np.abs(g["wdl"] - softmax(ref_v)).max() < 1e-5


def test_fp8_quantisation_matches_torch_e4m3():
    torch = pytest.importorskip("torch")
    x = np.random.default_rng(0).standard_normal(20000).astype(np.float32) * 50
    x = np.concatenate([x, [0.0, -0.0, 448.0, -448.0, 1e-9, 0.001953125, 0.0029296875, 600.0]]).astype(np.float32)
    ours = weights.e4m3_round(x)
    ref = torch.from_numpy(np.clip(x, -448, 448)).to(torch.float8_e4m3fn).float().numpy()
    assert (ours == ref).all()
    w = np.random.default_rng(1).standard_normal((64, 32)).astype(np.float32) * 0.02
    codes, scale = weights.fp8_quantize(w)
    assert np.abs(codes).max() == 448.0
    assert np.abs(codes * scale - w).max() <= np.abs(w).max() * 2 ** -4
