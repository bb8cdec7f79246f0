"""Runtime guarantees of the evaluator library on the GPU, through the C ABI:

* the passes on one context are ordered on the device even when they are enqueued on different
  streams with no synchronisation in between (the reference serialises its backend under one
  mutex and synchronises every call, src/net/cuda/mod.rs:932-973);
* the multi-device evaluator (`mrn_group_*`) returns what one context returns, in input order;
* a GEMM whose bounded waits run out reports MRN_ERR_DEVICE_FAULT and leaves the GPU context
  serving the next pass (the reference's error contract: a failing network stops the search with
  its error, nothing is substituted, src/net/mod.rs:284-288, src/search/mod.rs:794-797). The wait
  runs out because the test GEMM's producer issues no loads, so no copy or MMA is ever in flight.
"""

import ctypes

import numpy as np
import pytest

import oracle
from marina_b200 import _lib, chess, model, weights
from marina_b200.network import B200Network, GroupNetwork, NetworkError

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

WDL_TOL, PRIOR_TOL = 2e-2, 3e-2


@pytest.fixture(scope="module")
def nano():
    arch = model.nano()
    w = weights.random_init(arch, seed=0)
    boards, legal, counts, _ = chess.random_positions(61, 96, 0, 80)
    return arch, w, boards, legal, counts


def test_passes_on_two_streams_and_the_host_path_are_ordered(cuda, nano):
    """mrn_evaluate_device on stream A, then on stream B, then mrn_evaluate (the context's own
    stream), then again on A -- with different batches and no synchronisation in between. Each
    result equals the one the same batch gives on its own."""
    arch, w, boards, legal, counts = nano
    net = B200Network(arch, w, device=0, max_batch=96, precision="bf16")
    halves = [(boards[:48], legal[:48]), (boards[48:], legal[48:])]
    alone = [net.evaluate_packed(b, l) for b, l in halves]
    sa, sb = torch.cuda.Stream(cuda), torch.cuda.Stream(cuda)
    dev = [(torch.from_numpy(b).to(cuda), torch.from_numpy(l).to(cuda)) for b, l in halves]
    outs = [(torch.full((48, 224), float("nan"), device=cuda), torch.full((48, 3), float("nan"), device=cuda))
            for _ in range(3)]
    torch.cuda.synchronize()
    for rep in range(3):
        net.evaluate_device(48, dev[0][0].data_ptr(), dev[0][1].data_ptr(), outs[0][0].data_ptr(),
                            outs[0][1].data_ptr(), sa.cuda_stream)
        net.evaluate_device(48, dev[1][0].data_ptr(), dev[1][1].data_ptr(), outs[1][0].data_ptr(),
                            outs[1][1].data_ptr(), sb.cuda_stream)
        host_p, host_w = net.evaluate_packed(*halves[0])
        net.evaluate_device(48, dev[1][0].data_ptr(), dev[1][1].data_ptr(), outs[2][0].data_ptr(),
                            outs[2][1].data_ptr(), sa.cuda_stream)
        torch.cuda.synchronize()
        assert net.status_word() == 0
        assert np.array_equal(host_p, alone[0][0]) and np.array_equal(host_w, alone[0][1]), rep
        for (p, wd), half in zip(outs, (0, 1, 1)):
            assert np.array_equal(p.cpu().numpy(), alone[half][0]), (rep, half)
            assert np.array_equal(wd.cpu().numpy(), alone[half][1]), (rep, half)
    net.close()


@pytest.mark.parametrize("n_devices", [1, 2, 3])
def test_group_matches_one_context(cuda, nano, n_devices):
    """A group of contexts (all on device 0 here: a device may be listed more than once) gives each
    position the answer one context gives it, in input order, for batches that split evenly, unevenly
    and into fewer positions than devices, and for batches of several max_batch chunks (shards taken
    from the shared queue); a failing shard is reported with its device and positions."""
    arch, w, boards, legal, counts = nano
    one = B200Network(arch, w, device=0, max_batch=96, precision="bf16")
    group = GroupNetwork(arch, w, [0] * n_devices, max_batch=96, precision="bf16")
    assert str(n_devices) in group.describe()
    for n in (96, 95, 2, 1):
        p1, w1 = one.evaluate_packed(boards[:n], legal[:n])
        pg, wg = group.evaluate_packed(boards[:n], legal[:n])
        assert np.abs(p1 - pg).max() <= 1e-6 and np.abs(w1 - wg).max() <= 1e-6, n
        assert all((pg[i, counts[i]:] == 0).all() for i in range(n))
    leaves = [(boards[i], legal[i, :counts[i]].tolist()) for i in range(10)]
    evs = group.evaluate(leaves)
    assert [len(e.priors) for e in evs] == list(counts[:10])
    big_b, big_l = np.concatenate([boards] * 4), np.concatenate([legal] * 4)
    for n in (97, 250, 384):  # 2, 3 and 4 chunks of max_batch, the last ragged or full
        pg, wg = group.evaluate_packed(big_b[:n], big_l[:n])
        for a in range(0, n, 96):
            p1, w1 = one.evaluate_packed(big_b[a:min(n, a + 96)], big_l[a:min(n, a + 96)])
            assert np.abs(p1 - pg[a:a + len(p1)]).max() <= 1e-6 and np.abs(w1 - wg[a:a + len(w1)]).max() <= 1e-6, n
    bad_l = big_l[:250].copy()
    bad_l[150, 0] = 5000  # an action index outside [0, 4672) in the second chunk
    with pytest.raises(NetworkError) as e:
        group.evaluate_packed(big_b[:250], bad_l)
    assert e.value.code == 7 and "device 0" in str(e.value), str(e.value)
    lo, hi = (int(x) for x in str(e.value).split("positions [")[1].split(")")[0].split(", "))
    assert lo <= 150 < hi, str(e.value)
    pg, wg = group.evaluate_packed(big_b[:96], big_l[:96])  # the group serves the next call
    p1, w1 = one.evaluate_packed(big_b[:96], big_l[:96])
    assert np.abs(p1 - pg).max() <= 1e-6 and np.abs(w1 - wg).max() <= 1e-6
    group.close()
    one.close()


def test_bounded_wait_expiry_reports_a_device_fault_and_the_context_recovers(cuda, nano):
    arch, w, boards, legal, counts = nano
    net = B200Network(arch, w, device=0, max_batch=96, precision="bf16")
    before_p, before_w = net.evaluate_packed(boards, legal)
    test = _lib.load_test()
    m, n, k = 65 * 4, 256, 512
    a = torch.randn(m, k, device=cuda).to(torch.bfloat16)
    b = (torch.randn(n, k, device=cuda) * 0.05).to(torch.bfloat16)
    bias = torch.zeros(n, device=cuda)
    out = torch.zeros(m, n, device=cuda, dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    import time

    def plain():
        status.zero_()
        rc = test.mrn_test_gemm(0, 0, -1, a.data_ptr(), b.data_ptr(), bias.data_ptr(), out.data_ptr(), n, m, n, k,
                                1.0, 1.0, ctypes.c_void_p(status.data_ptr()), ctypes.c_void_p(stream))
        torch.cuda.synchronize()
        assert rc == 0 and int(status.item()) == 0
        ref = a.float() @ b.float().T
        assert float((out.float() - ref).abs().max()) <= float(ref.abs().max()) * 2 ** -7 + 1e-3

    plain()  # loads the test library's kernels before anything is timed
    status.zero_()
    t0 = time.perf_counter()
    rc = test.mrn_test_gemm_wait_expiry(1_000_000, a.data_ptr(), b.data_ptr(), bias.data_ptr(), out.data_ptr(), m,
                                        n, k, ctypes.c_void_p(status.data_ptr()), ctypes.c_void_p(stream))
    elapsed = time.perf_counter() - t0
    msg = test.mrn_test_last_error().decode()
    assert rc == 6, (rc, msg)  # MRN_ERR_DEVICE_FAULT
    assert int(status.item()) in (2, 3), msg  # the MMA issuer's or the epilogue's wait gave up
    assert "gave up" in msg
    assert elapsed < 1.0, elapsed  # the 1 ms limit, not the 2 s default
    # The same GEMM with the default limit and loads issued runs clean afterwards ...
    plain()
    # ... and the evaluator's context serves the same answers, which meet the oracle bounds.
    after_p, after_w = net.evaluate_packed(boards, legal)
    assert np.array_equal(before_p, after_p) and np.array_equal(before_w, after_w)
    ref_p, ref_w = oracle.OracleNetwork(arch, w, threads=8).evaluate(boards, legal)
    prior = max(float(np.abs(after_p[i, :c] - ref_p[i, :c]).max()) for i, c in enumerate(counts))
    assert prior <= PRIOR_TOL and float(np.abs(after_w - ref_w).max()) <= WDL_TOL
    assert net.status_word() == 0
    net.close()
