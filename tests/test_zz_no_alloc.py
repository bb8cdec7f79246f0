"""`mrn_evaluate_device_static` -- the forward pass for callers that cannot allocate device
memory once running (their device memory belongs to another allocator, or an allocation
could stall a latency-critical thread) -- against `mrn_evaluate_device`, the entry point that
uses the context's own buffers, through the C ABI.

The static entry point keeps every intermediate buffer in one 8 MiB array compiled into the
library and shared by all calls on a device, so it is called twice in a row here to show that
the second call does not depend on what the first left in the array, and that neither call
changes the device's free memory. Both entry points run
the same kernels on the same inputs, so they agree to 1e-6 (the tolerance this suite uses for
GPU-to-GPU comparisons). This file sorts last so a failure here does not stop the rest of the
suite; it also runs on its own in a fresh process."""

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from marina_b200 import _lib, chess, model, weights  # noqa: E402
from marina_b200.network import B200Network, NetworkError  # noqa: E402

pytestmark = pytest.mark.gpu


def _card(name):
    from pathlib import Path

    return model.Architecture.from_json((Path(model.__file__).parent / "cards" / f"{name}.json").read_text())


@pytest.mark.parametrize("net,precision,n,limit", [("nano", "bf16", 8, 33), ("small", "fp8", 17, 17),
                                                   ("small", "fp8w", 12, 12), ("small", "fp8x2", 12, 12)])
def test_static_scratch_forward_matches_the_allocating_entry_point(net, precision, n, limit):
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    arch = _card(net)
    w = weights.random_init(arch, seed=0)
    boards, legal, counts, _ = chess.random_positions(23, n, 0, 80)
    ev = B200Network(arch, w, device=0, max_batch=n, precision=precision)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream(dev)
    db, dl = torch.from_numpy(boards).to(dev), torch.from_numpy(legal).to(dev)
    ref_p, ref_w = torch.empty((n, 224), device=dev), torch.empty((n, 3), device=dev)
    torch.cuda.synchronize()
    ev.evaluate_device(n, db.data_ptr(), dl.data_ptr(), ref_p.data_ptr(), ref_w.data_ptr(), stream.cuda_stream)
    stream.synchronize()
    assert ev.status_word() == 0
    for call in range(2):
        out_p = torch.full((n, 224), float("nan"), device=dev)
        out_w = torch.full((n, 3), float("nan"), device=dev)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info(dev)[0]
        ev.evaluate_device_static(n, db.data_ptr(), dl.data_ptr(), out_p.data_ptr(), out_w.data_ptr(),
                                  stream.cuda_stream)
        stream.synchronize()
        free_after = torch.cuda.mem_get_info(dev)[0]
        # The property the entry point exists for: no device memory is allocated by the call
        # (the array and the kernels were loaded by mrn_create), the first call included.
        assert free_after == free_before, (call, free_before - free_after)
        assert ev.status_word() == 0, call
        assert float((out_p - ref_p).abs().max()) <= 1e-6, call
        assert float((out_w - ref_w).abs().max()) <= 1e-6, call
        p = out_p.cpu().numpy()
        assert all(abs(p[i, :counts[i]].sum() - 1) < 1e-4 and (p[i, counts[i]:] == 0).all() for i in range(n))

    # The limit is the array's capacity for this network; one more position is refused.
    big = limit + 1
    bb, bl, _, _ = chess.random_positions(29, big, 0, 80)
    dbb, dbl = torch.from_numpy(bb).to(dev), torch.from_numpy(bl).to(dev)
    bp, bw = torch.empty((big, 224), device=dev), torch.empty((big, 3), device=dev)
    with pytest.raises(NetworkError) as e:
        ev.evaluate_device_static(big, dbb.data_ptr(), dbl.data_ptr(), bp.data_ptr(), bw.data_ptr(), stream.cuda_stream)
    assert e.value.code == 3 and f"the {limit} that fit" in str(e.value)
    # n = 0 is a no-op; the context still serves the allocating entry point afterwards
    ev.evaluate_device_static(0, db.data_ptr(), dl.data_ptr(), ref_p.data_ptr(), ref_w.data_ptr(), stream.cuda_stream)
    ev.evaluate_device(n, db.data_ptr(), dl.data_ptr(), ref_p.data_ptr(), ref_w.data_ptr(), stream.cuda_stream)
    stream.synchronize()
    assert ev.status_word() == 0
    ev.close()


def test_the_entry_point_is_exported():
    assert hasattr(_lib.load(), "mrn_evaluate_device_static")
    assert isinstance(ctypes.cast(_lib.load().mrn_evaluate_device_static, ctypes.c_void_p).value, int)
