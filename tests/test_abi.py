"""The C-ABI libraries load and export every symbol their headers declare, and the
evaluator's argument checks run (and fail cleanly) without a GPU."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from marina_b200 import _lib, chess, model, weights
from marina_b200.network import B200Network, NetworkError

ROOT = Path(__file__).resolve().parents[1]


def _declared(header: str, macro: str) -> list[str]:
    text = (ROOT / "include" / header).read_text()
    return re.findall(macro + r"\s+[\w\s\*]*?\b(m\w+)\(", text)


def test_evaluator_exports_every_declared_symbol():
    names = _declared("marina_b200.h", "MRN_API")
    assert "mrn_create" in names and "mrn_evaluate" in names and len(names) >= 12
    lib = _lib.load()
    for name in names:
        assert hasattr(lib, name), name
    assert set(_lib.EXPORTS) >= set(names)


def test_evaluator_exports_nothing_but_the_header():
    """The drop-in library exports exactly the evaluator ABI: no test hooks."""
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.split()[1:2] == ["T"]}
    mrn = {name for name in exported if name.startswith("mrn_")}
    assert mrn == set(_declared("marina_b200.h", "MRN_API")), mrn ^ set(_declared("marina_b200.h", "MRN_API"))
    assert not any(name.startswith("mrn_test") for name in exported)


def test_test_library_exports_every_declared_symbol():
    names = _declared("marina_b200_test.h", "MRN_TEST_API")
    assert "mrn_test_gemm_wait_expiry" in names
    lib = _lib.load_test()
    for name in names:
        assert hasattr(lib, name), name
    assert set(_lib.TEST_EXPORTS) == set(names)


def test_group_entry_points_refuse_bad_arguments():
    """mrn_group_create checks its device list before touching a device; mrn_group_evaluate
    refuses a NULL group; both messages come back through mrn_group_last_error(NULL)."""
    lib = _lib.load()
    arch = model.Architecture(64, 1, 2, 128)
    from marina_b200.network import c_arch, c_weights

    ca, amax = c_arch(arch)
    cw, layers = c_weights(weights.random_init(arch))
    out = ctypes.c_void_p()
    assert lib.mrn_group_create(ctypes.byref(ca), ctypes.byref(cw), None, 0, 8, 0, ctypes.byref(out)) == 1
    assert b"at least one device" in lib.mrn_group_last_error(None)
    devs = (ctypes.c_int * 1)(0)
    assert lib.mrn_group_create(ctypes.byref(ca), ctypes.byref(cw), devs, 1, 0, 0, ctypes.byref(out)) == 1
    assert b"max_batch" in lib.mrn_group_last_error(None)
    assert lib.mrn_group_evaluate(None, 1, None, None, None, None) == 1
    assert b"group is NULL" in lib.mrn_group_last_error(None)
    assert lib.mrn_group_size(None) == 0 and lib.mrn_group_context(None, 0) is None


def test_chess_library_exports_every_declared_symbol():
    names = _declared("marina_chess.h", "MRC_API")
    lib = chess.load()
    assert len(names) >= 13
    for name in names:
        assert hasattr(lib, name), name


def _create(arch, w, precision="bf16"):
    return B200Network(arch, w, device=0, max_batch=8, precision=precision)


def test_unsupported_architectures_are_refused_before_touching_a_device():
    w_arch = model.Architecture(192, 1, 4, 768)  # head dim 48
    with pytest.raises(NetworkError) as e:
        _create(w_arch, weights.random_init(w_arch))
    assert e.value.code == 5 and "head dimension 48" in str(e.value)
    arch = model.nano()
    arch.fp8_amax = None
    with pytest.raises(NetworkError) as e:
        _create(arch, weights.random_init(arch), precision="fp8")
    assert e.value.code == 1 and "calibration" in str(e.value)


def test_non_finite_weights_are_refused():
    arch = model.Architecture(64, 1, 2, 128)
    w = weights.random_init(arch)
    w.tensors["encoder.layers.0.linear1.weight"][3, 5] = np.nan
    with pytest.raises(NetworkError) as e:
        _create(arch, w)
    assert e.value.code == 1 and "linear1.weight" in str(e.value)


def test_create_without_a_cuda_device_reports_an_error(monkeypatch):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    arch = model.Architecture(64, 1, 2, 128)
    with pytest.raises(NetworkError) as e:
        _create(arch, weights.random_init(arch))
    assert e.value.code in (2, 5)


def test_precision_names():
    arch = model.Architecture(64, 1, 2, 128)
    with pytest.raises(ValueError):
        B200Network(arch, weights.random_init(arch), precision="fp32")


def test_host_entry_points_refuse_a_null_context():
    """mrn_evaluate and mrn_evaluate_f16 reject a NULL context before any CUDA call, and the
    message is readable through mrn_last_error(NULL)."""
    lib = _lib.load()
    boards = np.zeros((1, _lib.BOARD_BYTES), dtype=np.uint8)
    legal = np.full((1, _lib.MAX_LEGAL), -1, dtype=np.int32)
    wdl = np.zeros((1, 3), dtype=np.float32)
    b = boards.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8))
    lg = legal.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))
    w = wdl.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    p32 = np.zeros((1, _lib.MAX_LEGAL), dtype=np.float32)
    p16 = np.zeros((1, _lib.MAX_LEGAL), dtype=np.float16)
    assert lib.mrn_evaluate(None, 1, b, lg, p32.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), w) == 1
    assert b"context is NULL" in lib.mrn_last_error(None)
    assert lib.mrn_evaluate_f16(None, 1, b, lg, p16.ctypes.data, w) == 1
    assert b"context is NULL" in lib.mrn_last_error(None)
