"""ctypes binding of ``libmarina_b200.so`` (the C ABI in ``include/marina_b200.h``) and of the
GPU test-suite's ``libmarina_b200_test.so`` (``include/marina_b200_test.h``).

The libraries are loaded from the package directory, where ``marina_b200.build`` puts them.
There is no fallback: a missing or unloadable library raises ``ImportError`` here, so a
caller never silently runs anything but the CUDA path.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_double, c_float, c_int, c_int32, c_uint8, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmarina_b200.so"
TEST_LIB_PATH = Path(__file__).resolve().parent / "libmarina_b200_test.so"

BOARD_BYTES = 66
MAX_LEGAL = 224
POLICY_PLANES = 73
ACTIONS = 64 * POLICY_PLANES
WDL = 3

PRECISION_BF16 = 0
PRECISION_FP8_WEIGHTS = 1
PRECISION_FP8 = 2
PRECISION_FP8_X2 = 3
PRECISIONS = {"bf16": PRECISION_BF16, "fp8w": PRECISION_FP8_WEIGHTS, "fp8": PRECISION_FP8,
              "fp8x2": PRECISION_FP8_X2}

PROFILE_SLOTS = ("embed", "layernorm", "gemm", "attention", "heads")

# Every symbol each header declares; `tests/test_abi.py` checks the libraries export exactly these.
EXPORTS = (
    "mrn_create", "mrn_evaluate", "mrn_evaluate_f16", "mrn_logits", "mrn_evaluate_device", "mrn_status_word",
    "mrn_profile", "mrn_launches_per_forward", "mrn_describe", "mrn_last_error", "mrn_destroy",
    "mrn_group_create", "mrn_group_evaluate", "mrn_group_size", "mrn_group_context", "mrn_group_describe",
    "mrn_group_last_error", "mrn_group_destroy",
    "mrn_evaluate_device_static",
)
TEST_EXPORTS = ("mrn_test_gemm", "mrn_test_gemm_wait_expiry", "mrn_test_attention", "mrn_test_layernorm",
                "mrn_test_last_error")


class MrnLinear(ctypes.Structure):
    _fields_ = [("weight", POINTER(c_float)), ("bias", POINTER(c_float))]


class MrnNorm(ctypes.Structure):
    _fields_ = [("weight", POINTER(c_float)), ("bias", POINTER(c_float))]


class MrnLayer(ctypes.Structure):
    _fields_ = [("norm1", MrnNorm), ("in_proj", MrnLinear), ("out_proj", MrnLinear),
                ("norm2", MrnNorm), ("linear1", MrnLinear), ("linear2", MrnLinear)]


class MrnWeights(ctypes.Structure):
    _fields_ = [("piece_embed", POINTER(c_float)), ("square_embed", POINTER(c_float)),
                ("state_embed", POINTER(c_float)), ("castling_proj", MrnLinear),
                ("en_passant_embed", POINTER(c_float)), ("layers", POINTER(MrnLayer)),
                ("final_norm", MrnNorm), ("policy_norm", MrnNorm), ("policy_proj", MrnLinear),
                ("value_norm", MrnNorm), ("value_ff1", MrnLinear), ("value_ff2", MrnLinear)]


class MrnArch(ctypes.Structure):
    _fields_ = [("d_model", c_int32), ("n_layers", c_int32), ("n_heads", c_int32), ("d_ff", c_int32),
                ("layer_norm_eps", c_float), ("gelu", c_int32), ("tokens", c_int32),
                ("square_token_start", c_int32), ("fp8_amax", POINTER(c_float))]


_lib = None
_test_lib = None

SIGNATURES = {
    "mrn_create": (c_int, [POINTER(MrnArch), POINTER(MrnWeights), c_int, c_int, c_int, POINTER(c_void_p)]),
    "mrn_evaluate": (c_int, [c_void_p, c_int, POINTER(c_uint8), POINTER(c_int32), POINTER(c_float), POINTER(c_float)]),
    "mrn_evaluate_f16": (c_int, [c_void_p, c_int, POINTER(c_uint8), POINTER(c_int32), c_void_p, POINTER(c_float)]),
    "mrn_logits": (c_int, [c_void_p, c_int, POINTER(c_uint8), POINTER(c_float), POINTER(c_float)]),
    "mrn_evaluate_device": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "mrn_evaluate_device_static": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "mrn_status_word": (c_int, [c_void_p, POINTER(c_int)]),
    "mrn_profile": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                            POINTER(c_float), POINTER(c_double), POINTER(c_int)]),
    "mrn_launches_per_forward": (c_int, [c_void_p, c_int]),
    "mrn_describe": (c_char_p, [c_void_p]),
    "mrn_last_error": (c_char_p, [c_void_p]),
    "mrn_destroy": (None, [c_void_p]),
    "mrn_group_create": (c_int, [POINTER(MrnArch), POINTER(MrnWeights), POINTER(c_int), c_int, c_int, c_int,
                                 POINTER(c_void_p)]),
    "mrn_group_evaluate": (c_int, [c_void_p, c_int, POINTER(c_uint8), POINTER(c_int32), POINTER(c_float),
                                   POINTER(c_float)]),
    "mrn_group_size": (c_int, [c_void_p]),
    "mrn_group_context": (c_void_p, [c_void_p, c_int]),
    "mrn_group_describe": (c_char_p, [c_void_p]),
    "mrn_group_last_error": (c_char_p, [c_void_p]),
    "mrn_group_destroy": (None, [c_void_p]),
}

TEST_SIGNATURES = {
    "mrn_test_gemm": (c_int, [c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                              c_int, c_float, c_float, c_void_p, c_void_p]),
    "mrn_test_gemm_wait_expiry": (c_int, [ctypes.c_ulonglong, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                          c_int, c_void_p, c_void_p]),
    "mrn_test_attention": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_float, c_void_p, c_void_p]),
    "mrn_test_layernorm": (c_int, [c_void_p, c_void_p, c_void_p, c_float, c_int, c_float, c_void_p, c_int, c_int,
                                   c_void_p]),
    "mrn_test_last_error": (c_char_p, []),
}


def _open(path: Path, signatures: dict) -> ctypes.CDLL:
    if not path.exists():
        raise ImportError(f"{path} is not built; run `python -m marina_b200.build`")
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in signatures.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    return lib


def load() -> ctypes.CDLL:
    """The evaluator library (declared signatures), loading it on first use."""
    global _lib
    if _lib is None:
        _lib = _open(LIB_PATH, SIGNATURES)
    return _lib


def load_test() -> ctypes.CDLL:
    """The GPU test-suite's kernel-level library, loading it on first use."""
    global _test_lib
    if _test_lib is None:
        _test_lib = _open(TEST_LIB_PATH, TEST_SIGNATURES)
    return _test_lib
