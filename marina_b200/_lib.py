"""ctypes binding of ``libmarina_b200.so`` (the C ABI in ``include/marina_b200.h``).

The library is loaded from the package directory, where ``marina_b200.build`` puts it.
There is no fallback: a missing or unloadable library raises ``ImportError`` here, so a
caller never silently runs anything but the CUDA path.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_double, c_float, c_int, c_int32, c_uint8, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmarina_b200.so"

BOARD_BYTES = 66
MAX_LEGAL = 224
POLICY_PLANES = 73
ACTIONS = 64 * POLICY_PLANES
WDL = 3

PRECISION_BF16 = 0
PRECISION_FP8_WEIGHTS = 1
PRECISION_FP8 = 2
PRECISIONS = {"bf16": PRECISION_BF16, "fp8w": PRECISION_FP8_WEIGHTS, "fp8": PRECISION_FP8}

PROFILE_SLOTS = ("embed", "layernorm", "gemm", "attention", "heads")

# Every symbol the header declares; `tests/test_abi.py` checks the library exports them.
EXPORTS = (
    "mrn_create", "mrn_evaluate", "mrn_evaluate_f16", "mrn_logits", "mrn_evaluate_device", "mrn_status_word",
    "mrn_profile", "mrn_launches_per_forward", "mrn_describe", "mrn_last_error", "mrn_destroy",
    "mrn_test_gemm", "mrn_test_gemm_ln", "mrn_test_gemm_norm", "mrn_test_mlp", "mrn_test_attention", "mrn_test_layernorm",
    "mrn_test_last_error",
    "mrn_evaluate_device_static",
)


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


def load() -> ctypes.CDLL:
    """The loaded library (declared signatures), loading it on first use."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is not built; run `python -m marina_b200.build`")
    lib = ctypes.CDLL(str(LIB_PATH))
    sig = {
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
        "mrn_test_gemm": (c_int, [c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                  c_float, c_float, c_void_p, c_void_p]),
        "mrn_test_gemm_ln": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                     c_int, c_int, c_int, c_float, c_float, c_float, c_void_p, c_void_p]),
        "mrn_test_gemm_norm": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_float, c_float, c_void_p, c_void_p,
                                       c_void_p, c_int, c_int, c_int, c_int, c_float, c_float, c_void_p, c_void_p]),
        "mrn_test_mlp": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                 c_int, c_float, c_float, c_float, c_void_p, c_void_p]),
        "mrn_test_attention": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_float, c_void_p, c_void_p]),
        "mrn_test_layernorm": (c_int, [c_void_p, c_void_p, c_void_p, c_float, c_int, c_float, c_void_p, c_int, c_int,
                                       c_void_p]),
        "mrn_test_last_error": (c_char_p, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib
