"""CPU oracle for Marina's batched transformer forward -- TEST INFRASTRUCTURE ONLY.

ctypes binding of ``oracle/_build/liboracle.so``, the plain-C restatement of the reference's
fp32 CPU backend (src/net/cpu.rs:48-184; see ``marina_oracle.h``). Only ``tests/``,
``__graft_entry__.smoke()`` and the benchmark's CPU-baseline / reference legs use it, and only
as the checker or the timed CPU baseline, never on the product path.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, Structure, c_float, c_int, c_int32, c_uint8

import numpy as np

from . import build as _build


class _Linear(Structure):
    _fields_ = [("weight", POINTER(c_float)), ("bias", POINTER(c_float))]


class _Norm(Structure):
    _fields_ = [("weight", POINTER(c_float)), ("bias", POINTER(c_float))]


class _Layer(Structure):
    _fields_ = [("norm1", _Norm), ("in_proj", _Linear), ("out_proj", _Linear), ("norm2", _Norm),
                ("linear1", _Linear), ("linear2", _Linear)]


class _Weights(Structure):
    _fields_ = [("piece_embed", POINTER(c_float)), ("square_embed", POINTER(c_float)),
                ("state_embed", POINTER(c_float)), ("castling_proj", _Linear),
                ("en_passant_embed", POINTER(c_float)), ("layers", POINTER(_Layer)), ("final_norm", _Norm),
                ("policy_norm", _Norm), ("policy_proj", _Linear), ("value_norm", _Norm), ("value_ff1", _Linear),
                ("value_ff2", _Linear)]


class _Arch(Structure):
    _fields_ = [("d_model", c_int32), ("n_layers", c_int32), ("n_heads", c_int32), ("d_ff", c_int32),
                ("layer_norm_eps", c_float), ("gelu", c_int32), ("tokens", c_int32),
                ("square_token_start", c_int32)]


_lib = None


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(_build.build()))
        f = POINTER(c_float)
        lib.oracle_logits.argtypes = [POINTER(_Arch), POINTER(_Weights), c_int, POINTER(c_uint8), f, f, f, c_int]
        lib.oracle_evaluate.argtypes = [POINTER(_Arch), POINTER(_Weights), c_int, POINTER(c_uint8), POINTER(c_int32),
                                        f, f, c_int]
        for name in ("oracle_exp_fast", "oracle_erf", "oracle_gelu", "oracle_gelu_tanh"):
            getattr(lib, name).argtypes = [c_float]
            getattr(lib, name).restype = c_float
        lib.oracle_softmax.argtypes = [f, c_int]
        lib.oracle_softmax.restype = None
        lib.oracle_layer_norm.argtypes = [f, f, f, f, c_int, c_int, c_float]
        lib.oracle_layer_norm.restype = None
        lib.oracle_sgemm_nt.argtypes = [c_int, c_int, c_int, f, f, f]
        lib.oracle_sgemm_nt.restype = None
        lib.oracle_linear.argtypes = [f, f, f, f, c_int, c_int, c_int, c_int]
        lib.oracle_linear.restype = None
        _lib = lib
    return _lib


def fp(a: np.ndarray):
    return a.ctypes.data_as(POINTER(c_float))


class OracleNetwork:
    """The reference CPU backend, restated: `logits` and `evaluate` over packed boards."""

    def __init__(self, arch, weights, threads: int = 1):
        self.arch, self.weights, self.threads = arch, weights, threads
        w = weights
        lin = lambda a, b: _Linear(w.ptr(a), w.ptr(b))  # noqa: E731
        nrm = lambda p: _Norm(w.ptr(p + ".weight"), w.ptr(p + ".bias"))  # noqa: E731
        self._layers = (_Layer * arch.n_layers)()
        for i in range(arch.n_layers):
            p = f"encoder.layers.{i}."
            self._layers[i] = _Layer(nrm(p + "norm1"), lin(p + "self_attn.in_proj_weight", p + "self_attn.in_proj_bias"),
                                     lin(p + "self_attn.out_proj.weight", p + "self_attn.out_proj.bias"),
                                     nrm(p + "norm2"), lin(p + "linear1.weight", p + "linear1.bias"),
                                     lin(p + "linear2.weight", p + "linear2.bias"))
        self._w = _Weights(w.ptr("piece_embed.weight"), w.ptr("square_embed.weight"), w.ptr("state_embed"),
                           lin("castling_proj.weight", "castling_proj.bias"), w.ptr("en_passant_embed.weight"),
                           ctypes.cast(self._layers, POINTER(_Layer)), nrm("final_norm"), nrm("policy_head.norm"),
                           lin("policy_head.proj.weight", "policy_head.proj.bias"), nrm("value_head.norm"),
                           lin("value_head.ff.0.weight", "value_head.ff.0.bias"),
                           lin("value_head.ff.2.weight", "value_head.ff.2.bias"))
        self._arch = _Arch(arch.d_model, arch.n_layers, arch.n_heads, arch.d_ff, arch.layer_norm_eps, arch.gelu,
                           arch.tokens, arch.square_token_start)

    def logits(self, boards: np.ndarray, with_amax: bool = False):
        """Raw policy logits [n, 4672], WDL logits [n, 3] (and the per-layer activation maxima)."""
        boards = np.ascontiguousarray(boards, dtype=np.uint8)
        n = boards.shape[0]
        policy = np.zeros((n, 64 * 73), dtype=np.float32)
        value = np.zeros((n, 3), dtype=np.float32)
        amax = np.zeros((self.arch.n_layers, 4), dtype=np.float32) if with_amax else None
        rc = load().oracle_logits(ctypes.byref(self._arch), ctypes.byref(self._w), n,
                                  boards.ctypes.data_as(POINTER(c_uint8)), fp(policy), fp(value),
                                  fp(amax) if amax is not None else None, self.threads)
        if rc != 0:
            raise ValueError("oracle_logits rejected its input")
        return (policy, value, amax) if with_amax else (policy, value)

    def evaluate(self, boards: np.ndarray, legal: np.ndarray):
        """Priors [n, 224] (softmax over each position's legal slots) and WDL [n, 3]."""
        boards = np.ascontiguousarray(boards, dtype=np.uint8)
        legal = np.ascontiguousarray(legal, dtype=np.int32)
        n = boards.shape[0]
        priors = np.zeros((n, 224), dtype=np.float32)
        wdl = np.zeros((n, 3), dtype=np.float32)
        rc = load().oracle_evaluate(ctypes.byref(self._arch), ctypes.byref(self._w), n,
                                    boards.ctypes.data_as(POINTER(c_uint8)), legal.ctypes.data_as(POINTER(c_int32)),
                                    fp(priors), fp(wdl), self.threads)
        if rc != 0:
            raise ValueError("oracle_evaluate rejected its input")
        return priors, wdl


def calibrate(arch, weights, boards: np.ndarray, threads: int = 1) -> list[list[float]]:
    """The FP8 calibration the reference's card carries: per layer, the largest |value| of
    norm1 out, attention out, norm2 out and GELU out over `boards` (src/net/model.rs:87-95)."""
    _, _, amax = OracleNetwork(arch, weights, threads).logits(boards, with_amax=True)
    return amax.astype(float).tolist()
