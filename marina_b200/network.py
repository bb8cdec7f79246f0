"""The evaluator behind the reference's ``Network`` trait (src/net/mod.rs:264-296), in Python.

``B200Network`` is the drop-in for ``CudaNetwork`` (src/net/cuda/mod.rs:225-1012): it
owns one library context (``mrn_ctx``) on one GPU, packs leaves the way the reference's CUDA
backend does (src/net/cuda/mod.rs:946-967) and slices each position's priors out of the
224-slot output (:994-999). ``GroupNetwork`` implements the same trait over several GPUs
through the library's own multi-device evaluator (``mrn_group_*``: contiguous shards, one
per GPU, evaluated at the same time by native per-device threads and written back in
order); ``ShardedNetwork`` does the same from Python threads over any replicas. No
collective is involved: the positions are independent. Errors surface as ``NetworkError``; nothing is ever substituted for a
network's answer (src/net/mod.rs:284-288).
"""

from __future__ import annotations

import ctypes
import threading
from abc import ABC, abstractmethod
from concurrent.futures import ThreadPoolExecutor
from ctypes import POINTER, c_double, c_float, c_int, c_int32, c_uint8, c_void_p
from dataclasses import dataclass
from typing import Sequence

import numpy as np

from . import _lib
from .model import Architecture
from .weights import Weights

MAX_LEGAL = _lib.MAX_LEGAL
BOARD_BYTES = _lib.BOARD_BYTES


class NetworkError(RuntimeError):
    """A backend that can no longer evaluate (`NetworkError`, src/net/mod.rs:284-288)."""

    def __init__(self, message: str, code: int = 0):
        super().__init__(message)
        self.code = code


@dataclass
class Evaluation:
    """What the network says about one position, from the side to move
    (src/net/mod.rs:264-279)."""

    priors: np.ndarray  # one prior per legal move, in the leaf's move order, summing to 1
    wdl: tuple[float, float, float]

    def value(self) -> float:
        return self.wdl[0] - self.wdl[2]


# A leaf: (66-byte encoded board, legal action indices in move order), the packed form of
# the reference's `Leaf = (&EncodedBoard, &LegalActions)` (src/net/mod.rs:281-282).
Leaf = tuple


class Network(ABC):
    @abstractmethod
    def evaluate(self, batch: Sequence[Leaf]) -> list[Evaluation]:
        """One `Evaluation` per input, in order; priors cover exactly the legal moves."""

    @abstractmethod
    def describe(self) -> str:
        """Human-readable description for `info string` at load time."""


def pack(batch: Sequence[Leaf]) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Boards [n, 66] uint8, legal [n, 224] int32 (-1 padded) and move counts, as
    `CudaNetwork::forward` packs its pinned buffers (src/net/cuda/mod.rs:946-967)."""
    n = len(batch)
    boards = np.zeros((n, BOARD_BYTES), dtype=np.uint8)
    legal = np.full((n, MAX_LEGAL), -1, dtype=np.int32)
    counts = np.zeros(n, dtype=np.int32)
    for p, (board, actions) in enumerate(batch):
        boards[p] = np.frombuffer(bytes(board), dtype=np.uint8) if not isinstance(board, np.ndarray) else board
        acts = np.asarray(actions, dtype=np.int64)
        if len(acts) > MAX_LEGAL:
            raise NetworkError(f"position with {len(acts)} legal moves exceeds MAX_LEGAL {MAX_LEGAL}",
                               code=4)
        legal[p, :len(acts)] = acts
        counts[p] = len(acts)
    return boards, legal, counts


def unpack(priors: np.ndarray, wdl: np.ndarray, counts: np.ndarray) -> list[Evaluation]:
    return [Evaluation(priors[p, :counts[p]].copy(), (float(wdl[p, 0]), float(wdl[p, 1]), float(wdl[p, 2])))
            for p in range(len(counts))]


def _f32p(a: np.ndarray):
    return a.ctypes.data_as(POINTER(c_float))


def c_weights(w: Weights):
    """(mrn_weights, mrn_layer array) pointing into `w`'s arrays (keep `w` alive)."""
    L = _lib.MrnLinear
    N = _lib.MrnNorm
    lin = lambda wn, bn: L(w.ptr(wn), w.ptr(bn))  # noqa: E731
    nrm = lambda p: N(w.ptr(p + ".weight"), w.ptr(p + ".bias"))  # noqa: E731
    layers = (_lib.MrnLayer * w.arch.n_layers)()
    for i in range(w.arch.n_layers):
        p = f"encoder.layers.{i}."
        layers[i] = _lib.MrnLayer(
            nrm(p + "norm1"), lin(p + "self_attn.in_proj_weight", p + "self_attn.in_proj_bias"),
            lin(p + "self_attn.out_proj.weight", p + "self_attn.out_proj.bias"), nrm(p + "norm2"),
            lin(p + "linear1.weight", p + "linear1.bias"), lin(p + "linear2.weight", p + "linear2.bias"))
    cw = _lib.MrnWeights(
        w.ptr("piece_embed.weight"), w.ptr("square_embed.weight"), w.ptr("state_embed"),
        lin("castling_proj.weight", "castling_proj.bias"), w.ptr("en_passant_embed.weight"),
        ctypes.cast(layers, POINTER(_lib.MrnLayer)), nrm("final_norm"), nrm("policy_head.norm"),
        lin("policy_head.proj.weight", "policy_head.proj.bias"), nrm("value_head.norm"),
        lin("value_head.ff.0.weight", "value_head.ff.0.bias"), lin("value_head.ff.2.weight", "value_head.ff.2.bias"))
    return cw, layers


def c_arch(arch: Architecture):
    amax = None
    if arch.fp8_amax is not None:
        amax = np.ascontiguousarray(np.asarray(arch.fp8_amax, dtype=np.float32).reshape(-1))
    ca = _lib.MrnArch(arch.d_model, arch.n_layers, arch.n_heads, arch.d_ff, arch.layer_norm_eps, arch.gelu,
                      arch.tokens, arch.square_token_start, _f32p(amax) if amax is not None else None)
    return ca, amax


class B200Network(Network):
    """One GPU's evaluator: `CudaNetwork::new(arch, &weights, ordinal, max_batch, fp8)`
    (src/net/cuda/mod.rs:276-493) with `precision` one of "bf16", "fp8w" (e4m3 weights,
    bf16 activations), "fp8" (e4m3 weights and activations) or "fp8x2" (e4m3 weights,
    activations as two e4m3 terms each)."""

    def __init__(self, arch: Architecture, weights: Weights, device: int = 0, max_batch: int = 1024,
                 precision: str = "fp8w"):
        self._lib = _lib.load()
        if precision not in _lib.PRECISIONS:
            raise ValueError(f"precision {precision!r}: one of {sorted(_lib.PRECISIONS)}")
        self.arch, self.device, self.max_batch, self.precision = arch, device, max_batch, precision
        ca, amax = c_arch(arch)
        cw, layers = c_weights(weights)
        ctx = c_void_p()
        rc = self._lib.mrn_create(ctypes.byref(ca), ctypes.byref(cw), device, max_batch,
                                  _lib.PRECISIONS[precision], ctypes.byref(ctx))
        del amax, layers
        if rc != 0:
            raise NetworkError(f"b200 backend failed to load: {self._lib.mrn_last_error(None).decode()}", rc)
        self._ctx = ctx
        self._lock = threading.Lock()

    # -- the trait --------------------------------------------------------------------------
    def evaluate(self, batch: Sequence[Leaf]) -> list[Evaluation]:
        boards, legal, counts = pack(batch)
        priors, wdl = self.evaluate_packed(boards, legal)
        return unpack(priors, wdl, counts)

    def describe(self) -> str:
        return self._lib.mrn_describe(self._ctx).decode()

    # -- packed / raw entry points ---------------------------------------------------------
    def _check(self, rc: int, what: str):
        if rc != 0:
            raise NetworkError(f"b200 {what} failed: {self._lib.mrn_last_error(self._ctx).decode()}", rc)

    def evaluate_packed(self, boards: np.ndarray, legal: np.ndarray, priors: np.ndarray | None = None,
                        wdl: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray]:
        """`mrn_evaluate` on packed host arrays: boards [n, 66] uint8, legal [n, 224] int32.
        Returns priors [n, 224] and wdl [n, 3] (written into `priors` / `wdl` when given)."""
        boards = np.ascontiguousarray(boards, dtype=np.uint8)
        legal = np.ascontiguousarray(legal, dtype=np.int32)
        n = boards.shape[0]
        if boards.shape != (n, BOARD_BYTES) or legal.shape != (n, MAX_LEGAL):
            raise ValueError("boards must be [n, 66] and legal [n, 224]")
        if priors is None:
            priors = np.empty((n, MAX_LEGAL), dtype=np.float32)
        if wdl is None:
            wdl = np.empty((n, 3), dtype=np.float32)
        rc = self._lib.mrn_evaluate(self._ctx, n, boards.ctypes.data_as(POINTER(c_uint8)),
                                    legal.ctypes.data_as(POINTER(c_int32)), _f32p(priors), _f32p(wdl))
        self._check(rc, "forward")
        return priors, wdl

    def evaluate_packed_f16(self, boards: np.ndarray, legal: np.ndarray, priors: np.ndarray | None = None,
                            wdl: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray]:
        """`mrn_evaluate_f16`: as `evaluate_packed`, with the priors returned as float16 [n, 224]
        (half the bytes copied back from the GPU; written into `priors` / `wdl` when given)."""
        boards = np.ascontiguousarray(boards, dtype=np.uint8)
        legal = np.ascontiguousarray(legal, dtype=np.int32)
        n = boards.shape[0]
        if boards.shape != (n, BOARD_BYTES) or legal.shape != (n, MAX_LEGAL):
            raise ValueError("boards must be [n, 66] and legal [n, 224]")
        if priors is None:
            priors = np.empty((n, MAX_LEGAL), dtype=np.float16)
        if wdl is None:
            wdl = np.empty((n, 3), dtype=np.float32)
        if priors.dtype != np.float16 or priors.shape != (n, MAX_LEGAL) or not priors.flags.c_contiguous:
            raise ValueError("priors must be a C-contiguous float16 [n, 224] array")
        rc = self._lib.mrn_evaluate_f16(self._ctx, n, boards.ctypes.data_as(POINTER(c_uint8)),
                                        legal.ctypes.data_as(POINTER(c_int32)), priors.ctypes.data, _f32p(wdl))
        self._check(rc, "forward")
        return priors, wdl

    def logits(self, boards: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
        """Raw policy logits [n, 4672] and WDL logits [n, 3] (`CpuNetwork::logits`)."""
        boards = np.ascontiguousarray(boards, dtype=np.uint8)
        n = boards.shape[0]
        policy = np.empty((n, _lib.ACTIONS), dtype=np.float32)
        value = np.empty((n, 3), dtype=np.float32)
        rc = self._lib.mrn_logits(self._ctx, n, boards.ctypes.data_as(POINTER(c_uint8)), _f32p(policy), _f32p(value))
        self._check(rc, "logits")
        return policy, value

    def evaluate_device(self, n: int, boards_ptr: int, legal_ptr: int, priors_ptr: int, wdl_ptr: int,
                        stream: int | None = None) -> None:
        """Enqueue a forward pass on device-resident buffers (device pointers) on `stream`."""
        rc = self._lib.mrn_evaluate_device(self._ctx, n, c_void_p(boards_ptr), c_void_p(legal_ptr),
                                           c_void_p(priors_ptr), c_void_p(wdl_ptr), c_void_p(stream or 0))
        self._check(rc, "device forward")

    def evaluate_device_static(self, n: int, boards_ptr: int, legal_ptr: int, priors_ptr: int, wdl_ptr: int,
                               stream: int | None = None) -> None:
        """`evaluate_device` without any device allocation: the pass's intermediates live in the
        library's static 8 MiB device array, so it serves callers that must not allocate once
        running, for small batches (see `mrn_evaluate_device_static`). Calls whose GPU work
        overlaps share that array and race; serialise them."""
        rc = self._lib.mrn_evaluate_device_static(self._ctx, n, c_void_p(boards_ptr), c_void_p(legal_ptr),
                                                  c_void_p(priors_ptr), c_void_p(wdl_ptr), c_void_p(stream or 0))
        self._check(rc, "static-scratch forward")

    def status_word(self) -> int:
        word = c_int()
        self._check(self._lib.mrn_status_word(self._ctx, ctypes.byref(word)), "status")
        return word.value

    def profile(self, n: int, boards_ptr: int, legal_ptr: int, priors_ptr: int, wdl_ptr: int,
                stream: int | None = None) -> dict:
        """Per kernel class: device ms, algorithmic FLOPs and launches of one eager pass."""
        k = len(_lib.PROFILE_SLOTS)
        times = (c_float * k)()
        flops = (c_double * k)()
        launches = (c_int * k)()
        rc = self._lib.mrn_profile(self._ctx, n, c_void_p(boards_ptr), c_void_p(legal_ptr), c_void_p(priors_ptr),
                                   c_void_p(wdl_ptr), c_void_p(stream or 0), times, flops, launches)
        self._check(rc, "profile")
        return {name: {"ms": times[i], "flops": flops[i], "launches": launches[i]}
                for i, name in enumerate(_lib.PROFILE_SLOTS)}

    def launches_per_forward(self, n: int) -> int:
        return int(self._lib.mrn_launches_per_forward(self._ctx, n))

    def close(self) -> None:
        if getattr(self, "_ctx", None):
            self._lib.mrn_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class GroupNetwork(Network):
    """`Network` over one weight replica per listed device through `mrn_group_create` /
    `mrn_group_evaluate`: every batch is cut into contiguous shards (sizes differing by at most
    one position), evaluated at the same time by the library's per-device threads and written
    into the outputs in input order. A batch larger than `max_batch` runs as consecutive
    `max_batch` chunks whose shards the threads take as they become free. A failing shard raises
    `NetworkError` naming its device and positions."""

    def __init__(self, arch: Architecture, weights: Weights, devices: Sequence[int], max_batch: int = 1024,
                 precision: str = "fp8w"):
        self._lib = _lib.load()
        if precision not in _lib.PRECISIONS:
            raise ValueError(f"precision {precision!r}: one of {sorted(_lib.PRECISIONS)}")
        self.arch, self.devices, self.max_batch, self.precision = arch, list(devices), max_batch, precision
        ca, amax = c_arch(arch)
        cw, layers = c_weights(weights)
        devs = (c_int * len(self.devices))(*self.devices)
        group = c_void_p()
        rc = self._lib.mrn_group_create(ctypes.byref(ca), ctypes.byref(cw), devs, len(self.devices), max_batch,
                                        _lib.PRECISIONS[precision], ctypes.byref(group))
        del amax, layers
        if rc != 0:
            raise NetworkError(f"b200 group failed to load: {self._lib.mrn_group_last_error(None).decode()}", rc)
        self._group = group

    def evaluate(self, batch: Sequence[Leaf]) -> list[Evaluation]:
        boards, legal, counts = pack(batch)
        priors, wdl = self.evaluate_packed(boards, legal)
        return unpack(priors, wdl, counts)

    def evaluate_packed(self, boards: np.ndarray, legal: np.ndarray, priors: np.ndarray | None = None,
                        wdl: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray]:
        """`mrn_group_evaluate` on packed host arrays (see `B200Network.evaluate_packed`)."""
        boards = np.ascontiguousarray(boards, dtype=np.uint8)
        legal = np.ascontiguousarray(legal, dtype=np.int32)
        n = boards.shape[0]
        if boards.shape != (n, BOARD_BYTES) or legal.shape != (n, MAX_LEGAL):
            raise ValueError("boards must be [n, 66] and legal [n, 224]")
        if priors is None:
            priors = np.empty((n, MAX_LEGAL), dtype=np.float32)
        if wdl is None:
            wdl = np.empty((n, 3), dtype=np.float32)
        rc = self._lib.mrn_group_evaluate(self._group, n, boards.ctypes.data_as(POINTER(c_uint8)),
                                          legal.ctypes.data_as(POINTER(c_int32)), _f32p(priors), _f32p(wdl))
        if rc != 0:
            raise NetworkError(f"b200 group forward failed: {self._lib.mrn_group_last_error(self._group).decode()}",
                               rc)
        return priors, wdl

    def describe(self) -> str:
        return self._lib.mrn_group_describe(self._group).decode()

    def close(self) -> None:
        if getattr(self, "_group", None):
            self._lib.mrn_group_destroy(self._group)
            self._group = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ShardedNetwork(Network):
    """`Network` over one replica per GPU: each batch is cut into contiguous shards (one per
    replica, sizes differing by at most one), evaluated concurrently by per-GPU evaluator
    threads, and concatenated in order. The first shard error is raised as `NetworkError`."""

    def __init__(self, replicas: Sequence[Network]):
        if not replicas:
            raise ValueError("no replicas")
        self.replicas = list(replicas)
        self._pool = ThreadPoolExecutor(max_workers=len(self.replicas), thread_name_prefix="marina-b200-gpu")

    @staticmethod
    def shards(n: int, k: int) -> list[tuple[int, int]]:
        base, extra = divmod(n, k)
        out, start = [], 0
        for i in range(k):
            size = base + (1 if i < extra else 0)
            out.append((start, start + size))
            start += size
        return out

    def evaluate(self, batch: Sequence[Leaf]) -> list[Evaluation]:
        spans = [s for s in self.shards(len(batch), len(self.replicas))]
        futures = [self._pool.submit(r.evaluate, batch[a:b]) for r, (a, b) in zip(self.replicas, spans) if b > a]
        out: list[Evaluation] = []
        error = None
        for f in futures:
            try:
                out.extend(f.result())
            except Exception as e:  # noqa: BLE001 - re-raised below as the trait's error type
                error = error or e
        if error is not None:
            raise error if isinstance(error, NetworkError) else NetworkError(str(error))
        return out

    def _packed(self, method: str, prior_dtype, boards: np.ndarray, legal: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
        """Packed batches: each replica writes its shard straight into its rows of the outputs."""
        n = boards.shape[0]
        priors = np.empty((n, MAX_LEGAL), dtype=prior_dtype)
        wdl = np.empty((n, 3), dtype=np.float32)
        spans = self.shards(n, len(self.replicas))
        futures = [self._pool.submit(getattr(r, method), boards[a:b], legal[a:b], priors[a:b], wdl[a:b])
                   for r, (a, b) in zip(self.replicas, spans) if b > a]
        error = None
        for f in futures:
            try:
                f.result()
            except Exception as e:  # noqa: BLE001 - re-raised below as the trait's error type
                error = error or e
        if error is not None:
            raise error if isinstance(error, NetworkError) else NetworkError(str(error))
        return priors, wdl

    def evaluate_packed(self, boards: np.ndarray, legal: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
        return self._packed("evaluate_packed", np.float32, boards, legal)

    def evaluate_packed_f16(self, boards: np.ndarray, legal: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
        return self._packed("evaluate_packed_f16", np.float16, boards, legal)

    def describe(self) -> str:
        return f"{len(self.replicas)} replicas: " + "; ".join(r.describe() for r in self.replicas)
