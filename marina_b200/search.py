"""Batched PUCT search over the evaluator (ctypes binding of ``mrs_search``,
``include/marina_search.h``): the nodes/s measurement of the reference's search loop
(src/search/mod.rs:667-835), with each GPU's evaluator driven by worker threads in C++."""

from __future__ import annotations

import ctypes
from ctypes import POINTER, Structure, c_double, c_float, c_int, c_int32, c_uint64, c_void_p

from . import chess

EVAL_FN = ctypes.CFUNCTYPE(c_int, c_void_p, c_int, POINTER(ctypes.c_uint8), POINTER(c_int32), POINTER(c_float),
                           POINTER(c_float))


class Params(Structure):
    _fields_ = [("cpuct", c_float), ("fpu_reduction", c_float), ("batch", c_int32), ("batch_ramp", c_int32),
                ("collision_budget_pct", c_int32)]


class Summary(Structure):
    _fields_ = [("nodes", c_uint64), ("network_evals", c_uint64), ("batches", c_uint64), ("collisions", c_uint64),
                ("max_depth", c_uint64), ("tree_nodes", c_uint64), ("seconds", c_double), ("best_action", c_int32),
                ("error", c_int32)]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


def default_params(batch: int = 256) -> Params:
    """cpuct 1.75 and FPU reduction 0.25 (the reference's defaults for a network directory,
    src/options.rs:303-307), batch ramp 4 and a 100% collision budget (:292-296)."""
    return Params(1.75, 0.25, batch, 4, 100)


def search(roots: list, node_limit: int, evaluators: list, workers_per_evaluator: int = 2,
           params: Params | None = None, visits: bool = False):
    """Search every root position to `node_limit` nodes. `evaluators` is a list of
    (function pointer, context) pairs: the C function `mrn_evaluate` with an `mrn_ctx` per
    GPU, or an `EVAL_FN` callback with any context. Returns (per-root summaries, total); with
    `visits`, each per-root summary also holds "root_visits": {action index: visits} over the
    root's children (`mrs_search_visits`)."""
    lib = chess.load()
    if not hasattr(lib, "_mrs_ready"):
        lib.mrs_search.argtypes = [POINTER(chess.Position), c_int, c_uint64, POINTER(Params), c_void_p,
                                   POINTER(c_void_p), c_int, c_int, POINTER(Summary), POINTER(Summary)]
        lib.mrs_search.restype = c_int
        lib.mrs_search_visits.argtypes = lib.mrs_search.argtypes + [POINTER(c_int32), POINTER(ctypes.c_uint32)]
        lib.mrs_search_visits.restype = c_int
        lib._mrs_ready = True
    params = params or default_params()
    n = len(roots)
    arr = (chess.Position * n)(*roots)
    fns = {ctypes.cast(f, c_void_p).value for f, _ in evaluators}
    if len(fns) != 1:
        raise ValueError("all evaluators must share one function")
    ctxs = (c_void_p * len(evaluators))(*[c for _, c in evaluators])
    per_root = (Summary * n)()
    total = Summary()
    if visits:
        acts = (c_int32 * (n * 224))()
        vis = (ctypes.c_uint32 * (n * 224))()
        rc = lib.mrs_search_visits(arr, n, node_limit, ctypes.byref(params), c_void_p(fns.pop()), ctxs,
                                   len(evaluators), workers_per_evaluator, per_root, ctypes.byref(total), acts, vis)
    else:
        rc = lib.mrs_search(arr, n, node_limit, ctypes.byref(params), c_void_p(fns.pop()), ctxs, len(evaluators),
                            workers_per_evaluator, per_root, ctypes.byref(total))
    if rc != 0:
        raise RuntimeError(f"search failed (network error {rc})")
    out = [s.as_dict() for s in per_root]
    if visits:
        for i, d in enumerate(out):
            d["root_visits"] = {int(acts[i * 224 + k]): int(vis[i * 224 + k]) for k in range(224)
                                if acts[i * 224 + k] >= 0}
    return out, total.as_dict()
