"""The batched PUCT harness driving the B200 evaluator through the C ABI (`mrn_evaluate` as the
search's network function): node limits, legal best moves, and per-root determinism."""

import ctypes

import pytest

from marina_b200 import _lib, chess, model, search, weights
from marina_b200.network import B200Network

pytestmark = pytest.mark.gpu


def test_search_on_the_gpu_is_deterministic_per_root():
    arch = model.nano()
    w = weights.random_init(arch, seed=0)
    nets = [B200Network(arch, w, max_batch=512, precision="bf16") for _ in range(2)]
    fn = ctypes.cast(_lib.load().mrn_evaluate, ctypes.c_void_p).value
    evaluators = [(fn, n._ctx.value) for n in nets]
    _, _, _, fens = chess.random_positions(5, 6, 0, 80, fens=True)
    roots = [chess.from_fen(f) for f in fens]
    a, ta = search.search(roots, 3000, evaluators, 2, search.default_params(64))
    b, tb = search.search(roots, 3000, evaluators, 2, search.default_params(64))
    assert ta["error"] == 0 and ta["nodes"] >= 6 * 3000
    for root, x, y in zip(roots, a, b):
        assert x["best_action"] in chess.legal_actions(root).tolist()
        for key in ("nodes", "network_evals", "collisions", "tree_nodes", "best_action"):
            assert x[key] == y[key], (key, x, y)
