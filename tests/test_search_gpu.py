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


def _oracle_evaluator(arch, w):
    """The oracle (the C restatement of the reference's CPU backend) as a search network."""
    import numpy as np

    import oracle

    net = oracle.OracleNetwork(arch, w, threads=8)

    @search.EVAL_FN
    def evaluate(ctx, n, boards, legal, priors, wdl):
        b = np.ctypeslib.as_array(boards, shape=(n, 66)).copy()
        lg = np.ctypeslib.as_array(legal, shape=(n, 224)).copy()
        p, v = net.evaluate(b, lg)
        np.ctypeslib.as_array(priors, shape=(n, 224))[:] = p
        np.ctypeslib.as_array(wdl, shape=(n, 3))[:] = v
        return 0

    return evaluate


def test_search_with_the_gpu_evaluator_matches_the_oracle_evaluator():
    """The same roots searched (one gathering thread, so each search is deterministic) once with the
    B200 evaluator and once with the oracle: the root visit distributions -- what the reference's
    search picks its move from (src/search/mod.rs:1131-1155) -- agree, and so do the chosen moves
    wherever the oracle search's choice is clear."""
    import numpy as np

    arch = model.nano()
    w = weights.random_init(arch, seed=0)
    _, _, _, fens = chess.random_positions(11, 6, 0, 80, fens=True)
    roots = [chess.from_fen(f) for f in fens]
    params = search.default_params(32)
    gpu = B200Network(arch, w, max_batch=256, precision="bf16")
    fn = ctypes.cast(_lib.load().mrn_evaluate, ctypes.c_void_p).value
    ours, _ = search.search(roots, 800, [(fn, gpu._ctx.value)], 1, params, visits=True)
    ref, _ = search.search(roots, 800, [(_oracle_evaluator(arch, w), None)], 1, params, visits=True)
    clear = 0
    for root, a, b in zip(roots, ours, ref):
        assert set(a["root_visits"]) == set(b["root_visits"]) == set(chess.legal_actions(root).tolist())
        acts = sorted(b["root_visits"])
        va = np.array([a["root_visits"][x] for x in acts], dtype=np.float64)
        vb = np.array([b["root_visits"][x] for x in acts], dtype=np.float64)
        tv = 0.5 * np.abs(va / va.sum() - vb / vb.sum()).sum()
        print(root, "total variation", round(tv, 4), "best", a["best_action"], b["best_action"])
        assert tv <= 0.02, tv
        top2 = np.sort(vb)[-2:]
        if len(vb) > 1 and top2[1] >= 1.2 * top2[0]:
            clear += 1
            assert a["best_action"] == b["best_action"]
    assert clear >= 1
    gpu.close()
