"""The batched PUCT harness on the CPU with a fake network (uniform priors, value from the
board), checking the search bookkeeping the reference's tests check
(src/search/mod.rs:1560, :1631-1647): node limits are met, every virtual visit is released,
collisions are counted, and the chosen move is legal."""

import ctypes

import numpy as np
import pytest

from marina_b200 import chess, search

calls = []


@search.EVAL_FN
def uniform_net(ctx, n, boards, legal, priors, wdl):
    calls.append(n)
    lg = np.ctypeslib.as_array(legal, shape=(n, 224))
    pr = np.ctypeslib.as_array(priors, shape=(n, 224))
    wd = np.ctypeslib.as_array(wdl, shape=(n, 3))
    counts = (lg >= 0).sum(1, keepdims=True)
    pr[:] = np.where(lg >= 0, 1.0 / np.maximum(counts, 1), 0.0)
    bd = np.ctypeslib.as_array(boards, shape=(n, 66)).astype(np.float32)
    wd[:, 0] = 0.3 + 0.01 * (bd[:, :64] > 6).sum(1) / 16
    wd[:, 1] = 0.4
    wd[:, 2] = 1 - wd[:, 0] - wd[:, 1]
    return 0


def test_search_meets_node_limits_and_picks_legal_moves():
    roots = [chess.startpos(), chess.from_fen("r3k2r/p1ppqpb1/bn2pnp1/3PN3/1p2P3/2N2Q1p/PPPBBPPP/R3K2R w KQkq - 0 1"),
             chess.from_fen("8/1P2k3/8/8/8/8/4K1p1/8 w - - 0 1")]
    calls.clear()
    per_root, total = search.search(roots, 3000, [(uniform_net, None)], workers_per_evaluator=2,
                                    params=search.default_params(64))
    assert total["error"] == 0
    for root, s in zip(roots, per_root):
        assert 3000 <= s["nodes"] < 3000 + 64
        assert s["network_evals"] <= s["nodes"]
        assert s["best_action"] in chess.legal_actions(root).tolist()
        assert s["tree_nodes"] > s["network_evals"]
    assert total["nodes"] == sum(s["nodes"] for s in per_root)
    assert max(calls) <= 2 * 64  # each worker sends at most its roots' batches in one call
    assert total["collisions"] > 0


def test_mate_in_one_root_is_found_without_the_network_deciding():
    # White mates with Ra8#: a terminal child backs up -1 for Black, i.e. +1 for White.
    root = chess.from_fen("6k1/5ppp/8/8/8/8/8/R5K1 w - - 0 1")
    per_root, _ = search.search([root], 2000, [(uniform_net, None)], workers_per_evaluator=1,
                                params=search.default_params(32))
    mate = chess.encode_move(root, chess.parse_uci(root, "a1a8"))
    assert per_root[0]["best_action"] == mate


def test_terminal_root_uses_no_network_slot():
    calls.clear()
    stalemate = chess.from_fen("7k/5Q2/6K1/8/8/8/8/8 b - - 0 1")
    per_root, _ = search.search([stalemate], 100, [(uniform_net, None)], workers_per_evaluator=1,
                                params=search.default_params(16))
    assert per_root[0]["network_evals"] == 0 and per_root[0]["nodes"] >= 100 and not calls


def _summary_keys(s):
    return {k: s[k] for k in ("nodes", "network_evals", "batches", "collisions", "max_depth", "tree_nodes",
                              "best_action", "error")}


def test_one_worker_search_is_deterministic():
    """With one gathering thread and a deterministic network, two searches of the same roots
    visit the same tree (the reference checks determinism at src/search/mod.rs:1690)."""
    roots = [chess.startpos(), chess.from_fen("r1bqkbnr/pppp1ppp/2n5/4p3/4P3/5N2/PPPP1PPP/RNBQKB1R w KQkq - 2 3")]
    runs = [search.search(roots, 1500, [(uniform_net, None)], workers_per_evaluator=1,
                          params=search.default_params(32))[0] for _ in range(2)]
    assert [_summary_keys(s) for s in runs[0]] == [_summary_keys(s) for s in runs[1]]


@search.EVAL_FN
def failing_net(ctx, n, boards, legal, priors, wdl):
    return 6


def test_a_network_error_stops_the_search_and_is_reported():
    """A network call that fails ends the search with that error code, as `NetworkFailed` does
    in the reference (src/search/mod.rs:794-797); nothing is substituted for the evaluation."""
    with pytest.raises(RuntimeError, match="network error 6"):
        search.search([chess.startpos()], 1000, [(failing_net, None)], workers_per_evaluator=1,
                      params=search.default_params(16))


def test_root_visit_distribution():
    """mrs_search_visits returns every legal root move once, with the visits the search gave it:
    they add up to the root's visits (one per node but the root's own), the most visited is the
    best move, and one-thread searches repeat exactly."""
    root = chess.from_fen("r3k2r/p1ppqpb1/bn2pnp1/3PN3/1p2P3/2N2Q1p/PPPBBPPP/R3K2R w KQkq - 0 1")
    runs = [search.search([root], 1500, [(uniform_net, None)], workers_per_evaluator=1,
                          params=search.default_params(32), visits=True)[0][0] for _ in range(2)]
    a, b = runs
    assert a["root_visits"] == b["root_visits"]
    assert sorted(a["root_visits"]) == sorted(chess.legal_actions(root).tolist())
    assert sum(a["root_visits"].values()) == a["nodes"] - 1
    assert max(a["root_visits"], key=a["root_visits"].get) == a["best_action"] or \
        a["root_visits"][a["best_action"]] == max(a["root_visits"].values())
