"""The position library against the reference's encoding known-answer tests
(src/encoding/action.rs:194-251, src/encoding/board.rs:208-281) and standard perft counts."""

import numpy as np
import pytest

from marina_b200 import chess


def test_perft_startpos():
    p = chess.startpos()
    assert [chess.perft(p, d) for d in (1, 2, 3, 4)] == [20, 400, 8902, 197281]


@pytest.mark.parametrize("fen,counts", [
    ("r3k2r/p1ppqpb1/bn2pnp1/3PN3/1p2P3/2N2Q1p/PPPBBPPP/R3K2R w KQkq - 0 1", [48, 2039, 97862]),
    ("8/2p5/3p4/KP5r/1R3p1k/8/4P1P1/8 w - - 0 1", [14, 191, 2812, 43238]),
    ("r3k2r/Pppp1ppp/1b3nbN/nP6/BBP1P3/q4N2/Pp1P2PP/R2Q1RK1 w kq - 0 1", [6, 264, 9467]),
    ("rnbq1k1r/pp1Pbppp/2p5/8/2B5/8/PPP1NnPP/RNBQK2R w KQ - 1 8", [44, 1486, 62379]),
])
def test_perft_positions(fen, counts):
    p = chess.from_fen(fen)
    assert [chess.perft(p, d + 1) for d in range(len(counts))] == counts


def _action(pos, uci):
    return chess.encode_move(pos, chess.parse_uci(pos, uci))


def test_hand_checked_actions():
    """src/encoding/action.rs:194-212."""
    start = chess.startpos()
    assert _action(start, "e2e4") == 12 * 73 + 1
    assert _action(start, "g1f3") == 6 * 73 + 63
    black = chess.play_uci(start, "e2e4")
    assert _action(black, "e7e5") == 11 * 73 + 1
    castle = chess.from_fen("r3k2r/8/8/8/8/8/8/R3K2R w KQkq - 0 1")
    assert _action(castle, "e1g1") == 4 * 73 + 15
    promo = chess.from_fen("8/1P2k3/8/8/8/8/4K1p1/8 w - - 0 1")
    assert _action(promo, "b7b8q") == 49 * 73
    assert _action(promo, "b7b8n") == 49 * 73 + 64 + 3
    assert _action(promo, "b7b8r") == 49 * 73 + 64 + 5


ROUND_TRIP_FENS = [
    chess.STARTPOS,
    "r3k2r/pppq1ppp/2npbn2/4p3/4P3/2NPBN2/PPPQ1PPP/R3K2R w KQkq - 4 9",
    "r3k2r/pppq1ppp/2npbn2/4p3/4P3/2NPBN2/PPPQ1PPP/R4RK1 b kq - 5 9",
    "rnbqkbnr/ppp2ppp/8/3pP3/8/8/PPPP1PPP/RNBQKBNR w KQkq d6 0 3",
    "8/1P2k3/8/8/8/8/4K1p1/8 w - - 0 1",
    "8/1P2k3/8/8/8/8/4K1p1/8 b - - 0 1",
    "7k/8/5K1R/8/8/8/8/8 b - - 0 1",
]


@pytest.mark.parametrize("fen", ROUND_TRIP_FENS)
def test_every_legal_move_round_trips(fen):
    """src/encoding/action.rs:214-241: distinct actions that decode to their moves."""
    p = chess.from_fen(fen)
    moves = chess.legal_moves(p)
    actions = chess.legal_actions(p)
    assert len(actions) == len(moves)
    assert len(set(actions.tolist())) == len(actions)
    for m, a in zip(moves, actions):
        assert 0 <= a < 64 * 73
        assert chess.decode_action(p, int(a)) == m


def test_decode_rejects_off_board_and_illegal():
    """src/encoding/action.rs:243-251."""
    p = chess.startpos()
    assert chess.decode_action(p, 64 * 73) is None
    assert chess.decode_action(p, 7 * 7) is None
    assert chess.decode_action(p, 12 * 73 + 2) is None


def test_startpos_tokens_from_both_sides():
    """src/encoding/board.rs:222-250."""
    white = chess.encode_board(chess.startpos())
    assert white[0:8].tolist() == [4, 2, 3, 5, 6, 3, 2, 4]
    assert white[8:16].tolist() == [1] * 8
    assert white[48:56].tolist() == [7] * 8
    assert white[56:64].tolist() == [10, 8, 9, 11, 12, 9, 8, 10]
    assert white[64] == 0b1111 and white[65] == 0
    black = chess.encode_board(chess.play_uci(chess.startpos(), "e2e4"))
    assert black[0:8].tolist() == [4, 2, 3, 6, 5, 3, 2, 4]
    e4 = 4 + 3 * 8
    assert black[63 - e4] == 7 and 63 - e4 == 3 + 4 * 8  # e4 appears on d5 as an opponent pawn
    assert black[65] == 3 + 1  # file D + 1


def test_en_passant_is_set_after_any_double_push():
    """src/encoding/board.rs:252-263."""
    g = chess.play_uci(chess.startpos(), "e2e4 e7e5")
    assert chess.encode_board(g)[65] == 4 + 1
    g = chess.from_fen("rnbqkbnr/pppp1ppp/8/4p3/4P3/8/PPPP1PPP/RNBQKBNR w KQkq - 0 2")
    assert chess.encode_board(g)[65] == 0


def test_castling_bits_are_relative_to_the_mover():
    """src/encoding/board.rs:265-270: own queenside | opp kingside."""
    g = chess.from_fen("r3k2r/8/8/8/8/8/8/R3K2R b Kq - 0 1")
    assert chess.encode_board(g)[64] == 2 | 4


def test_fen_round_trip_and_play():
    p = chess.play_uci(chess.startpos(), "e2e4 c7c5 g1f3")
    assert chess.to_fen(p) == "rnbqkbnr/pp1ppppp/8/2p5/4P3/5N2/PPPP1PPP/RNBQKB1R b KQkq - 1 2"
    with pytest.raises(ValueError):
        chess.from_fen("not a fen")
    with pytest.raises(ValueError):
        chess.parse_uci(chess.startpos(), "e2e5")


def test_position_with_218_moves_fits_max_legal():
    p = chess.from_fen("R6R/3Q4/1Q4Q1/4Q3/2Q4Q/Q4Q2/pp1Q4/kBNN1KB1 w - - 0 1")
    assert len(chess.legal_actions(p)) == 218


def test_random_positions_are_deterministic_and_legal():
    b1, l1, c1, fens = chess.random_positions(1, 200, 0, 80, threads=4, fens=True)
    b2, l2, c2, _ = chess.random_positions(1, 200, 0, 80, threads=1)
    assert (b1 == b2).all() and (l1 == l2).all() and (c1 == c2).all()
    assert (c1 > 0).all()
    for i in range(0, 200, 17):
        p = chess.from_fen(fens[i])
        assert (chess.encode_board(p) == b1[i]).all()
        assert chess.legal_actions(p).tolist() == l1[i, :c1[i]].tolist()
        assert (l1[i, c1[i]:] == -1).all()
    b3, *_ = chess.random_positions(2, 200)
    assert not (b3 == b1).all()
