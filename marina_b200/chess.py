"""Positions for the evaluator's inputs: ctypes binding of ``libmarina_chess.so``
(``include/marina_chess.h``).

Mirrors what the reference's search hands its network: the 66-byte ``EncodedBoard``
packing (src/encoding/board.rs:142-192, src/net/cuda/mod.rs:951-956) and the 73-plane
action index of each legal move (src/encoding/action.rs:47-83, 138-156), plus seeded
random-playout positions for synthetic leaf batches.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_int, c_int8, c_int32, c_uint8, c_uint16, c_uint64
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "libmarina_chess.so"
MAX_LEGAL = 224
STARTPOS = "rnbqkbnr/pppppppp/8/8/8/8/PPPPPPPP/RNBQKBNR w KQkq - 0 1"


class Position(ctypes.Structure):
    _fields_ = [("board", c_int8 * 64), ("turn", c_int8), ("castling", c_uint8), ("ep", c_int8),
                ("pad", c_uint8), ("halfmove", c_uint16), ("fullmove", c_uint16)]

    def copy(self) -> "Position":
        p = Position()
        ctypes.pointer(p)[0] = self
        return p


class Move(ctypes.Structure):
    _fields_ = [("from_", c_uint8), ("to", c_uint8), ("promotion", c_uint8), ("flags", c_uint8)]

    def uci(self) -> str:
        sq = lambda s: "abcdefgh"[s % 8] + str(s // 8 + 1)  # noqa: E731
        promo = {0: "", 2: "n", 3: "b", 4: "r", 5: "q"}[self.promotion]
        return sq(self.from_) + sq(self.to) + promo

    def __eq__(self, other):
        return isinstance(other, Move) and (self.from_, self.to, self.promotion) == (other.from_, other.to, other.promotion)

    def __repr__(self):
        return f"Move({self.uci()})"


_lib = None


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is not built; run `python -m marina_b200.build`")
    lib = ctypes.CDLL(str(LIB_PATH))
    P = POINTER(Position)
    lib.mrc_from_fen.argtypes = [c_char_p, P]
    lib.mrc_startpos.argtypes = [P]
    lib.mrc_legal_moves.argtypes = [P, POINTER(Move)]
    lib.mrc_play.argtypes = [P, Move]
    lib.mrc_play.restype = None
    lib.mrc_in_check.argtypes = [P]
    lib.mrc_parse_uci.argtypes = [P, c_char_p, POINTER(Move)]
    lib.mrc_perft.argtypes = [P, c_int]
    lib.mrc_perft.restype = c_uint64
    lib.mrc_encode_board.argtypes = [P, POINTER(c_uint8)]
    lib.mrc_encode_board.restype = None
    lib.mrc_encode_move.argtypes = [P, Move]
    lib.mrc_legal_actions.argtypes = [P, POINTER(c_int32), c_int]
    lib.mrc_decode_action.argtypes = [P, c_int, POINTER(Move)]
    lib.mrc_random_positions.argtypes = [c_uint64, c_int, c_int, c_int, POINTER(c_uint8), POINTER(c_int32),
                                         POINTER(c_int32), c_char_p, c_int]
    lib.mrc_to_fen.argtypes = [P, c_char_p]
    lib.mrc_to_fen.restype = None
    _lib = lib
    return lib


def from_fen(fen: str) -> Position:
    p = Position()
    if load().mrc_from_fen(fen.encode(), ctypes.byref(p)) != 0:
        raise ValueError(f"malformed FEN: {fen!r}")
    return p


def startpos() -> Position:
    return from_fen(STARTPOS)


def to_fen(pos: Position) -> str:
    buf = ctypes.create_string_buffer(128)
    load().mrc_to_fen(ctypes.byref(pos), buf)
    return buf.value.decode()


def legal_moves(pos: Position) -> list[Move]:
    moves = (Move * 256)()
    n = load().mrc_legal_moves(ctypes.byref(pos), moves)
    return [Move(m.from_, m.to, m.promotion, m.flags) for m in moves[:n]]


def play(pos: Position, move: Move) -> Position:
    q = pos.copy()
    load().mrc_play(ctypes.byref(q), move)
    return q


def parse_uci(pos: Position, uci: str) -> Move:
    m = Move()
    if load().mrc_parse_uci(ctypes.byref(pos), uci.encode(), ctypes.byref(m)) != 0:
        raise ValueError(f"{uci} is not legal in {to_fen(pos)}")
    return m


def play_uci(pos: Position, moves: str) -> Position:
    for uci in moves.split():
        pos = play(pos, parse_uci(pos, uci))
    return pos


def in_check(pos: Position) -> bool:
    return bool(load().mrc_in_check(ctypes.byref(pos)))


def perft(pos: Position, depth: int) -> int:
    return int(load().mrc_perft(ctypes.byref(pos), depth))


def encode_board(pos: Position) -> np.ndarray:
    """The 66-byte network board: 64 canonical piece tokens, castling bits, en passant."""
    out = np.zeros(66, dtype=np.uint8)
    load().mrc_encode_board(ctypes.byref(pos), out.ctypes.data_as(POINTER(c_uint8)))
    return out


def encode_move(pos: Position, move: Move) -> int:
    return int(load().mrc_encode_move(ctypes.byref(pos), move))


def legal_actions(pos: Position) -> np.ndarray:
    """Action index of every legal move, in generation order (`LegalActions`)."""
    buf = np.full(256, -1, dtype=np.int32)
    n = load().mrc_legal_actions(ctypes.byref(pos), buf.ctypes.data_as(POINTER(c_int32)), 256)
    return buf[:n].copy()


def decode_action(pos: Position, action: int) -> Move | None:
    m = Move()
    if load().mrc_decode_action(ctypes.byref(pos), int(action), ctypes.byref(m)) != 0:
        return None
    return m


def random_positions(seed: int, count: int, min_ply: int = 0, max_ply: int = 80, threads: int | None = None,
                     fens: bool = False):
    """`count` seeded random-playout positions (uniform ply count in [min_ply, max_ply],
    uniform legal moves, positions without legal moves redrawn). Returns ``(boards [n, 66]
    uint8, legal [n, 224] int32 padded with -1, legal_count [n] int32, fens or None)``."""
    boards = np.zeros((count, 66), dtype=np.uint8)
    legal = np.full((count, MAX_LEGAL), -1, dtype=np.int32)
    counts = np.zeros(count, dtype=np.int32)
    fen_buf = ctypes.create_string_buffer(100 * count) if fens else None
    rc = load().mrc_random_positions(seed, count, min_ply, max_ply, boards.ctypes.data_as(POINTER(c_uint8)),
                                     legal.ctypes.data_as(POINTER(c_int32)), counts.ctypes.data_as(POINTER(c_int32)),
                                     fen_buf, threads or os.cpu_count() or 1)
    if rc != 0:
        raise ValueError("bad arguments to random_positions")
    fen_list = None
    if fens:
        raw = fen_buf.raw
        fen_list = [raw[i * 100:(i + 1) * 100].split(b"\0", 1)[0].decode() for i in range(count)]
    return boards, legal, counts, fen_list
