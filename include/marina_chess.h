/*
 * marina_chess: host-side positions for the evaluator's inputs.
 *
 * A legal move generator for standard chess plus the reference's network encoding of a
 * position: the 66-byte board of the CUDA upload (64 canonical piece tokens, castling
 * bits, en-passant file + 1; src/encoding/board.rs:142-192, src/net/cuda/mod.rs:951-956)
 * and the 73-plane action index of every legal move (src/encoding/action.rs:47-83,
 * 138-156). It stands in for the reference's move generator (the shakmaty crate, which is
 * not part of the reference tree) so that synthetic leaf batches can be produced the way
 * the search produces them (src/search/mod.rs:1077-1083).
 */
#ifndef MARINA_CHESS_H
#define MARINA_CHESS_H

#include <stdint.h>

#if defined(__GNUC__)
#define MRC_API __attribute__((visibility("default")))
#else
#define MRC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define MRC_MAX_MOVES 256

/* Absolute squares a1 = 0 ... h8 = 63. `board` holds 0 for empty, +1..+6 for white
 * pawn, knight, bishop, rook, queen, king and -1..-6 for black. */
typedef struct mrc_position {
  int8_t board[64];
  int8_t turn;      /* 0 white to move, 1 black to move */
  uint8_t castling; /* absolute rights: 1 white O-O, 2 white O-O-O, 4 black O-O, 8 black O-O-O */
  int8_t ep;        /* en-passant target square after any double push, or -1 */
  uint8_t pad;
  uint16_t halfmove;
  uint16_t fullmove;
} mrc_position;

/* A move: from/to squares (the king's own squares for castling, e1g1), promotion 0 or the
 * piece type 2..5 (knight, bishop, rook, queen). */
typedef struct mrc_move {
  uint8_t from;
  uint8_t to;
  uint8_t promotion;
  uint8_t flags; /* 1 capture, 2 en passant, 4 castle, 8 double push */
} mrc_move;

/* 0 on success, -1 on a malformed FEN (4 or 6 fields). */
MRC_API int mrc_from_fen(const char* fen, mrc_position* out);
MRC_API void mrc_startpos(mrc_position* out);
/* Legal moves in generation order; returns the count (<= MRC_MAX_MOVES). */
MRC_API int mrc_legal_moves(const mrc_position* pos, mrc_move* moves);
MRC_API void mrc_play(mrc_position* pos, mrc_move move);
/* 1 when the side to move is in check. */
MRC_API int mrc_in_check(const mrc_position* pos);
/* Parse "e2e4" / "e7e8q" against the legal moves of `pos`; 0 on success, -1 if not legal. */
MRC_API int mrc_parse_uci(const mrc_position* pos, const char* uci, mrc_move* out);
/* Leaf nodes of the legal move tree to `depth` plies. */
MRC_API uint64_t mrc_perft(const mrc_position* pos, int depth);

/* The 66-byte network board (`EncodedBoard` pieces, castling, en_passant). */
MRC_API void mrc_encode_board(const mrc_position* pos, uint8_t* board66);
/* Action index (canonical from square * 73 + plane) of a legal move (`encode_move`,
 * src/encoding/action.rs:73-83); -1 if the move has no plane. */
MRC_API int mrc_encode_move(const mrc_position* pos, mrc_move move);
/* Action indices of every legal move in generation order into `actions` (capacity `cap`),
 * the `LegalActions` of the position; returns the number of legal moves (may exceed cap,
 * in which case only `cap` are written). */
MRC_API int mrc_legal_actions(const mrc_position* pos, int32_t* actions, int cap);
/* The legal move an action index denotes (`decode_action`, src/encoding/action.rs:85-114);
 * 0 on success, -1 if none. */
MRC_API int mrc_decode_action(const mrc_position* pos, int action, mrc_move* out);

/* `count` positions, each from a uniform-random legal playout of a uniform-random number of
 * plies in [min_ply, max_ply] from the start position; a playout that reaches a position
 * without legal moves is redrawn. Position i depends only on (seed, i), so the output does
 * not depend on `threads`. Writes count x 66 board bytes, count x 224 legal action slots
 * (-1 padded) and the legal count per position; `fens` (may be NULL) receives count x 100
 * bytes of NUL-terminated FEN. Returns 0, or -1 on bad arguments. */
MRC_API int mrc_random_positions(uint64_t seed, int count, int min_ply, int max_ply, uint8_t* boards,
                                 int32_t* legal, int32_t* legal_count, char* fens, int threads);

/* FEN of `pos` into `out` (>= 100 bytes). */
MRC_API void mrc_to_fen(const mrc_position* pos, char* out);

#ifdef __cplusplus
}
#endif

#endif /* MARINA_CHESS_H */
