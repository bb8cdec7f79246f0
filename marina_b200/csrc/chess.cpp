// Legal move generation (copy-make with a king-safety test), the reference network's
// position encoding, and seeded random playouts. See include/marina_chess.h.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "marina_chess.h"

namespace {

enum : int { P = 1, N = 2, B = 3, R = 4, Q = 5, K = 6 };

inline int file_of(int s) { return s & 7; }
inline int rank_of(int s) { return s >> 3; }
inline bool on_board(int f, int r) { return f >= 0 && f < 8 && r >= 0 && r < 8; }
inline int sq(int f, int r) { return r * 8 + f; }

const int kKnight[8][2] = {{1, 2}, {2, 1}, {2, -1}, {1, -2}, {-1, -2}, {-2, -1}, {-2, 1}, {-1, 2}};
const int kKing[8][2] = {{0, 1}, {1, 1}, {1, 0}, {1, -1}, {0, -1}, {-1, -1}, {-1, 0}, {-1, 1}};
const int kRook[4][2] = {{0, 1}, {1, 0}, {0, -1}, {-1, 0}};
const int kBishop[4][2] = {{1, 1}, {1, -1}, {-1, -1}, {-1, 1}};

// Is square `s` attacked by a piece of colour `by` (0 white, 1 black)?
bool attacked(const mrc_position& p, int s, int by) {
  const int sign = by == 0 ? 1 : -1;
  const int f = file_of(s), r = rank_of(s);
  // Pawns: a white pawn on (f', r') attacks (f'±1, r'+1).
  const int pr = r - sign;
  for (int df : {-1, 1})
    if (on_board(f + df, pr) && p.board[sq(f + df, pr)] == sign * P) return true;
  for (auto& d : kKnight)
    if (on_board(f + d[0], r + d[1]) && p.board[sq(f + d[0], r + d[1])] == sign * N) return true;
  for (auto& d : kKing)
    if (on_board(f + d[0], r + d[1]) && p.board[sq(f + d[0], r + d[1])] == sign * K) return true;
  for (auto& d : kRook) {
    int ff = f + d[0], rr = r + d[1];
    while (on_board(ff, rr)) {
      const int pc = p.board[sq(ff, rr)];
      if (pc != 0) {
        if (pc == sign * R || pc == sign * Q) return true;
        break;
      }
      ff += d[0];
      rr += d[1];
    }
  }
  for (auto& d : kBishop) {
    int ff = f + d[0], rr = r + d[1];
    while (on_board(ff, rr)) {
      const int pc = p.board[sq(ff, rr)];
      if (pc != 0) {
        if (pc == sign * B || pc == sign * Q) return true;
        break;
      }
      ff += d[0];
      rr += d[1];
    }
  }
  return false;
}

int king_square(const mrc_position& p, int color) {
  const int k = color == 0 ? K : -K;
  for (int s = 0; s < 64; ++s)
    if (p.board[s] == k) return s;
  return -1;
}

void apply(mrc_position& p, const mrc_move& m) {
  const int us = p.turn;
  const int sign = us == 0 ? 1 : -1;
  const int piece = p.board[m.from];
  const int type = piece * sign;
  const bool capture = p.board[m.to] != 0 || (m.flags & 2);
  p.board[m.to] = m.promotion ? static_cast<int8_t>(sign * m.promotion) : static_cast<int8_t>(piece);
  p.board[m.from] = 0;
  if (m.flags & 2) p.board[m.to - 8 * sign] = 0;  // the pawn taken en passant
  if (m.flags & 4) {
    // The rook jumps over the king: h-file rook to f, a-file rook to d.
    const int r = rank_of(m.from);
    if (file_of(m.to) == 6) {
      p.board[sq(5, r)] = p.board[sq(7, r)];
      p.board[sq(7, r)] = 0;
    } else {
      p.board[sq(3, r)] = p.board[sq(0, r)];
      p.board[sq(0, r)] = 0;
    }
  }
  // Castling rights: lost when the king moves, or a rook leaves or is taken on its corner.
  if (type == K) p.castling &= us == 0 ? ~3u : ~12u;
  for (int s : {static_cast<int>(m.from), static_cast<int>(m.to)}) {
    if (s == 7) p.castling &= ~1u;
    if (s == 0) p.castling &= ~2u;
    if (s == 63) p.castling &= ~4u;
    if (s == 56) p.castling &= ~8u;
  }
  p.ep = (m.flags & 8) ? static_cast<int8_t>(m.from + 8 * sign) : static_cast<int8_t>(-1);
  p.halfmove = (type == P || capture) ? 0 : static_cast<uint16_t>(p.halfmove + 1);
  if (us == 1) p.fullmove++;
  p.turn = static_cast<int8_t>(1 - us);
}

int pseudo_moves(const mrc_position& p, mrc_move* out) {
  int n = 0;
  const int us = p.turn, them = 1 - us;
  const int sign = us == 0 ? 1 : -1;
  auto push = [&](int from, int to, int promo, int flags) {
    out[n++] = mrc_move{static_cast<uint8_t>(from), static_cast<uint8_t>(to), static_cast<uint8_t>(promo),
                        static_cast<uint8_t>(flags)};
  };
  auto enemy = [&](int pc) { return pc * sign < 0; };
  for (int s = 0; s < 64; ++s) {
    const int pc = p.board[s];
    if (pc * sign <= 0) continue;
    const int type = pc * sign;
    const int f = file_of(s), r = rank_of(s);
    if (type == P) {
      const int r1 = r + sign;
      const int promo_rank = us == 0 ? 7 : 0;
      const int start_rank = us == 0 ? 1 : 6;
      auto pawn_to = [&](int to, int flags) {
        if (rank_of(to) == promo_rank) {
          for (int pr : {Q, R, B, N}) push(s, to, pr, flags);
        } else {
          push(s, to, 0, flags);
        }
      };
      if (on_board(f, r1) && p.board[sq(f, r1)] == 0) {
        pawn_to(sq(f, r1), 0);
        const int r2 = r + 2 * sign;
        if (r == start_rank && p.board[sq(f, r2)] == 0) push(s, sq(f, r2), 0, 8);
      }
      for (int df : {-1, 1}) {
        if (!on_board(f + df, r1)) continue;
        const int to = sq(f + df, r1);
        if (enemy(p.board[to]))
          pawn_to(to, 1);
        else if (to == p.ep && p.board[to] == 0 && p.board[to - 8 * sign] == -sign * P)
          push(s, to, 0, 1 | 2);
      }
    } else if (type == N || type == K) {
      for (auto& d : (type == N ? kKnight : kKing)) {
        const int ff = f + d[0], rr = r + d[1];
        if (!on_board(ff, rr)) continue;
        const int to = sq(ff, rr);
        if (p.board[to] == 0)
          push(s, to, 0, 0);
        else if (enemy(p.board[to]))
          push(s, to, 0, 1);
      }
      if (type == K) {
        const int home = us == 0 ? 4 : 60;
        const int rook = sign * R;
        const unsigned ks = us == 0 ? 1u : 4u, qs = us == 0 ? 2u : 8u;
        if (s == home && !attacked(p, home, them)) {
          if ((p.castling & ks) && p.board[home + 3] == rook && p.board[home + 1] == 0 && p.board[home + 2] == 0 &&
              !attacked(p, home + 1, them) && !attacked(p, home + 2, them))
            push(s, home + 2, 0, 4);
          if ((p.castling & qs) && p.board[home - 4] == rook && p.board[home - 1] == 0 && p.board[home - 2] == 0 &&
              p.board[home - 3] == 0 && !attacked(p, home - 1, them) && !attacked(p, home - 2, them))
            push(s, home - 2, 0, 4);
        }
      }
    } else {
      const bool diag = type == B || type == Q;
      const bool orth = type == R || type == Q;
      for (int dir = 0; dir < 8; ++dir) {
        const int* d = dir < 4 ? kRook[dir] : kBishop[dir - 4];
        if ((dir < 4 && !orth) || (dir >= 4 && !diag)) continue;
        int ff = f + d[0], rr = r + d[1];
        while (on_board(ff, rr)) {
          const int to = sq(ff, rr);
          if (p.board[to] == 0) {
            push(s, to, 0, 0);
          } else {
            if (enemy(p.board[to])) push(s, to, 0, 1);
            break;
          }
          ff += d[0];
          rr += d[1];
        }
      }
    }
  }
  return n;
}

// ---- encoding (src/encoding/board.rs, src/encoding/action.rs) -------------------------
inline int canonical(int s, int turn) { return turn == 0 ? s : 63 - s; }

// Plane of a canonical displacement; -1 when there is none.
int plane_of(int dfile, int drank, int promotion) {
  static const int kQueenDirs[8][2] = {{0, 1}, {1, 1}, {1, 0}, {1, -1}, {0, -1}, {-1, -1}, {-1, 0}, {-1, 1}};
  if (promotion == N || promotion == B || promotion == R) {
    if (drank != 1 || dfile < -1 || dfile > 1) return -1;
    const int piece = promotion == N ? 0 : promotion == B ? 1 : 2;
    return 64 + (dfile + 1) * 3 + piece;
  }
  for (int i = 0; i < 8; ++i)
    if (kKnight[i][0] == dfile && kKnight[i][1] == drank) return 56 + i;
  const int adf = dfile < 0 ? -dfile : dfile, adr = drank < 0 ? -drank : drank;
  const int dist = adf > adr ? adf : adr;
  if (dist == 0 || !(dfile == 0 || drank == 0 || adf == adr)) return -1;
  const int ux = dfile / dist, uy = drank / dist;
  for (int i = 0; i < 8; ++i)
    if (kQueenDirs[i][0] == ux && kQueenDirs[i][1] == uy) return i * 7 + (dist - 1);
  return -1;
}

uint64_t splitmix64(uint64_t& x) {
  uint64_t z = (x += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Uniform integer in [0, n) from the stream (n small; rejection keeps it unbiased).
uint32_t uniform(uint64_t& state, uint32_t n) {
  const uint64_t limit = UINT64_MAX - UINT64_MAX % n;
  uint64_t v;
  do v = splitmix64(state);
  while (v >= limit);
  return static_cast<uint32_t>(v % n);
}

}  // namespace

extern "C" {

MRC_API void mrc_startpos(mrc_position* out) {
  mrc_from_fen("rnbqkbnr/pppppppp/8/8/8/8/PPPPPPPP/RNBQKBNR w KQkq - 0 1", out);
}

MRC_API int mrc_from_fen(const char* fen, mrc_position* out) {
  mrc_position p;
  memset(&p, 0, sizeof(p));
  p.ep = -1;
  p.fullmove = 1;
  const char* c = fen;
  int r = 7, f = 0;
  for (; *c && *c != ' '; ++c) {
    if (*c == '/') {
      if (f != 8) return -1;
      --r;
      f = 0;
      continue;
    }
    if (*c >= '1' && *c <= '8') {
      f += *c - '0';
      if (f > 8) return -1;
      continue;
    }
    const char* kinds = "pnbrqk";
    const char lower = static_cast<char>(*c | 0x20);
    const char* k = strchr(kinds, lower);
    if (!k || f > 7 || r < 0) return -1;
    const int type = static_cast<int>(k - kinds) + 1;
    p.board[sq(f, r)] = static_cast<int8_t>((*c == lower) ? -type : type);
    ++f;
  }
  if (r != 0 || f != 8 || *c != ' ') return -1;
  ++c;
  if (*c == 'w')
    p.turn = 0;
  else if (*c == 'b')
    p.turn = 1;
  else
    return -1;
  ++c;
  if (*c != ' ') return -1;
  ++c;
  for (; *c && *c != ' '; ++c) {
    switch (*c) {
      case 'K': p.castling |= 1; break;
      case 'Q': p.castling |= 2; break;
      case 'k': p.castling |= 4; break;
      case 'q': p.castling |= 8; break;
      case '-': break;
      default: return -1;
    }
  }
  if (*c != ' ') return -1;
  ++c;
  if (*c == '-') {
    ++c;
  } else if (*c >= 'a' && *c <= 'h' && (c[1] == '3' || c[1] == '6')) {
    p.ep = static_cast<int8_t>(sq(*c - 'a', c[1] - '1'));
    c += 2;
  } else {
    return -1;
  }
  if (*c == ' ') {
    int half = 0, full = 1;
    if (sscanf(c, " %d %d", &half, &full) != 2) return -1;
    p.halfmove = static_cast<uint16_t>(half);
    p.fullmove = static_cast<uint16_t>(full);
  } else if (*c != 0) {
    return -1;
  }
  *out = p;
  return 0;
}

MRC_API void mrc_to_fen(const mrc_position* p, char* out) {
  char* o = out;
  for (int r = 7; r >= 0; --r) {
    int empty = 0;
    for (int f = 0; f < 8; ++f) {
      const int pc = p->board[sq(f, r)];
      if (pc == 0) {
        ++empty;
        continue;
      }
      if (empty) *o++ = static_cast<char>('0' + empty);
      empty = 0;
      const char ch = " pnbrqk"[pc < 0 ? -pc : pc];
      *o++ = pc > 0 ? static_cast<char>(ch - 32) : ch;
    }
    if (empty) *o++ = static_cast<char>('0' + empty);
    if (r) *o++ = '/';
  }
  *o++ = ' ';
  *o++ = p->turn == 0 ? 'w' : 'b';
  *o++ = ' ';
  if (!p->castling) *o++ = '-';
  if (p->castling & 1) *o++ = 'K';
  if (p->castling & 2) *o++ = 'Q';
  if (p->castling & 4) *o++ = 'k';
  if (p->castling & 8) *o++ = 'q';
  *o++ = ' ';
  if (p->ep < 0) {
    *o++ = '-';
  } else {
    *o++ = static_cast<char>('a' + file_of(p->ep));
    *o++ = static_cast<char>('1' + rank_of(p->ep));
  }
  snprintf(o, 20, " %u %u", p->halfmove, p->fullmove);
}

MRC_API int mrc_in_check(const mrc_position* p) {
  const int k = king_square(*p, p->turn);
  return k >= 0 && attacked(*p, k, 1 - p->turn) ? 1 : 0;
}

MRC_API int mrc_legal_moves(const mrc_position* p, mrc_move* moves) {
  mrc_move pseudo[MRC_MAX_MOVES];
  const int n = pseudo_moves(*p, pseudo);
  int legal = 0;
  for (int i = 0; i < n; ++i) {
    mrc_position q = *p;
    apply(q, pseudo[i]);
    const int k = king_square(q, p->turn);
    if (k >= 0 && !attacked(q, k, q.turn)) moves[legal++] = pseudo[i];
  }
  return legal;
}

MRC_API void mrc_play(mrc_position* p, mrc_move m) { apply(*p, m); }

MRC_API int mrc_parse_uci(const mrc_position* p, const char* uci, mrc_move* out) {
  if (strlen(uci) < 4) return -1;
  const int from = sq(uci[0] - 'a', uci[1] - '1');
  const int to = sq(uci[2] - 'a', uci[3] - '1');
  int promo = 0;
  if (uci[4]) {
    const char* k = strchr("nbrq", uci[4]);
    if (!k) return -1;
    promo = static_cast<int>(k - "nbrq") + N;
  }
  mrc_move moves[MRC_MAX_MOVES];
  const int n = mrc_legal_moves(p, moves);
  for (int i = 0; i < n; ++i)
    if (moves[i].from == from && moves[i].to == to && moves[i].promotion == promo) {
      *out = moves[i];
      return 0;
    }
  return -1;
}

MRC_API uint64_t mrc_perft(const mrc_position* p, int depth) {
  mrc_move moves[MRC_MAX_MOVES];
  const int n = mrc_legal_moves(p, moves);
  if (depth <= 1) return depth == 1 ? static_cast<uint64_t>(n) : 1;
  uint64_t total = 0;
  for (int i = 0; i < n; ++i) {
    mrc_position q = *p;
    apply(q, moves[i]);
    total += mrc_perft(&q, depth - 1);
  }
  return total;
}

// src/encoding/board.rs:142-192: pieces in the side-to-move frame (rotated 180 degrees for
// Black), own pieces 1-6, opponent 7-12; castling bits own K, own Q, opp K, opp Q; en
// passant = canonical file of the target square + 1 (the target exists after every double
// push).
MRC_API void mrc_encode_board(const mrc_position* p, uint8_t* out) {
  const int turn = p->turn;
  const int sign = turn == 0 ? 1 : -1;
  for (int s = 0; s < 64; ++s) {
    const int pc = p->board[s];
    uint8_t token = 0;
    if (pc != 0) {
      const int type = pc < 0 ? -pc : pc;
      token = static_cast<uint8_t>(pc * sign > 0 ? type : type + 6);
    }
    out[canonical(s, turn)] = token;
  }
  const unsigned own_k = turn == 0 ? 1u : 4u, own_q = turn == 0 ? 2u : 8u;
  const unsigned opp_k = turn == 0 ? 4u : 1u, opp_q = turn == 0 ? 8u : 2u;
  uint8_t c = 0;
  if (p->castling & own_k) c |= 1;
  if (p->castling & own_q) c |= 2;
  if (p->castling & opp_k) c |= 4;
  if (p->castling & opp_q) c |= 8;
  out[64] = c;
  out[65] = p->ep < 0 ? 0 : static_cast<uint8_t>(file_of(canonical(p->ep, turn)) + 1);
}

// src/encoding/action.rs:73-83.
MRC_API int mrc_encode_move(const mrc_position* p, mrc_move m) {
  const int from = canonical(m.from, p->turn), to = canonical(m.to, p->turn);
  const int plane = plane_of(file_of(to) - file_of(from), rank_of(to) - rank_of(from), m.promotion);
  return plane < 0 ? -1 : from * 73 + plane;
}

MRC_API int mrc_legal_actions(const mrc_position* p, int32_t* actions, int cap) {
  mrc_move moves[MRC_MAX_MOVES];
  const int n = mrc_legal_moves(p, moves);
  for (int i = 0; i < n && i < cap; ++i) actions[i] = mrc_encode_move(p, moves[i]);
  return n;
}

// src/encoding/action.rs:85-114: the legal move with the action's squares; a ray move of a
// pawn onto the last rank is the queen promotion.
MRC_API int mrc_decode_action(const mrc_position* p, int action, mrc_move* out) {
  if (action < 0 || action >= 64 * 73) return -1;
  mrc_move moves[MRC_MAX_MOVES];
  const int n = mrc_legal_moves(p, moves);
  for (int i = 0; i < n; ++i)
    if (mrc_encode_move(p, moves[i]) == action) {
      *out = moves[i];
      return 0;
    }
  return -1;
}

MRC_API int mrc_random_positions(uint64_t seed, int count, int min_ply, int max_ply, uint8_t* boards, int32_t* legal,
                                 int32_t* legal_count, char* fens, int threads) {
  if (count < 0 || min_ply < 0 || max_ply < min_ply || !boards || !legal || !legal_count) return -1;
  if (threads < 1) threads = 1;
  auto one = [&](int i) {
    uint64_t state = seed * 0xD1B54A32D192ED03ull + static_cast<uint64_t>(i) * 0x9E3779B97F4A7C15ull + 1;
    splitmix64(state);
    mrc_move moves[MRC_MAX_MOVES];
    for (;;) {
      mrc_position p;
      mrc_startpos(&p);
      const int plies = min_ply + static_cast<int>(uniform(state, static_cast<uint32_t>(max_ply - min_ply + 1)));
      bool dead = false;
      for (int k = 0; k < plies; ++k) {
        const int n = mrc_legal_moves(&p, moves);
        if (n == 0) {
          dead = true;
          break;
        }
        apply(p, moves[uniform(state, static_cast<uint32_t>(n))]);
      }
      if (dead) continue;
      int32_t* slots = legal + static_cast<size_t>(i) * 224;
      const int n = mrc_legal_actions(&p, slots, 224);
      if (n == 0) continue;  // terminal (mate or stalemate): redraw
      for (int k = n; k < 224; ++k) slots[k] = -1;
      legal_count[i] = n;
      mrc_encode_board(&p, boards + static_cast<size_t>(i) * 66);
      if (fens) mrc_to_fen(&p, fens + static_cast<size_t>(i) * 100);
      return;
    }
  };
  if (threads == 1 || count < 64) {
    for (int i = 0; i < count; ++i) one(i);
    return 0;
  }
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t)
    pool.emplace_back([&, t] {
      for (int i = t; i < count; i += threads) one(i);
    });
  for (auto& th : pool) th.join();
  return 0;
}

}  // extern "C"
