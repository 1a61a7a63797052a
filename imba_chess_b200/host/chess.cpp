// Worker-side chess for search inference, as a CPython extension (_chess):
// legal move generation, the UCI-sorted legal-id projection onto the static
// move vocabulary and the board-state encoding of a position, which the
// search worker computes for every expanded node before it sends a wave.
//
// Reference behaviour restated here:
//   * legal-id projection: src/imba_chess/eval/actor_worker.py:230-264
//     (generate legal moves, castling as the king's two-square UCI move,
//     keep moves present in the vocabulary, sort the (uci, id) pairs by UCI);
//   * castling UCI normalisation: src/imba_chess/eval/cozy_bridge.py:91-100;
//   * static move vocabulary: src/imba_chess/data/move_vocab.py:124-155
//     (<pad> 0, <start> 1, then for every from-square a1..h8 the queen-ray and
//     knight targets of an empty board in square order, then the 176 pawn
//     promotions; 1,970 tokens);
//   * board-state encoding: src/imba_chess/data/board_state.py:26-45, :94-129
//     (piece ids 1-6 white P N B R Q K, 7-12 black, 0 empty, square a1 = 0;
//     turn 0 white / 1 black; castle bits K 1, Q 2, k 4, q 8; en-passant
//     file + 1 in "legal" mode only when a legal en-passant capture exists,
//     the FEN square in "fen" mode, a pseudo-legal capturer in "xfen" mode;
//     half- and full-move counters clamped to a maximum and divided by the
//     bucket size).
//
// Board: 64 signed bytes (piece codes as above), side to move, castle bits,
// en-passant target square (-1: none), half- and full-move counters.
// Legality: a pseudo-legal move is legal when, after it is made, the mover's
// king is not attacked; castling also requires the king's start and
// crossing squares to be unattacked.
#define PY_SSIZE_T_CLEAN
#include <Python.h>

#include <algorithm>
#include <array>
#include <cstdint>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

namespace {

enum { EMPTY = 0, WP = 1, WN, WB, WR, WQ, WK, BP, BN, BB, BR, BQ, BK };

struct Pos {
  int8_t sq[64];
  int stm = 0;     // 0 white, 1 black
  int castle = 0;  // 1 K, 2 Q, 4 k, 8 q
  int ep = -1;     // en-passant target square
  int halfmove = 0, fullmove = 1;
};

struct Move {
  int8_t from, to, promo;  // promo: piece type 2 N, 3 B, 4 R, 5 Q (0: none)
  uint8_t flags;           // 1 en passant, 2 castling, 4 double push
};

inline int color_of(int p) { return p >= BP ? 1 : 0; }
inline int type_of(int p) { return p >= BP ? p - 6 : p; }  // 1 P .. 6 K
inline int make_piece(int color, int type) { return color ? type + 6 : type; }
inline int file_of(int s) { return s & 7; }
inline int rank_of(int s) { return s >> 3; }
inline bool on_board(int f, int r) { return f >= 0 && f < 8 && r >= 0 && r < 8; }

const int kKnight[8][2] = {{1, 2}, {2, 1}, {2, -1}, {1, -2}, {-1, -2}, {-2, -1}, {-2, 1}, {-1, 2}};
const int kKing[8][2] = {{1, 0}, {1, 1}, {0, 1}, {-1, 1}, {-1, 0}, {-1, -1}, {0, -1}, {1, -1}};
const int kDiag[4][2] = {{1, 1}, {1, -1}, {-1, 1}, {-1, -1}};
const int kOrth[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};

// Is square s attacked by a piece of colour `by`?
bool attacked(const Pos& p, int s, int by) {
  const int f = file_of(s), r = rank_of(s);
  const int dr = by ? 1 : -1;  // a pawn of `by` attacks from one rank behind s, seen from its side
  for (int df = -1; df <= 1; df += 2) {
    const int ff = f + df, rr = r + dr;
    if (on_board(ff, rr) && p.sq[rr * 8 + ff] == make_piece(by, 1)) return true;
  }
  for (const auto& d : kKnight) {
    const int ff = f + d[0], rr = r + d[1];
    if (on_board(ff, rr) && p.sq[rr * 8 + ff] == make_piece(by, 2)) return true;
  }
  for (const auto& d : kKing) {
    const int ff = f + d[0], rr = r + d[1];
    if (on_board(ff, rr) && p.sq[rr * 8 + ff] == make_piece(by, 6)) return true;
  }
  for (int k = 0; k < 2; ++k) {
    const auto* dirs = k ? kOrth : kDiag;
    const int slider = k ? 4 : 3;  // rook : bishop
    for (int i = 0; i < 4; ++i) {
      int ff = f + dirs[i][0], rr = r + dirs[i][1];
      while (on_board(ff, rr)) {
        const int q = p.sq[rr * 8 + ff];
        if (q != EMPTY) {
          if (color_of(q) == by && (type_of(q) == slider || type_of(q) == 5)) return true;
          break;
        }
        ff += dirs[i][0];
        rr += dirs[i][1];
      }
    }
  }
  return false;
}

int king_square(const Pos& p, int color) {
  const int k = make_piece(color, 6);
  for (int s = 0; s < 64; ++s)
    if (p.sq[s] == k) return s;
  return -1;
}

void pseudo_moves(const Pos& p, std::vector<Move>& out) {
  const int c = p.stm, them = c ^ 1;
  auto add = [&](int from, int to, int promo, int flags) {
    out.push_back(Move{(int8_t)from, (int8_t)to, (int8_t)promo, (uint8_t)flags});
  };
  for (int s = 0; s < 64; ++s) {
    const int q = p.sq[s];
    if (q == EMPTY || color_of(q) != c) continue;
    const int t = type_of(q), f = file_of(s), r = rank_of(s);
    if (t == 1) {
      const int dir = c ? -1 : 1, start = c ? 6 : 1, last = c ? 0 : 7;
      auto pawn_to = [&](int to, int flags) {
        if (rank_of(to) == last) {
          for (int pr = 5; pr >= 2; --pr) add(s, to, pr, flags);
        } else {
          add(s, to, 0, flags);
        }
      };
      const int r1 = r + dir;
      if (r1 >= 0 && r1 < 8 && p.sq[r1 * 8 + f] == EMPTY) {
        pawn_to(r1 * 8 + f, 0);
        const int r2 = r + 2 * dir;
        if (r == start && p.sq[r2 * 8 + f] == EMPTY) add(s, r2 * 8 + f, 0, 4);
      }
      for (int df = -1; df <= 1; df += 2) {
        const int ff = f + df;
        if (!on_board(ff, r1)) continue;
        const int to = r1 * 8 + ff, v = p.sq[to];
        if (v != EMPTY && color_of(v) == them) pawn_to(to, 0);
        else if (v == EMPTY && to == p.ep) add(s, to, 0, 1);
      }
    } else if (t == 2 || t == 6) {
      const auto* d = t == 2 ? kKnight : kKing;
      for (int i = 0; i < 8; ++i) {
        const int ff = f + d[i][0], rr = r + d[i][1];
        if (!on_board(ff, rr)) continue;
        const int v = p.sq[rr * 8 + ff];
        if (v == EMPTY || color_of(v) == them) add(s, rr * 8 + ff, 0, 0);
      }
    } else {
      for (int k = 0; k < 2; ++k) {
        if (k == 0 && t == 4) continue;  // rook: no diagonals
        if (k == 1 && t == 3) continue;  // bishop: no orthogonals
        const auto* dirs = k ? kOrth : kDiag;
        for (int i = 0; i < 4; ++i) {
          int ff = f + dirs[i][0], rr = r + dirs[i][1];
          while (on_board(ff, rr)) {
            const int v = p.sq[rr * 8 + ff];
            if (v == EMPTY) {
              add(s, rr * 8 + ff, 0, 0);
            } else {
              if (color_of(v) == them) add(s, rr * 8 + ff, 0, 0);
              break;
            }
            ff += dirs[i][0];
            rr += dirs[i][1];
          }
        }
      }
    }
  }
  // Castling: rights, king and rook in place, empty squares between, and
  // the king's start, crossing and destination squares unattacked.
  const int base = c ? 56 : 0, king = make_piece(c, 6), rook = make_piece(c, 4);
  if (p.sq[base + 4] == king) {
    const int short_bit = c ? 4 : 1, long_bit = c ? 8 : 2;
    if ((p.castle & short_bit) && p.sq[base + 7] == rook && p.sq[base + 5] == EMPTY && p.sq[base + 6] == EMPTY &&
        !attacked(p, base + 4, them) && !attacked(p, base + 5, them) && !attacked(p, base + 6, them))
      add(base + 4, base + 6, 0, 2);
    if ((p.castle & long_bit) && p.sq[base] == rook && p.sq[base + 1] == EMPTY && p.sq[base + 2] == EMPTY &&
        p.sq[base + 3] == EMPTY && !attacked(p, base + 4, them) && !attacked(p, base + 3, them) &&
        !attacked(p, base + 2, them))
      add(base + 4, base + 2, 0, 2);
  }
}

Pos make_move(const Pos& p, const Move& m) {
  Pos n = p;
  const int c = p.stm, q = p.sq[m.from];
  const bool capture = p.sq[m.to] != EMPTY || (m.flags & 1);
  n.sq[m.to] = m.promo ? make_piece(c, m.promo) : q;
  n.sq[m.from] = EMPTY;
  if (m.flags & 1) n.sq[rank_of(m.from) * 8 + file_of(m.to)] = EMPTY;  // the pawn taken en passant
  if (m.flags & 2) {                                                    // the rook's half of castling
    const int base = c ? 56 : 0;
    if (m.to == base + 6) {
      n.sq[base + 5] = n.sq[base + 7];
      n.sq[base + 7] = EMPTY;
    } else {
      n.sq[base + 3] = n.sq[base];
      n.sq[base] = EMPTY;
    }
  }
  if (type_of(q) == 6) n.castle &= c ? ~12 : ~3;
  for (int s : {(int)m.from, (int)m.to}) {
    if (s == 0) n.castle &= ~2;
    if (s == 7) n.castle &= ~1;
    if (s == 56) n.castle &= ~8;
    if (s == 63) n.castle &= ~4;
  }
  n.ep = (m.flags & 4) ? (m.from + m.to) / 2 : -1;
  n.halfmove = (type_of(q) == 1 || capture) ? 0 : p.halfmove + 1;
  if (c == 1) n.fullmove = p.fullmove + 1;
  n.stm = c ^ 1;
  return n;
}

void legal_moves(const Pos& p, std::vector<Move>& out) {
  std::vector<Move> pseudo;
  pseudo.reserve(64);
  pseudo_moves(p, pseudo);
  out.clear();
  for (const Move& m : pseudo) {
    const Pos n = make_move(p, m);
    const int k = king_square(n, p.stm);
    if (k >= 0 && !attacked(n, k, p.stm ^ 1)) out.push_back(m);
  }
}

uint64_t perft(const Pos& p, int depth) {
  std::vector<Move> moves;
  legal_moves(p, moves);
  if (depth <= 1) return depth == 1 ? moves.size() : 1;
  uint64_t total = 0;
  for (const Move& m : moves) total += perft(make_move(p, m), depth - 1);
  return total;
}

std::string square_name(int s) { return std::string{(char)('a' + file_of(s)), (char)('1' + rank_of(s))}; }

std::string uci_of(const Move& m) {
  std::string u = square_name(m.from) + square_name(m.to);
  if (m.promo) u += " nbrq"[m.promo - 1];
  return u;
}

// ---- static move vocabulary ----
struct Vocab {
  std::vector<std::string> tokens;
  std::unordered_map<std::string, int> ids;
};

const Vocab& vocab() {
  static Vocab v = [] {
    Vocab o;
    o.tokens = {"<pad>", "<start>"};
    for (int s = 0; s < 64; ++s) {
      bool target[64] = {};
      const int f = file_of(s), r = rank_of(s);
      for (const auto* dirs : {kDiag, kOrth})
        for (int i = 0; i < 4; ++i)
          for (int ff = f + dirs[i][0], rr = r + dirs[i][1]; on_board(ff, rr); ff += dirs[i][0], rr += dirs[i][1])
            target[rr * 8 + ff] = true;
      for (const auto& d : kKnight)
        if (on_board(f + d[0], r + d[1])) target[(r + d[1]) * 8 + f + d[0]] = true;
      for (int t = 0; t < 64; ++t)
        if (target[t]) o.tokens.push_back(square_name(s) + square_name(t));
    }
    for (const auto fr : {std::array<int, 2>{6, 7}, std::array<int, 2>{1, 0}})
      for (int f = 0; f < 8; ++f)
        for (int df = -1; df <= 1; ++df) {
          if (f + df < 0 || f + df > 7) continue;
          const std::string base = square_name(fr[0] * 8 + f) + square_name(fr[1] * 8 + f + df);
          for (char pc : {'q', 'r', 'b', 'n'}) o.tokens.push_back(base + pc);
        }
    for (size_t i = 0; i < o.tokens.size(); ++i) o.ids.emplace(o.tokens[i], (int)i);
    return o;
  }();
  return v;
}

// ---- FEN ----
bool parse_fen(const char* fen, Pos& p, std::string& err) {
  std::memset(p.sq, 0, sizeof(p.sq));
  const char* c = fen;
  int r = 7, f = 0;
  const char* names = "PNBRQKpnbrqk";
  for (; *c && *c != ' '; ++c) {
    if (*c == '/') {
      if (f != 8 || r == 0) return err = "bad FEN board", false;
      --r;
      f = 0;
    } else if (*c >= '1' && *c <= '8') {
      f += *c - '0';
      if (f > 8) return err = "bad FEN board", false;
    } else {
      const char* k = std::strchr(names, *c);
      if (!k || f > 7) return err = "bad FEN board", false;
      p.sq[r * 8 + f++] = (int8_t)(k - names + 1);
    }
  }
  if (r != 0 || f != 8) return err = "bad FEN board", false;
  auto field = [&](std::string& out) {
    while (*c == ' ') ++c;
    out.clear();
    while (*c && *c != ' ') out += *c++;
    return !out.empty();
  };
  std::string stm, cas, ep, hm, fm;
  if (!field(stm) || (stm != "w" && stm != "b")) return err = "bad FEN side to move", false;
  p.stm = stm == "b";
  p.castle = 0;
  if (field(cas) && cas != "-")
    for (char ch : cas) {
      const char* k = std::strchr("KQkq", ch);
      if (!k) return err = "bad FEN castling field", false;
      p.castle |= 1 << (k - "KQkq");
    }
  p.ep = -1;
  if (field(ep) && ep != "-") {
    if (ep.size() != 2 || ep[0] < 'a' || ep[0] > 'h' || ep[1] < '1' || ep[1] > '8')
      return err = "bad FEN en-passant square", false;
    p.ep = (ep[1] - '1') * 8 + (ep[0] - 'a');
  }
  p.halfmove = field(hm) ? std::atoi(hm.c_str()) : 0;
  p.fullmove = field(fm) ? std::atoi(fm.c_str()) : 1;
  if (king_square(p, 0) < 0 || king_square(p, 1) < 0) return err = "FEN without both kings", false;
  return true;
}

// The legal en-passant capture of the position, if any (used by the
// "legal" encoding mode and by the FEN writer).
bool has_legal_ep(const Pos& p, const std::vector<Move>& legal) {
  for (const Move& m : legal)
    if (m.flags & 1) return true;
  return false;
}

bool has_pseudo_ep(const Pos& p) {
  if (p.ep < 0) return false;
  const int c = p.stm, dir = c ? 1 : -1;  // capturers stand one rank behind the target, seen from the mover
  const int f = file_of(p.ep), r = rank_of(p.ep) + dir;
  if (r < 0 || r > 7) return false;
  for (int df = -1; df <= 1; df += 2)
    if (on_board(f + df, r) && p.sq[r * 8 + f + df] == make_piece(c, 1)) return true;
  return false;
}

std::string write_fen(const Pos& p, const std::vector<Move>& legal) {
  std::string o;
  const char* names = " PNBRQKpnbrqk";
  for (int r = 7; r >= 0; --r) {
    int empty = 0;
    for (int f = 0; f < 8; ++f) {
      const int q = p.sq[r * 8 + f];
      if (q == EMPTY) {
        ++empty;
        continue;
      }
      if (empty) o += (char)('0' + empty);
      empty = 0;
      o += names[q];
    }
    if (empty) o += (char)('0' + empty);
    if (r) o += '/';
  }
  o += p.stm ? " b " : " w ";
  std::string cas;
  for (int i = 0; i < 4; ++i)
    if (p.castle & (1 << i)) cas += "KQkq"[i];
  o += cas.empty() ? "-" : cas;
  o += ' ';
  o += (p.ep >= 0 && has_legal_ep(p, legal)) ? square_name(p.ep) : "-";
  o += ' ' + std::to_string(p.halfmove) + ' ' + std::to_string(p.fullmove);
  return o;
}

int bucket(int v, int max_v, int size) { return (v < 0 ? 0 : v > max_v ? max_v : v) / size; }

struct EncodeCfg {
  int ep_mode = 0;  // 0 legal, 1 fen, 2 xfen
  int half_max = 100, half_size = 2, full_max = 200, full_size = 2;
};

// side: turn, castle, ep file, halfmove bucket, fullmove bucket.
void encode(const Pos& p, const std::vector<Move>& legal, const EncodeCfg& cfg, uint8_t* piece, int32_t* side) {
  for (int s = 0; s < 64; ++s) piece[s] = (uint8_t)p.sq[s];
  int ep = 0;
  if (p.ep >= 0) {
    const bool ok = cfg.ep_mode == 1 ? true : cfg.ep_mode == 0 ? has_legal_ep(p, legal) : has_pseudo_ep(p);
    ep = ok ? file_of(p.ep) + 1 : 0;
  }
  side[0] = p.stm;
  side[1] = p.castle;
  side[2] = ep;
  side[3] = bucket(p.halfmove, cfg.half_max, cfg.half_size);
  side[4] = bucket(p.fullmove, cfg.full_max, cfg.full_size);
}

// UCI order as an integer: "f1 r1 f2 r2 [p]" compares character by
// character, i.e. by (from file, from rank, to file, to rank, promotion
// letter with none < b < n < q < r).
inline int uci_key(const Move& m) {
  static const int promo_rank[6] = {0, 0, 2, 1, 4, 3};  // none, -, n, b, r, q
  return (((file_of(m.from) * 8 + rank_of(m.from)) * 8 + file_of(m.to)) * 8 + rank_of(m.to)) * 5 +
         promo_rank[(int)m.promo];
}

// Vocabulary id of (from, to, promotion type), -1 when absent.
const std::vector<int>& id_table() {
  static std::vector<int> t = [] {
    std::vector<int> o(64 * 64 * 6, -1);
    for (int from = 0; from < 64; ++from)
      for (int to = 0; to < 64; ++to)
        for (int pr = 0; pr < 6; ++pr) {
          if (pr == 1) continue;
          const Move m{(int8_t)from, (int8_t)to, (int8_t)pr, 0};
          auto it = vocab().ids.find(uci_of(m));
          if (it != vocab().ids.end()) o[(from * 64 + to) * 6 + pr] = it->second;
        }
    return o;
  }();
  return t;
}

// Legal moves mapped to vocabulary ids, sorted by UCI: (key, id, move index).
void projection(const std::vector<Move>& legal, std::vector<std::array<int, 3>>& out) {
  const std::vector<int>& ids = id_table();
  out.clear();
  for (size_t i = 0; i < legal.size(); ++i) {
    const Move& m = legal[i];
    const int id = ids[(m.from * 64 + m.to) * 6 + m.promo];
    if (id >= 0) out.push_back({uci_key(m), id, (int)i});
  }
  std::sort(out.begin(), out.end());
}

// ---- Python bindings ----
bool get_pos(PyObject* fen_obj, Pos& p) {
  const char* fen = PyUnicode_AsUTF8(fen_obj);
  if (!fen) return false;
  std::string err;
  if (!parse_fen(fen, p, err)) {
    PyErr_Format(PyExc_ValueError, "%s: %s", err.c_str(), fen);
    return false;
  }
  return true;
}

bool parse_cfg(PyObject* kw, EncodeCfg& cfg) {
  if (!kw) return true;
  static const char* keys[] = {"en_passant", "halfmove_max", "halfmove_bucket_size", "fullmove_max",
                               "fullmove_bucket_size"};
  PyObject *k, *val;
  Py_ssize_t pos = 0;
  while (PyDict_Next(kw, &pos, &k, &val)) {
    const char* name = PyUnicode_AsUTF8(k);
    if (!name) return false;
    if (!std::strcmp(name, keys[0])) {
      const char* m = PyUnicode_AsUTF8(val);
      if (!m) return false;
      if (!std::strcmp(m, "legal")) cfg.ep_mode = 0;
      else if (!std::strcmp(m, "fen")) cfg.ep_mode = 1;
      else if (!std::strcmp(m, "xfen")) cfg.ep_mode = 2;
      else {
        PyErr_Format(PyExc_ValueError, "Unsupported en_passant mode: %s", m);
        return false;
      }
      continue;
    }
    int* dst = nullptr;
    if (!std::strcmp(name, keys[1])) dst = &cfg.half_max;
    else if (!std::strcmp(name, keys[2])) dst = &cfg.half_size;
    else if (!std::strcmp(name, keys[3])) dst = &cfg.full_max;
    else if (!std::strcmp(name, keys[4])) dst = &cfg.full_size;
    if (!dst) {
      PyErr_Format(PyExc_TypeError, "unexpected keyword argument '%s'", name);
      return false;
    }
    const long v = PyLong_AsLong(val);
    if (v == -1 && PyErr_Occurred()) return false;
    *dst = (int)v;
  }
  if (cfg.half_size <= 0) return PyErr_SetString(PyExc_ValueError, "halfmove_bucket_size must be > 0"), false;
  if (cfg.full_size <= 0) return PyErr_SetString(PyExc_ValueError, "fullmove_bucket_size must be > 0"), false;
  return true;
}

PyObject* py_perft(PyObject*, PyObject* args) {
  PyObject* fen;
  int depth;
  if (!PyArg_ParseTuple(args, "Ui", &fen, &depth)) return nullptr;
  Pos p;
  if (!get_pos(fen, p)) return nullptr;
  uint64_t n;
  Py_BEGIN_ALLOW_THREADS n = perft(p, depth);
  Py_END_ALLOW_THREADS return PyLong_FromUnsignedLongLong(n);
}

PyObject* py_vocab(PyObject*, PyObject*) {
  const Vocab& v = vocab();
  PyObject* out = PyList_New((Py_ssize_t)v.tokens.size());
  if (!out) return nullptr;
  for (size_t i = 0; i < v.tokens.size(); ++i) {
    PyObject* s = PyUnicode_FromStringAndSize(v.tokens[i].data(), (Py_ssize_t)v.tokens[i].size());
    if (!s) {
      Py_DECREF(out);
      return nullptr;
    }
    PyList_SET_ITEM(out, (Py_ssize_t)i, s);
  }
  return out;
}

PyObject* py_legal_projection(PyObject*, PyObject* args) {
  PyObject* fen;
  if (!PyArg_ParseTuple(args, "U", &fen)) return nullptr;
  Pos p;
  if (!get_pos(fen, p)) return nullptr;
  std::vector<Move> legal;
  legal_moves(p, legal);
  std::vector<std::array<int, 3>> proj;
  projection(legal, proj);
  PyObject* ids = PyList_New((Py_ssize_t)proj.size());
  PyObject* ucis = PyList_New((Py_ssize_t)proj.size());
  if (!ids || !ucis) {
    Py_XDECREF(ids);
    Py_XDECREF(ucis);
    return nullptr;
  }
  for (size_t i = 0; i < proj.size(); ++i) {
    PyList_SET_ITEM(ids, (Py_ssize_t)i, PyLong_FromLong(proj[i][1]));
    PyList_SET_ITEM(ucis, (Py_ssize_t)i, PyUnicode_FromString(uci_of(legal[proj[i][2]]).c_str()));
  }
  return Py_BuildValue("(NN)", ids, ucis);
}

PyObject* py_encode(PyObject*, PyObject* args, PyObject* kw) {
  PyObject* fen;
  if (!PyArg_ParseTuple(args, "U", &fen)) return nullptr;
  EncodeCfg cfg;
  if (!parse_cfg(kw, cfg)) return nullptr;
  Pos p;
  if (!get_pos(fen, p)) return nullptr;
  std::vector<Move> legal;
  legal_moves(p, legal);
  uint8_t piece[64];
  int32_t side[5];
  encode(p, legal, cfg, piece, side);
  PyObject* ids = PyList_New(64);
  if (!ids) return nullptr;
  for (int s = 0; s < 64; ++s) PyList_SET_ITEM(ids, s, PyLong_FromLong(piece[s]));
  return Py_BuildValue("(Niiiii)", ids, side[0], side[1], side[2], side[3], side[4]);
}

PyObject* py_push_uci(PyObject*, PyObject* args) {
  PyObject* fen;
  const char* uci;
  if (!PyArg_ParseTuple(args, "Us", &fen, &uci)) return nullptr;
  Pos p;
  if (!get_pos(fen, p)) return nullptr;
  std::vector<Move> legal;
  legal_moves(p, legal);
  for (const Move& m : legal)
    if (uci_of(m) == uci) {
      const Pos n = make_move(p, m);
      std::vector<Move> nl;
      legal_moves(n, nl);
      return PyUnicode_FromString(write_fen(n, nl).c_str());
    }
  PyErr_Format(PyExc_ValueError, "illegal move %s in %U", uci, fen);
  return nullptr;
}

// expand(fens, **cfg) -> (piece bytes [N*64], side bytes int32 [N, 5],
//                         legal_off bytes int32 [N + 1], legal_ids bytes int32)
// Every position's encoding and UCI-sorted legal vocabulary ids, packed as
// the wave request's arrays (one call per expanded search node batch).
PyObject* py_expand(PyObject*, PyObject* args, PyObject* kw) {
  PyObject* fens;
  if (!PyArg_ParseTuple(args, "O", &fens)) return nullptr;
  EncodeCfg cfg;
  if (!parse_cfg(kw, cfg)) return nullptr;
  PyObject* fast = PySequence_Fast(fens, "fens must be a sequence of FEN strings");
  if (!fast) return nullptr;
  const Py_ssize_t n = PySequence_Fast_GET_SIZE(fast);
  std::vector<uint8_t> piece((size_t)n * 64);
  std::vector<int32_t> side((size_t)n * 5), loff((size_t)n + 1, 0), lids;
  std::vector<Move> legal;
  std::vector<std::array<int, 3>> proj;
  for (Py_ssize_t i = 0; i < n; ++i) {
    Pos p;
    if (!get_pos(PySequence_Fast_GET_ITEM(fast, i), p)) {
      Py_DECREF(fast);
      return nullptr;
    }
    legal_moves(p, legal);
    encode(p, legal, cfg, piece.data() + 64 * i, side.data() + 5 * i);
    projection(legal, proj);
    for (const auto& e : proj) lids.push_back(e[1]);
    loff[i + 1] = (int32_t)lids.size();
  }
  Py_DECREF(fast);
  return Py_BuildValue("(y#y#y#y#)", reinterpret_cast<const char*>(piece.data()), (Py_ssize_t)piece.size(),
                       reinterpret_cast<const char*>(side.data()), (Py_ssize_t)(side.size() * 4),
                       reinterpret_cast<const char*>(loff.data()), (Py_ssize_t)(loff.size() * 4),
                       reinterpret_cast<const char*>(lids.data()), (Py_ssize_t)(lids.size() * 4));
}

PyMethodDef kMethods[] = {
    {"perft", py_perft, METH_VARARGS, "perft(fen, depth) -> leaf count of the legal move tree"},
    {"vocab", py_vocab, METH_NOARGS, "vocab() -> the static move vocabulary, id -> token"},
    {"legal_projection", py_legal_projection, METH_VARARGS,
     "legal_projection(fen) -> (vocab ids, UCIs) of the legal moves, sorted by UCI"},
    {"encode", reinterpret_cast<PyCFunction>(reinterpret_cast<void (*)(void)>(py_encode)),
     METH_VARARGS | METH_KEYWORDS,
     "encode(fen, **cfg) -> (piece_ids[64], turn, castle, ep_file, halfmove_bucket, fullmove_bucket)"},
    {"push_uci", py_push_uci, METH_VARARGS, "push_uci(fen, uci) -> FEN after the legal move"},
    {"expand", reinterpret_cast<PyCFunction>(reinterpret_cast<void (*)(void)>(py_expand)),
     METH_VARARGS | METH_KEYWORDS, "expand(fens, **cfg) -> packed encodings and legal-id CSR"},
    {nullptr, nullptr, 0, nullptr}};

PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_chess", "Worker-side chess: movegen, legal-id projection, encoding.",
                       -1, kMethods};

}  // namespace

PyMODINIT_FUNC PyInit__chess(void) { return PyModule_Create(&kModule); }
