// Host-side batch producer: tokenisation and tensorisation of pretraining
// games into the 10 per-sequence tensors of the training step.
//
// Restates, in native code, chessdecoder/dataloader/data.py:7-97
// (fen_to_position_tokens, game_to_token_ids) and the per-game body of
// chessdecoder/dataloader/loader.py:69-184 (random start among the valid
// starts, truncation, shifted board targets, move / value targets, block
// ids).  The two random decisions of the reference (board kept per ply, the
// start index) are taken by the caller with the reference's own generator
// and passed in, so the rows are identical to the reference's for the same
// seed.  Games are independent: they are spread over host threads.
//
// Castling rights follow the reference's python-chess semantics for standard
// chess: a right counts only if the FEN lists it, the king stands on its home
// square (e1 / e8) and the rook on the matching corner (h1 / a1 / h8 / a8).
#include "../../include/cdk.h"

#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <string_view>
#include <thread>
#include <unordered_map>
#include <vector>

namespace {

constexpr int kIgnore = -100;

struct Vocab {
  std::unordered_map<std::string, int32_t> index;
  std::vector<int32_t> to_board, to_move;
  int32_t pad = -1, start_pos = -1, end_pos = -1, empty = -1, wl_value = -1, d_value = -1;
  int32_t white_to_move = -1, black_to_move = -1, no_castling = -1, generic_move_board = -1;
  int32_t piece[2][6];  // [color][pawn knight bishop rook queen king]
  int32_t castling[16];  // by rights mask K=1 Q=2 k=4 q=8 (0 = no_castling_rights)

  int32_t find(std::string_view s) const {
    auto it = index.find(std::string(s));
    return it == index.end() ? -1 : it->second;
  }
};

int32_t piece_slot(char c) {
  switch (c) {
    case 'p': return 0;
    case 'n': return 1;
    case 'b': return 2;
    case 'r': return 3;
    case 'q': return 4;
    case 'k': return 5;
    default: return -1;
  }
}

// 68 position tokens of a FEN; false if the FEN is malformed.
bool fen_tokens(const Vocab& v, std::string_view fen, int32_t* out) {
  char board[64];
  std::memset(board, 0, sizeof(board));
  size_t i = 0;
  int rank = 7, file = 0;
  for (; i < fen.size() && fen[i] != ' '; ++i) {
    const char c = fen[i];
    if (c == '/') {
      if (file != 8 || rank == 0) return false;
      --rank;
      file = 0;
    } else if (c >= '1' && c <= '8') {
      file += c - '0';
      if (file > 8) return false;
    } else {
      const char lower = (char)(c | 0x20);
      if (piece_slot(lower) < 0 || file >= 8) return false;
      board[rank * 8 + file] = c;
      ++file;
    }
  }
  if (rank != 0 || file != 8 || i >= fen.size()) return false;
  ++i;  // side to move
  if (i >= fen.size() || (fen[i] != 'w' && fen[i] != 'b')) return false;
  const bool white = fen[i] == 'w';
  ++i;
  int rights = 0;
  if (i < fen.size() && fen[i] == ' ') {
    ++i;
    for (; i < fen.size() && fen[i] != ' '; ++i) {
      switch (fen[i]) {
        case 'K': rights |= 1; break;
        case 'Q': rights |= 2; break;
        case 'k': rights |= 4; break;
        case 'q': rights |= 8; break;
        case '-': break;
        default: return false;
      }
    }
  }
  // python-chess cleaning for standard chess: king home, rook on the corner
  if (board[4] != 'K') rights &= ~3;
  if (board[7] != 'R') rights &= ~1;
  if (board[0] != 'R') rights &= ~2;
  if (board[60] != 'k') rights &= ~12;
  if (board[63] != 'r') rights &= ~4;
  if (board[56] != 'r') rights &= ~8;
  out[0] = v.start_pos;
  for (int s = 0; s < 64; ++s) {
    const char c = board[s];
    if (c == 0) {
      out[1 + s] = v.empty;
    } else {
      const bool w = c >= 'A' && c <= 'Z';
      out[1 + s] = v.piece[w ? 0 : 1][piece_slot((char)(c | 0x20))];
    }
  }
  out[65] = v.end_pos;
  out[66] = v.castling[rights];
  out[67] = white ? v.white_to_move : v.black_to_move;
  return true;
}

struct MoveTarget {
  int64_t pos;
  int32_t best;  // full vocabulary index
};
struct ValueEntry {
  int64_t wl_pos, d_pos;
  float wl, d;
  bool valid;
};
struct Block {
  int64_t b0, b1;
};

struct GameIn {
  int64_t ply0, ply1;
  const char* fen_chars;
  const int64_t* fen_off;
  const char* played_chars;
  const int64_t* played_off;
  const char* best_chars;
  const int64_t* best_off;
  const double* q;
  const double* d;
  const uint8_t* include_board;
  int64_t start_choice;
};

struct RowOut {
  int64_t* ids;
  int64_t* board_t;
  int64_t* move_t;
  uint8_t* move_mask;
  uint8_t* wl_pos;
  uint8_t* d_pos;
  float* wl_t;
  float* d_t;
  uint8_t* valid;
  int64_t* block_id;
};

int tokenize_game(const Vocab& v, const GameIn& g, int64_t S, const RowOut& o, std::vector<int32_t>& seq,
                  std::vector<MoveTarget>& moves, std::vector<ValueEntry>& values, std::vector<Block>& blocks) {
  seq.clear();
  moves.clear();
  values.clear();
  blocks.clear();
  int32_t pos_tokens[68];
  // game_to_token_ids (chessdecoder/dataloader/data.py:50-97)
  for (int64_t p = g.ply0; p < g.ply1; ++p) {
    const bool include = p == g.ply0 || g.include_board[p] != 0;
    int64_t block_start = 0;
    if (include) {
      block_start = (int64_t)seq.size();
      std::string_view fen(g.fen_chars + g.fen_off[p], (size_t)(g.fen_off[p + 1] - g.fen_off[p]));
      if (!fen_tokens(v, fen, pos_tokens)) return -3;
      seq.insert(seq.end(), pos_tokens, pos_tokens + 68);
    }
    const int64_t plen = g.played_off[p + 1] - g.played_off[p];
    if (plen > 0) {  // `if played_move:` -- an empty / missing move adds nothing
      const int32_t mv = v.find(std::string_view(g.played_chars + g.played_off[p], (size_t)plen));
      const int32_t best = v.find(std::string_view(g.best_chars + g.best_off[p],
                                                   (size_t)(g.best_off[p + 1] - g.best_off[p])));
      if (mv < 0 || best < 0 || v.to_move[best] < 0) return -2;
      const int64_t move_idx = (int64_t)seq.size();
      seq.push_back(mv);
      if (include) blocks.push_back({block_start, move_idx});
      moves.push_back({move_idx, best});
      const int64_t wl_pos = (int64_t)seq.size();
      seq.push_back(v.wl_value);
      const int64_t d_pos = (int64_t)seq.size();
      seq.push_back(v.d_value);
      const bool ok = !std::isnan(g.q[p]) && !std::isnan(g.d[p]);
      values.push_back({wl_pos, d_pos, ok ? (float)g.q[p] : 0.f, ok ? (float)g.d[p] : 0.f, ok});
    }
  }
  // random start (loader.py:75-104): 0 or one past each D placeholder but the last
  const int64_t n_starts = values.empty() ? 1 : (int64_t)values.size();
  if (g.start_choice < 0 || g.start_choice >= n_starts) return -4;
  const int64_t start = g.start_choice == 0 ? 0 : values[g.start_choice - 1].d_pos + 1;
  int64_t n = (int64_t)seq.size() - start;
  // positions relative to the start; truncation (loader.py:106-124)
  std::vector<Block> adj;
  adj.reserve(blocks.size());
  for (const Block& b : blocks) {
    const int64_t a0 = b.b0 - start, a1 = b.b1 - start;
    if (a1 > 0 && a0 < n) adj.push_back({a0 > 0 ? a0 : 0, a1 < n ? a1 : n});
  }
  if (n > S) {
    n = S;
    std::vector<Block> cut;
    for (const Block& b : adj)
      if (b.b0 < S) cut.push_back({b.b0, b.b1 < S ? b.b1 : S});
    adj.swap(cut);
  }
  // value entries fully inside; move targets only where their values survived
  std::vector<ValueEntry> vals;
  for (const ValueEntry& e : values) {
    const int64_t w = e.wl_pos - start, d = e.d_pos - start;
    if (d >= 0 && w < S && d < S) vals.push_back({w, d, e.wl, e.d, e.valid});
  }
  // tensors (loader.py:126-184)
  for (int64_t i = 0; i < S; ++i) {
    o.ids[i] = i < n ? seq[start + i] : v.pad;
    o.board_t[i] = kIgnore;
    o.move_t[i] = kIgnore;
    o.move_mask[i] = 0;
    o.wl_pos[i] = 0;
    o.d_pos[i] = 0;
    o.wl_t[i] = 0.f;
    o.d_t[i] = 0.f;
    o.valid[i] = 0;
  }
  for (int64_t i = 0; i + 1 < n; ++i) {
    const int32_t b = v.to_board[o.ids[i + 1]];
    o.board_t[i] = b >= 0 ? b : kIgnore;
  }
  for (const MoveTarget& m : moves) {
    const int64_t mi = m.pos - start;
    if (mi < 0 || mi >= S) continue;
    bool has_value = false;  // wl_pos = move_idx + 1 among the surviving values
    for (const ValueEntry& e : vals)
      if (e.wl_pos - 1 == mi) {
        has_value = true;
        break;
      }
    if (!has_value) continue;
    const int64_t stm = mi - 1;
    if (stm >= 0 && stm < S) {
      o.board_t[stm] = v.generic_move_board;
      o.move_t[stm] = v.to_move[m.best];
      o.move_mask[stm] = 1;
    }
  }
  for (const ValueEntry& e : vals) {
    if (e.wl_pos < S) {
      o.wl_pos[e.wl_pos] = 1;
      o.wl_t[e.wl_pos] = e.wl;
      o.valid[e.wl_pos] = e.valid;
    }
    if (e.d_pos < S) {
      o.d_pos[e.d_pos] = 1;
      o.d_t[e.d_pos] = e.d;
      o.valid[e.d_pos] = e.valid;
    }
    const int64_t stm = e.wl_pos - 2;
    if (stm >= 0 && stm < S) {
      o.wl_t[stm] = e.wl;
      o.d_t[stm] = e.d;
      o.valid[stm] = e.valid;
    }
  }
  const int64_t nb = (int64_t)adj.size();
  for (int64_t i = 0; i < S; ++i) o.block_id[i] = i + nb;
  for (int64_t k = 0; k < nb; ++k)
    for (int64_t i = adj[k].b0; i < adj[k].b1; ++i) o.block_id[i] = k;
  return 0;
}

}  // namespace

extern "C" void* cdk_vocab_create(const char* chars, const int64_t* offsets, int64_t n_tokens,
                                  const int32_t* full_to_board, const int32_t* full_to_move) {
  if (!chars || !offsets || !full_to_board || !full_to_move || n_tokens <= 0) return nullptr;
  Vocab* v = new Vocab();
  v->to_board.assign(full_to_board, full_to_board + n_tokens);
  v->to_move.assign(full_to_move, full_to_move + n_tokens);
  for (int64_t t = 0; t < n_tokens; ++t)
    v->index.emplace(std::string(chars + offsets[t], (size_t)(offsets[t + 1] - offsets[t])), (int32_t)t);
  auto need = [&](const char* s) { return v->find(s); };
  v->pad = need("pad");
  v->start_pos = need("start_pos");
  v->end_pos = need("end_pos");
  v->empty = need("empty");
  v->wl_value = need("wl_value");
  v->d_value = need("d_value");
  v->white_to_move = need("white_to_move");
  v->black_to_move = need("black_to_move");
  v->no_castling = need("no_castling_rights");
  const int32_t gm = need("generic_move");
  v->generic_move_board = gm >= 0 ? v->to_board[gm] : -1;
  static const char* names[6] = {"pawn", "knight", "bishop", "rook", "queen", "king"};
  bool ok = v->pad >= 0 && v->start_pos >= 0 && v->end_pos >= 0 && v->empty >= 0 && v->wl_value >= 0 &&
            v->d_value >= 0 && v->white_to_move >= 0 && v->black_to_move >= 0 && v->no_castling >= 0 &&
            v->generic_move_board >= 0;
  for (int c = 0; c < 2; ++c)
    for (int k = 0; k < 6; ++k) {
      v->piece[c][k] = need((std::string(c == 0 ? "white_" : "black_") + names[k]).c_str());
      ok = ok && v->piece[c][k] >= 0;
    }
  for (int m = 0; m < 16; ++m) {
    std::string s;
    if (m & 1) s += 'K';
    if (m & 2) s += 'Q';
    if (m & 4) s += 'k';
    if (m & 8) s += 'q';
    v->castling[m] = m == 0 ? v->no_castling : need(s.c_str());
    ok = ok && v->castling[m] >= 0;
  }
  if (!ok) {
    delete v;
    return nullptr;
  }
  return v;
}

extern "C" void cdk_vocab_destroy(void* vocab) { delete reinterpret_cast<Vocab*>(vocab); }

extern "C" int cdk_tokenize_games(const void* vocab, int64_t n_games, const int64_t* game_offsets,
                                  const char* fen_chars, const int64_t* fen_offsets, const char* played_chars,
                                  const int64_t* played_offsets, const char* best_chars, const int64_t* best_offsets,
                                  const double* played_q, const double* played_d, const uint8_t* include_board,
                                  const int64_t* start_choice, int64_t max_seq_len, int32_t n_threads,
                                  int64_t* input_ids, int64_t* board_target_ids, int64_t* move_target_ids,
                                  uint8_t* move_mask, uint8_t* wl_positions, uint8_t* d_positions, float* wl_targets,
                                  float* d_targets, uint8_t* wdl_valid, int64_t* block_id) {
  if (!vocab || n_games < 0 || max_seq_len <= 0) return -1;
  if (n_games == 0) return 0;
  if (!game_offsets || !fen_chars || !fen_offsets || !played_chars || !played_offsets || !best_chars ||
      !best_offsets || !played_q || !played_d || !include_board || !start_choice || !input_ids ||
      !board_target_ids || !move_target_ids || !move_mask || !wl_positions || !d_positions || !wl_targets ||
      !d_targets || !wdl_valid || !block_id)
    return -1;
  const Vocab& v = *reinterpret_cast<const Vocab*>(vocab);
  const int64_t S = max_seq_len;
  int threads = n_threads > 0 ? n_threads : (int)std::thread::hardware_concurrency();
  if (threads < 1) threads = 1;
  if (threads > n_games) threads = (int)n_games;
  std::vector<int> status(threads, 0);
  auto work = [&](int t) {
    std::vector<int32_t> seq;
    std::vector<MoveTarget> moves;
    std::vector<ValueEntry> values;
    std::vector<Block> blocks;
    seq.reserve(4096);
    for (int64_t gi = t; gi < n_games; gi += threads) {
      GameIn g{game_offsets[gi], game_offsets[gi + 1], fen_chars, fen_offsets, played_chars, played_offsets,
               best_chars, best_offsets, played_q, played_d, include_board, start_choice[gi]};
      if (g.ply1 <= g.ply0) {
        status[t] = -5;  // a game without plies
        return;
      }
      RowOut o{input_ids + gi * S, board_target_ids + gi * S, move_target_ids + gi * S, move_mask + gi * S,
               wl_positions + gi * S, d_positions + gi * S, wl_targets + gi * S, d_targets + gi * S,
               wdl_valid + gi * S, block_id + gi * S};
      const int rc = tokenize_game(v, g, S, o, seq, moves, values, blocks);
      if (rc != 0) {
        status[t] = rc;
        return;
      }
    }
  };
  if (threads == 1) {
    work(0);
  } else {
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t) pool.emplace_back(work, t);
    for (auto& th : pool) th.join();
  }
  for (int s : status)
    if (s != 0) return s;
  return 0;
}
