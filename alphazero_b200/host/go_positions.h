// Go rules, input-plane encoder and seeded random-playout position generator.
//
// This is the synthetic-input producer for the network-evaluation path: it
// yields the same 17 binary planes the reference encoder writes
// (src/game.cpp:229-256, GoGame::encode) for positions reached by uniformly
// random legal moves from the empty board.  The rules follow the reference's
// GoGame exactly where they decide which moves are legal:
//   - pass is always legal unless the game is over (src/game.cpp:164-168);
//   - a point with an empty neighbour is always legal (src/game.cpp:189-194);
//   - otherwise captures are resolved, suicide is illegal and a move that
//     recreates the previous board is illegal (simple ko,
//     src/game.cpp:199-233);
//   - two consecutive passes end the game and area scoring decides the winner
//     (src/game.cpp:247-256, :258-315).
// History planes use the last 8 boards, most recent first, coloured relative
// to the player to move; plane 16 is all ones when black is to move.
#pragma once

#include <cstdint>
#include <vector>

namespace mgb {

constexpr int kMaxBoard = 19;
constexpr int kHistory = 8;
constexpr int kInputPlanes = 2 * kHistory + 1;  // 17

// History wire format of mg_forward_history (include/minigo_cuda.h): the
// board-history ring GoGame::encode reads (src/game.cpp:229-256), shipped as
// it is kept instead of as planes.  Word 0 holds the player to move (bits
// 0-1: 1 black, 2 white), the number h of valid boards (bits 4-7) and the
// ring slot of the current board (bits 8-10); slot top - i (mod kHistory)
// is the board i moves back, for i < h.  Then kHistory slots of
// history_slot_words(n) words, point p of a slot at bits 2 * (p % 16) and
// up of word p / 16 (0 empty, 1 black, 2 white).
constexpr int kMaxSlotWords = (kMaxBoard * kMaxBoard + 15) / 16;
inline int history_slot_words(int n) { return (n * n + 15) / 16; }
inline int history_words(int n) { return 1 + kHistory * history_slot_words(n); }

class GoPosition {
public:
    explicit GoPosition(int board_size = 19, float komi = 7.5f);

    void reset();
    bool legal(int action) const;  // action in [0, n*n]; n*n = pass
    void play(int action);         // caller guarantees legal(action)
    void encode(float* out) const; // kInputPlanes * n * n floats, plane-major
    // The same planes in the bit-packed wire format of mg_forward_packed:
    // element j = plane * n * n + point at bit j % 32 of word j / 32;
    // packed_words() words, the unused tail bits zero.
    void encode_bits(uint32_t* words) const;
    int packed_words() const { return (kInputPlanes * n_ * n_ + 31) / 32; }
    // out[a] = 1 if legal(a) else 0, for a in [0, n * n] (pass last).
    void legal_mask(uint8_t* out) const;
    // The position in the history wire format (history_words(size())
    // words): a copy of the packed ring, which play() keeps up to date one
    // board per move; the planes are expanded on the device.
    void encode_history(uint32_t* words) const;

    int size() const { return n_; }
    bool over() const { return over_; }
    int to_move() const { return to_move_; }  // 1 black, 2 white
    int winner() const { return winner_; }    // 0 draw/none, 1, 2
    int moves() const { return moves_; }
    const int8_t* board() const { return cells_; }

private:
    int n_;
    float komi_;
    int8_t cells_[kMaxBoard * kMaxBoard];
    int8_t prev_[kMaxBoard * kMaxBoard];
    bool has_prev_;
    int to_move_;
    int passes_;
    bool over_;
    int winner_;
    int moves_;
    // Circular store of the last kHistory boards; hist_len_ valid entries
    // ending at hist_top_ (the current board).
    int8_t hist_[kHistory][kMaxBoard * kMaxBoard];
    int hist_len_;
    int hist_top_;
    // The same ring at 2 bits per point (the history wire format's slots),
    // and the current board in that packing, updated stone by stone.
    uint32_t hist2_[kHistory][kMaxSlotWords];
    uint32_t cur2_[kMaxSlotWords];

    void set2(int p, int colour) {
        uint32_t& w = cur2_[p >> 4];
        const int sh = 2 * (p & 15);
        w = (w & ~(3u << sh)) | ((uint32_t)colour << sh);
    }

    int neighbours(int p, int* out) const;
    // Flood-fills the chain through p on `b`; returns its liberty count and
    // writes its points to `chain` (length in *len).
    int chain_liberties(const int8_t* b, int p, int* chain, int* len) const;
    void push_history();
    void decide_winner();
};

// Uniform draw in [0, range) from a 32-bit Mersenne Twister word by the
// multiply-shift map floor(r * range / 2^32): fully specified, so a harness
// around any other Go implementation can reproduce the same choices.
uint32_t draw_below(uint32_t r, uint32_t range);

// Writes n positions (kInputPlanes * board^2 floats each) to out.  Position i
// plays k_i = draw_below(rng(), max_moves + 1) random legal moves (pass
// included, stopping early if the game ends), drawing each move as
// legal_list[draw_below(rng(), legal_count)] where legal_list is the legal
// points in increasing index order followed by pass; rng is one
// std::mt19937 seeded with `seed` shared by all n positions.
void random_positions(int board, int n, uint32_t seed, int max_moves, float* out);
// The same positions in the history wire format, history_words(board) words
// each.
void random_histories(int board, int n, uint32_t seed, int max_moves, uint32_t* out);

}  // namespace mgb
