#include "go_positions.h"

#include <array>
#include <cstring>
#include <random>
#if defined(__SSE2__)
#include <emmintrin.h>
#endif

namespace mgb {

namespace {
// Orthogonal neighbours of every point, per board size (built once).
struct NeighbourTable {
    int8_t count[kMaxBoard * kMaxBoard];
    int16_t at[kMaxBoard * kMaxBoard][4];
};

const NeighbourTable& neighbour_table(int n) {
    static const std::array<NeighbourTable, kMaxBoard + 1> tables = [] {
        std::array<NeighbourTable, kMaxBoard + 1> t{};
        for (int b = 1; b <= kMaxBoard; ++b)
            for (int p = 0; p < b * b; ++p) {
                const int r = p / b, c = p % b;
                int k = 0;
                if (r > 0) t[b].at[p][k++] = (int16_t)(p - b);
                if (r < b - 1) t[b].at[p][k++] = (int16_t)(p + b);
                if (c > 0) t[b].at[p][k++] = (int16_t)(p - 1);
                if (c < b - 1) t[b].at[p][k++] = (int16_t)(p + 1);
                t[b].count[p] = (int8_t)k;
            }
        return t;
    }();
    return tables[n];
}

// ORs the low `nbits` bits of src (64-bit words, bit i of the sequence at
// bit i % 64 of word i / 64) into words[] starting at bit `dest`.
void or_bits(uint32_t* words, int nw, int dest, const uint64_t* src, int nbits) {
    for (int k = 0; k * 64 < nbits; ++k) {
        uint64_t v = src[k];
        const int left = nbits - k * 64;
        if (left < 64) v &= (uint64_t(1) << left) - 1;
        if (v == 0) continue;
        const int bit = dest + k * 64, off = bit >> 5, sh = bit & 31;
        const uint64_t lo = v << sh;
        words[off] |= (uint32_t)lo;
        if (off + 1 < nw) words[off + 1] |= (uint32_t)(lo >> 32);
        if (sh != 0 && off + 2 < nw) words[off + 2] |= (uint32_t)(v >> (64 - sh));
    }
}
}  // namespace

GoPosition::GoPosition(int board_size, float komi) : n_(board_size), komi_(komi) {
    reset();
}

void GoPosition::reset() {
    std::memset(cells_, 0, sizeof(cells_));
    std::memset(prev_, 0, sizeof(prev_));
    std::memset(hist_, 0, sizeof(hist_));
    std::memset(hist2_, 0, sizeof(hist2_));
    std::memset(cur2_, 0, sizeof(cur2_));
    has_prev_ = false;
    to_move_ = 1;
    passes_ = 0;
    over_ = false;
    winner_ = 0;
    moves_ = 0;
    hist_len_ = 0;
    hist_top_ = kHistory - 1;
    push_history();
}

int GoPosition::neighbours(int p, int* out) const {
    const NeighbourTable& t = neighbour_table(n_);
    const int k = t.count[p];
    for (int i = 0; i < k; ++i) out[i] = t.at[p][i];
    return k;
}

int GoPosition::chain_liberties(const int8_t* b, int p, int* chain, int* len) const {
    const int8_t colour = b[p];
    uint8_t seen[kMaxBoard * kMaxBoard];
    std::memset(seen, 0, sizeof(seen));
    // bit 0: in chain, bit 1: counted as a liberty
    int head = 0, tail = 0, libs = 0;
    chain[tail++] = p;
    seen[p] = 1;
    while (head < tail) {
        int q = chain[head++];
        int nb[4];
        int k = neighbours(q, nb);
        for (int i = 0; i < k; ++i) {
            int t = nb[i];
            if (b[t] == 0) {
                if (!(seen[t] & 2)) { seen[t] |= 2; ++libs; }
            } else if (b[t] == colour && !(seen[t] & 1)) {
                seen[t] |= 1;
                chain[tail++] = t;
            }
        }
    }
    *len = tail;
    return libs;
}

bool GoPosition::legal(int action) const {
    if (over_) return false;
    const int nn = n_ * n_;
    if (action == nn) return true;
    if (action < 0 || action > nn) return false;
    if (cells_[action] != 0) return false;
    int nb[4];
    int k = neighbours(action, nb);
    for (int i = 0; i < k; ++i)
        if (cells_[nb[i]] == 0) return true;

    // Every neighbour is occupied: resolve captures on a scratch board.
    int8_t trial[kMaxBoard * kMaxBoard];
    std::memcpy(trial, cells_, sizeof(trial));
    trial[action] = (int8_t)to_move_;
    const int8_t them = (int8_t)(3 - to_move_);
    int chain[kMaxBoard * kMaxBoard];
    int len = 0;
    for (int i = 0; i < k; ++i) {
        if (trial[nb[i]] != them) continue;
        if (chain_liberties(trial, nb[i], chain, &len) == 0)
            for (int j = 0; j < len; ++j) trial[chain[j]] = 0;
    }
    if (chain_liberties(trial, action, chain, &len) == 0) return false;  // suicide
    if (has_prev_) {
        bool same = true;
        for (int q = 0; q < nn && same; ++q) same = (trial[q] == prev_[q]);
        if (same) return false;  // recreates the previous board
    }
    return true;
}

void GoPosition::play(int action) {
    const int nn = n_ * n_;
    std::memcpy(prev_, cells_, sizeof(cells_));
    has_prev_ = true;
    if (action == nn || action < 0) {
        if (++passes_ >= 2) {
            over_ = true;
            decide_winner();
        }
    } else {
        passes_ = 0;
        cells_[action] = (int8_t)to_move_;
        set2(action, to_move_);
        const int8_t them = (int8_t)(3 - to_move_);
        int nb[4];
        int k = neighbours(action, nb);
        int chain[kMaxBoard * kMaxBoard];
        int len = 0;
        for (int i = 0; i < k; ++i) {
            if (cells_[nb[i]] != them) continue;
            if (chain_liberties(cells_, nb[i], chain, &len) == 0)
                for (int j = 0; j < len; ++j) {
                    cells_[chain[j]] = 0;
                    set2(chain[j], 0);
                }
        }
    }
    ++moves_;
    to_move_ = 3 - to_move_;
    push_history();
}

void GoPosition::push_history() {
    hist_top_ = (hist_top_ + 1) % kHistory;
    std::memcpy(hist_[hist_top_], cells_, sizeof(cells_));
    std::memcpy(hist2_[hist_top_], cur2_, sizeof(uint32_t) * (size_t)history_slot_words(n_));
    if (hist_len_ < kHistory) ++hist_len_;
}

void GoPosition::encode_history(uint32_t* words) const {
    const int sw = history_slot_words(n_);
    words[0] = (uint32_t)to_move_ | ((uint32_t)hist_len_ << 4) | ((uint32_t)hist_top_ << 8);
    for (int k = 0; k < kHistory; ++k)
        std::memcpy(words + 1 + k * sw, hist2_[k], sizeof(uint32_t) * (size_t)sw);
}

void GoPosition::encode(float* out) const {
    const int nn = n_ * n_;
    std::memset(out, 0, sizeof(float) * (size_t)kInputPlanes * nn);
    const int8_t us = (int8_t)to_move_, them = (int8_t)(3 - to_move_);
    for (int i = 0; i < hist_len_; ++i) {
        const int8_t* snap = hist_[(hist_top_ - i + kHistory) % kHistory];
        float* mine = out + (size_t)i * nn;
        float* theirs = out + (size_t)(kHistory + i) * nn;
        for (int q = 0; q < nn; ++q) {
            if (snap[q] == us) mine[q] = 1.0f;
            else if (snap[q] == them) theirs[q] = 1.0f;
        }
    }
    if (to_move_ == 1) {
        float* colour = out + (size_t)2 * kHistory * nn;
        for (int q = 0; q < nn; ++q) colour[q] = 1.0f;
    }
}

void GoPosition::encode_bits(uint32_t* words) const {
    const int nn = n_ * n_;
    const int nw = packed_words();
    std::memset(words, 0, sizeof(uint32_t) * (size_t)nw);
    auto set = [&](int j) { words[j >> 5] |= 1u << (j & 31); };
    const int8_t us = (int8_t)to_move_, them = (int8_t)(3 - to_move_);
    constexpr int kW64 = (kMaxBoard * kMaxBoard + 63) / 64;
    for (int i = 0; i < hist_len_; ++i) {
        const int8_t* snap = hist_[(hist_top_ - i + kHistory) % kHistory];
        // the snapshot's two planes as bit strings, then placed at their
        // plane offsets (which are not word-aligned)
        uint64_t mine[kW64] = {}, theirs[kW64] = {};
        int q = 0;
#if defined(__SSE2__)
        // 16 points per compare; q is a multiple of 16, so a group's 16 bits
        // never straddle two 64-bit words
        const __m128i vus = _mm_set1_epi8(us), vthem = _mm_set1_epi8(them);
        for (; q + 16 <= nn; q += 16) {
            const __m128i x = _mm_loadu_si128(reinterpret_cast<const __m128i*>(snap + q));
            mine[q >> 6] |= (uint64_t)(uint32_t)_mm_movemask_epi8(_mm_cmpeq_epi8(x, vus)) << (q & 63);
            theirs[q >> 6] |= (uint64_t)(uint32_t)_mm_movemask_epi8(_mm_cmpeq_epi8(x, vthem)) << (q & 63);
        }
#endif
        for (; q < nn; ++q) {
            mine[q >> 6] |= (uint64_t)(snap[q] == us) << (q & 63);
            theirs[q >> 6] |= (uint64_t)(snap[q] == them) << (q & 63);
        }
        or_bits(words, nw, i * nn, mine, nn);
        or_bits(words, nw, (kHistory + i) * nn, theirs, nn);
    }
    if (to_move_ == 1) {
        // plane 16: bits [16 * nn, 17 * nn) all set
        int j = 2 * kHistory * nn;
        const int end = j + nn;
        for (; j < end && (j & 31); ++j) set(j);
        for (; j + 32 <= end; j += 32) words[j >> 5] = 0xffffffffu;
        for (; j < end; ++j) set(j);
    }
}

void GoPosition::legal_mask(uint8_t* out) const {
    const int nn = n_ * n_;
    if (over_) {
        std::memset(out, 0, (size_t)nn + 1);
        return;
    }
    // legal()'s fast path inline: an empty point with an empty neighbour is
    // legal; only points whose neighbours are all occupied take the full test.
    const NeighbourTable& t = neighbour_table(n_);
    for (int a = 0; a < nn; ++a) {
        if (cells_[a] != 0) {
            out[a] = 0;
            continue;
        }
        bool open = false;
        for (int i = 0; i < t.count[a]; ++i) open |= cells_[t.at[a][i]] == 0;
        out[a] = (open || legal(a)) ? 1 : 0;
    }
    out[nn] = 1;
}

void GoPosition::decide_winner() {
    const int nn = n_ * n_;
    float area[3] = {0.f, 0.f, 0.f};
    for (int q = 0; q < nn; ++q) area[cells_[q]] += 1.0f;
    uint8_t seen[kMaxBoard * kMaxBoard];
    std::memset(seen, 0, sizeof(seen));
    int region[kMaxBoard * kMaxBoard];
    for (int s = 0; s < nn; ++s) {
        if (cells_[s] != 0 || seen[s]) continue;
        int head = 0, tail = 0;
        bool touch[3] = {false, false, false};
        region[tail++] = s;
        seen[s] = 1;
        while (head < tail) {
            int q = region[head++];
            int nb[4];
            int k = neighbours(q, nb);
            for (int i = 0; i < k; ++i) {
                int t = nb[i];
                if (cells_[t] == 0) {
                    if (!seen[t]) { seen[t] = 1; region[tail++] = t; }
                } else {
                    touch[cells_[t]] = true;
                }
            }
        }
        if (touch[1] && !touch[2]) area[1] += (float)tail;
        else if (touch[2] && !touch[1]) area[2] += (float)tail;
    }
    const float black = area[1], white = area[2] + komi_;
    winner_ = black > white ? 1 : (white > black ? 2 : 0);
}

uint32_t draw_below(uint32_t r, uint32_t range) {
    return (uint32_t)(((uint64_t)r * (uint64_t)range) >> 32);
}

namespace {
// The seeded random-playout procedure of random_positions; emit(i, g)
// receives position i.
template <typename Emit>
void random_playouts(int board, int n, uint32_t seed, int max_moves, Emit&& emit) {
    std::mt19937 rng(seed);
    const int nn = board * board;
    std::vector<int> legal_list;
    legal_list.reserve(nn + 1);
    for (int i = 0; i < n; ++i) {
        GoPosition g(board);
        const int k = (int)draw_below(rng(), (uint32_t)max_moves + 1u);
        for (int m = 0; m < k && !g.over(); ++m) {
            legal_list.clear();
            for (int a = 0; a < nn; ++a)
                if (g.legal(a)) legal_list.push_back(a);
            legal_list.push_back(nn);
            g.play(legal_list[draw_below(rng(), (uint32_t)legal_list.size())]);
        }
        emit(i, g);
    }
}
}  // namespace

void random_positions(int board, int n, uint32_t seed, int max_moves, float* out) {
    const size_t per = (size_t)kInputPlanes * board * board;
    random_playouts(board, n, seed, max_moves,
                    [&](int i, const GoPosition& g) { g.encode(out + (size_t)i * per); });
}

void random_histories(int board, int n, uint32_t seed, int max_moves, uint32_t* out) {
    const size_t per = (size_t)history_words(board);
    random_playouts(board, n, seed, max_moves,
                    [&](int i, const GoPosition& g) { g.encode_history(out + (size_t)i * per); });
}

}  // namespace mgb
