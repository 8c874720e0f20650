// FastSearch and GoPosition (alphazero_b200/host) against the reference's
// own src/mcts.cpp and src/game.cpp, compiled from the reference tree into
// this test: no GPU.
//   1. rules: random games played move by move on both boards give the
//      same board, legal moves, encoded planes (fp32 and bit-packed) and
//      winner;
//   2. search: one search thread, no root noise, the same deterministic
//      network on both sides: the root visit counts are identical;
//   3. the thread pool: 8 search threads complete the playouts (the root's
//      children hold between sims and sims + 7 visits) over repeated
//      searches;
//   4. an evaluation failure surfaces as an exception from search() and the
//      searcher keeps working;
//   5. the grouped mode (the playouts of a round evaluated as one group on
//      the calling thread): with one playout per round it visits exactly
//      what the reference's single-threaded search does; with 16 it
//      completes exactly the requested playouts; failures surface as in 4.
// Exit code 0 = pass.
#include "fast_search.h"
#include "go_positions.h"

#include "batch_evaluator.h"
#include "config.h"
#include "game.h"
#include "mcts.h"

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <stdexcept>
#include <thread>
#include <vector>

#define CHECK(c)                                                                       \
    do {                                                                               \
        if (!(c)) {                                                                    \
            std::fprintf(stderr, "CHECK failed %s:%d: %s\n", __FILE__, __LINE__, #c); \
            std::abort();                                                              \
        }                                                                              \
    } while (0)

namespace {

std::vector<float> unpack(const uint32_t* w, int n) {
    std::vector<float> out(n);
    for (int j = 0; j < n; ++j) out[j] = (float)((w[j >> 5] >> (j & 31)) & 1u);
    return out;
}

// A deterministic stand-in network over the fp32 planes: a position hash
// picks the policy weights and the value.
void fake_net(const std::vector<float>& planes, int actions, std::vector<float>& policy, float& value) {
    uint32_t h = 2166136261u;
    for (size_t j = 0; j < planes.size(); ++j)
        if (planes[j] != 0.0f) h = (h ^ (uint32_t)j) * 16777619u;
    policy.assign(actions, 0.0f);
    float sum = 0.0f;
    for (int a = 0; a < actions; ++a) {
        policy[a] = 1.0f + (float)((h >> (a % 24)) % 97u) / 97.0f;
        sum += policy[a];
    }
    for (auto& p : policy) p /= sum;
    value = (float)((int)(h % 201u) - 100) / 100.0f;
}

class FakeBatch : public minigo::BatchEvaluator {
public:
    explicit FakeBatch(int actions) : actions_(actions) {}
    std::vector<Result> evaluate(const std::vector<std::vector<float>>& states) override {
        std::vector<Result> out;
        for (const auto& s : states) {
            Result r;
            fake_net(s, actions_, r.first, r.second);
            out.push_back(std::move(r));
        }
        return out;
    }

private:
    int actions_;
};

class FakePacked : public mgb::PackedEvaluator {
public:
    FakePacked(int board, int fail_at = -1) : board_(board), fail_at_(fail_at) {}
    std::atomic<int> calls{0};
    std::atomic<int> delay_us{0};
    void evaluate_packed(const uint32_t* words, int n_words, float* policy, float* value) override {
        const int n = 17 * board_ * board_;
        CHECK(n_words == (n + 31) / 32);
        const int c = calls.fetch_add(1);
        if (c == fail_at_) throw std::runtime_error("injected evaluation failure");
        if (delay_us.load()) std::this_thread::sleep_for(std::chrono::microseconds(delay_us.load()));
        std::vector<float> p;
        float v;
        fake_net(unpack(words, n), board_ * board_ + 1, p, v);
        std::copy(p.begin(), p.end(), policy);
        *value = v;
    }

private:
    int board_, fail_at_;
};

void check_rules(int board, int games, uint32_t seed) {
    std::mt19937 rng(seed);
    const int nn = board * board;
    std::vector<float> ref_legal, ref_enc, enc(17 * nn);
    std::vector<uint8_t> legal(nn + 1);
    std::vector<uint32_t> words;
    for (int g = 0; g < games; ++g) {
        minigo::GoGame ref(board, 7.5f);
        mgb::GoPosition pos(board, 7.5f);
        words.assign(pos.packed_words(), 0);
        for (int m = 0; m < 4 * nn && !ref.game_over; ++m) {
            for (int q = 0; q < nn; ++q) CHECK((int)ref.board[q / board][q % board] == (int)pos.board()[q]);
            CHECK(ref.current_player == pos.to_move());
            ref.get_legal_moves(ref_legal);
            pos.legal_mask(legal.data());
            std::vector<int> moves;
            for (int a = 0; a <= nn; ++a) {
                CHECK((ref_legal[a] != 0.0f) == (legal[a] != 0));
                if (legal[a]) moves.push_back(a);
            }
            ref.encode(ref_enc);
            pos.encode(enc.data());
            CHECK(ref_enc == enc);
            pos.encode_bits(words.data());
            CHECK(unpack(words.data(), 17 * nn) == ref_enc);
            for (int j = 17 * nn; j < pos.packed_words() * 32; ++j) CHECK(((words[j >> 5] >> (j & 31)) & 1u) == 0);
            // pass rarely, so that games run long and reach captures and ko
            int a = moves[rng() % moves.size()];
            if (a == nn && moves.size() > 1 && rng() % 8) a = moves[rng() % (moves.size() - 1)];
            ref.play(a == nn ? minigo::PASS_MOVE : a);
            pos.play(a);
            CHECK(ref.game_over == pos.over());
        }
        if (ref.game_over) CHECK((int)ref.winner == pos.winner());
    }
}

void check_search_parity(int board, int sims, uint32_t seed, bool grouped = false) {
    const int actions = board * board + 1;
    std::mt19937 rng(seed);
    FakeBatch ref_eval(actions);
    FakePacked fast_eval(board);
    minigo::Config cfg;
    cfg.board_size = board;
    cfg.num_simulations = sims;
    cfg.num_search_threads = 1;
    minigo::MCTS ref_mcts(&ref_eval, cfg);
    mgb::SearchParams sp;
    sp.simulations = sims;
    sp.threads = 1;
    sp.grouped = grouped;
    mgb::FastSearch fast(&fast_eval, board, sp, 7);
    minigo::GoGame ref(board, 7.5f);
    mgb::GoPosition pos(board, 7.5f);
    int compared = 0;
    for (int m = 0; m < 24 && !ref.game_over; ++m) {
        std::vector<float> rv, fv;
        ref_mcts.search(ref, rv, sims, false);
        fast.search(pos, fv, false);
        CHECK(rv.size() == fv.size());
        for (size_t a = 0; a < rv.size(); ++a) {
            if (rv[a] != fv[a]) {
                std::fprintf(stderr, "board %d move %d action %zu: reference %g visits, fast %g\n", board, m,
                             a, rv[a], fv[a]);
                std::abort();
            }
        }
        ++compared;
        // continue the game with a random legal move
        std::vector<float> legal;
        ref.get_legal_moves(legal);
        std::vector<int> moves;
        for (int a = 0; a < actions; ++a)
            if (legal[a] != 0.0f) moves.push_back(a);
        const int a = moves[rng() % moves.size()];
        ref.play(a == actions - 1 ? minigo::PASS_MOVE : a);
        pos.play(a);
    }
    CHECK(compared > 0);
}

void check_pool(int board, int sims, int threads, bool grouped = false) {
    FakePacked ev(board);
    ev.delay_us = 20;
    mgb::SearchParams sp;
    sp.simulations = sims;
    sp.threads = threads;
    sp.grouped = grouped;
    mgb::FastSearch fast(&ev, board, sp, 11);
    mgb::GoPosition pos(board, 7.5f);
    for (int m = 0; m < 6; ++m) {
        std::vector<float> visits, pi;
        fast.search(pos, visits, true);
        double total = 0;
        for (float v : visits) total += v;
        if (grouped) CHECK(total == sims);  // a round never overshoots
        else CHECK(total >= sims && total <= sims + threads - 1);
        const int a = fast.get_action(pos, pi, 1.0f, true);
        CHECK(a >= 0 && a <= board * board && pos.legal(a));
        pos.play(a);
    }
}

void check_failure(int board, bool grouped = false) {
    FakePacked ev(board, 40);
    mgb::SearchParams sp;
    sp.simulations = 100;
    sp.threads = 4;
    sp.grouped = grouped;
    mgb::FastSearch fast(&ev, board, sp, 3);
    mgb::GoPosition pos(board, 7.5f);
    std::vector<float> visits;
    bool threw = false;
    try {
        fast.search(pos, visits, false);
    } catch (const std::runtime_error& e) {
        threw = std::string(e.what()).find("injected") != std::string::npos;
    }
    CHECK(threw);
    fast.search(pos, visits, false);  // the searcher still works
    double total = 0;
    for (float v : visits) total += v;
    CHECK(total >= 100 && total <= 103);
}

}  // namespace

int main() {
    check_rules(9, 40, 1);
    check_rules(19, 6, 2);
    std::printf("rules ok\n");
    check_search_parity(9, 300, 3);
    check_search_parity(19, 200, 4);
    std::printf("search parity ok\n");
    check_pool(9, 400, 8);
    check_pool(19, 300, 8);
    std::printf("pool ok\n");
    check_failure(9);
    std::printf("failure ok\n");
    check_search_parity(9, 300, 5, true);
    check_search_parity(19, 200, 6, true);
    check_pool(9, 400, 16, true);
    check_pool(19, 300, 16, true);
    check_failure(9, true);
    std::printf("grouped ok\n");
    std::printf("fast search tests passed\n");
    return 0;
}
