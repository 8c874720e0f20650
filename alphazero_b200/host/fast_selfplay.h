// Self-play workers on FastSearch (the same move loop as selfplay_loop.h,
// src/mcts.cpp:470-495: temperature 1 for the first 30 moves and 0 after,
// Dirichlet noise at the root, the trajectory step's encode, the move), with
// positions encoded straight to the bit-packed wire format.
#pragma once

#include "fast_search.h"
#include "go_positions.h"
#include "selfplay_window.h"

#include <atomic>
#include <cstdint>
#include <functional>
#include <vector>

namespace mgb_selfplay {

struct FastGameParams {
    int board = 19;
    float komi = 7.5f;
    int max_moves = 19 * 19 * 2;   // Config::max_moves_per_game
    int temperature_threshold = 30;
    mgb::SearchParams search;
    uint64_t seed = 1;
};

inline Window run_fast(mgb::PackedEvaluator* evaluator, const FastGameParams& p, int workers,
                       double warmup_s, double measure_s,
                       const std::function<void(Counters&)>& nn_counters) {
    std::atomic<uint64_t> next_seed{p.seed};
    auto worker = [&](const std::atomic<bool>& stop, std::atomic<uint64_t>& moves,
                      std::atomic<uint64_t>& games) {
        mgb::FastSearch search(evaluator, p.board, p.search, next_seed.fetch_add(1));
        std::vector<uint32_t> step;
        while (!stop.load(std::memory_order_relaxed)) {
            mgb::GoPosition game(p.board, p.komi);
            step.resize(game.packed_words());
            while (!stop.load(std::memory_order_relaxed) && !game.over() && game.moves() < p.max_moves) {
                const float temp = game.moves() < p.temperature_threshold ? 1.0f : 0.0f;
                std::vector<float> pi;
                const int action = search.get_action(game, pi, temp, true);
                game.encode_bits(step.data());
                game.play(action);
                moves.fetch_add(1, std::memory_order_relaxed);
            }
            if (game.over() || game.moves() >= p.max_moves) games.fetch_add(1, std::memory_order_relaxed);
        }
    };
    return run_window(workers, warmup_s, measure_s, worker, nn_counters);
}

}  // namespace mgb_selfplay
