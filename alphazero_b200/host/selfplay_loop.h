// Time-bounded self-play over any BatchEvaluator, for the end-to-end
// self-play measurement (19x19 games, 800 simulations per move, many game
// workers each with its own multi-threaded search).
//
// Each worker runs the move loop of the reference's self_play_game
// (src/mcts.cpp:470-495) through the reference's own MCTS (compiled from the
// reference tree; the reference headers config.h / game.h / mcts.h are on the
// include path): temperature 1 for the first temperature_threshold moves and
// 0 after, Dirichlet noise at the root, the trajectory step's encode, then
// the move.  A finished game starts a new one.  Training records (the 8-fold
// augmentation and the file write at the end of a game) are not produced:
// they happen once per game, not per simulation.
//
#pragma once

#include "selfplay_window.h"

#include "config.h"
#include "game.h"
#include "mcts.h"

#include <atomic>
#include <cstdint>
#include <functional>
#include <vector>

namespace mgb_selfplay {

// Runs `workers` self-play workers of the reference's search over
// `evaluator` (see run_window).
inline Window run(minigo::BatchEvaluator* evaluator, const minigo::Config& config, int workers,
                  double warmup_s, double measure_s,
                  const std::function<void(Counters&)>& nn_counters,
                  const std::function<void()>& on_stop = {}) {
    const int action_size = config.action_size();
    auto worker = [&](const std::atomic<bool>& stop, std::atomic<uint64_t>& moves,
                      std::atomic<uint64_t>& games) {
        minigo::MCTS mcts(evaluator, config);
        while (!stop.load(std::memory_order_relaxed)) {
            minigo::GoGame game(config.board_size, config.komi);
            while (!stop.load(std::memory_order_relaxed) && !game.game_over &&
                   game.move_count < config.max_moves_per_game) {
                const float temp = game.move_count < config.temperature_threshold ? 1.0f : 0.0f;
                std::vector<float> pi;
                const int action = mcts.get_action(game, pi, temp, -1, true);
                std::vector<float> state;
                game.encode(state);
                game.play(action == action_size - 1 ? minigo::PASS_MOVE : action);
                moves.fetch_add(1, std::memory_order_relaxed);
            }
            if (game.game_over || game.move_count >= config.max_moves_per_game)
                games.fetch_add(1, std::memory_order_relaxed);
        }
    };
    return run_window(workers, warmup_s, measure_s, worker, nn_counters, on_stop);
}

}  // namespace mgb_selfplay
