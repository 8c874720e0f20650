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
// The loop runs until the caller's window closes; the counters are sampled
// at the start and the end of the measured window so warm-up (first-call
// allocations, thread start-up, CUDA graph capture) stays outside it.
#pragma once

#include "config.h"
#include "game.h"
#include "mcts.h"

#include <atomic>
#include <chrono>
#include <cstdint>
#include <functional>
#include <thread>
#include <vector>

namespace mgb_selfplay {

struct Counters {
    uint64_t moves = 0;         // searches completed (one per move played)
    uint64_t games = 0;         // games finished
    uint64_t nn_positions = 0;  // positions the evaluator's engine(s) computed
    uint64_t nn_batches = 0;    // engine calls
    uint64_t gpu_launches = 0;  // kernel launches of those calls (0 on a CPU engine)
    uint64_t engine_ns = 0;     // evaluator server time in engine calls (all servers)
    uint64_t scatter_ns = 0;    // evaluator server time returning results (all servers)
    uint64_t pack_ns = 0;       // part of engine_ns spent packing planes to bits
};

struct Window {
    double seconds = 0.0;
    Counters begin, end;
};

// Runs `workers` self-play workers over `evaluator` for warmup_s + measure_s
// seconds and returns the counters at both ends of the measured window.
// `nn_counters` fills the nn_* and gpu_launches fields.  After
// the window the workers finish the search they are in; `on_stop` (if set)
// runs first, e.g. to make a slow engine answer at once so that those
// searches end quickly.
inline Window run(minigo::BatchEvaluator* evaluator, const minigo::Config& config, int workers,
                  double warmup_s, double measure_s,
                  const std::function<void(Counters&)>& nn_counters,
                  const std::function<void()>& on_stop = {}) {
    std::atomic<bool> stop{false};
    std::atomic<uint64_t> moves{0}, games{0};
    const int action_size = config.action_size();

    auto worker = [&]() {
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

    auto sample = [&](Counters& c) {
        c.moves = moves.load();
        c.games = games.load();
        nn_counters(c);
    };

    std::vector<std::thread> pool;
    pool.reserve(workers);
    for (int i = 0; i < workers; ++i) pool.emplace_back(worker);

    Window w;
    std::this_thread::sleep_for(std::chrono::duration<double>(warmup_s));
    const auto t0 = std::chrono::steady_clock::now();
    sample(w.begin);
    std::this_thread::sleep_for(std::chrono::duration<double>(measure_s));
    sample(w.end);
    w.seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    stop.store(true);
    if (on_stop) on_stop();
    for (auto& t : pool) t.join();
    return w;
}

}  // namespace mgb_selfplay
