// Time-bounded self-play measurement: `workers` game workers play until the
// measured window closes; counters are sampled at both ends of the window so
// warm-up (first-call allocations, thread start-up, CUDA graph capture)
// stays outside it.  The worker body (which search, which board) is the
// caller's: selfplay_loop.h runs the reference's MCTS, fast_selfplay.h the
// FastSearch.
#pragma once

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
    uint64_t scatter_ns = 0;    // evaluator time returning results (all servers)
    uint64_t pack_ns = 0;       // part of engine_ns spent packing planes to bits
};

struct Window {
    double seconds = 0.0;
    Counters begin, end;
};

// One game worker: plays moves until `stop`, adding 1 to `moves` per search
// completed and to `games` per game finished.
using Worker = std::function<void(const std::atomic<bool>& stop, std::atomic<uint64_t>& moves,
                                  std::atomic<uint64_t>& games)>;

// Runs `workers` copies of `worker` for warmup_s + measure_s seconds and
// returns the counters at both ends of the measured window.  `nn_counters`
// fills the nn_* / gpu_launches / *_ns fields.  After the window the workers
// finish the search they are in; `on_stop` (if set) runs first, e.g. to make
// a slow engine answer at once so that those searches end quickly.
inline Window run_window(int workers, double warmup_s, double measure_s, const Worker& worker,
                         const std::function<void(Counters&)>& nn_counters,
                         const std::function<void()>& on_stop = {}) {
    std::atomic<bool> stop{false};
    std::atomic<uint64_t> moves{0}, games{0};
    auto sample = [&](Counters& c) {
        c.moves = moves.load();
        c.games = games.load();
        nn_counters(c);
    };
    std::vector<std::thread> pool;
    pool.reserve(workers);
    for (int i = 0; i < workers; ++i) pool.emplace_back([&] { worker(stop, moves, games); });

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
