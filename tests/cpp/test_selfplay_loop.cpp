// The time-bounded self-play loop (alphazero_b200/host/selfplay_loop.h)
// driving the reference's own MCTS (src/mcts.cpp, src/game.cpp, compiled from
// the reference tree) through a ShardedEvaluator over two fake engines: no
// GPU.  Checks that searches complete inside the measured window, that every
// evaluation of the window went through the engines, and that both shards
// received work.  Exit code 0 = pass.
#include "gpu_evaluator.h"
#include "selfplay_loop.h"

#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

using namespace minigo;

#define CHECK(c)                                                                       \
    do {                                                                               \
        if (!(c)) {                                                                    \
            std::fprintf(stderr, "CHECK failed %s:%d: %s\n", __FILE__, __LINE__, #c); \
            std::abort();                                                              \
        }                                                                              \
    } while (0)

// Uniform policy over the actions, value from the colour plane: enough for
// the search to run real games.
class UniformEngine : public InferenceEngine {
public:
    explicit UniformEngine(int board) {
        board_size = board;
        input_channels = 17;
        num_filters = 8;
        num_res_blocks = 1;
    }
    std::atomic<long> calls{0}, positions{0};
    void load_model(const std::string&) override {}
    std::string backend_name() const override { return "uniform"; }
    std::pair<std::vector<float>, float> predict(const std::vector<float>& st) override {
        const int hw = board_size * board_size;
        CHECK((int)st.size() == 17 * hw);
        std::vector<float> p(hw + 1, 1.0f / (hw + 1));
        return {p, st[16 * hw] > 0.5f ? 0.1f : -0.1f};
    }
    std::vector<std::pair<std::vector<float>, float>> predict_batch(
        const std::vector<std::vector<float>>& states) override {
        calls.fetch_add(1);
        positions.fetch_add((long)states.size());
        std::vector<std::pair<std::vector<float>, float>> out;
        for (const auto& s : states) out.push_back(predict(s));
        return out;
    }
};

int main() {
    const int board = 9, sims = 48;
    UniformEngine e0(board), e1(board);
    ShardedEvaluator ev({&e0, &e1}, 64);

    Config config;
    config.board_size = board;
    config.max_moves_per_game = board * board * 2;
    config.num_search_threads = 4;
    config.num_simulations = sims;
    config.max_batch_size = 64;

    auto nn = [&](mgb_selfplay::Counters& c) {
        c.nn_positions = ev.shard(0).positions() + ev.shard(1).positions();
        c.nn_batches = ev.shard(0).batches() + ev.shard(1).batches();
    };
    const mgb_selfplay::Window w = mgb_selfplay::run(&ev, config, 6, 0.5, 1.5, nn);

    const uint64_t moves = w.end.moves - w.begin.moves;
    const uint64_t pos = w.end.nn_positions - w.begin.nn_positions;
    std::printf("window %.2f s: %llu moves, %llu games, %llu positions in %llu batches\n", w.seconds,
                (unsigned long long)moves, (unsigned long long)(w.end.games - w.begin.games),
                (unsigned long long)pos,
                (unsigned long long)(w.end.nn_batches - w.begin.nn_batches));
    CHECK(w.seconds >= 1.4 && w.seconds < 5.0);
    CHECK(moves > 0);
    // every search evaluates its root plus (up to) one leaf per simulation
    CHECK(pos > 0 && pos <= (moves + 12) * (uint64_t)(sims + config.num_search_threads + 1));
    CHECK(e0.positions.load() > 0 && e1.positions.load() > 0);
    CHECK(ev.shard(0).failed_batches() == 0 && ev.shard(1).failed_batches() == 0);
    CHECK((long)(ev.shard(0).positions() + ev.shard(1).positions()) ==
          e0.positions.load() + e1.positions.load());
    std::printf("selfplay loop ok\n");
    return 0;
}
