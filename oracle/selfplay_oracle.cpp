// ORACLE - test infrastructure only: the CPU arm of the end-to-end self-play
// measurement.  The reference's own stack as its selfplay binary runs it
// with the Eigen backend (src/main_selfplay.cpp:66-84): src/mcts.cpp,
// src/game.cpp, src/nn_evaluator.cpp and src/onnx_loader.cpp compiled
// unmodified from the reference tree, with the engine replaced by the C
// restatement of src/eigen_engine.cpp (eigen_restated.c; Eigen3 is absent, so
// the reference engine itself does not compile).  Like the reference engine
// it evaluates a batch as a serial loop on one core (threads = 1,
// include/inference_engine.h:25-32).  Built by oracle/Makefile into
// oracle/_ref/selfplay_oracle; same flags and JSON line as selfplay_cuda
// (alphazero_b200/host/selfplay_main.cpp).
#include "eigen_restated.h"
#include "nn_evaluator.h"
#include "onnx_loader.h"
#include "selfplay_loop.h"

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

using namespace minigo;

namespace {

class OracleEngine : public InferenceEngine {
public:
    std::atomic<uint64_t> positions{0}, batches{0};
    // Set once the measured window is over: batches are answered with a
    // uniform policy and value 0 at once, so the searches in progress (which
    // would need minutes of one-core evaluation) end promptly.
    std::atomic<bool> drain{false};

    ~OracleEngine() override { orc_free(net_); }

    void load_model(const std::string& path) override {
        net_ = orc_new();
        for (const auto& t : onnx_parser::parse_onnx_file(path)) {
            const std::vector<float> v = t.get_floats();
            orc_set(net_, t.name.c_str(), t.dims.data(), (int)t.dims.size(), v.data());
        }
        char err[256] = {0};
        if (orc_finalize(net_, err, sizeof(err)) != 0) throw std::runtime_error(err);
        int actions = 0;
        orc_info(net_, &board_size, &input_channels, &num_filters, &num_res_blocks, &actions);
        actions_ = actions;
    }

    std::pair<std::vector<float>, float> predict(const std::vector<float>& state) override {
        return predict_batch({state})[0];
    }

    std::vector<std::pair<std::vector<float>, float>> predict_batch(
        const std::vector<std::vector<float>>& states) override {
        const int n = (int)states.size();
        if (n == 0) return {};
        if (drain.load())
            return std::vector<std::pair<std::vector<float>, float>>(
                n, {std::vector<float>(actions_, 1.0f / actions_), 0.0f});
        const size_t per = states[0].size();
        std::vector<float> in((size_t)n * per), probs((size_t)n * actions_), values(n);
        for (int i = 0; i < n; ++i) std::memcpy(in.data() + i * per, states[i].data(), per * 4);
        if (orc_predict_batch(net_, in.data(), n, ORC_LITERAL, 1, probs.data(), nullptr,
                              values.data()) != 0)
            throw std::runtime_error("oracle predict failed");
        std::vector<std::pair<std::vector<float>, float>> out(n);
        for (int i = 0; i < n; ++i)
            out[i] = {std::vector<float>(probs.begin() + (size_t)i * actions_,
                                         probs.begin() + (size_t)(i + 1) * actions_),
                      values[i]};
        positions.fetch_add((uint64_t)n);
        batches.fetch_add(1);
        return out;
    }

    std::string backend_name() const override { return "eigen (C restatement)"; }

private:
    orc_net* net_ = nullptr;
    int actions_ = 0;
};

}  // namespace

int main(int argc, char** argv) {
    std::string model;
    int workers = 64, search_threads = 16, sims = 800, max_batch = 512;
    double warmup_s = 5.0, measure_s = 20.0;
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        if (i + 1 >= argc) {
            std::fprintf(stderr, "missing value after %s\n", a.c_str());
            return 2;
        }
        const char* v = argv[++i];
        if (a == "--model") model = v;
        else if (a == "--workers") workers = std::atoi(v);
        else if (a == "--search-threads") search_threads = std::atoi(v);
        else if (a == "--sims") sims = std::atoi(v);
        else if (a == "--max-batch") max_batch = std::atoi(v);
        else if (a == "--warmup-seconds") warmup_s = std::atof(v);
        else if (a == "--seconds") measure_s = std::atof(v);
        else if (a == "--gpus" || a == "--precision") continue;  // accepted, unused
        else {
            std::fprintf(stderr, "unknown argument %s\n", a.c_str());
            return 2;
        }
    }
    if (model.empty()) {
        std::fprintf(stderr, "usage: selfplay_oracle --model M.onnx ...\n");
        return 2;
    }
    try {
        OracleEngine engine;
        engine.load_model(model);
        NNEvaluator evaluator(&engine, max_batch);

        Config config;
        config.board_size = engine.board_size;
        config.input_channels = engine.input_channels;
        config.num_filters = engine.num_filters;
        config.num_res_blocks = engine.num_res_blocks;
        config.max_moves_per_game = config.board_size * config.board_size * 2;
        config.num_search_threads = search_threads;
        config.num_simulations = sims;
        config.max_batch_size = max_batch;

        auto nn = [&](mgb_selfplay::Counters& c) {
            c.nn_positions = engine.positions.load();
            c.nn_batches = engine.batches.load();
        };
        const mgb_selfplay::Window w = mgb_selfplay::run(
            &evaluator, config, workers, warmup_s, measure_s, nn, [&] { engine.drain = true; });
        const double moves = (double)(w.end.moves - w.begin.moves);
        const double pos = (double)(w.end.nn_positions - w.begin.nn_positions);
        const double bat = (double)(w.end.nn_batches - w.begin.nn_batches);
        std::printf(
            "{\"visits_per_s\": %.3f, \"nn_positions_per_s\": %.3f, \"moves_per_s\": %.4f, "
            "\"mean_batch\": %.2f, \"seconds\": %.3f, \"moves\": %.0f, \"games_finished\": %llu, "
            "\"gpus\": 0, \"workers\": %d, \"search_threads\": %d, \"sims\": %d, "
            "\"max_batch\": %d, \"board\": %d, \"filters\": %d, \"blocks\": %d, "
            "\"host_threads\": %u, \"failed_batches\": 0}\n",
            moves * sims / w.seconds, pos / w.seconds, moves / w.seconds, bat > 0 ? pos / bat : 0.0,
            w.seconds, moves, (unsigned long long)(w.end.games - w.begin.games), workers,
            search_threads, sims, max_batch, config.board_size, config.num_filters,
            config.num_res_blocks, std::thread::hardware_concurrency());
        std::fflush(stdout);
    } catch (const std::exception& e) {
        std::fprintf(stderr, "selfplay_oracle: %s\n", e.what());
        return 1;
    }
    return 0;
}
