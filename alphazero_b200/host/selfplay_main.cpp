// selfplay_cuda: end-to-end self-play throughput of this backend.
//
// The reference's own search (src/mcts.cpp, src/game.cpp, compiled unmodified
// from the reference tree) plays games through a ShardedEvaluator: one
// GpuEvaluator batching server and one CudaEngine per GPU, weights replicated,
// each search thread bound to one GPU round-robin.  This is what the
// reference's selfplay binary runs once the backend is wired in
// (src/main_selfplay.cpp:66-84 with create_engine returning a CudaEngine),
// minus the game-record file writes.
//
//   selfplay_cuda --model M.onnx [--gpus N] [--workers 64] [--search-threads 16]
//                 [--sims 800] [--max-batch 512] [--warmup-seconds 10]
//                 [--seconds 30] [--precision bf16|fp16|fp32]
//                 [--servers-per-gpu K] [--search reference|fast|grouped]
//
// --search fast replaces the reference's search with FastSearch
// (fast_search.h: the same algorithm at a lower host cost per visit, boards
// encoded straight to the bit-packed wire format).  --search grouped runs
// FastSearch's grouped mode: each game worker's search-threads concurrent
// playouts as rounds on the worker's own thread, a round's leaves evaluated
// as one group (SearchParams::grouped).
//
//   selfplay_cuda --model M.onnx --search fast --games N [--records DIR] ...
//
// plays N whole games instead of a timed window, like the reference's
// selfplay binary (src/main_selfplay.cpp:86-122), and writes each game's
// 8-fold augmented training records to DIR/game_<i>.bin in its format.
// With K > 1 each GPU gets K engines (each its own weights copy, stream and
// buffers) and K batching servers, so one server's host work (gathering the
// batch, waking its clients) overlaps another's GPU work.
//
// Prints one JSON line: MCTS visits/s (searches completed in the measured
// window x simulations per search), NN positions/s and mean batch size.
#include "cuda_engine.h"
#include "fast_selfplay.h"
#include "gpu_evaluator.h"
#include "selfplay_loop.h"
#include "selfplay_records.h"

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <thread>
#include <vector>

using namespace minigo;

int main(int argc, char** argv) {
    std::string model;
    int gpus = 1, workers = 64, search_threads = 16, sims = 800, max_batch = 512, per_gpu = 1;
    double warmup_s = 10.0, measure_s = 30.0;
    CudaEngine::Precision prec = CudaEngine::kBf16;
    bool fast = false, grouped = false;
    int games = 0;
    std::string records_dir;
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        auto next = [&]() -> const char* {
            if (i + 1 >= argc) {
                std::fprintf(stderr, "missing value after %s\n", a.c_str());
                std::exit(2);
            }
            return argv[++i];
        };
        if (a == "--model") model = next();
        else if (a == "--gpus") gpus = std::atoi(next());
        else if (a == "--workers") workers = std::atoi(next());
        else if (a == "--search-threads") search_threads = std::atoi(next());
        else if (a == "--sims") sims = std::atoi(next());
        else if (a == "--max-batch") max_batch = std::atoi(next());
        else if (a == "--servers-per-gpu") per_gpu = std::atoi(next());
        else if (a == "--games") games = std::atoi(next());
        else if (a == "--records") records_dir = next();
        else if (a == "--search") {
            const std::string v = next();
            if (v != "fast" && v != "reference" && v != "grouped") {
                std::fprintf(stderr, "--search takes reference, fast or grouped\n");
                return 2;
            }
            fast = v != "reference";
            grouped = v == "grouped";
        }
        else if (a == "--warmup-seconds") warmup_s = std::atof(next());
        else if (a == "--seconds") measure_s = std::atof(next());
        else if (a == "--precision") {
            const std::string p = next();
            prec = p == "fp16" ? CudaEngine::kFp16 : (p == "fp32" ? CudaEngine::kFp32 : CudaEngine::kBf16);
        } else {
            std::fprintf(stderr, "unknown argument %s\n", a.c_str());
            return 2;
        }
    }
    if (model.empty() || gpus < 1 || workers < 1 || search_threads < 1 || sims < 1 || max_batch < 1 ||
        per_gpu < 1) {
        std::fprintf(stderr, "usage: selfplay_cuda --model M.onnx [--gpus N] ...\n");
        return 2;
    }
    try {
        std::vector<std::unique_ptr<CudaEngine>> engines;
        std::vector<InferenceEngine*> raw;
        for (int k = 0; k < per_gpu; ++k)
            for (int d = 0; d < gpus; ++d) {
                engines.push_back(std::make_unique<CudaEngine>(d, prec, false, max_batch));
                engines.back()->load_model(model);
                raw.push_back(engines.back().get());
            }
        ShardedEvaluator evaluator(raw, max_batch);

        Config config;
        config.board_size = engines[0]->board_size;
        config.input_channels = engines[0]->input_channels;
        config.num_filters = engines[0]->num_filters;
        config.num_res_blocks = engines[0]->num_res_blocks;
        config.max_moves_per_game = config.board_size * config.board_size * 2;
        config.num_search_threads = search_threads;
        config.num_simulations = sims;
        config.max_batch_size = max_batch;

        auto nn = [&](mgb_selfplay::Counters& c) {
            c.nn_positions = c.nn_batches = c.gpu_launches = c.engine_ns = c.scatter_ns = 0;
            for (size_t s = 0; s < evaluator.shards(); ++s) {
                c.nn_positions += evaluator.shard(s).positions();
                c.nn_batches += evaluator.shard(s).batches();
                c.engine_ns += evaluator.shard(s).engine_ns();
                c.scatter_ns += evaluator.shard(s).scatter_ns();
            }
            for (const auto& e : engines) {
                c.gpu_launches += e->kernel_launches();
                c.pack_ns += e->pack_ns();
            }
        };
        if (games > 0) {
            if (!fast) {
                std::fprintf(stderr, "--games needs --search fast\n");
                return 2;
            }
            mgb::SearchParams sp;
            sp.simulations = sims;
            sp.c_puct = config.c_puct;
            sp.dirichlet_alpha = config.dirichlet_alpha;
            sp.dirichlet_epsilon = config.dirichlet_epsilon;
            sp.threads = search_threads;
            sp.grouped = grouped;
            std::atomic<int> next_game{0};
            std::atomic<uint64_t> moves{0}, records{0};
            const auto t0 = std::chrono::steady_clock::now();
            std::vector<std::thread> pool;
            for (int i = 0; i < workers; ++i)
                pool.emplace_back([&, i] {
                    mgb::FastSearch search(&evaluator, config.board_size, sp, 1000 + (uint64_t)i);
                    for (int g; (g = next_game.fetch_add(1)) < games;) {
                        auto recs = mgb::self_play_game(search, config.board_size, config.komi,
                                                        config.max_moves_per_game,
                                                        config.temperature_threshold);
                        moves += recs.size() / 8;
                        records += recs.size();
                        if (!records_dir.empty())
                            mgb::write_records(records_dir + "/game_" + std::to_string(g) + ".bin", recs);
                    }
                });
            for (auto& t : pool) t.join();
            const double secs =
                std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
            std::printf("{\"games\": %d, \"seconds\": %.3f, \"moves\": %llu, \"records\": %llu, "
                        "\"visits_per_s\": %.3f, \"seconds_per_game\": %.3f}\n",
                        games, secs, (unsigned long long)moves.load(), (unsigned long long)records.load(),
                        (double)moves.load() * sims / secs, secs / games);
            std::fflush(stdout);
            return 0;
        }
        mgb_selfplay::Window w;
        if (fast) {
            mgb_selfplay::FastGameParams fp;
            fp.board = config.board_size;
            fp.komi = config.komi;
            fp.max_moves = config.max_moves_per_game;
            fp.temperature_threshold = config.temperature_threshold;
            fp.search.simulations = sims;
            fp.search.c_puct = config.c_puct;
            fp.search.dirichlet_alpha = config.dirichlet_alpha;
            fp.search.dirichlet_epsilon = config.dirichlet_epsilon;
            fp.search.threads = search_threads;
            fp.search.grouped = grouped;
            w = mgb_selfplay::run_fast(&evaluator, fp, workers, warmup_s, measure_s, nn);
        } else {
            w = mgb_selfplay::run(&evaluator, config, workers, warmup_s, measure_s, nn);
        }

        const double moves = (double)(w.end.moves - w.begin.moves);
        const double pos = (double)(w.end.nn_positions - w.begin.nn_positions);
        const double bat = (double)(w.end.nn_batches - w.begin.nn_batches);
        uint64_t failed = 0;
        for (size_t s = 0; s < evaluator.shards(); ++s) failed += evaluator.shard(s).failed_batches();
        std::printf(
            "{\"visits_per_s\": %.3f, \"nn_positions_per_s\": %.3f, \"moves_per_s\": %.4f, "
            "\"mean_batch\": %.2f, \"seconds\": %.3f, \"moves\": %.0f, \"games_finished\": %llu, "
            "\"search\": \"%s\", \"gpus\": %d, \"servers_per_gpu\": %d, \"workers\": %d, \"search_threads\": %d, \"sims\": %d, "
            "\"max_batch\": %d, \"board\": %d, \"filters\": %d, \"blocks\": %d, "
            "\"host_threads\": %u, \"failed_batches\": %llu, \"gpu_launches\": %llu, "
            "\"server_engine_frac\": %.3f, \"server_pack_frac\": %.3f, \"server_scatter_frac\": %.3f}\n",
            moves * sims / w.seconds, pos / w.seconds, moves / w.seconds, bat > 0 ? pos / bat : 0.0,
            w.seconds, moves, (unsigned long long)(w.end.games - w.begin.games), grouped ? "grouped" : (fast ? "fast" : "reference"),
            gpus, per_gpu, workers,
            search_threads, sims, max_batch, config.board_size, config.num_filters,
            config.num_res_blocks, std::thread::hardware_concurrency(),
            (unsigned long long)failed,
            (unsigned long long)(w.end.gpu_launches - w.begin.gpu_launches),
            (double)(w.end.engine_ns - w.begin.engine_ns) * 1e-9 / w.seconds / evaluator.shards(),
            (double)(w.end.pack_ns - w.begin.pack_ns) * 1e-9 / w.seconds / evaluator.shards(),
            (double)(w.end.scatter_ns - w.begin.scatter_ns) * 1e-9 / w.seconds / evaluator.shards());
        std::fflush(stdout);
    } catch (const std::exception& e) {
        std::fprintf(stderr, "selfplay_cuda: %s\n", e.what());
        return 1;
    }
    return 0;
}
