// CudaEngine and ShardedEvaluator on a real GPU (device 0).
//   test_cuda_engine <model.onnx> <states.f32> <n> <out.f32>
// Writes n rows of (policy[action_size], value) for the Python side to check
// against the oracle, and checks the C++ interfaces on the way.
#include "cuda_engine.h"
#include "gpu_evaluator.h"

#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <stdexcept>
#include <thread>
#include <vector>

using namespace minigo;

#define CHECK(c)                                                                     \
    do {                                                                             \
        if (!(c)) {                                                                  \
            std::fprintf(stderr, "CHECK failed %s:%d: %s\n", __FILE__, __LINE__, #c); \
            std::exit(1);                                                            \
        }                                                                            \
    } while (0)

static float maxdiff(const std::vector<float>& a, const std::vector<float>& b) {
    if (a.size() != b.size()) return INFINITY;
    float m = 0;
    for (size_t i = 0; i < a.size(); ++i) m = std::fmax(m, std::fabs(a[i] - b[i]));
    return m;
}

int main(int argc, char** argv) {
    if (argc != 5) return 2;
    const int n = std::atoi(argv[3]);
    CudaEngine eng(0);
    CHECK(eng.backend_name() == "cuda");
    bool threw = false;
    try {
        eng.load_model("/nonexistent/model.onnx");
    } catch (const std::runtime_error& ex) {
        threw = std::string(ex.what()).find("Cannot open model file") != std::string::npos;
    }
    CHECK(threw);
    eng.load_model(argv[1]);
    CHECK(eng.board_size == 19 && eng.input_channels == 17 && eng.num_filters == 128 &&
          eng.num_res_blocks == 3);
    const int per = 17 * 361;
    std::vector<float> flat((size_t)n * per);
    std::ifstream(argv[2], std::ios::binary).read(reinterpret_cast<char*>(flat.data()),
                                                   flat.size() * sizeof(float));
    std::vector<std::vector<float>> states(n);
    for (int i = 0; i < n; ++i) states[i].assign(flat.begin() + (size_t)i * per, flat.begin() + (size_t)(i + 1) * per);

    CHECK(eng.predict_batch({}).empty());
    auto batch = eng.predict_batch(states);
    CHECK((int)batch.size() == n);
    for (int i = 0; i < n; i += 13) {
        auto one = eng.predict(states[i]);
        CHECK(maxdiff(one.first, batch[i].first) < 1e-5f && std::fabs(one.second - batch[i].second) < 1e-5f);
    }
    {
        std::ofstream out(argv[4], std::ios::binary);
        for (auto& r : batch) {
            out.write(reinterpret_cast<const char*>(r.first.data()), r.first.size() * sizeof(float));
            out.write(reinterpret_cast<const char*>(&r.second), sizeof(float));
        }
    }

    // Two replicas on this GPU behind one sharded evaluator, driven by
    // concurrent search threads; every result must match the direct batch.
    CudaEngine e1(0), e2(0);
    e1.load_model(argv[1]);
    e2.load_model(argv[1]);
    ShardedEvaluator sh({&e1, &e2}, 64);
    const int T = 16;
    std::atomic<int> bad{0};
    std::vector<std::thread> th;
    for (int t = 0; t < T; ++t)
        th.emplace_back([&, t] {
            NNResultBuf buf;
            for (int i = t; i < n; i += T) {
                auto r = sh.evaluate_with_buf(buf, states[i]);
                if (maxdiff(r.first, batch[i].first) > 1e-5f || std::fabs(r.second - batch[i].second) > 1e-5f)
                    bad++;
            }
        });
    for (auto& x : th) x.join();
    CHECK(bad == 0);
    CHECK(sh.shard(0).positions() + sh.shard(1).positions() == (uint64_t)n);
    CHECK(sh.shard(0).positions() > 0 && sh.shard(1).positions() > 0);
    auto all = sh.evaluate(states);
    for (int i = 0; i < n; ++i) CHECK(maxdiff(all[i].first, batch[i].first) < 1e-5f);

    // Bit-packed requests (evaluate_packed, the FastSearch path), alone and
    // mixed into batches with fp32-plane requests, give the same results.
    std::vector<std::vector<uint32_t>> words(n, std::vector<uint32_t>((per + 31) / 32));
    for (int i = 0; i < n; ++i) CHECK(CudaEngine::pack_planes(states[i].data(), per, words[i].data()));
    std::atomic<int> bad_packed{0};
    th.clear();
    for (int t = 0; t < T; ++t)
        th.emplace_back([&, t] {
            NNResultBuf buf;
            std::vector<float> p(362);
            float v = 0.0f;
            for (int i = t; i < n; i += T) {
                if ((i + t) % 2) {
                    sh.evaluate_packed(words[i].data(), (int)words[i].size(), p.data(), &v);
                    if (maxdiff(p, batch[i].first) > 1e-5f || std::fabs(v - batch[i].second) > 1e-5f) bad_packed++;
                } else {
                    auto r = sh.evaluate_with_buf(buf, states[i]);
                    if (maxdiff(r.first, batch[i].first) > 1e-5f) bad_packed++;
                }
            }
        });
    for (auto& x : th) x.join();
    CHECK(bad_packed == 0);
    std::printf("sharded ok: %llu + %llu positions\n", (unsigned long long)sh.shard(0).positions(),
                (unsigned long long)sh.shard(1).positions());
    return 0;
}
