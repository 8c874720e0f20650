// Host-side tests of the batching servers (GpuEvaluator, ShardedEvaluator)
// with a fake engine: no GPU.  Exit code 0 = pass; failures print and abort.
#include "gpu_evaluator.h"

#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <set>
#include <stdexcept>
#include <thread>
#include <vector>

using namespace minigo;

#define CHECK(c)                                                              \
    do {                                                                      \
        if (!(c)) {                                                           \
            std::fprintf(stderr, "CHECK failed %s:%d: %s\n", __FILE__, __LINE__, #c); \
            std::abort();                                                     \
        }                                                                     \
    } while (0)

// Deterministic stand-in: policy[a] = (a + 1) * s / norm, value = tanh(s),
// with s = sum(state) / size.  Records batch sizes; can fail on request.
class FakeEngine : public InferenceEngine {
public:
    int actions = 10;
    std::atomic<int> fail_next{0};
    std::atomic<int> delay_us{0};
    std::mutex mu;
    std::vector<int> batch_sizes;
    std::atomic<int> in_flight{0};
    std::atomic<bool> overlapped{false};

    void load_model(const std::string&) override {}
    std::string backend_name() const override { return "fake"; }

    static std::pair<std::vector<float>, float> expected(const std::vector<float>& st, int actions) {
        double s = 0;
        for (float x : st) s += x;
        s /= std::max<size_t>(1, st.size());
        std::vector<float> p(actions);
        double norm = 0;
        for (int a = 0; a < actions; ++a) norm += (a + 1) * (1.0 + s);
        for (int a = 0; a < actions; ++a) p[a] = (float)((a + 1) * (1.0 + s) / norm);
        return {p, (float)std::tanh(s)};
    }

    std::pair<std::vector<float>, float> predict(const std::vector<float>& st) override {
        return expected(st, actions);
    }

    std::vector<std::pair<std::vector<float>, float>> predict_batch(
        const std::vector<std::vector<float>>& states) override {
        if (in_flight.fetch_add(1) != 0) overlapped = true;  // engine must be single-threaded
        {
            std::lock_guard<std::mutex> lock(mu);
            batch_sizes.push_back((int)states.size());
        }
        if (delay_us.load() > 0) std::this_thread::sleep_for(std::chrono::microseconds(delay_us.load()));
        if (fail_next.load() > 0) {
            fail_next.fetch_sub(1);
            in_flight.fetch_sub(1);
            throw std::runtime_error("injected engine failure");
        }
        std::vector<std::pair<std::vector<float>, float>> out;
        for (auto& s : states) out.push_back(expected(s, actions));
        in_flight.fetch_sub(1);
        return out;
    }
};

static std::vector<float> state_for(int thread, int i) {
    std::vector<float> s(37);
    for (size_t k = 0; k < s.size(); ++k) s[k] = (float)((thread * 131 + i * 7 + (int)k) % 11) / 10.0f;
    return s;
}

static bool same(const BatchEvaluator::Result& r, const std::vector<float>& st, int actions) {
    auto e = FakeEngine::expected(st, actions);
    if (r.first.size() != e.first.size() || r.second != e.second) return false;
    for (size_t a = 0; a < e.first.size(); ++a)
        if (r.first[a] != e.first[a]) return false;
    return true;
}

static void test_many_search_threads() {
    FakeEngine eng;
    eng.delay_us = 200;
    GpuEvaluator ev(&eng, 16);
    const int T = 48, N = 60;
    std::vector<std::thread> th;
    std::atomic<int> bad{0};
    for (int t = 0; t < T; ++t)
        th.emplace_back([&, t] {
            NNResultBuf buf;  // one buffer per search thread, reused
            for (int i = 0; i < N; ++i) {
                auto st = state_for(t, i);
                auto r = ev.evaluate_with_buf(buf, st);
                if (!same(r, st, eng.actions)) bad++;
            }
        });
    for (auto& x : th) x.join();
    CHECK(bad == 0);
    CHECK(ev.positions() == (uint64_t)T * N);
    CHECK(ev.largest_batch() <= 16);
    CHECK(ev.largest_batch() > 1);  // concurrent submissions were batched
    CHECK(!eng.overlapped);
    int total = 0;
    for (int b : eng.batch_sizes) total += b;
    CHECK(total == T * N);
}

static void test_failure_reaches_clients() {
    FakeEngine eng;
    GpuEvaluator ev(&eng, 8);
    eng.fail_next = 1;
    bool threw = false;
    try {
        ev.evaluate_single(state_for(1, 1));
    } catch (const std::runtime_error& ex) {
        threw = std::string(ex.what()).find("injected engine failure") != std::string::npos;
    }
    CHECK(threw);
    CHECK(ev.failed_batches() == 1);
    // the evaluator keeps serving after a failed batch
    auto st = state_for(2, 3);
    CHECK(same(ev.evaluate_single(st), st, eng.actions));
    // batch API
    eng.fail_next = 1;
    threw = false;
    try {
        ev.evaluate({state_for(0, 0), state_for(0, 1)});
    } catch (const std::runtime_error&) {
        threw = true;
    }
    CHECK(threw);
    auto ok = ev.evaluate({state_for(0, 0), state_for(0, 1), state_for(0, 2)});
    CHECK(ok.size() == 3 && same(ok[2], state_for(0, 2), eng.actions));
    CHECK(ev.evaluate({}).empty());
}

static void test_sharded() {
    FakeEngine e0, e1, e2;
    e0.delay_us = e1.delay_us = e2.delay_us = 100;
    ShardedEvaluator sh({&e0, &e1, &e2}, 32);
    CHECK(sh.shards() == 3);
    const int T = 30, N = 40;
    std::vector<int> shard_of(T, -1);
    std::atomic<int> bad{0}, moved{0};
    std::vector<std::thread> th;
    for (int t = 0; t < T; ++t)
        th.emplace_back([&, t] {
            NNResultBuf buf;
            shard_of[t] = sh.shard_of_this_thread();
            for (int i = 0; i < N; ++i) {
                auto st = state_for(t, i);
                if (!same(sh.evaluate_with_buf(buf, st), st, 10)) bad++;
                if (sh.shard_of_this_thread() != shard_of[t]) moved++;
            }
        });
    for (auto& x : th) x.join();
    CHECK(bad == 0 && moved == 0);
    std::map<int, int> per;
    for (int s : shard_of) per[s]++;
    CHECK(per.size() == 3);
    for (auto& kv : per) CHECK(kv.second == T / 3);  // round-robin assignment
    for (size_t s = 0; s < 3; ++s) CHECK(sh.shard(s).positions() == (uint64_t)(T / 3) * N);
    // batch API split across shards keeps order
    std::vector<std::vector<float>> batch;
    for (int i = 0; i < 25; ++i) batch.push_back(state_for(99, i));
    auto r = sh.evaluate(batch);
    CHECK(r.size() == 25);
    for (int i = 0; i < 25; ++i) CHECK(same(r[i], batch[i], 10));
    // a failure in one shard surfaces
    e1.fail_next = 1;
    bool threw = false;
    try {
        sh.evaluate(batch);
    } catch (const std::runtime_error&) {
        threw = true;
    }
    CHECK(threw);
}

static void test_shutdown_drains_queue() {
    FakeEngine eng;
    eng.delay_us = 2000;
    std::atomic<int> done{0};
    std::vector<std::thread> th;
    {
        GpuEvaluator ev(&eng, 4);
        for (int t = 0; t < 12; ++t)
            th.emplace_back([&, t] {
                NNResultBuf buf;
                auto st = state_for(t, 0);
                if (same(ev.evaluate_with_buf(buf, st), st, eng.actions)) done++;
            });
        for (auto& x : th) x.join();
    }
    CHECK(done == 12);
}

int main() {
    test_many_search_threads();
    test_failure_reaches_clients();
    test_sharded();
    test_shutdown_drains_queue();
    std::printf("evaluator tests passed\n");
    return 0;
}
