// Training records (alphazero_b200/host/selfplay_records.h) against the
// reference's own self-play (src/mcts.cpp compiled from the reference tree):
//   1. augmentation: for every move of a reference self-play game, the
//      reference's first record of the move is the untransformed sample, and
//      DihedralAugmenter applied to it reproduces all 8 of the reference's
//      records bit for bit;
//   2. a FastSearch game's records have the reference's shape (8 per move,
//      17 x n^2 binary planes, n^2 + 1 probabilities, values +-1 / 0 from the
//      mover's side) and are written to argv[1] in the reference selfplay's
//      file format (read back by the Python side with scripts/train.py's
//      reader).
// Exit code 0 = pass; prints the record count written.
#include "fast_search.h"
#include "selfplay_records.h"

#include "batch_evaluator.h"
#include "config.h"
#include "mcts.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#define CHECK(c)                                                                       \
    do {                                                                               \
        if (!(c)) {                                                                    \
            std::fprintf(stderr, "CHECK failed %s:%d: %s\n", __FILE__, __LINE__, #c); \
            std::abort();                                                              \
        }                                                                              \
    } while (0)

namespace {

// Position-dependent but deterministic policy, so that the search policy
// differs between points and a wrong permutation shows.
void fake_net(const float* planes, int n_planes_floats, int actions, float* policy, float* value) {
    uint32_t h = 2166136261u;
    for (int j = 0; j < n_planes_floats; ++j)
        if (planes[j] != 0.0f) h = (h ^ (uint32_t)j) * 16777619u;
    float sum = 0.0f;
    for (int a = 0; a < actions; ++a) {
        policy[a] = 1.0f + (float)((h + 7u * (uint32_t)a) % 13u);
        sum += policy[a];
    }
    for (int a = 0; a < actions; ++a) policy[a] /= sum;
    *value = (float)((int)(h % 101u) - 50) / 50.0f;
}

class FakeBatch : public minigo::BatchEvaluator {
public:
    explicit FakeBatch(int actions) : actions_(actions) {}
    std::vector<Result> evaluate(const std::vector<std::vector<float>>& states) override {
        std::vector<Result> out;
        for (const auto& s : states) {
            Result r;
            r.first.resize(actions_);
            fake_net(s.data(), (int)s.size(), actions_, r.first.data(), &r.second);
            out.push_back(std::move(r));
        }
        return out;
    }

private:
    int actions_;
};

class FakePacked : public mgb::PackedEvaluator {
public:
    explicit FakePacked(int board) : board_(board) {}
    void evaluate_packed(const uint32_t* w, int, float* policy, float* value) override {
        const int n = 17 * board_ * board_;
        std::vector<float> planes(n);
        for (int j = 0; j < n; ++j) planes[j] = (float)((w[j >> 5] >> (j & 31)) & 1u);
        fake_net(planes.data(), n, board_ * board_ + 1, policy, value);
    }

private:
    int board_;
};

}  // namespace

int main(int argc, char** argv) {
    if (argc != 2) return 2;
    const int board = 5, nn = board * board;

    // 1. the reference's records against DihedralAugmenter
    minigo::Config cfg;
    cfg.board_size = board;
    cfg.num_simulations = 24;
    cfg.num_search_threads = 1;
    cfg.max_moves_per_game = 2 * nn;
    FakeBatch ref_eval(nn + 1);
    mgb::DihedralAugmenter aug(board, 17);
    int moves_checked = 0;
    for (int game = 0; game < 3; ++game) {
        auto ref = minigo::self_play_game(&ref_eval, cfg);
        CHECK(!ref.empty() && ref.size() % 8 == 0);
        for (size_t k = 0; k < ref.size(); k += 8) {
            std::vector<mgb::TrainingRecord> mine;
            aug.augment(ref[k].state.data(), ref[k].policy.data(), ref[k].value, mine);
            CHECK(mine.size() == 8);
            for (int t = 0; t < 8; ++t) {
                CHECK(mine[t].state == ref[k + t].state);
                CHECK(mine[t].policy == ref[k + t].policy);
                CHECK(mine[t].value == ref[k + t].value);
            }
            ++moves_checked;
        }
    }
    std::printf("augmentation matches the reference on %d moves\n", moves_checked);

    // 2. a FastSearch game's records, written in the reference's format
    FakePacked ev(board);
    mgb::SearchParams sp;
    sp.simulations = 24;
    sp.threads = 2;
    mgb::FastSearch search(&ev, board, sp, 5);
    auto recs = mgb::self_play_game(search, board, 7.5f, 2 * nn, 30);
    CHECK(!recs.empty() && recs.size() % 8 == 0);
    for (size_t k = 0; k < recs.size(); ++k) {
        const auto& r = recs[k];
        CHECK(r.state.size() == (size_t)17 * nn && r.policy.size() == (size_t)nn + 1);
        for (float x : r.state) CHECK(x == 0.0f || x == 1.0f);
        double s = 0;
        for (float p : r.policy) s += p;
        CHECK(std::fabs(s - 1.0) < 1e-5);
        CHECK(r.value == 0.0f || r.value == 1.0f || r.value == -1.0f);
        CHECK(r.value == recs[k - k % 8].value);
    }
    mgb::write_records(argv[1], recs);
    std::printf("records %zu\n", recs.size());
    std::printf("records tests passed\n");
    return 0;
}
