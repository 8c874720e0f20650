#include "selfplay_records.h"

#include <cstdio>
#include <memory>
#include <stdexcept>

namespace mgb {

DihedralAugmenter::DihedralAugmenter(int board_size, int planes)
    : n_(board_size), planes_(planes), dest_((size_t)8 * board_size * board_size) {
    const int n = n_, nn = n * n;
    for (int rot = 0; rot < 4; ++rot)
        for (int flip = 0; flip < 2; ++flip) {
            int* d = dest_.data() + (size_t)(rot * 2 + flip) * nn;
            for (int r = 0; r < n; ++r)
                for (int c = 0; c < n; ++c) {
                    int tr = r, tc = c;
                    for (int k = 0; k < rot; ++k) {
                        const int t = tr;
                        tr = tc;
                        tc = n - 1 - t;
                    }
                    if (flip) tc = n - 1 - tc;
                    d[r * n + c] = tr * n + tc;
                }
        }
}

void DihedralAugmenter::augment(const float* state, const float* policy, float value,
                                std::vector<TrainingRecord>& out) const {
    const int nn = n_ * n_;
    for (int t = 0; t < 8; ++t) {
        const int* d = dest_.data() + (size_t)t * nn;
        TrainingRecord rec;
        rec.state.resize((size_t)planes_ * nn);
        rec.policy.resize(nn + 1);
        rec.value = value;
        for (int ch = 0; ch < planes_; ++ch) {
            const float* src = state + (size_t)ch * nn;
            float* dst = rec.state.data() + (size_t)ch * nn;
            for (int p = 0; p < nn; ++p) dst[d[p]] = src[p];
        }
        for (int p = 0; p < nn; ++p) rec.policy[d[p]] = policy[p];
        rec.policy[nn] = policy[nn];
        out.push_back(std::move(rec));
    }
}

std::vector<TrainingRecord> self_play_game(FastSearch& search, int board_size, float komi,
                                           int max_moves, int temperature_threshold) {
    struct Step {
        std::vector<float> state, policy;
        int player;
    };
    GoPosition game(board_size, komi);
    const int nn = board_size * board_size;
    std::vector<Step> trajectory;
    while (!game.over() && game.moves() < max_moves) {
        const float temp = game.moves() < temperature_threshold ? 1.0f : 0.0f;
        Step step;
        const int action = search.get_action(game, step.policy, temp, true);
        step.state.resize((size_t)kInputPlanes * nn);
        game.encode(step.state.data());
        step.player = game.to_move();
        trajectory.push_back(std::move(step));
        game.play(action);
    }
    while (!game.over()) game.play(nn);  // pass until the game ends
    DihedralAugmenter aug(board_size, kInputPlanes);
    std::vector<TrainingRecord> records;
    records.reserve(trajectory.size() * 8);
    for (const auto& s : trajectory) {
        const float value = game.winner() == 0 ? 0.0f : (game.winner() == s.player ? 1.0f : -1.0f);
        aug.augment(s.state.data(), s.policy.data(), value, records);
    }
    return records;
}

void write_records(const std::string& path, const std::vector<TrainingRecord>& records) {
    std::unique_ptr<FILE, int (*)(FILE*)> f(std::fopen(path.c_str(), "wb"), &std::fclose);
    if (!f) throw std::runtime_error("cannot write " + path);
    bool ok = true;
    auto put = [&](const void* p, size_t bytes) { ok &= std::fwrite(p, 1, bytes, f.get()) == bytes; };
    const int32_t n = (int32_t)records.size();
    put(&n, 4);
    for (const auto& r : records) {
        const int32_t ss = (int32_t)r.state.size(), ps = (int32_t)r.policy.size();
        put(&ss, 4);
        put(r.state.data(), sizeof(float) * r.state.size());
        put(&ps, 4);
        put(r.policy.data(), sizeof(float) * r.policy.size());
        put(&r.value, sizeof(float));
    }
    if (!ok) throw std::runtime_error("short write to " + path);
}

}  // namespace mgb
