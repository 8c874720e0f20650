// Self-play training records: the step after evaluation in the training
// loop.  A finished game's trajectory (encoded state, search policy, player
// to move per move) becomes 8 records per move, the 8 symmetries of the
// board, valued +1 / -1 / 0 by the winner from the mover's side
// (src/mcts.cpp:377-467), written in the reference selfplay binary's file
// format (src/main_selfplay.cpp:17-32), which scripts/train.py:33-55 reads.
#pragma once

#include "fast_search.h"
#include "go_positions.h"

#include <cstdint>
#include <string>
#include <vector>

namespace mgb {

struct TrainingRecord {
    std::vector<float> state;   // planes x board^2, plane-major
    std::vector<float> policy;  // board^2 + 1 (pass last)
    float value = 0.0f;
};

// The 8 symmetries in the reference's order (src/mcts.cpp:377-420): for
// rot = 0..3 and flip = 0..1, a point (r, c) is rotated `rot` times by
// (r, c) -> (c, n - 1 - r), then mirrored c -> n - 1 - c when flip is set;
// the planes and the policy move with it, the pass probability stays.
class DihedralAugmenter {
public:
    DihedralAugmenter(int board_size, int planes);
    // Appends the 8 records of one sample to `out`.
    void augment(const float* state, const float* policy, float value,
                 std::vector<TrainingRecord>& out) const;

private:
    int n_, planes_;
    std::vector<int> dest_;  // [8][n*n]: where point p lands under symmetry t
};

// A whole self-play game on `search` (src/mcts.cpp:443-467): moves until the
// game ends or max_moves, temperature 1 for the first temperature_threshold
// moves and 0 after, root noise on; then passes until the game is over and
// the records of every move, augmented.
std::vector<TrainingRecord> self_play_game(FastSearch& search, int board_size, float komi,
                                           int max_moves, int temperature_threshold);

// The reference selfplay's binary file: int32 record count, then per record
// int32 state size, the state floats, int32 policy size, the policy floats,
// float value (little-endian as written by the host).  Throws
// std::runtime_error if the file cannot be written.
void write_records(const std::string& path, const std::vector<TrainingRecord>& records);

}  // namespace mgb
