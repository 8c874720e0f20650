// Evaluation of positions already in the bit-packed wire format, for a
// search that encodes its boards straight to bits (mgb::GoPosition::
// encode_bits) instead of the reference's 24.5 KB fp32 planes
// (src/game.cpp:229-256).  GpuEvaluator and ShardedEvaluator implement it
// next to the reference's BatchEvaluator interface.
#pragma once

#include <cstdint>

namespace mgb {

class PackedEvaluator {
public:
    virtual ~PackedEvaluator() = default;
    // Evaluates one position (17 planes of board^2 points, element j at bit
    // j % 32 of word j / 32; n_words words) and blocks until it is done:
    // `policy` receives board^2 + 1 softmax probabilities, `value` the tanh
    // value.  Throws std::runtime_error if the evaluation failed.
    virtual void evaluate_packed(const uint32_t* words, int n_words, float* policy,
                                 float* value) = 0;

    // Evaluates n positions (words[i], n_words words each) as one group and
    // blocks until every one is done: policies[i] receives position i's
    // probabilities, values[i] its value.  Throws std::runtime_error if an
    // evaluation failed.  The default evaluates them one after another.
    virtual void evaluate_packed_group(const uint32_t* const* words, int n, int n_words,
                                       float* const* policies, float* values) {
        for (int i = 0; i < n; ++i) evaluate_packed(words[i], n_words, policies[i], &values[i]);
    }
};

}  // namespace mgb
