// The reference's engine and evaluator interfaces, as the CUDA backend's C++
// host code sees them.
//
// Built inside the reference tree (-DMGB_USE_REFERENCE_HEADERS) the
// reference's own headers are used.  Built standalone
// (this repository's tests) the same declarations are restated here; they
// must stay layout- and signature-identical to
//   include/inference_engine.h:14-41   InferenceEngine
//   include/batch_evaluator.h:18-33    NNResultBuf
//   include/batch_evaluator.h:38-68    BatchEvaluator
// because the reference's MCTS (src/mcts.cpp) calls evaluators through them.
#pragma once

#ifdef MGB_USE_REFERENCE_HEADERS
#include "batch_evaluator.h"
#include "inference_engine.h"
#else

#include <condition_variable>
#include <memory>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

namespace minigo {

// A backend evaluating encoded positions (17 planes x board^2 fp32) into a
// softmax policy over board^2 + 1 actions and a tanh value.
class InferenceEngine {
public:
    virtual ~InferenceEngine() = default;
    virtual void load_model(const std::string& model_path) = 0;
    virtual std::pair<std::vector<float>, float> predict(const std::vector<float>& state) = 0;
    virtual std::vector<std::pair<std::vector<float>, float>> predict_batch(
        const std::vector<std::vector<float>>& states) {
        std::vector<std::pair<std::vector<float>, float>> out;
        out.reserve(states.size());
        for (const auto& s : states) out.push_back(predict(s));
        return out;
    }
    virtual std::string backend_name() const = 0;

    int board_size = 9;
    int input_channels = 17;
    int num_filters = 64;
    int num_res_blocks = 5;
};

// One search thread's pending evaluation: the state it submits, the
// rendezvous with the evaluator's server thread, and the result slot.
struct NNResultBuf {
    const float* state_data = nullptr;
    int state_size = 0;

    std::mutex mu;
    std::condition_variable cv;
    bool done = false;

    std::vector<float> policy;
    float value = 0.0f;

    void reset() { done = false; }
};

// Evaluation service used by the search.
class BatchEvaluator {
public:
    virtual ~BatchEvaluator() = default;
    using Result = std::pair<std::vector<float>, float>;

    virtual std::vector<Result> evaluate(const std::vector<std::vector<float>>& states) = 0;

    virtual Result evaluate_with_buf(NNResultBuf& buf, const std::vector<float>& state) {
        (void)buf;
        auto results = evaluate({state});
        return std::move(results[0]);
    }

    virtual Result evaluate_single(const std::vector<float>& state) {
        auto results = evaluate({state});
        return std::move(results[0]);
    }
};

}  // namespace minigo

#endif  // MGB_USE_REFERENCE_HEADERS
