// CudaEngine: the B200 backend behind the reference's InferenceEngine
// interface (include/inference_engine.h:14-41), implemented over the C ABI of
// include/minigo_cuda.h.  One instance owns one network on one GPU and, like
// every reference engine, is not thread-safe: one evaluator thread drives it.
#pragma once

#include "minigo_api.h"

#include <cstddef>
#include <cstdint>
#include <string>
#include <utility>
#include <vector>

struct mg_engine;

namespace minigo {

class CudaEngine : public InferenceEngine {
public:
    enum Precision { kBf16 = 0, kFp16 = 1, kFp32 = 2 };

    // Creates the engine on `device`; throws std::runtime_error if no usable
    // sm_100 GPU is there (there is no CPU fallback).
    explicit CudaEngine(int device = 0, Precision precision = kBf16, bool eigen_compat = false,
                        int max_batch = 1024);
    ~CudaEngine() override;
    CudaEngine(const CudaEngine&) = delete;
    CudaEngine& operator=(const CudaEngine&) = delete;

    // Reads the .onnx initializers, infers the architecture and sets
    // board_size / input_channels / num_filters / num_res_blocks; throws
    // std::runtime_error ("Cannot open model file: ...", "Missing tensor:
    // ...") like the reference engines.
    void load_model(const std::string& model_path) override;

    std::pair<std::vector<float>, float> predict(const std::vector<float>& state) override;

    // An empty batch returns {} (src/opencl_engine.cpp:724).
    std::vector<std::pair<std::vector<float>, float>> predict_batch(
        const std::vector<std::vector<float>>& states) override;

    std::string backend_name() const override { return "cuda"; }

    // Batch evaluation for evaluators: n state pointers of state_size floats
    // each.  Binary states (the encoder's planes) are packed to bits while
    // gathered and shipped in the packed wire format; otherwise the fp32
    // planes are gathered straight into the engine's pinned input buffer.
    // Results land in policy (n x action_size) and value (n).
    void predict_raw(const float* const* states, int n, int state_size, float* policy,
                     float* value);

    int device() const { return device_; }
    int action_size() const { return action_size_; }

private:
    void check(int rc, const char* what) const;

    mg_engine* h_ = nullptr;
    int device_ = 0;
    int action_size_ = 0;
    std::vector<float> policy_scratch_, value_scratch_;
    std::vector<uint32_t> bits_;
};

}  // namespace minigo
