// CudaEngine: the B200 backend behind the reference's InferenceEngine
// interface (include/inference_engine.h:14-41), implemented over the C ABI of
// include/minigo_cuda.h.  One instance owns one network on one GPU and, like
// every reference engine, is not thread-safe: one evaluator thread drives it.
#pragma once

#include "minigo_api.h"

#include <atomic>
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

    // As predict_raw for states already in the bit-packed wire format
    // (words_per_position() words each, see pack_planes): gathered straight
    // into the engine's pinned buffer (mg_host_bits) and shipped as is.
    void predict_bits(const uint32_t* const* bits, int n, float* policy, float* value);

    // The same without waiting (mg_submit_packed): gathers n <= max batch
    // positions into one of two page-locked input buffers of this object,
    // enqueues the evaluation with results into policy / value (page-locked,
    // e.g. mg_host_alloc) and returns a ticket for wait_submitted.  At most
    // two submissions may be outstanding.  wait_submitted may run on another
    // thread than submit_bits; it throws std::runtime_error if the
    // evaluation failed.
    int submit_bits(const uint32_t* const* bits, int n, float* policy, float* value);
    void wait_submitted(int ticket);

    // Packs one state's binary planes (`size` floats, each 0 or 1) into
    // (size + 31) / 32 words, element j at bit j % 32 of word j / 32; false
    // if some value is neither 0 nor 1 (the words are then unspecified).
    static bool pack_planes(const float* state, int size, uint32_t* words);
    int words_per_position() const { return (input_channels * board_size * board_size + 31) / 32; }

    int device() const { return device_; }
    int max_batch() const;  // positions per engine call (mg_max_batch)
    int action_size() const { return action_size_; }
    // Kernel launches of this library made by predict / predict_batch /
    // predict_raw so far (readable from any thread).
    uint64_t kernel_launches() const { return launches_.load(std::memory_order_relaxed); }
    // Host time (ns) predict_raw spent packing binary planes into bits.
    uint64_t pack_ns() const { return pack_ns_.load(std::memory_order_relaxed); }

private:
    void check(int rc, const char* what) const;
    void count_launches(int n);

    mg_engine* h_ = nullptr;
    uint32_t* submit_in_[2] = {nullptr, nullptr};  // page-locked inputs of submit_bits
    int submit_next_ = 0;
    int device_ = 0;
    int action_size_ = 0;
    std::vector<float> policy_scratch_, value_scratch_;
    std::atomic<uint64_t> launches_{0}, pack_ns_{0};
};

}  // namespace minigo
