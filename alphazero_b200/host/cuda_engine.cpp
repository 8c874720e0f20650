#include "cuda_engine.h"

#include "../../include/minigo_cuda.h"

#include <algorithm>
#include <cstring>
#include <stdexcept>

namespace minigo {

CudaEngine::CudaEngine(int device, Precision precision, bool eigen_compat, int max_batch)
    : device_(device) {
    h_ = mg_create(device, eigen_compat ? MG_FLAG_EIGEN_COMPAT : 0);
    if (h_ == nullptr) throw std::runtime_error(std::string("CUDA backend: ") + mg_create_error());
    check(mg_set_max_batch(h_, max_batch), "mg_set_max_batch");
    check(mg_set_precision(h_, (int)precision), "mg_set_precision");
}

CudaEngine::~CudaEngine() { mg_destroy(h_); }

void CudaEngine::check(int rc, const char* what) const {
    if (rc != MG_OK) {
        const char* msg = mg_last_error(h_);
        throw std::runtime_error(std::string(what) + ": " + (msg && *msg ? msg : "failed"));
    }
}

void CudaEngine::load_model(const std::string& model_path) {
    if (mg_load_onnx(h_, model_path.c_str()) != MG_OK) throw std::runtime_error(mg_last_error(h_));
    check(mg_get_info(h_, &board_size, &input_channels, &num_filters, &num_res_blocks, &action_size_),
          "mg_get_info");
}

namespace {
// Packs one state's binary planes into words (bit j % 32 of word j / 32);
// false if some value is neither 0 nor 1.
bool pack_state(const float* s, int size, uint32_t* w) {
    const int words = (size + 31) / 32;
    for (int k = 0; k < words; ++k) {
        uint32_t v = 0;
        const int lo = k * 32, hi = std::min(size, lo + 32);
        for (int j = lo; j < hi; ++j) {
            const float x = s[j];
            v |= (uint32_t)(x == 1.0f) << (j - lo);
            if (x != 0.0f && x != 1.0f) return false;
        }
        w[k] = v;
    }
    return true;
}
}  // namespace

void CudaEngine::predict_raw(const float* const* states, int n, int state_size, float* policy,
                             float* value) {
    if (n <= 0) return;
    const int expect = input_channels * board_size * board_size;
    if (state_size != expect)
        throw std::invalid_argument("state has " + std::to_string(state_size) + " floats, expected " +
                                    std::to_string(expect));
    // Encoded positions are binary planes: ship them bit-packed (32x fewer
    // bytes over PCIe), unless some state is not binary.
    const int words = (state_size + 31) / 32;
    bits_.resize((size_t)n * words);
    bool binary = true;
    for (int i = 0; i < n && binary; ++i) binary = pack_state(states[i], state_size, bits_.data() + (size_t)i * words);
    if (binary) {
        check(mg_forward_packed(h_, bits_.data(), n, policy, value, nullptr), "mg_forward_packed");
        return;
    }
    float* pinned = mg_host_input(h_);
    if (pinned == nullptr) throw std::runtime_error(std::string("mg_host_input: ") + mg_last_error(h_));
    const int cap = mg_max_batch(h_);
    for (int base = 0; base < n; base += cap) {
        const int m = std::min(cap, n - base);
        for (int i = 0; i < m; ++i)
            std::memcpy(pinned + (size_t)i * state_size, states[base + i], sizeof(float) * state_size);
        check(mg_forward(h_, pinned, m, policy + (size_t)base * action_size_, value + base, nullptr),
              "mg_forward");
    }
}

std::vector<std::pair<std::vector<float>, float>> CudaEngine::predict_batch(
    const std::vector<std::vector<float>>& states) {
    std::vector<std::pair<std::vector<float>, float>> out;
    if (states.empty()) return out;
    const int n = (int)states.size();
    std::vector<const float*> ptrs(n);
    for (int i = 0; i < n; ++i) {
        if ((int)states[i].size() != (int)states[0].size())
            throw std::invalid_argument("states of different sizes in one batch");
        ptrs[i] = states[i].data();
    }
    policy_scratch_.resize((size_t)n * action_size_);
    value_scratch_.resize(n);
    predict_raw(ptrs.data(), n, (int)states[0].size(), policy_scratch_.data(), value_scratch_.data());
    out.reserve(n);
    for (int i = 0; i < n; ++i)
        out.emplace_back(std::vector<float>(policy_scratch_.begin() + (size_t)i * action_size_,
                                            policy_scratch_.begin() + (size_t)(i + 1) * action_size_),
                         value_scratch_[i]);
    return out;
}

std::pair<std::vector<float>, float> CudaEngine::predict(const std::vector<float>& state) {
    auto r = predict_batch({state});
    return std::move(r[0]);
}

}  // namespace minigo
