#include "cuda_engine.h"

#include "../../include/minigo_cuda.h"

#include <algorithm>
#include <chrono>
#if defined(__SSE2__)
#include <emmintrin.h>
#endif
#include <cstring>
#include <stdexcept>
#if defined(MGB_USE_REFERENCE_HEADERS)
#include "onnx_loader.h"
#endif

namespace minigo {

CudaEngine::CudaEngine(int device, Precision precision, bool eigen_compat, int max_batch)
    : device_(device) {
    h_ = mg_create(device, eigen_compat ? MG_FLAG_EIGEN_COMPAT : 0);
    if (h_ == nullptr) throw std::runtime_error(std::string("CUDA backend: ") + mg_create_error());
    check(mg_set_max_batch(h_, max_batch), "mg_set_max_batch");
    check(mg_set_precision(h_, (int)precision), "mg_set_precision");
}

CudaEngine::~CudaEngine() {
    mg_destroy(h_);
    mg_host_free(submit_in_[0]);
    mg_host_free(submit_in_[1]);
}

void CudaEngine::check(int rc, const char* what) const {
    if (rc != MG_OK) {
        const char* msg = mg_last_error(h_);
        throw std::runtime_error(std::string(what) + ": " + (msg && *msg ? msg : "failed"));
    }
}

void CudaEngine::count_launches(int n) {
    const int k = mg_launches_per_forward(h_, n);
    if (k > 0) launches_.fetch_add((uint64_t)k, std::memory_order_relaxed);
}

void CudaEngine::load_model(const std::string& model_path) {
#if defined(MGB_USE_REFERENCE_HEADERS)
    // Built inside the reference tree: the model goes through the
    // reference's own loader, onnx_parser::parse_onnx_file
    // (src/onnx_loader.cpp:183), as its Eigen / OpenCL / Metal engines load it
    // (it throws "Cannot open model file: ..."), and the parsed initializers
    // go to the device through mg_load_weights.  Non-FLOAT tensors
    // (num_batches_tracked) are passed without values, as mg_load_onnx does.
    const std::vector<onnx_parser::OnnxTensor> parsed = onnx_parser::parse_onnx_file(model_path);
    std::vector<std::vector<float>> values(parsed.size());
    std::vector<mg_tensor> tensors(parsed.size());
    for (size_t i = 0; i < parsed.size(); ++i) {
        const onnx_parser::OnnxTensor& t = parsed[i];
        if (t.data_type == 0 || t.data_type == 1) values[i] = t.get_floats();
        if (!values[i].empty() && (int64_t)values[i].size() != t.total_elements())
            throw std::runtime_error("tensor " + t.name + " holds " + std::to_string(values[i].size()) +
                                     " values for " + std::to_string(t.total_elements()) + " elements");
        tensors[i].name = t.name.c_str();
        tensors[i].dims = t.dims.data();
        tensors[i].ndims = (int)t.dims.size();
        tensors[i].data = values[i].empty() ? nullptr : values[i].data();
    }
    if (mg_load_weights(h_, tensors.data(), (int)tensors.size()) != MG_OK)
        throw std::runtime_error(mg_last_error(h_));
#else
    if (mg_load_onnx(h_, model_path.c_str()) != MG_OK) throw std::runtime_error(mg_last_error(h_));
#endif
    check(mg_get_info(h_, &board_size, &input_channels, &num_filters, &num_res_blocks, &action_size_),
          "mg_get_info");
}

bool CudaEngine::pack_planes(const float* s, int size, uint32_t* w) {
    const int words = (size + 31) / 32;
    int k = 0;
#if defined(__SSE2__)
    // Whole words four floats at a time: bits from (x == 1), and every
    // lane must be 0 or 1.
    const __m128 one = _mm_set1_ps(1.0f), zero = _mm_setzero_ps();
    for (; k < size / 32; ++k) {
        uint32_t v = 0;
        int ok = 0xF;
        for (int q = 0; q < 8; ++q) {
            const __m128 x = _mm_loadu_ps(s + k * 32 + q * 4);
            const __m128 is1 = _mm_cmpeq_ps(x, one);
            v |= (uint32_t)_mm_movemask_ps(is1) << (4 * q);
            ok &= _mm_movemask_ps(_mm_or_ps(is1, _mm_cmpeq_ps(x, zero)));
        }
        if (ok != 0xF) return false;
        w[k] = v;
    }
#endif
    for (; k < words; ++k) {
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

void CudaEngine::predict_bits(const uint32_t* const* bits, int n, float* policy, float* value) {
    if (n <= 0) return;
    uint32_t* pinned = mg_host_bits(h_);
    if (pinned == nullptr) check(MG_E_DEVICE, "mg_host_bits");
    const int words = words_per_position();
    const int cap = mg_max_batch(h_);
    for (int base = 0; base < n; base += cap) {
        const int m = std::min(cap, n - base);
        for (int i = 0; i < m; ++i)
            std::memcpy(pinned + (size_t)i * words, bits[base + i], sizeof(uint32_t) * words);
        check(mg_forward_packed(h_, pinned, m, policy + (size_t)base * action_size_, value + base, nullptr),
              "mg_forward_packed");
        count_launches(m);
    }
}

int CudaEngine::submit_bits(const uint32_t* const* bits, int n, float* policy, float* value) {
    const int words = words_per_position();
    const int cap = mg_max_batch(h_);
    if (n < 1 || n > cap) throw std::invalid_argument("submit_bits: batch size out of range");
    uint32_t*& in = submit_in_[submit_next_];
    if (in == nullptr) {
        in = static_cast<uint32_t*>(mg_host_alloc((size_t)cap * words * sizeof(uint32_t)));
        if (in == nullptr) throw std::runtime_error("page-locked input buffer could not be allocated");
    }
    for (int i = 0; i < n; ++i) std::memcpy(in + (size_t)i * words, bits[i], sizeof(uint32_t) * words);
    int ticket = -1;
    check(mg_submit_packed(h_, in, n, policy, value, &ticket), "mg_submit_packed");
    submit_next_ ^= 1;
    count_launches(n);
    return ticket;
}

int CudaEngine::max_batch() const { return mg_max_batch(h_); }

void CudaEngine::wait_submitted(int ticket) {
    const int rc = mg_wait_submitted(h_, ticket);
    if (rc == MG_E_DEVICE) throw std::runtime_error("mg_wait_submitted: a kernel gave up waiting");
    if (rc != MG_OK) throw std::runtime_error("mg_wait_submitted failed (" + std::to_string(rc) + ")");
}

void CudaEngine::predict_raw(const float* const* states, int n, int state_size, float* policy,
                             float* value) {
    if (n <= 0) return;
    const int expect = input_channels * board_size * board_size;
    if (state_size != expect)
        throw std::invalid_argument("state has " + std::to_string(state_size) + " floats, expected " +
                                    std::to_string(expect));
    // Encoded positions are binary planes: packed straight into the
    // engine's pinned buffer and shipped bit-packed (32x fewer bytes over
    // PCIe); a chunk with a non-binary state goes as fp32 planes instead.
    const int words = (state_size + 31) / 32;
    const int cap = mg_max_batch(h_);
    for (int base = 0; base < n; base += cap) {
        const int m = std::min(cap, n - base);
        uint32_t* pinned_bits = mg_host_bits(h_);
        if (pinned_bits == nullptr) check(MG_E_DEVICE, "mg_host_bits");
        bool binary = true;
        const auto t0 = std::chrono::steady_clock::now();
        for (int i = 0; i < m && binary; ++i)
            binary = pack_planes(states[base + i], state_size, pinned_bits + (size_t)i * words);
        pack_ns_.fetch_add((uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                               std::chrono::steady_clock::now() - t0)
                               .count(),
                           std::memory_order_relaxed);
        if (binary) {
            check(mg_forward_packed(h_, pinned_bits, m, policy + (size_t)base * action_size_, value + base,
                                    nullptr),
                  "mg_forward_packed");
        } else {
            float* pinned = mg_host_input(h_);
            if (pinned == nullptr) check(MG_E_DEVICE, "mg_host_input");
            for (int i = 0; i < m; ++i)
                std::memcpy(pinned + (size_t)i * state_size, states[base + i], sizeof(float) * state_size);
            check(mg_forward(h_, pinned, m, policy + (size_t)base * action_size_, value + base, nullptr),
                  "mg_forward");
        }
        count_launches(m);
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
