#include "gpu_evaluator.h"

#include "cuda_engine.h"

#include "../../include/minigo_cuda.h"

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cmath>
#include <limits>
#include <stdexcept>
#include <unordered_map>
#include <utility>

namespace minigo {

GpuEvaluator::GpuEvaluator(InferenceEngine* engine, int max_batch_size)
    : engine_(engine), cuda_(dynamic_cast<CudaEngine*>(engine)), max_batch_(max_batch_size) {
    if (engine_ == nullptr || max_batch_ < 1) throw std::invalid_argument("GpuEvaluator: bad arguments");
    queue_.reserve(max_batch_);
    if (const char* s = std::getenv("MG_EVAL_IN_FLIGHT")) max_in_flight_ = std::atoi(s) >= 2 ? 2 : 1;
    if (const char* s = std::getenv("MG_EVAL_OVERLAP_MIN")) overlap_min_ = (size_t)std::max(0, std::atoi(s));
    server_ = std::thread(&GpuEvaluator::server_loop, this);
    completer_ = std::thread(&GpuEvaluator::completion_loop, this);
}

void GpuEvaluator::reserve(Slot& slot, size_t n, size_t actions) {
    if (n <= slot.capacity) return;
    mg_host_free(slot.policy);
    mg_host_free(slot.value);
    slot.policy = static_cast<float*>(mg_host_alloc(n * actions * sizeof(float)));
    slot.value = static_cast<float*>(mg_host_alloc(n * sizeof(float)));
    if (slot.policy == nullptr || slot.value == nullptr) {
        mg_host_free(slot.policy);
        mg_host_free(slot.value);
        slot.policy = slot.value = nullptr;
        slot.capacity = 0;
        throw std::runtime_error("page-locked result buffers could not be allocated");
    }
    slot.capacity = n;
}

GpuEvaluator::~GpuEvaluator() {
    {
        std::lock_guard<std::mutex> lock(mu_);
        stop_ = true;
    }
    cv_.notify_all();
    server_.join();  // drains the queue, then tells the completion thread
    completer_.join();
    for (Slot& s : slots_) {
        mg_host_free(s.policy);
        mg_host_free(s.value);
    }
}

BatchEvaluator::Result GpuEvaluator::take_result(NNResultBuf& buf) {
    if (buf.policy.empty()) {
        std::string why;
        {
            std::lock_guard<std::mutex> lock(mu_);
            why = last_error_;
        }
        throw std::runtime_error("batched evaluation failed: " + why);
    }
    // Copied, not moved: the buffer keeps its capacity, so the server's next
    // result for this client (the search reuses one buffer per thread) is a
    // plain copy without an allocation on the server thread, and the
    // client's copy allocates on its own thread.
    return {buf.policy, buf.value};
}

void GpuEvaluator::enqueue(const Pending* items, size_t n) {
    {
        std::lock_guard<std::mutex> lock(mu_);
        queue_.insert(queue_.end(), items, items + n);
    }
    cv_.notify_all();
}

BatchEvaluator::Result GpuEvaluator::evaluate_with_buf(NNResultBuf& buf,
                                                      const std::vector<float>& state) {
    buf.done = false;
    buf.state_data = state.data();
    buf.state_size = (int)state.size();
    Pending p{&buf, nullptr};
    if (cuda_ != nullptr) {
        // The client blocks below until its result is back, so its
        // thread-local words stay valid while the server reads them.
        thread_local std::vector<uint32_t> words;
        words.resize((state.size() + 31) / 32);
        if (CudaEngine::pack_planes(state.data(), (int)state.size(), words.data())) p.bits = words.data();
    }
    enqueue(&p, 1);
    {
        std::unique_lock<std::mutex> lock(buf.mu);
        buf.cv.wait(lock, [&] { return buf.done; });
    }
    return take_result(buf);
}

void GpuEvaluator::evaluate_packed(const uint32_t* words, int n_words, float* policy, float* value) {
    if (cuda_ == nullptr) throw std::logic_error("evaluate_packed needs a CudaEngine");
    const int size = cuda_->input_channels * cuda_->board_size * cuda_->board_size;
    if (n_words != (size + 31) / 32)
        throw std::invalid_argument("packed state has " + std::to_string(n_words) + " words, expected " +
                                    std::to_string((size + 31) / 32));
    // One buffer per client thread, as the reference's search keeps one per
    // search thread (src/mcts.cpp:133).
    thread_local NNResultBuf buf;
    buf.done = false;
    buf.state_data = nullptr;
    buf.state_size = size;
    Pending p{&buf, words};
    enqueue(&p, 1);
    {
        std::unique_lock<std::mutex> lock(buf.mu);
        buf.cv.wait(lock, [&] { return buf.done; });
    }
    if (buf.policy.empty()) (void)take_result(buf);  // throws with the server's error
    std::copy(buf.policy.begin(), buf.policy.end(), policy);
    *value = buf.value;
}

void GpuEvaluator::evaluate_packed_group(const uint32_t* const* words, int n, int n_words,
                                         float* const* policies, float* values) {
    if (cuda_ == nullptr) throw std::logic_error("evaluate_packed_group needs a CudaEngine");
    if (n <= 0) return;
    const int size = cuda_->input_channels * cuda_->board_size * cuda_->board_size;
    if (n_words != (size + 31) / 32)
        throw std::invalid_argument("packed state has " + std::to_string(n_words) + " words, expected " +
                                    std::to_string((size + 31) / 32));
    // One buffer per group member, kept per client thread.
    thread_local std::vector<std::unique_ptr<NNResultBuf>> bufs;
    thread_local std::vector<Pending> items;
    while ((int)bufs.size() < n) bufs.push_back(std::make_unique<NNResultBuf>());
    items.resize(n);
    for (int i = 0; i < n; ++i) {
        NNResultBuf& b = *bufs[i];
        b.done = false;
        b.state_data = nullptr;
        b.state_size = size;
        items[i] = {&b, words[i]};
    }
    enqueue(items.data(), (size_t)n);
    bool failed = false;
    for (int i = 0; i < n; ++i) {
        NNResultBuf& b = *bufs[i];
        {
            // Usually only the first wait sleeps: the group is served by one
            // or two batches.
            std::unique_lock<std::mutex> lock(b.mu);
            b.cv.wait(lock, [&] { return b.done; });
        }
        if (b.policy.empty()) {
            failed = true;
            continue;
        }
        std::copy(b.policy.begin(), b.policy.end(), policies[i]);
        values[i] = b.value;
    }
    if (failed) {
        std::lock_guard<std::mutex> lock(mu_);
        throw std::runtime_error("batched evaluation failed: " + last_error_);
    }
}

BatchEvaluator::Result GpuEvaluator::evaluate_single(const std::vector<float>& state) {
    NNResultBuf buf;
    return evaluate_with_buf(buf, state);
}

std::vector<BatchEvaluator::Result> GpuEvaluator::evaluate(
    const std::vector<std::vector<float>>& states) {
    if (states.empty()) return {};
    const size_t n = states.size();
    std::vector<std::unique_ptr<NNResultBuf>> bufs(n);
    std::vector<std::vector<uint32_t>> words(cuda_ != nullptr ? n : 0);
    std::vector<Pending> items(n);
    for (size_t i = 0; i < n; ++i) {
        bufs[i] = std::make_unique<NNResultBuf>();
        bufs[i]->state_data = states[i].data();
        bufs[i]->state_size = (int)states[i].size();
        items[i] = {bufs[i].get(), nullptr};
        if (cuda_ != nullptr) {
            words[i].resize((states[i].size() + 31) / 32);
            if (CudaEngine::pack_planes(states[i].data(), (int)states[i].size(), words[i].data()))
                items[i].bits = words[i].data();
        }
    }
    enqueue(items.data(), n);
    std::vector<Result> out;
    out.reserve(n);
    bool failed = false;
    for (size_t i = 0; i < n; ++i) {
        std::unique_lock<std::mutex> lock(bufs[i]->mu);
        bufs[i]->cv.wait(lock, [&] { return bufs[i]->done; });
        failed |= bufs[i]->policy.empty();
        out.emplace_back(std::move(bufs[i]->policy), bufs[i]->value);
    }
    if (failed) {
        std::lock_guard<std::mutex> lock(mu_);
        throw std::runtime_error("batched evaluation failed: " + last_error_);
    }
    return out;
}

void GpuEvaluator::run_batch(Slot& slot) {
    std::vector<Pending>& batch = slot.batch;
    const int n = (int)batch.size();
    const auto t0 = std::chrono::steady_clock::now();
    if (cuda_ != nullptr) {
        const int a = cuda_->action_size();
        const int size = batch[0].buf->state_size;
        bool packed = size == cuda_->input_channels * cuda_->board_size * cuda_->board_size;
        for (const auto& p : batch) packed &= p.bits != nullptr && p.buf->state_size == size;
        reserve(slot, (size_t)std::max(n, max_batch_), (size_t)a);
        if (packed) {
            bit_ptrs_.resize(n);
            for (int i = 0; i < n; ++i) bit_ptrs_[i] = batch[i].bits;
            cuda_->predict_bits(bit_ptrs_.data(), n, slot.policy, slot.value);
        } else {
            // Mixed batch: fp32 planes for all; packed-only requests
            // (evaluate_packed) are unpacked first.
            ptrs_.resize(n);
            int unpack = 0;
            for (const auto& p : batch) unpack += p.buf->state_data == nullptr;
            unpacked_.resize((size_t)unpack * size);
            for (int i = 0, u = 0; i < n; ++i) {
                if (batch[i].buf->state_data != nullptr) {
                    ptrs_[i] = batch[i].buf->state_data;
                    continue;
                }
                float* dst = unpacked_.data() + (size_t)u++ * size;
                for (int j = 0; j < size; ++j) dst[j] = (float)((batch[i].bits[j >> 5] >> (j & 31)) & 1u);
                ptrs_[i] = dst;
            }
            cuda_->predict_raw(ptrs_.data(), n, size, slot.policy, slot.value);
        }
    } else {
        std::vector<std::vector<float>> states;
        states.reserve(n);
        for (const auto& p : batch) states.emplace_back(p.buf->state_data, p.buf->state_data + p.buf->state_size);
        slot.results = engine_->predict_batch(states);
        if ((int)slot.results.size() != n) throw std::runtime_error("engine returned a short batch");
    }
    engine_ns_.fetch_add((uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                             std::chrono::steady_clock::now() - t0)
                             .count());
}

void GpuEvaluator::hand_back(Slot& slot) {
    const auto t0 = std::chrono::steady_clock::now();
    const int n = (int)slot.batch.size();
    const size_t a = cuda_ != nullptr ? (size_t)cuda_->action_size() : 0;
    for (int i = 0; i < n; ++i) {
        NNResultBuf* buf = slot.batch[i].buf;
        std::lock_guard<std::mutex> lock(buf->mu);
        if (cuda_ != nullptr) {
            buf->policy.assign(slot.policy + i * a, slot.policy + (i + 1) * a);
            buf->value = slot.value[i];
        } else {
            buf->policy = std::move(slot.results[i].first);
            buf->value = slot.results[i].second;
        }
        buf->done = true;
        // Notify under the lock: once the client sees `done` it may return
        // and destroy its buffer (and condition variable).
        buf->cv.notify_one();
    }
    slot.batch.clear();
    slot.results.clear();
    scatter_ns_.fetch_add((uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                              std::chrono::steady_clock::now() - t0)
                              .count());
}

void GpuEvaluator::fail_batch(std::vector<Pending>& batch) {
    // Wake every client of the batch with an empty policy: each one turns
    // that into an exception on its own thread.
    for (const auto& p : batch) {
        NNResultBuf* buf = p.buf;
        std::lock_guard<std::mutex> lock(buf->mu);
        if (!buf->done) {
            buf->policy.clear();
            buf->value = std::numeric_limits<float>::quiet_NaN();
            buf->done = true;
            buf->cv.notify_one();
        }
    }
    batch.clear();
}

bool GpuEvaluator::submittable(const std::vector<Pending>& batch) const {
    if (cuda_ == nullptr || batch.empty() || (int)batch.size() > max_batch_ ||
        (int)batch.size() > cuda_->max_batch())
        return false;
    const int size = cuda_->input_channels * cuda_->board_size * cuda_->board_size;
    for (const auto& p : batch)
        if (p.bits == nullptr || p.buf->state_size != size) return false;
    return true;
}

void GpuEvaluator::server_loop() {
    std::vector<Pending> batch;
    batch.reserve(max_batch_);
    for (uint64_t k = 0;; ++k) {
        {
            std::unique_lock<std::mutex> lock(mu_);
            // The in-flight limit holds even while stopping (two pinned input
            // buffers); a stop only drops the wait for a full second batch.
            cv_.wait(lock, [&] {
                if (queue_.empty()) return stop_;
                if (in_flight_ >= max_in_flight_) return false;
                return in_flight_ == 0 || stop_ ||
                       queue_.size() >= std::min((size_t)max_batch_,
                                                 overlap_min_ > 0 ? overlap_min_ : last_batch_);
            });
            if (queue_.empty()) break;  // stopping, nothing left
            const int n = std::min((int)queue_.size(), max_batch_);
            batch.assign(queue_.begin(), queue_.begin() + n);
            queue_.erase(queue_.begin(), queue_.begin() + n);
            ++in_flight_;  // until the completion thread has waited for it
            last_batch_ = (size_t)n;
        }
        const int si = (int)(k % kSlots);
        Slot& slot = slots_[si];
        {
            // The completion thread may still be handing back the batch
            // that used this slot kSlots batches ago.
            std::unique_lock<std::mutex> lock(cmu_);
            ccv_.wait(lock, [&] { return !slot.busy; });
        }
        slot.batch.swap(batch);
        slot.ticket = -1;
        try {
            const int n = (int)slot.batch.size();
            if (submittable(slot.batch)) {
                reserve(slot, (size_t)max_batch_, (size_t)cuda_->action_size());
                const auto t0 = std::chrono::steady_clock::now();
                bit_ptrs_.resize(n);
                for (int i = 0; i < n; ++i) bit_ptrs_[i] = slot.batch[i].bits;
                slot.ticket = cuda_->submit_bits(bit_ptrs_.data(), n, slot.policy, slot.value);
                engine_ns_.fetch_add((uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                                         std::chrono::steady_clock::now() - t0)
                                         .count());
            } else {
                run_batch(slot);  // synchronous (fp32 planes, mixed or other engines)
            }
            batches_.fetch_add(1);
            positions_.fetch_add(n);
            int seen = largest_.load();
            while (n > seen && !largest_.compare_exchange_weak(seen, n)) {
            }
            {
                std::lock_guard<std::mutex> lock(cmu_);
                slot.busy = true;
                posted_.push_back(si);
            }
            ccv_.notify_all();
        } catch (const std::exception& ex) {
            failed_.fetch_add(1);
            {
                std::lock_guard<std::mutex> lock(mu_);
                last_error_ = ex.what();
                --in_flight_;
            }
            fail_batch(slot.batch);
        }
        batch.clear();
    }
    {
        std::lock_guard<std::mutex> lock(cmu_);
        done_ = true;
    }
    ccv_.notify_all();
}

void GpuEvaluator::completion_loop() {
    while (true) {
        int si;
        {
            std::unique_lock<std::mutex> lock(cmu_);
            ccv_.wait(lock, [this] { return !posted_.empty() || done_; });
            if (posted_.empty()) break;  // done_ and nothing left
            si = posted_.front();
            posted_.erase(posted_.begin());
        }
        Slot& slot = slots_[si];
        bool ok = true;
        if (slot.ticket >= 0) {
            // Submissions complete in order: wait for this one on the GPU.
            const auto t0 = std::chrono::steady_clock::now();
            try {
                cuda_->wait_submitted(slot.ticket);
            } catch (const std::exception& ex) {
                ok = false;
                failed_.fetch_add(1);
                std::lock_guard<std::mutex> lock(mu_);
                last_error_ = ex.what();
            }
            engine_ns_.fetch_add((uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                                     std::chrono::steady_clock::now() - t0)
                                     .count());
        }
        {
            // Its place in flight is free before the clients are woken, so
            // the server can submit the next batch meanwhile.
            std::lock_guard<std::mutex> lock(mu_);
            --in_flight_;
        }
        cv_.notify_all();
        if (ok) hand_back(slot);
        else fail_batch(slot.batch);
        {
            std::lock_guard<std::mutex> lock(cmu_);
            slot.busy = false;
        }
        ccv_.notify_all();
    }
}

// ---------------------------------------------------------------------------

namespace {
std::atomic<uint64_t> g_sharded_ids{1};
}

ShardedEvaluator::ShardedEvaluator(const std::vector<InferenceEngine*>& engines, int max_batch_size)
    : id_(g_sharded_ids.fetch_add(1)) {
    if (engines.empty()) throw std::invalid_argument("ShardedEvaluator: no engines");
    for (auto* e : engines) shards_.push_back(std::make_unique<GpuEvaluator>(e, max_batch_size));
}

std::unique_ptr<ShardedEvaluator> ShardedEvaluator::create_cuda(const std::string& model_path,
                                                                const std::vector<int>& devices,
                                                                int max_batch_size) {
    std::vector<std::unique_ptr<InferenceEngine>> owned;
    std::vector<InferenceEngine*> raw;
    for (int d : devices) {
        auto e = std::make_unique<CudaEngine>(d, CudaEngine::kBf16, false, max_batch_size);
        e->load_model(model_path);
        raw.push_back(e.get());
        owned.push_back(std::move(e));
    }
    auto s = std::make_unique<ShardedEvaluator>(raw, max_batch_size);
    s->owned_engines_ = std::move(owned);
    return s;
}

ShardedEvaluator::~ShardedEvaluator() {
    shards_.clear();  // servers stop before the engines they drive
    owned_engines_.clear();
}

int ShardedEvaluator::shard_of_this_thread() {
    thread_local std::unordered_map<uint64_t, int> assigned;
    auto it = assigned.find(id_);
    if (it != assigned.end()) return it->second;
    const int s = (int)(next_.fetch_add(1) % shards_.size());
    assigned.emplace(id_, s);
    return s;
}

BatchEvaluator::Result ShardedEvaluator::evaluate_with_buf(NNResultBuf& buf,
                                                          const std::vector<float>& state) {
    return shards_[shard_of_this_thread()]->evaluate_with_buf(buf, state);
}

void ShardedEvaluator::evaluate_packed(const uint32_t* words, int n_words, float* policy, float* value) {
    shards_[shard_of_this_thread()]->evaluate_packed(words, n_words, policy, value);
}

void ShardedEvaluator::evaluate_packed_group(const uint32_t* const* words, int n, int n_words,
                                             float* const* policies, float* values) {
    shards_[shard_of_this_thread()]->evaluate_packed_group(words, n, n_words, policies, values);
}

BatchEvaluator::Result ShardedEvaluator::evaluate_single(const std::vector<float>& state) {
    return shards_[shard_of_this_thread()]->evaluate_single(state);
}

std::vector<BatchEvaluator::Result> ShardedEvaluator::evaluate(
    const std::vector<std::vector<float>>& states) {
    const size_t n = states.size(), k = shards_.size();
    if (n == 0) return {};
    if (k == 1 || n == 1) return shards_[shard_of_this_thread()]->evaluate(states);
    std::vector<std::vector<Result>> parts(k);
    std::vector<std::string> errors(k);
    std::vector<std::thread> workers;
    for (size_t s = 0; s < k; ++s) {
        const size_t lo = n * s / k, hi = n * (s + 1) / k;
        if (lo == hi) continue;
        workers.emplace_back([&, s, lo, hi] {
            try {
                std::vector<std::vector<float>> slice(states.begin() + lo, states.begin() + hi);
                parts[s] = shards_[s]->evaluate(slice);
            } catch (const std::exception& ex) {
                errors[s] = ex.what();
            }
        });
    }
    for (auto& w : workers) w.join();
    for (auto& e : errors)
        if (!e.empty()) throw std::runtime_error(e);
    std::vector<Result> out;
    out.reserve(n);
    for (auto& p : parts)
        for (auto& r : p) out.push_back(std::move(r));
    return out;
}

}  // namespace minigo
