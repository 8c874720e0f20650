// Batching servers for the network evaluation path.
//
// GpuEvaluator is the reference's NNEvaluator (src/nn_evaluator.cpp:6-140)
// for one engine: search threads push an NNResultBuf, one server thread pops
// up to max_batch of them with no timeout or minimum (the batch size follows
// the number of concurrent search threads), runs one batched evaluation and
// wakes each client.  Three differences:
//   * a failed batch is reported to its clients: evaluate_with_buf /
//     evaluate / evaluate_single throw std::runtime_error on the calling
//     thread, where the reference returned an empty policy that the search
//     then indexed out of bounds (src/nn_evaluator.cpp:117-125,
//     src/mcts.cpp:59-64);
//   * with a CudaEngine, each client packs its own state's binary planes
//     into the bit-packed wire format (1/32 of the fp32 bytes) on its own
//     thread before queueing it, and the server only gathers those words
//     into the engine's pinned buffer: the reference's server thread copies
//     every 24.5 KB fp32 state twice (src/nn_evaluator.cpp:108-112 plus the
//     engine's flatten), and packing on the server thread alone took 60% of
//     its time at 19x19 with 1024 search threads;
//   * handing results back is pipelined with the next engine call: the
//     server thread forms batch k+1 and runs it on the engine while a
//     completion thread copies batch k's results into the clients' buffers
//     and wakes them (waking a sleeping client is a futex call of a few
//     microseconds, half the server's time at 19x19 batch 512 when it was
//     done inline);
//   * with a CudaEngine, bit-packed batches are submitted without waiting
//     (CudaEngine::submit_bits): the server gathers and submits the next
//     batch while the GPU still computes the previous one, so the GPU does
//     not idle through each batch's gather, copies and synchronisation.  A
//     second batch is submitted while one is in flight only once at least
//     as many requests are queued as that batch holds, so batches do not
//     shrink (else the server waits for the GPU, then takes whatever is
//     queued, as the reference's server does); the completion thread waits
//     for each submission in order, frees its place in flight, then wakes
//     its clients.  Measured on 2 GPUs with 24 host threads, FastSearch
//     self-play 697k -> 763k visits/s;
//   * a client is woken while its buffer's mutex is held: the reference
//     notifies after unlocking (src/nn_evaluator.cpp:127-137), so a client
//     that sees `done` can return and destroy its stack NNResultBuf while
//     notify_one still runs on its condition variable (found by
//     ThreadSanitizer in this repository's tests).
//
// ShardedEvaluator runs one GpuEvaluator per GPU (weights replicated, no
// collective) and assigns each search thread to one of them round-robin on
// its first call, so the MCTS code (src/mcts.cpp) uses it unchanged through
// the BatchEvaluator interface.
#pragma once

#include "minigo_api.h"
#include "packed_evaluator.h"

#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace minigo {

class CudaEngine;

class GpuEvaluator : public BatchEvaluator, public mgb::PackedEvaluator {
public:
    GpuEvaluator(InferenceEngine* engine, int max_batch_size);
    ~GpuEvaluator() override;
    GpuEvaluator(const GpuEvaluator&) = delete;
    GpuEvaluator& operator=(const GpuEvaluator&) = delete;

    std::vector<Result> evaluate(const std::vector<std::vector<float>>& states) override;
    Result evaluate_with_buf(NNResultBuf& buf, const std::vector<float>& state) override;
    Result evaluate_single(const std::vector<float>& state) override;
    // A position already in the bit-packed wire format (CudaEngine only):
    // queued like evaluate_with_buf, with no fp32 planes at all.
    void evaluate_packed(const uint32_t* words, int n_words, float* policy, float* value) override;
    // A group of packed positions queued together (one lock, one wake-up of
    // the server); the calling thread sleeps once for the whole group.
    void evaluate_packed_group(const uint32_t* const* words, int n, int n_words,
                               float* const* policies, float* values) override;

    // Counters (for batching statistics and tests).
    uint64_t batches() const { return batches_.load(); }
    uint64_t positions() const { return positions_.load(); }
    int largest_batch() const { return largest_.load(); }
    uint64_t failed_batches() const { return failed_.load(); }
    // Time (ns) in the engine call (server thread: gather, H2D, forward,
    // D2H) and in handing results back to the clients (completion thread:
    // copy + wake-up).
    uint64_t engine_ns() const { return engine_ns_.load(); }
    uint64_t scatter_ns() const { return scatter_ns_.load(); }

private:
    // A queued request: the client's buffer and, with a CudaEngine, its
    // state packed to bits (null if it is not binary).
    struct Pending {
        NNResultBuf* buf;
        const uint32_t* bits;
    };
    // One batch between the server and the completion thread.
    struct Slot {
        std::vector<Pending> batch;
        // CudaEngine results, flat, in page-locked memory (mg_host_alloc)
        // so that the engine's result copies are direct DMA; grown on demand.
        float* policy = nullptr;
        float* value = nullptr;
        size_t capacity = 0;               // positions policy / value hold
        std::vector<Result> results;       // other engines' results
        bool busy = false;                 // posted, not yet handed back
        int ticket = -1;                   // submitted without waiting (CudaEngine), else -1
    };
    static constexpr int kSlots = 4;       // in flight (2), being handed back, being formed
    // Batches submitted and not yet waited for (1 or 2; MG_EVAL_IN_FLIGHT),
    // and the queued requests that let a second one go in flight
    // (MG_EVAL_OVERLAP_MIN; 0, the default, means the size of the batch in
    // flight).
    int max_in_flight_ = 2;
    size_t overlap_min_ = 0;
    size_t last_batch_ = 1;  // size of the last batch taken (guarded by mu_)
    // True if this batch goes to the engine as a submission (bit-packed,
    // CudaEngine, one chunk).
    bool submittable(const std::vector<Pending>& batch) const;
    static void reserve(Slot& slot, size_t n, size_t actions);
    void server_loop();
    void completion_loop();
    void run_batch(Slot& slot);
    void hand_back(Slot& slot);
    void fail_batch(std::vector<Pending>& batch);
    void enqueue(const Pending* items, size_t n);
    Result take_result(NNResultBuf& buf);

    InferenceEngine* engine_;
    CudaEngine* cuda_;  // engine_ when it is a CudaEngine, else null
    int max_batch_;

    std::mutex mu_;
    std::condition_variable cv_;
    std::vector<Pending> queue_;
    bool stop_ = false;
    std::string last_error_;  // guarded by mu_

    std::vector<const float*> ptrs_;
    std::vector<const uint32_t*> bit_ptrs_;
    std::vector<float> unpacked_;  // fp32 planes of packed-only requests in a mixed batch

    Slot slots_[kSlots];
    int in_flight_ = 0;  // submitted batches not yet waited for (guarded by mu_)
    std::mutex cmu_;  // guards slots_[*].busy, posted_, done_
    std::condition_variable ccv_;
    std::vector<int> posted_;  // slots waiting for the completion thread
    bool done_ = false;        // the server has exited

    std::atomic<uint64_t> batches_{0}, positions_{0}, failed_{0};
    std::atomic<uint64_t> engine_ns_{0}, scatter_ns_{0};
    std::atomic<int> largest_{0};
    std::thread server_, completer_;
};

class ShardedEvaluator : public BatchEvaluator, public mgb::PackedEvaluator {
public:
    // One GpuEvaluator per engine (the engines stay owned by the caller).
    ShardedEvaluator(const std::vector<InferenceEngine*>& engines, int max_batch_size);

    // Owning convenience: one CudaEngine per device, all loading model_path.
    static std::unique_ptr<ShardedEvaluator> create_cuda(const std::string& model_path,
                                                         const std::vector<int>& devices,
                                                         int max_batch_size);

    ~ShardedEvaluator() override;

    // Splits the batch into contiguous slices, one per shard, evaluated
    // concurrently; results keep the input order.
    std::vector<Result> evaluate(const std::vector<std::vector<float>>& states) override;
    // Routed to the calling thread's shard.
    Result evaluate_with_buf(NNResultBuf& buf, const std::vector<float>& state) override;
    Result evaluate_single(const std::vector<float>& state) override;
    void evaluate_packed(const uint32_t* words, int n_words, float* policy, float* value) override;
    void evaluate_packed_group(const uint32_t* const* words, int n, int n_words,
                               float* const* policies, float* values) override;

    size_t shards() const { return shards_.size(); }
    GpuEvaluator& shard(size_t i) { return *shards_[i]; }
    // Shard the calling thread is assigned to (assigning it on first use).
    int shard_of_this_thread();

private:
    std::vector<std::unique_ptr<InferenceEngine>> owned_engines_;
    std::vector<std::unique_ptr<GpuEvaluator>> shards_;
    std::atomic<uint32_t> next_{0};
    uint64_t id_;
};

}  // namespace minigo
