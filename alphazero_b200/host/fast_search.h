// Multi-threaded MCTS for self-play over a PackedEvaluator.
//
// The search algorithm is the reference's (src/mcts.cpp:126-325,
// include/mcts.h): PUCT selection with virtual loss, one playout per search
// thread at a time, a node claimed for expansion by a compare-and-swap
// (UNEVALUATED -> EXPANDING), collisions with a node another thread is
// evaluating revert their virtual losses and retry without counting, the
// policy masked to the legal moves and renormalised, Dirichlet noise at the
// root, terminal positions valued by the winner, backup with alternating
// sign.  Selection, masking and backup use the same float expressions in the
// same order, so a single-threaded search without noise visits exactly what
// the reference's does (tested).
//
// What differs is the cost per visit, which bounds end-to-end self-play on
// the host:
//   * a node's children are one array of the legal moves only, carved at
//     expansion out of the expanding thread's node arena, which is reset
//     once per search and keeps its memory (the reference makes one heap
//     node per legal move, frees the tree after every move, and scans all
//     board^2 + 1 slots on every selection);
//   * the square root of the parent's visits is taken once per selection,
//     not once per child;
//   * positions are encoded straight to the bit-packed wire format (768
//     bytes at 19x19) and evaluated through PackedEvaluator, instead of a
//     24.5 KB fp32 encode that the evaluator then packs;
//   * the search threads are a pool kept for the searcher's lifetime (the
//     reference creates and joins num_search_threads - 1 threads per move,
//     src/mcts.cpp:284-319).
#pragma once

#include "go_positions.h"
#include "packed_evaluator.h"

#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <exception>
#include <memory>
#include <mutex>
#include <random>
#include <thread>
#include <vector>

namespace mgb {

struct SearchParams {
    int simulations = 800;          // Config::num_simulations
    float c_puct = 1.5f;            // Config::c_puct
    float dirichlet_alpha = 0.03f;  // Config::dirichlet_alpha
    float dirichlet_epsilon = 0.25f;
    int threads = 16;               // Config::num_search_threads
    // false: `threads` search threads (a pool), as the reference runs them.
    // true: the same number of concurrent playouts as one group on the
    // calling thread: each round selects up to `threads` leaves with virtual
    // loss (a leaf already in the round ends the round early), evaluates
    // them through one evaluate_packed_group call, then expands them and
    // backs them up.  The arithmetic is the same; what changes is that a
    // round's playouts start together, and the host pays one sleep and one
    // wake-up per round instead of one per playout.
    bool grouped = false;
};

class FastSearch {
public:
    FastSearch(PackedEvaluator* evaluator, int board_size, const SearchParams& params,
               uint64_t seed);
    ~FastSearch();
    FastSearch(const FastSearch&) = delete;
    FastSearch& operator=(const FastSearch&) = delete;

    // MCTS::search: runs params.simulations playouts from `pos`; visits[a]
    // = visit count of root action a (board^2 + 1 entries).
    void search(const GoPosition& pos, std::vector<float>& visits, bool add_noise);

    // MCTS::get_action (src/mcts.cpp:327-359): search, then the most visited
    // action at temperature 0, else a draw from visits^(1/temperature).
    int get_action(const GoPosition& pos, std::vector<float>& policy, float temperature,
                   bool add_noise);

    uint64_t playouts() const { return playouts_.load(std::memory_order_relaxed); }

    struct Node;

private:
    // Bump allocator of child arrays, one per search thread: blocks are
    // kept across searches and reused from the start of each search.
    struct Arena {
        std::vector<std::unique_ptr<unsigned char[]>> blocks;
        size_t block = 0, used = 0;
        Node* take(int n);
        void reset() { block = used = 0; }
    };

    void worker_loop(int tid);
    void playouts_from_root(int tid);
    void grouped_playouts();
    Node* select_child(Node* node) const;
    void expand(Node* node, float* policy, const uint8_t* legal, Arena& arena);
    void backup(std::vector<Node*>& path, float value);
    static void revert(std::vector<Node*>& path);
    void add_dirichlet_noise(Node* root);

    PackedEvaluator* evaluator_;
    int board_, actions_, words_;
    SearchParams params_;
    std::mt19937 rng_;

    // The current search, shared with the pool.
    const GoPosition* pos_ = nullptr;
    Node* root_ = nullptr;
    std::atomic<int> sims_done_{0};
    std::atomic<uint64_t> playouts_{0};

    std::mutex mu_;
    std::condition_variable cv_;
    uint64_t generation_ = 0;  // one per search
    int finished_ = 0;         // pool threads done with the current search
    bool stop_ = false;
    std::exception_ptr error_;  // first evaluation failure of the current search
    std::vector<Arena> arenas_;  // [0] the caller's thread, [1 + i] pool thread i
    std::vector<std::thread> pool_;

    // Per-member storage of a grouped round (grouped mode only).
    struct Group {
        std::vector<std::vector<Node*>> paths;
        std::vector<Node*> leaves;
        std::vector<uint32_t> words;
        std::vector<float> policy, values;
        std::vector<uint8_t> legal;
        std::vector<const uint32_t*> word_ptrs;
        std::vector<float*> policy_ptrs;
    } group_;
};

}  // namespace mgb
